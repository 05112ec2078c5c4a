/* glypr_cuda.h — C ABI of libglypr_cuda.so, the B200 (sm_100a) backend for glypr's
 * EmbeddingGemma text path: token ids -> 24-layer encoder (Q8_0 or BF16 weights) -> masked
 * mean-pool -> dense head -> L2 -> Matryoshka truncation.
 *
 * Conventions (mirroring glypr-core, crates/glypr-core/src):
 *   - every function returns an int status, GLP_OK (0) on success; on failure no partial
 *     output is written and glp_last_error() returns a message for the calling thread
 *     (anyhow/candle errors in the reference, e.g. lib.rs:970-976, model.rs:500-506);
 *   - the caller owns all buffers it passes; the context owns the weights (immutable after
 *     glp_open, like EmbeddingGemma2Model in model.rs:14-26);
 *   - one host thread at a time may call into a given context (the reference drives one
 *     embedder from one worker thread, glypr-server/src/engine.rs:216-253); internally a
 *     context runs one worker thread per device.
 *   - pointers named d_* are device pointers on the context's device `dev_index`; functions
 *     taking a `stream` (a cudaStream_t, NULL = legacy default stream) are stream-ordered
 *     and return before the work completes.
 */
#ifndef GLYPR_CUDA_H_
#define GLYPR_CUDA_H_

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLP_OK 0
#define GLP_ERR_INVALID_ARG 1
#define GLP_ERR_IO 2
#define GLP_ERR_FORMAT 3
#define GLP_ERR_UNSUPPORTED 4
#define GLP_ERR_CUDA 5
#define GLP_ERR_OOM 6
#define GLP_ERR_DEVICE 7        /* a kernel's bounded wait expired (device status word) */
#define GLP_ERR_CONTEXT_LIMIT 8 /* sequence longer than the model's context_length */

#define GLP_MAX_DEVICES 16

typedef struct glp_ctx glp_ctx;

typedef struct glp_options {
  int64_t max_batch_tokens; /* tokens per device launch chunk; 0 = 262144 */
  int max_batch_seqs;       /* sequences per chunk; 0 = 4096 */
  int device_memory_limit_mib; /* device memory the context may take on each device; 0 = no limit.
                                * glp_open fails with GLP_ERR_OOM before touching any device when
                                * the model's plan (weights, RoPE tables, one launch chunk, load
                                * staging) exceeds it; later growth of the host-API staging
                                * buffers past it fails the same way */
  int reserved[5];
} glp_options;

typedef struct glp_model_info_t {
  int n_layers, hidden, ffn, n_heads, n_kv_heads, head_dim, vocab;
  int embedding_dim;  /* embedding_length_out */
  int max_position;   /* context_length */
  int sliding_window; /* 512, fixed as in config.rs:191 */
  int weight_type;    /* ggml type id of the linears: 8 = Q8_0, 30 = BF16 */
  int n_devices;
  int64_t device_bytes; /* device memory the context holds on its first device (bytes requested) */
} glp_model_info_t;

typedef struct glp_timing {
  int n_devices;
  float device_ms[GLP_MAX_DEVICES]; /* per device: CUDA events from first H2D to last D2H */
} glp_timing;

/* Parse a GGUF file with glypr's key/tensor schema (config.rs:76-213, model.rs:244-488)
 * and upload one weight replica to each listed device.  Replaces
 * GlyprEmbedder::load_gguf / load_gguf_q8 (lib.rs:176-229). */
int glp_open(const char* gguf_path, const int* device_ids, int n_devices, const glp_options* opt,
             glp_ctx** out);

/* Release every device allocation of the context.  NULL is a no-op. */
void glp_close(glp_ctx* ctx);

/* Thread-local message of the last failed call on this thread ("" if none). */
const char* glp_last_error(void);

/* Model hyperparameters as parsed from the GGUF (TextConfig, config.rs:8-60). */
int glp_model_info(const glp_ctx* ctx, glp_model_info_t* info);

/* Embed a right-padded batch of token ids: ids [n_seq * max_len] (pad id ignored),
 * lengths [n_seq].  Writes out [n_seq * out_dim] f32, L2-normalised; out_dim < embedding_dim
 * applies Matryoshka truncation + renormalisation.  Host buffers; sequences are sharded
 * across the context's devices in contiguous ranges balanced by token count.
 * Replaces EmbeddingGemma2Model::forward + pool_and_normalize (model.rs:498-510, 654-705)
 * as driven by GlyprEmbedder::embed_batch / profile_encode_batch (lib.rs:731-952, 994-1068).
 * Errors: lengths[i] > context_length -> GLP_ERR_CONTEXT_LIMIT ("exceeds model
 * max_position_embeddings", model.rs:500-506); ids outside [0, vocab) -> GLP_ERR_INVALID_ARG. */
int glp_embed_tokens(glp_ctx* ctx, const int32_t* ids, const int32_t* lengths, int n_seq, int max_len,
                     int out_dim, float* out, glp_timing* timing);

/* The sharding of glp_embed_tokens over caller-supplied executors instead of the context's
 * devices (other backends; the host tests drive the coordinator through it without a GPU):
 * contiguous shards balanced by token count, one host thread per executor, executor i gets
 * shard i as a right-padded batch (glp_batch_fn, declared below).  The embeddings reach `out`
 * only when every executor has succeeded; otherwise `out` is untouched and the first failing
 * executor's status is returned ("executor i: <its message>").  No counterpart function in the
 * reference, whose embed_batch runs one device (lib.rs:731-952); its server fails every request
 * of a failed batch and returns no partial result (glypr-server/src/engine.rs:308-325). */
typedef int (*glp_batch_fn)(void* user, const int32_t* ids, const int32_t* lengths, int n_seq, int max_len,
                            int out_dim, float* out);
int glp_embed_tokens_sharded(const glp_batch_fn* fns, void* const* users, int n_executors, int embedding_dim,
                             const int32_t* ids, const int32_t* lengths, int n_seq, int max_len, int out_dim,
                             float* out);

/* Device-resident variant on one device: d_ids = packed valid tokens of all sequences,
 * d_cu_seqlens [n_seq + 1] device offsets into d_ids, h_cu_seqlens the same offsets on the
 * host (used to cut launch chunks); d_out [n_seq * out_dim] f32.  Stream-ordered; the ids
 * are not range-checked (the host variant checks them). */
int glp_embed_packed_device(glp_ctx* ctx, int dev_index, const int32_t* d_ids, const int32_t* d_cu_seqlens,
                            const int32_t* h_cu_seqlens, int n_seq, int out_dim, float* d_out, void* stream);

/* Status word of the device kernels' bounded waits on device dev_index (0 = none); a
 * non-zero value is also reported by the next glp_embed_* call as GLP_ERR_DEVICE. */
int glp_device_status(glp_ctx* ctx, int dev_index, int* status);

/* What a device status code means (static string; codes as glp_device_status and
 * glp_kernel_status report them; unknown codes have a text too).  No reference counterpart
 * (candle reports device errors as strings). */
const char* glp_status_text(int status);

/* ---- per-kernel profiling (the reference's forward_profiled, profile.rs:55-430, done with
 * CUDA events on the launching stream instead of wall clock + device sync) ---- */

#define GLP_PROFILE_KINDS 14

typedef struct glp_profile {
  int n_kinds;
  const char* names[GLP_PROFILE_KINDS]; /* static strings owned by the library */
  int64_t launches[GLP_PROFILE_KINDS];  /* kernel launches per kind since the last read */
  double total_ms[GLP_PROFILE_KINDS];   /* summed event time (0 unless timing is enabled) */
  double flops[GLP_PROFILE_KINDS];      /* algorithmic FLOPs summed over the launches */
  double bytes[GLP_PROFILE_KINDS];      /* algorithmic HBM bytes summed over the launches */
  int64_t total_launches;
} glp_profile;

/* enable = 1: bracket every kernel launch on device dev_index with CUDA events; 0: only
 * count launches.  Resets the counters either way. */
int glp_profile_enable(glp_ctx* ctx, int dev_index, int enable);

/* Synchronise the recorded events and return the per-kind totals since the last
 * enable/read, then reset them. */
int glp_profile_read(glp_ctx* ctx, int dev_index, glp_profile* out);

/* ---- dynamic-batching engine (glypr-server's inference engine, engine.rs:157-325) ---- */

typedef struct glp_engine glp_engine;

/* A batch executor (glp_batch_fn, declared above): embed n_seq right-padded sequences (ids
 * [n_seq * max_len], lengths [n_seq]) into out [n_seq * out_dim] f32; returns GLP_OK or an
 * error status. */

/* Start an engine over a model context: one worker thread forms batches of up to max_batch
 * requests as the reference's worker does (block for the first, drain what is pending, yield
 * once, drain again; engine.rs:216-245) and runs each through glp_embed_tokens, which shards
 * it across the context's devices.  queue_capacity bounds the waiting requests (0 = 1024,
 * the reference's channel size).  While the engine runs, it is the context's only caller. */
int glp_engine_create(glp_ctx* ctx, int max_batch, int queue_capacity, glp_engine** out);

/* The same engine over a caller-supplied executor of width embedding_dim (other backends;
 * the host tests drive the batching logic through it). */
int glp_engine_create_with_executor(glp_batch_fn fn, void* user, int embedding_dim, int max_batch,
                                    int queue_capacity, glp_engine** out);

/* Embed one sequence of len token ids through the engine; blocks until its batch is done and
 * may be called from any number of threads at once (EngineHandle::embed, engine.rs:120-150).
 * truncate_dim in (0, embedding_dim) returns the Matryoshka truncation (first truncate_dim
 * values renormalised, util.rs:6-29) in out [truncate_dim]; 0 (or >= embedding_dim) the full
 * out [embedding_dim].  A failed batch fails each of its requests ("Batch inference error:
 * ..."); after glp_engine_destroy has begun, calls fail with "Inference worker is not
 * running". */
int glp_engine_embed(glp_engine* e, const int32_t* ids, int len, int truncate_dim, float* out);

/* Requests answered, batches run and the largest batch so far. */
int glp_engine_stats(glp_engine* e, int64_t* requests, int64_t* batches, int* largest_batch);

/* Answer every queued request, stop the worker and free the engine (NULL is a no-op).  No
 * call may use the engine after this returns. */
void glp_engine_destroy(glp_engine* e);

/* ---- text front end: GGUF tokenizer and task prompts (tokenizer.rs, task.rs) ---- */

typedef struct glp_tokenizer glp_tokenizer;

/* Sequence forms of a text (token ids 0 = pad, 1 = EOS, 2 = BOS, tokenizer.rs:588-590). */
#define GLP_TOKENS_BARE 0     /* the BPE ids alone (Tokenizer::encode on the text) */
#define GLP_TOKENS_SINGLE 1   /* BOS + ids + EOS, BOS only when the first id is not 2 and EOS only
                               * when the last is not 1: GlyprTokenizer::encode (tokenizer.rs:162-177),
                               * the single-text path (embed_text / embed_query, lib.rs:967-968) */
#define GLP_TOKENS_SEQUENCE 2 /* BOS + ids + EOS always: encode_modality_sequence for a text part
                               * (tokenizer.rs:454-566), the batch and server path (lib.rs:833) */
#define GLP_DEFAULT_MAX_SEQ_LEN 8320 /* DEFAULT_MAX_SEQ_LEN = 8192 + 128 (lib.rs:47) */

/* The tokenizer GlyprTokenizer::from_gguf_metadata builds (tokenizer.rs:77-138) from the
 * GGUF's tokenizer.ggml.tokens and tokenizer.ggml.merges: BPE with byte fallback and fused
 * "<unk>", spaces normalised to U+2581.  Errors: a missing key or a non-array value
 * (GLP_ERR_FORMAT, the reference's messages), a merge whose parts or concatenation are not
 * tokens ("BPE build error: Token `x` out of vocabulary"). */
int glp_tokenizer_from_gguf(const char* gguf_path, glp_tokenizer** out);

/* The same from in-memory arrays (NUL-terminated UTF-8 tokens; merges as "left right"). */
int glp_tokenizer_from_vocab(const char* const* tokens, int n_tokens, const char* const* merges, int n_merges,
                             glp_tokenizer** out);

void glp_tokenizer_free(glp_tokenizer* tok);

/* Vocabulary entries and merges in use. */
int glp_tokenizer_info(const glp_tokenizer* tok, int* n_tokens, int* n_merges);

/* Token ids of one UTF-8 text in a GLP_TOKENS_* form into ids[cap]; *n_ids = the count (also
 * when the buffer is too small, which fails with GLP_ERR_INVALID_ARG).  A form never yields
 * more than 3 * text_len + 2 ids (a space with no token falls back to the 3 bytes of
 * U+2581).  A character with no token, no byte tokens and no "<unk>" fails with
 * "Encode error: Unk token `<unk>` not found in the vocabulary". */
int glp_tokenize(const glp_tokenizer* tok, const char* text, size_t text_len, int form, int32_t* ids, int cap,
                 int* n_ids);

/* A batch of texts tokenised on n_threads host threads (0 = all cores), packed back to back:
 * text i's ids are ids[offsets[i] .. offsets[i+1]) (offsets [n_texts + 1]).  ids_cap =
 * 3 * sum(text_lens) + 2 * n_texts always suffices.  limit > 0 fails the first text (in order)
 * with more ids with GLP_ERR_CONTEXT_LIMIT ("Batch item i sequence length (n tokens) exceeds
 * maximum context limit (limit tokens)", encode_batch_padded_with_limit, tokenizer.rs:182-222);
 * an empty batch fails with "Cannot encode an empty batch". */
int glp_tokenize_batch(const glp_tokenizer* tok, const char* const* texts, const size_t* text_lens, int n_texts,
                       int form, int limit, int n_threads, int32_t* ids, size_t ids_cap, int64_t* offsets);

/* Prompt formatting into out[cap] (NUL-terminated; *n_out = the length without the NUL, also
 * when out is too small).  glp_format_query: the task's prompt from GlyprTokenizer's table,
 * else "task: <task lowercased> | query: " (tokenizer.rs:13-64, 144-152); glp_format_document:
 * "title: <title or none> | text: " (tokenizer.rs:154-160); glp_task_format:
 * Task::from_name_and_title(task, title).format_text(text) (task.rs:21-73), task NULL = Raw. */
int glp_format_query(const char* query, size_t query_len, const char* task, char* out, size_t cap, size_t* n_out);
int glp_format_document(const char* content, size_t content_len, const char* title, char* out, size_t cap,
                        size_t* n_out);
int glp_task_format(const char* task, const char* title, const char* text, size_t text_len, char* out, size_t cap,
                    size_t* n_out);

/* Texts -> embeddings: tokenise in `form` (GLP_TOKENS_SINGLE for the reference's single-text
 * calls, GLP_TOKENS_SEQUENCE for its batch calls), check max_seq_len (0 = 8320) with the
 * reference's message for that path (lib.rs:969-976, 837-844, 551-558), then glp_embed_tokens.
 * Texts are embedded as given: apply the prompt formatters first. */
int glp_embed_texts(glp_ctx* ctx, const glp_tokenizer* tok, const char* const* texts, const size_t* text_lens,
                    int n_texts, int form, int max_seq_len, int out_dim, float* out);

/* One text request through the engine, as the server's text items go (handlers.rs:88-92,
 * engine.rs:296-325): Task::from_name_and_title(task, title) formats it (task NULL = Raw),
 * GLP_TOKENS_SEQUENCE tokenises it on the calling thread, then glp_engine_embed.  Longer than
 * 8320 ids: GLP_ERR_CONTEXT_LIMIT before it is queued. */
int glp_engine_embed_text(glp_engine* e, const glp_tokenizer* tok, const char* text, size_t text_len, const char* task,
                          const char* title, int truncate_dim, float* out);

/* ---- kernel-level entry points (microbenchmarks and tests; current device) ---- */

/* Bit-exact Q8_0 dequantisation: out[32*b + j] = f32(d_b) * q_b[j] for n_blocks 34-byte
 * blocks {fp16 d; int8 qs[32]} (ggml block_q8_0; metal_kernels/fused_ops.metal:568-581,
 * candle QTensor::dequantize used at model.rs:35-36). */
int glp_q8_0_dequant(const void* d_blocks, int64_t n_blocks, float* d_out, void* stream);

/* y[M, N] = x[M, K] (bf16, row-major) * dequant(W[N, K])^T, W as raw Q8_0 rows of K/32
 * blocks; y f32 (y_is_f32 = 1) or bf16.  K % 64 == 0, N % 128 == 0.  The Q8_0 matmul behind
 * LinearOp::forward (linear.rs:150-172; Metal fused_metal_q8_0_matmul,
 * metal_kernels/mod.rs:1271-1394).  Up to M = 8192 (and for a 16-byte aligned W) one launch
 * streams the raw rows by TMA and dequantises them in shared memory in front of the tcgen05
 * MMA; for larger M, where that measures slower, W is dequantised into a context-free scratch
 * buffer owned by the library (cached per device) and the bf16 tcgen05 GEMM runs. */
int glp_q8_0_gemm(const void* d_q8_w, int N, int K, const void* d_x_bf16, int M, void* d_y, int y_is_f32,
                  void* stream);

/* The Q8_0 GEMM above for callers that cannot allocate device memory (no counterpart in the
 * reference): code running where cudaMalloc is unavailable or must not be called, such as
 * inside a host callback, under a caller-owned memory pool or fixed memory budget, or from a
 * framework that forbids allocations after start-up.  The dequantised weight goes into a
 * fixed scratch array inside the library (6 MiB per GPU that loads the library, held until
 * the process exits), so N * K must be at most 3,145,728; larger weights are rejected with
 * GLP_ERR_INVALID_ARG.  The call allocates nothing and frees nothing.  The first call on a
 * device looks up the array's device address; make that first call before any stream
 * capture.  All calls on a device share the array: calls that overlap on the GPU (other
 * streams, other host threads) race on it.  Each call overwrites every scratch element it
 * reads, so nothing needs to be cleared between calls.  A bounded wait that expired inside its
 * kernel is reported by glp_kernel_status (which reads the call's status word with symbol
 * copies, allocating nothing). */
int glp_q8_0_gemm_noalloc(const void* d_q8_w, int N, int K, const void* d_x_bf16, int M, void* d_y, int y_is_f32,
                          void* stream);

/* Status of the kernel-level entry points above and below (glp_q8_0_gemm, glp_bf16_gemm,
 * glp_flash_attention, glp_q8_0_gemm_noalloc and the fused-epilogue GEMMs) on CUDA device
 * `device`: they are stream-ordered and return before their kernels run, so a kernel whose
 * bounded wait expired (its output then undefined) is reported here.  Synchronises the device,
 * then reads and clears the status words of these entry points: *status = the code recorded
 * since the last read (0 = none), and a recorded code returns GLP_ERR_DEVICE with
 * glp_status_text(code) in glp_last_error().  Allocates nothing (the no-allocation entry
 * point's word is read with symbol copies).  The model path (glp_embed_*) has its own word per
 * context: glp_device_status. */
int glp_kernel_status(int device, int* status);

/* Failure-detection self-test on CUDA device `device`: one kernel waits, with the bounded wait
 * every pipeline kernel uses, on a barrier nobody arrives at; after limit_us microseconds
 * (at most 2,000,000) the wait gives up, records status 6 in the kernel-level word and the
 * kernel returns normally.  Returns GLP_OK once the kernel has finished; glp_kernel_status then
 * reports GLP_ERR_DEVICE with status 6, and the device stays usable.  No reference counterpart. */
int glp_selftest_wait_timeout(int device, int limit_us);

/* Same GEMM on an already dequantised bf16 weight [N, K] (the model path's layout). */
int glp_bf16_gemm(const void* d_w_bf16, int N, int K, const void* d_x_bf16, int M, void* d_y, int y_is_f32,
                  void* stream);

/* The MLP's gate/up projection with the GeGLU in its epilogue (MLP::forward, mlp.rs:31-70;
 * cpu_simd/geglu.rs:6-18 with its +-10 clamp): out[M, F] = gelu_tanh(x Wg^T) * (x Wu^T), x f16
 * [M, K], Wg and Wu f16 [F, K], out f16; F % 128 == 0, K % 64 == 0.  Each call interleaves the
 * two weights per 128 rows into library scratch (cached per device; the model path does that
 * once at load), then runs the fused GEMM. */
int glp_gate_up_geglu(const void* d_w_gate, const void* d_w_up, int F, int K, const void* d_x, int M, void* d_out,
                      void* stream);

/* The attention block's QKV projection with the per-head norms and RoPE in its epilogue
 * (SelfAttention::forward, attention/mod.rs:166-213; rope.rs:14-106): y = x Wqkv^T over
 * (Hq + 2 Hkv) heads of 256, then per head RMSNorm (eps; gain q_gain on query heads, k_gain on
 * key heads, none on value heads) and NeoX RoPE at positions pos[M] with base theta on the
 * query and key heads.  x f16 [M, K], Wqkv f16 [(Hq + 2 Hkv) * 256, K] (q, then k, then v rows),
 * gains f32 [256] (16-byte aligned), out f16 [M, (Hq + 2 Hkv) * 256]; positions must lie in
 * [0, max_pos).  The cos/sin table for (theta, max_pos) is built once per device (rope.rs
 * values) and kept until the process exits. */
int glp_qkv_norm_rope(const void* d_w_qkv, int n_q_heads, int n_kv_heads, int K, const void* d_x, int M,
                      const float* d_q_gain, const float* d_k_gain, const int32_t* d_pos, double theta, int max_pos,
                      float eps, void* d_out, void* stream);

/* Flash attention over packed qkv (f16 [T, (Hq + 2 Hkv) * 256], per-head normed + RoPE'd)
 * for n_seq sequences at d_cu_seqlens; window > 0 applies |i - j| <= window.  Writes
 * d_out f16 [T, Hq * 256].  The AttentionBackend::compute_attention seam
 * (attention/traits.rs:37-46, AttentionMode::CudaFlash at attention/mod.rs:255-262). */
int glp_flash_attention(const void* d_qkv, const int32_t* d_cu_seqlens, int n_seq, int max_len, int n_q_heads,
                        int n_kv_heads, int head_dim, int window, void* d_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GLYPR_CUDA_H_ */
