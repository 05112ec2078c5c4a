"""Host-side mirror of glypr-core's embedder API over ``libglypr_cuda.so`` (ctypes).

Names and behaviour follow the reference facade (crates/glypr-core/src/lib.rs):
``GlyprEmbedder.load_gguf`` / ``load_gguf_q8`` (lib.rs:176-229), ``embed_batch`` on token-id
inputs (lib.rs:731-952), ``truncate_mrl`` / ``l2_normalize`` / ``cosine_similarity``
(util.rs:6-41).  Errors surface as :class:`GlyprError` carrying the library's message (the
reference's ``anyhow`` errors, e.g. "exceeds model max_position_embeddings",
model.rs:500-506).

There is no CPU fallback: if the CUDA library cannot be loaded or no GPU is visible, the
calls fail loudly.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import List, Optional, Sequence, Union

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_NAME = "libglypr_cuda.so"

GLP_OK = 0
GLP_ERR_INVALID_ARG = 1
GLP_ERR_IO = 2
GLP_ERR_FORMAT = 3
GLP_ERR_UNSUPPORTED = 4
GLP_ERR_CUDA = 5
GLP_ERR_OOM = 6
GLP_ERR_DEVICE = 7
GLP_ERR_CONTEXT_LIMIT = 8
GLP_MAX_DEVICES = 16

GLP_PROFILE_KINDS = 14

# Every symbol include/glypr_cuda.h declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "glp_open", "glp_close", "glp_last_error", "glp_model_info", "glp_embed_tokens",
    "glp_embed_packed_device", "glp_device_status", "glp_profile_enable", "glp_profile_read",
    "glp_q8_0_dequant", "glp_q8_0_gemm", "glp_q8_0_gemm_noalloc", "glp_bf16_gemm", "glp_flash_attention",
    "glp_engine_create", "glp_engine_create_with_executor", "glp_engine_embed", "glp_engine_stats",
    "glp_engine_destroy", "glp_tokenizer_from_gguf", "glp_tokenizer_from_vocab", "glp_tokenizer_free",
    "glp_tokenizer_info", "glp_tokenize", "glp_tokenize_batch", "glp_format_query", "glp_format_document",
    "glp_task_format", "glp_embed_texts", "glp_engine_embed_text", "glp_embed_tokens_sharded",
    "glp_kernel_status", "glp_status_text", "glp_selftest_wait_timeout", "glp_gate_up_geglu",
    "glp_qkv_norm_rope",
)

# sequence forms of a text (include/glypr_cuda.h GLP_TOKENS_*)
GLP_TOKENS_BARE = 0      # the BPE ids alone
GLP_TOKENS_SINGLE = 1    # GlyprTokenizer::encode: BOS/EOS added unless already there (tokenizer.rs:162-177)
GLP_TOKENS_SEQUENCE = 2  # encode_modality_sequence for a text: BOS + ids + EOS (tokenizer.rs:454-566)
GLP_DEFAULT_MAX_SEQ_LEN = 8320

# int (*glp_batch_fn)(void* user, const int32_t* ids, const int32_t* lengths, int n_seq, int max_len,
#                     int out_dim, float* out)
BATCH_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32),
                            ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                            ctypes.POINTER(ctypes.c_float))


class GlyprError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[glp error {code}] {message}")
        self.code = code
        self.message = message


class GlpOptions(ctypes.Structure):
    _fields_ = [("max_batch_tokens", ctypes.c_int64), ("max_batch_seqs", ctypes.c_int),
                ("device_memory_limit_mib", ctypes.c_int), ("reserved", ctypes.c_int * 5)]


class GlpModelInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "n_layers", "hidden", "ffn", "n_heads", "n_kv_heads", "head_dim", "vocab", "embedding_dim",
        "max_position", "sliding_window", "weight_type", "n_devices")] + [("device_bytes", ctypes.c_int64)]


class GlpTiming(ctypes.Structure):
    _fields_ = [("n_devices", ctypes.c_int), ("device_ms", ctypes.c_float * GLP_MAX_DEVICES)]


class GlpProfile(ctypes.Structure):
    _fields_ = [("n_kinds", ctypes.c_int), ("names", ctypes.c_char_p * GLP_PROFILE_KINDS),
                ("launches", ctypes.c_int64 * GLP_PROFILE_KINDS),
                ("total_ms", ctypes.c_double * GLP_PROFILE_KINDS),
                ("flops", ctypes.c_double * GLP_PROFILE_KINDS),
                ("bytes", ctypes.c_double * GLP_PROFILE_KINDS),
                ("total_launches", ctypes.c_int64)]

    def as_dict(self) -> dict:
        return {self.names[k].decode(): {"launches": int(self.launches[k]), "ms": float(self.total_ms[k]),
                                         "flops": float(self.flops[k]), "bytes": float(self.bytes[k])}
                for k in range(self.n_kinds)}


_lib = None
_lib_lock = threading.Lock()


def library_path() -> str:
    return os.path.join(_HERE, _LIB_NAME)


def load_library(path: Optional[str] = None) -> ctypes.CDLL:
    """Load (once) the CUDA library; raises if it has not been built."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        p = path or library_path()
        if not os.path.exists(p):
            raise GlyprError(GLP_ERR_IO, f"{p} not built (run glypr_b200/build.py)")
        L = ctypes.CDLL(p)
        P, I, I64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        L.glp_last_error.restype = ctypes.c_char_p
        L.glp_open.argtypes = [ctypes.c_char_p, P, I, P, ctypes.POINTER(P)]
        L.glp_close.argtypes = [P]
        L.glp_close.restype = None
        L.glp_model_info.argtypes = [P, P]
        L.glp_embed_tokens.argtypes = [P, P, P, I, I, I, P, P]
        L.glp_embed_packed_device.argtypes = [P, I, P, P, P, I, I, P, P]
        L.glp_device_status.argtypes = [P, I, P]
        L.glp_profile_enable.argtypes = [P, I, I]
        L.glp_profile_read.argtypes = [P, I, P]
        L.glp_q8_0_dequant.argtypes = [P, I64, P, P]
        L.glp_q8_0_gemm.argtypes = [P, I, I, P, I, P, I, P]
        L.glp_q8_0_gemm_noalloc.argtypes = [P, I, I, P, I, P, I, P]
        L.glp_bf16_gemm.argtypes = [P, I, I, P, I, P, I, P]
        L.glp_flash_attention.argtypes = [P, P, I, I, I, I, I, I, P, P]
        L.glp_engine_create.argtypes = [P, I, I, ctypes.POINTER(P)]
        L.glp_engine_create_with_executor.argtypes = [BATCH_FN, P, I, I, I, ctypes.POINTER(P)]
        L.glp_engine_embed.argtypes = [P, P, I, I, P]
        L.glp_engine_stats.argtypes = [P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                                       ctypes.POINTER(ctypes.c_int)]
        L.glp_engine_destroy.argtypes = [P]
        L.glp_engine_destroy.restype = None
        CP, SZ = ctypes.c_char_p, ctypes.c_size_t
        L.glp_tokenizer_from_gguf.argtypes = [CP, ctypes.POINTER(P)]
        L.glp_tokenizer_from_vocab.argtypes = [P, I, P, I, ctypes.POINTER(P)]
        L.glp_tokenizer_free.argtypes = [P]
        L.glp_tokenizer_free.restype = None
        L.glp_tokenizer_info.argtypes = [P, ctypes.POINTER(I), ctypes.POINTER(I)]
        L.glp_tokenize.argtypes = [P, CP, SZ, I, P, I, ctypes.POINTER(I)]
        L.glp_tokenize_batch.argtypes = [P, P, P, I, I, I, I, P, SZ, P]
        L.glp_format_query.argtypes = [CP, SZ, CP, P, SZ, ctypes.POINTER(SZ)]
        L.glp_format_document.argtypes = [CP, SZ, CP, P, SZ, ctypes.POINTER(SZ)]
        L.glp_task_format.argtypes = [CP, CP, CP, SZ, P, SZ, ctypes.POINTER(SZ)]
        L.glp_embed_texts.argtypes = [P, P, P, P, I, I, I, I, P]
        L.glp_engine_embed_text.argtypes = [P, P, CP, SZ, CP, CP, I, P]
        L.glp_embed_tokens_sharded.argtypes = [P, P, I, I, P, P, I, I, I, P]
        L.glp_kernel_status.argtypes = [I, ctypes.POINTER(I)]
        L.glp_status_text.argtypes = [I]
        L.glp_status_text.restype = ctypes.c_char_p
        L.glp_selftest_wait_timeout.argtypes = [I, I]
        L.glp_gate_up_geglu.argtypes = [P, P, I, I, P, I, P, P]
        L.glp_qkv_norm_rope.argtypes = [P, I, I, I, P, I, P, P, P, ctypes.c_double, I, ctypes.c_float, P, P]
        _lib = L
        return L


def check(rc: int) -> None:
    if rc != GLP_OK:
        msg = load_library().glp_last_error().decode(errors="replace")
        raise GlyprError(rc, msg)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------------------------------
# util.rs equivalents (host side, f32)
# ---------------------------------------------------------------------------------------

def l2_normalize(v: np.ndarray) -> np.ndarray:
    """util.rs:22-29 (a zero vector is returned unchanged)."""
    v = np.asarray(v, dtype=np.float32)
    n = np.float32(np.sqrt(np.sum(v * v, dtype=np.float32)))
    return v.copy() if n == 0 else (v / n).astype(np.float32)


def truncate_mrl(embedding: np.ndarray, target_dim: int) -> np.ndarray:
    """util.rs:6-19: first ``target_dim`` values, L2-renormalised."""
    embedding = np.asarray(embedding, dtype=np.float32)
    if target_dim == 0:
        raise ValueError("Target Matryoshka dimension cannot be 0")
    if target_dim > embedding.shape[-1]:
        raise ValueError(f"Target dimension {target_dim} exceeds embedding dimension {embedding.shape[-1]}")
    return l2_normalize(embedding[..., :target_dim])


def cosine_similarity(a: np.ndarray, b: np.ndarray) -> float:
    """util.rs:32-41."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    na, nb = float(np.sqrt((a * a).sum())), float(np.sqrt((b * b).sum()))
    if na == 0 or nb == 0:
        return 0.0
    return float(np.clip((a * b).sum() / (na * nb), -1.0, 1.0))


# ---------------------------------------------------------------------------------------
# the embedder
# ---------------------------------------------------------------------------------------

class GlyprEmbedder:
    """A loaded model replicated on one or more GPUs (one weight copy per device)."""

    def __init__(self, handle: int, path: str, devices: Sequence[int]):
        self._h = ctypes.c_void_p(handle)
        self.path = path
        self.devices = list(devices)
        info = GlpModelInfo()
        check(load_library().glp_model_info(self._h, ctypes.byref(info)))
        self.info = info

    # reference: GlyprEmbedder::load_gguf(path, device) / load_gguf_q8 (lib.rs:176-229)
    @classmethod
    def load_gguf(cls, path: str, devices: Optional[Sequence[int]] = None,
                  max_batch_tokens: int = 0, max_batch_seqs: int = 0,
                  device_memory_limit_mib: int = 0) -> "GlyprEmbedder":
        L = load_library()
        devs = list(devices) if devices is not None else []
        arr = (ctypes.c_int * max(1, len(devs)))(*devs) if devs else None
        opt = GlpOptions(max_batch_tokens=max_batch_tokens, max_batch_seqs=max_batch_seqs,
                         device_memory_limit_mib=device_memory_limit_mib)
        out = ctypes.c_void_p()
        check(L.glp_open(path.encode(), arr, len(devs), ctypes.byref(opt), ctypes.byref(out)))
        return cls(out.value, path, devs or [-1])

    load_gguf_q8 = load_gguf

    def close(self) -> None:
        if self._h and self._h.value:
            load_library().glp_close(self._h)
            self._h = ctypes.c_void_p(None)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def embedding_dim(self) -> int:
        return self.info.embedding_dim

    @property
    def max_position(self) -> int:
        return self.info.max_position

    def embed_tokens(self, ids: np.ndarray, lengths: np.ndarray, out_dim: Optional[int] = None,
                     timing: Optional[GlpTiming] = None) -> np.ndarray:
        """Right-padded ids [n_seq, max_len] + lengths -> L2-normalised [n_seq, out_dim] f32."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        if ids.ndim != 2:
            raise ValueError("ids must be [n_seq, max_len]")
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        n, s = ids.shape
        od = int(out_dim or self.embedding_dim)
        out = np.empty((n, od), dtype=np.float32)
        check(load_library().glp_embed_tokens(self._h, _ptr(ids), _ptr(lengths), n, s, od, _ptr(out),
                                              ctypes.byref(timing) if timing is not None else None))
        return out

    # reference: embed_batch(inputs, truncate_dim) -> Vec<Vec<f32>> (lib.rs:731-952), here on
    # token-id lists (the tokenizer is outside this backend's boundary)
    def embed_batch(self, token_ids: Sequence[Sequence[int]], truncate_dim: Optional[int] = None
                    ) -> List[np.ndarray]:
        if len(token_ids) == 0:
            return []
        lens = np.array([len(t) for t in token_ids], dtype=np.int32)
        s = int(lens.max()) if len(lens) else 0
        ids = np.zeros((len(token_ids), max(s, 1)), dtype=np.int32)
        for i, t in enumerate(token_ids):
            ids[i, :len(t)] = np.asarray(t, dtype=np.int32)
        emb = self.embed_tokens(ids[:, :max(s, 1)] if s else ids, lens, truncate_dim)
        return [e for e in emb]

    def embed_text_ids(self, ids: Sequence[int], truncate_dim: Optional[int] = None) -> np.ndarray:
        return self.embed_batch([ids], truncate_dim)[0]

    # text entry points (lib.rs:504-517, 655-723): prompt formatting + tokenisation on the host,
    # then the same device path as embed_tokens
    def embed_texts(self, tokenizer: "Tokenizer", texts: Sequence[str], form: int = GLP_TOKENS_SEQUENCE,
                    truncate_dim: Optional[int] = None, max_seq_len: int = 0) -> np.ndarray:
        """Formatted texts -> [n, dim] (glp_embed_texts).  ``form``: GLP_TOKENS_SINGLE as the
        reference's single-text calls tokenise, GLP_TOKENS_SEQUENCE as its batch calls do."""
        enc = [t.encode("utf-8") for t in texts]
        if not enc:
            return np.zeros((0, int(truncate_dim or self.embedding_dim)), dtype=np.float32)
        bufs = (ctypes.c_char_p * len(enc))(*enc)
        lens = (ctypes.c_size_t * len(enc))(*[len(b) for b in enc])
        od = int(truncate_dim or self.embedding_dim)
        out = np.empty((len(enc), od), dtype=np.float32)
        check(load_library().glp_embed_texts(self._h, tokenizer._h, ctypes.cast(bufs, ctypes.c_void_p),
                                             ctypes.cast(lens, ctypes.c_void_p), len(enc), form, max_seq_len, od,
                                             _ptr(out)))
        return out

    def embed_text(self, tokenizer: "Tokenizer", text: str, task: Optional[str] = None,
                   title: Optional[str] = None, truncate_dim: Optional[int] = None) -> np.ndarray:
        """``embed_text(text, Task)`` (lib.rs:506-509): task.rs formatting, single-text tokens."""
        return self.embed_texts(tokenizer, [task_format(task, title, text)], GLP_TOKENS_SINGLE, truncate_dim)[0]

    def embed_query(self, tokenizer: "Tokenizer", query: str, task: str = "search_query",
                    truncate_dim: Optional[int] = None) -> np.ndarray:
        """lib.rs:663-671: GlyprTokenizer::format_query, single-text tokens."""
        return self.embed_texts(tokenizer, [format_query(query, task)], GLP_TOKENS_SINGLE, truncate_dim)[0]

    def embed_document(self, tokenizer: "Tokenizer", content: str, title: Optional[str] = None,
                       truncate_dim: Optional[int] = None) -> np.ndarray:
        """lib.rs:673-681: GlyprTokenizer::format_document, single-text tokens."""
        return self.embed_texts(tokenizer, [format_document(content, title)], GLP_TOKENS_SINGLE, truncate_dim)[0]

    def embed_batch_queries(self, tokenizer: "Tokenizer", queries: Sequence[str], task: str = "search_query",
                            truncate_dim: Optional[int] = None) -> np.ndarray:
        """lib.rs:693-705: formatted queries through the batch path."""
        return self.embed_texts(tokenizer, [format_query(q, task) for q in queries], GLP_TOKENS_SEQUENCE,
                                truncate_dim)

    def embed_batch_documents(self, tokenizer: "Tokenizer", contents: Sequence[str],
                              titles: Optional[Sequence[str]] = None,
                              truncate_dim: Optional[int] = None) -> np.ndarray:
        """lib.rs:707-723: formatted documents through the batch path."""
        docs = [format_document(c, titles[i] if titles is not None else None) for i, c in enumerate(contents)]
        return self.embed_texts(tokenizer, docs, GLP_TOKENS_SEQUENCE, truncate_dim)

    # device-resident path (stream-ordered; pointers are raw device addresses)
    def embed_packed_device(self, d_ids: int, d_cu: int, h_cu: np.ndarray, n_seq: int, out_dim: int,
                            d_out: int, stream: int = 0, dev_index: int = 0) -> None:
        h_cu = np.ascontiguousarray(h_cu, dtype=np.int32)
        check(load_library().glp_embed_packed_device(self._h, dev_index, ctypes.c_void_p(d_ids),
                                                     ctypes.c_void_p(d_cu), _ptr(h_cu), n_seq, out_dim,
                                                     ctypes.c_void_p(d_out), ctypes.c_void_p(stream)))

    def profile_enable(self, enable: bool = True, dev_index: int = 0) -> None:
        check(load_library().glp_profile_enable(self._h, dev_index, int(enable)))

    def profile_read(self, dev_index: int = 0) -> dict:
        prof = GlpProfile()
        check(load_library().glp_profile_read(self._h, dev_index, ctypes.byref(prof)))
        out = prof.as_dict()
        out["_total_launches"] = int(prof.total_launches)
        return out

    def device_status(self, dev_index: int = 0) -> int:
        st = ctypes.c_int(0)
        check(load_library().glp_device_status(self._h, dev_index, ctypes.byref(st)))
        return st.value


# ---------------------------------------------------------------------------------------
# kernel-level entry points (raw device pointers)
# ---------------------------------------------------------------------------------------

def q8_0_dequant(d_blocks: int, n_blocks: int, d_out: int, stream: int = 0) -> None:
    check(load_library().glp_q8_0_dequant(ctypes.c_void_p(d_blocks), n_blocks, ctypes.c_void_p(d_out),
                                          ctypes.c_void_p(stream)))


def q8_0_gemm(d_w: int, n: int, k: int, d_x: int, m: int, d_y: int, y_is_f32: bool, stream: int = 0) -> None:
    check(load_library().glp_q8_0_gemm(ctypes.c_void_p(d_w), n, k, ctypes.c_void_p(d_x), m, ctypes.c_void_p(d_y),
                                       int(y_is_f32), ctypes.c_void_p(stream)))


def q8_0_gemm_noalloc(d_w: int, n: int, k: int, d_x: int, m: int, d_y: int, y_is_f32: bool, stream: int = 0) -> None:
    """glp_q8_0_gemm_noalloc: the same GEMM with its scratch in the library's fixed array."""
    check(load_library().glp_q8_0_gemm_noalloc(ctypes.c_void_p(d_w), n, k, ctypes.c_void_p(d_x), m,
                                               ctypes.c_void_p(d_y), int(y_is_f32), ctypes.c_void_p(stream)))


def kernel_status(device: int = 0) -> int:
    """glp_kernel_status: read and clear the kernel-level entry points' status word (raises
    GlyprError with GLP_ERR_DEVICE when a bounded wait expired)."""
    st = ctypes.c_int(0)
    check(load_library().glp_kernel_status(device, ctypes.byref(st)))
    return st.value


def status_text(status: int) -> str:
    return load_library().glp_status_text(int(status)).decode()


def selftest_wait_timeout(device: int = 0, limit_us: int = 1000) -> None:
    """glp_selftest_wait_timeout: a kernel whose bounded wait runs out on purpose."""
    check(load_library().glp_selftest_wait_timeout(device, limit_us))


def embed_tokens_sharded(executors, embedding_dim: int, ids: np.ndarray, lengths: np.ndarray,
                         out_dim: Optional[int] = None, out: Optional[np.ndarray] = None) -> np.ndarray:
    """glp_embed_tokens_sharded over Python executors ``fn(ids, lengths, out_dim) -> [n, out_dim]``
    (an executor fails its shard by raising)."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    lengths = np.ascontiguousarray(lengths, dtype=np.int32)
    n, s = ids.shape
    od = int(out_dim or embedding_dim)
    if out is None:
        out = np.empty((n, od), dtype=np.float32)

    def wrap(fn):
        def trampoline(user, p_ids, p_lengths, m, max_len, o_dim, p_out):
            try:
                a = np.ctypeslib.as_array(p_ids, shape=(m * max(max_len, 1),)).reshape(m, max(max_len, 1))
                lens = np.ctypeslib.as_array(p_lengths, shape=(m,))
                res = np.asarray(fn(a[:, :max_len].copy(), lens.copy(), o_dim), dtype=np.float32)
                np.ctypeslib.as_array(p_out, shape=(m * o_dim,))[:] = res.reshape(-1)
                return GLP_OK
            except Exception:
                return GLP_ERR_INVALID_ARG
        return BATCH_FN(trampoline)

    keep = [wrap(f) for f in executors]
    fns = (BATCH_FN * len(keep))(*keep)
    check(load_library().glp_embed_tokens_sharded(ctypes.cast(fns, ctypes.c_void_p), None, len(keep),
                                                  embedding_dim, _ptr(ids), _ptr(lengths), n, s, od, _ptr(out)))
    return out


def bf16_gemm(d_w: int, n: int, k: int, d_x: int, m: int, d_y: int, y_is_f32: bool, stream: int = 0) -> None:
    check(load_library().glp_bf16_gemm(ctypes.c_void_p(d_w), n, k, ctypes.c_void_p(d_x), m, ctypes.c_void_p(d_y),
                                       int(y_is_f32), ctypes.c_void_p(stream)))


def gate_up_geglu(d_wg: int, d_wu: int, f: int, k: int, d_x: int, m: int, d_out: int, stream: int = 0) -> None:
    check(load_library().glp_gate_up_geglu(ctypes.c_void_p(d_wg), ctypes.c_void_p(d_wu), f, k, ctypes.c_void_p(d_x),
                                           m, ctypes.c_void_p(d_out), ctypes.c_void_p(stream)))


def qkv_norm_rope(d_w: int, n_q_heads: int, n_kv_heads: int, k: int, d_x: int, m: int, d_q_gain: int,
                  d_k_gain: int, d_pos: int, theta: float, max_pos: int, eps: float, d_out: int,
                  stream: int = 0) -> None:
    check(load_library().glp_qkv_norm_rope(ctypes.c_void_p(d_w), n_q_heads, n_kv_heads, k, ctypes.c_void_p(d_x), m,
                                           ctypes.c_void_p(d_q_gain), ctypes.c_void_p(d_k_gain),
                                           ctypes.c_void_p(d_pos), float(theta), max_pos, float(eps),
                                           ctypes.c_void_p(d_out), ctypes.c_void_p(stream)))


def flash_attention(d_qkv: int, d_cu: int, n_seq: int, max_len: int, n_q_heads: int, n_kv_heads: int,
                    head_dim: int, window: int, d_out: int, stream: int = 0) -> None:
    check(load_library().glp_flash_attention(ctypes.c_void_p(d_qkv), ctypes.c_void_p(d_cu), n_seq, max_len,
                                             n_q_heads, n_kv_heads, head_dim, window, ctypes.c_void_p(d_out),
                                             ctypes.c_void_p(stream)))


# ---------------------------------------------------------------------------------------
# dynamic-batching engine (glypr-server's inference engine, engine.rs:157-325)
# ---------------------------------------------------------------------------------------

class InferenceEngine:
    """Blocking, thread-safe embedding of single sequences, batched by one worker thread.

    ``InferenceEngine(embedder, max_batch_size)`` runs batches through the model context
    (glp_engine_create); ``InferenceEngine.with_executor(fn, dim, max_batch_size)`` through a
    Python batch function ``fn(ids [n, max_len] int32, lengths [n], out_dim) -> [n, out_dim]``
    (glp_engine_create_with_executor; it raises to fail the batch).  ``embed(ids, truncate_dim)``
    may be called from many threads at once and mirrors EngineHandle::embed (engine.rs:120-150).
    """

    def __init__(self, embedder: Optional["GlyprEmbedder"] = None, max_batch_size: int = 32,
                 queue_capacity: int = 0, _executor=None, _dim: int = 0):
        L = load_library()
        self._h = ctypes.c_void_p()
        self._keep = None
        self._cv = threading.Condition()
        self._active = 0      # calls between the closed check and their return
        self._closed = False
        self._embedder = embedder  # the context must outlive the engine
        if embedder is not None:
            check(L.glp_engine_create(embedder._h, max_batch_size, queue_capacity, ctypes.byref(self._h)))
            self.dim = embedder.embedding_dim
        else:
            def trampoline(user, ids, lengths, n, max_len, out_dim, out):
                try:
                    a = np.ctypeslib.as_array(ids, shape=(n * max(max_len, 1),)).reshape(n, max(max_len, 1))
                    lens = np.ctypeslib.as_array(lengths, shape=(n,))
                    res = np.asarray(_executor(a[:, :max_len].copy(), lens.copy(), out_dim), dtype=np.float32)
                    np.ctypeslib.as_array(out, shape=(n * out_dim,))[:] = res.reshape(-1)
                    return GLP_OK
                except Exception:  # the batch fails; every request of it gets the error
                    return GLP_ERR_INVALID_ARG
            self._keep = BATCH_FN(trampoline)  # the callback must outlive the engine
            check(L.glp_engine_create_with_executor(self._keep, None, _dim, max_batch_size, queue_capacity,
                                                    ctypes.byref(self._h)))
            self.dim = _dim

    @classmethod
    def with_executor(cls, fn, dim: int, max_batch_size: int = 32, queue_capacity: int = 0) -> "InferenceEngine":
        return cls(None, max_batch_size, queue_capacity, _executor=fn, _dim=dim)

    def embed(self, ids, truncate_dim: Optional[int] = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        d = self.dim if not truncate_dim or truncate_dim >= self.dim else int(truncate_dim)
        out = np.empty(d, dtype=np.float32)
        with self._cv:
            if self._closed:
                raise GlyprError(GLP_ERR_INVALID_ARG, "Inference worker is not running")
            self._active += 1
        try:
            check(load_library().glp_engine_embed(self._h, _ptr(ids), ids.size, 0 if d == self.dim else d,
                                                  _ptr(out)))
        finally:
            with self._cv:
                self._active -= 1
                self._cv.notify_all()
        return out

    def embed_text(self, tokenizer: "Tokenizer", text: str, task: Optional[str] = None,
                   title: Optional[str] = None, truncate_dim: Optional[int] = None) -> np.ndarray:
        """A server-style text request (glp_engine_embed_text): task.rs formatting, sequence
        tokens on this thread, then the batching queue."""
        d = self.dim if not truncate_dim or truncate_dim >= self.dim else int(truncate_dim)
        out = np.empty(d, dtype=np.float32)
        b = text.encode("utf-8")
        with self._cv:
            if self._closed:
                raise GlyprError(GLP_ERR_INVALID_ARG, "Inference worker is not running")
            self._active += 1
        try:
            check(load_library().glp_engine_embed_text(
                self._h, tokenizer._h, b, len(b), task.encode("utf-8") if task is not None else None,
                title.encode("utf-8") if title is not None else None, 0 if d == self.dim else d, _ptr(out)))
        finally:
            with self._cv:
                self._active -= 1
                self._cv.notify_all()
        return out

    def stats(self) -> dict:
        r, b, m = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        check(load_library().glp_engine_stats(self._h, ctypes.byref(r), ctypes.byref(b), ctypes.byref(m)))
        return {"requests": r.value, "batches": b.value, "largest_batch": m.value}

    def close(self) -> None:
        """Reject new calls, let the calls in flight finish, then stop the worker."""
        with self._cv:
            self._closed = True
            self._cv.wait_for(lambda: self._active == 0)
        if self._h:
            load_library().glp_engine_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# ---------------------------------------------------------------------------------------
# text front end (tokenizer.rs, task.rs)
# ---------------------------------------------------------------------------------------

def _format(fn, *args) -> str:
    n = ctypes.c_size_t()
    cap = 256
    while True:
        buf = ctypes.create_string_buffer(cap)
        rc = fn(*args, buf, cap, ctypes.byref(n))
        if rc == GLP_OK:
            return buf.raw[:n.value].decode("utf-8")
        if n.value + 1 <= cap:
            check(rc)
        cap = n.value + 1


def format_query(query: str, task: str) -> str:
    """GlyprTokenizer::format_query (tokenizer.rs:144-152)."""
    q = query.encode("utf-8")
    return _format(load_library().glp_format_query, q, len(q), task.encode("utf-8"))


def format_document(content: str, title: Optional[str] = None) -> str:
    """GlyprTokenizer::format_document (tokenizer.rs:154-160)."""
    c = content.encode("utf-8")
    return _format(load_library().glp_format_document, c, len(c),
                   title.encode("utf-8") if title is not None else None)


def task_format(task: Optional[str], title: Optional[str], text: str) -> str:
    """Task::from_name_and_title(task, title).format_text(text) (task.rs:21-73); None = Raw."""
    t = text.encode("utf-8")
    return _format(load_library().glp_task_format, task.encode("utf-8") if task is not None else None,
                   title.encode("utf-8") if title is not None else None, t, len(t))


class Tokenizer:
    """GlyprTokenizer over the library's C++ BPE (glp_tokenizer_*).

    ``Tokenizer.from_gguf(path)`` reads ``tokenizer.ggml.tokens`` / ``tokenizer.ggml.merges``
    (tokenizer.rs:77-138); ``Tokenizer.from_vocab(tokens, merges)`` takes the two arrays.
    ``encode(text)`` is GlyprTokenizer::encode (BOS/EOS unless present); ``encode(text, form)``
    gives the other sequence forms; ``encode_batch`` tokenises on all host threads;
    ``encode_batch_padded`` mirrors encode_batch_padded_with_limit (tokenizer.rs:182-222).
    """

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle

    @classmethod
    def from_gguf(cls, path: str) -> "Tokenizer":
        h = ctypes.c_void_p()
        check(load_library().glp_tokenizer_from_gguf(path.encode(), ctypes.byref(h)))
        return cls(h)

    @classmethod
    def from_vocab(cls, tokens: Sequence[str], merges: Sequence[str]) -> "Tokenizer":
        tb = [t.encode("utf-8") for t in tokens]
        mb = [m.encode("utf-8") for m in merges]
        ta = (ctypes.c_char_p * max(len(tb), 1))(*tb)
        ma = (ctypes.c_char_p * max(len(mb), 1))(*mb)
        h = ctypes.c_void_p()
        check(load_library().glp_tokenizer_from_vocab(ctypes.cast(ta, ctypes.c_void_p), len(tb),
                                                      ctypes.cast(ma, ctypes.c_void_p), len(mb), ctypes.byref(h)))
        return cls(h)

    def close(self) -> None:
        if self._h:
            load_library().glp_tokenizer_free(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> dict:
        n, m = ctypes.c_int(), ctypes.c_int()
        check(load_library().glp_tokenizer_info(self._h, ctypes.byref(n), ctypes.byref(m)))
        return {"tokens": n.value, "merges": m.value}

    def encode(self, text: str, form: int = GLP_TOKENS_SINGLE) -> List[int]:
        b = text.encode("utf-8")
        ids = np.empty(3 * len(b) + 2, dtype=np.int32)
        n = ctypes.c_int()
        check(load_library().glp_tokenize(self._h, b, len(b), form, _ptr(ids), ids.size, ctypes.byref(n)))
        return ids[:n.value].tolist()

    def encode_batch(self, texts: Sequence[str], form: int = GLP_TOKENS_SINGLE, limit: int = 0,
                     n_threads: int = 0) -> List[np.ndarray]:
        enc = [t.encode("utf-8") for t in texts]
        n = len(enc)
        bufs = (ctypes.c_char_p * max(n, 1))(*enc)
        lens = (ctypes.c_size_t * max(n, 1))(*[len(b) for b in enc])
        cap = 3 * sum(len(b) for b in enc) + 2 * n
        ids = np.empty(max(cap, 1), dtype=np.int32)
        off = np.zeros(n + 1, dtype=np.int64)
        check(load_library().glp_tokenize_batch(self._h, ctypes.cast(bufs, ctypes.c_void_p),
                                                ctypes.cast(lens, ctypes.c_void_p), n, form, limit, n_threads,
                                                _ptr(ids), cap, _ptr(off)))
        return [ids[off[i]:off[i + 1]].copy() for i in range(n)]

    def encode_batch_padded(self, texts: Sequence[str], limit: int = 0):
        """(ids [B, L] right-padded with 0, mask [B, L]) like encode_batch_padded_with_limit."""
        rows = self.encode_batch(texts, GLP_TOKENS_SINGLE, limit)
        width = max(len(r) for r in rows)
        ids = np.zeros((len(rows), width), dtype=np.int32)
        mask = np.zeros((len(rows), width), dtype=np.int32)
        for i, r in enumerate(rows):
            ids[i, :len(r)] = r
            mask[i, :len(r)] = 1
        return ids, mask

    def format_query(self, query: str, task: str) -> str:
        return format_query(query, task)

    def format_document(self, content: str, title: Optional[str] = None) -> str:
        return format_document(content, title)
