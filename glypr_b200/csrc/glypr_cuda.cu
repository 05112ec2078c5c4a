// libglypr_cuda.so: host side of the B200 embedding path and its C ABI (include/glypr_cuda.h).
//
// Host responsibilities (the C++ counterpart of glypr-core's Rust facade):
//   * GGUF -> TextConfig with the reference's keys and defaults (config.rs:76-250)
//   * weight upload: one replica per device; Q8_0 linears dequantised once on the device
//     into fused bf16 layouts (QKV concatenated as in try_concat, linear.rs:82-148; gate/up
//     interleaved per 128 rows for the GeGLU epilogue); token table kept as raw Q8_0 blocks
//   * per-device forward over packed sequences in launch chunks (model.rs:498-578 +
//     pool_and_normalize 654-705), one worker thread and stream per device, contiguous
//     sequence shards (no collective: embeddings are copied back per device).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <unordered_map>
#include <vector>

#include "attention_tc.cuh"
#include "attention_d512.cuh"
#include "attention_pair.cuh"
#include "gemm.cuh"
#include "gguf.h"
#include "glypr_cuda.h"
#include "ple.cuh"
#include "q8gemm.cuh"
#include "rowops.cuh"

using glp::GemmParams;

namespace {

thread_local std::string t_err;

int fail(int code, const std::string& msg) {
  t_err = msg;
  return code;
}

#define GLP_CUDA(expr)                                                                         \
  do {                                                                                         \
    cudaError_t e_ = (expr);                                                                   \
    if (e_ != cudaSuccess)                                                                     \
      return fail(e_ == cudaErrorMemoryAllocation ? GLP_ERR_OOM : GLP_ERR_CUDA,                \
                  std::string(#expr) + ": " + cudaGetErrorString(e_));                         \
  } while (0)

#define GLP_TRY(expr)         \
  do {                        \
    int rc_ = (expr);         \
    if (rc_ != GLP_OK) return rc_; \
  } while (0)

// ------------------------------------------------------------------------------ TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Encoded maps by their arguments.  A map holds the address, shape, strides, box and layout and
// nothing of the data, so the map made for the same arguments stays valid (also for memory
// freed and allocated again at the same address); the standalone entry points build the same
// few maps on every call, and a lookup costs less than an encode.  Bounded: emptied when full.
struct MapKey {
  const void* base;
  int64_t a, b, c;
  int box, kind;
  bool operator==(const MapKey& o) const {
    return base == o.base && a == o.a && b == o.b && c == o.c && box == o.box && kind == o.kind;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.base);
    for (int64_t v : {k.a, k.b, k.c, static_cast<int64_t>(k.box), static_cast<int64_t>(k.kind)})
      h = h * 1000003u ^ std::hash<int64_t>()(v);
    return h;
  }
};
struct MapCache {
  std::mutex mu;
  std::unordered_map<MapKey, CUtensorMap, MapKeyHash> maps;
  bool get(const MapKey& k, CUtensorMap* out) {
    std::lock_guard<std::mutex> lk(mu);
    const auto it = maps.find(k);
    if (it == maps.end()) return false;
    *out = it->second;
    return true;
  }
  void put(const MapKey& k, const CUtensorMap& m) {
    std::lock_guard<std::mutex> lk(mu);
    if (maps.size() >= 1024) maps.clear();
    maps.emplace(k, m);
  }
};
MapCache g_maps;

// 2-D 16-bit row-major [rows, cols] tensor, box = 64 columns (one 128-byte swizzle row) x
// box_rows rows, 128B swizzle, out-of-bounds rows read as zero.  f16 = true for the model
// path's operands, false for bf16.
int make_map16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows, bool f16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GLP_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (driver too old?)");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_elems * 2) % 16 || cols % 64)
    return fail(GLP_ERR_INVALID_ARG, "TMA operand must be 16-byte aligned with K % 64 == 0");
  const MapKey key{base, rows, cols, ld_elems, box_rows, f16 ? 1 : 0};
  if (g_maps.get(key, m)) return GLP_OK;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_elems * 2)};
  const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GLP_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  g_maps.put(key, *m);
  return GLP_OK;
}

int sm_count();

// Launch attention over packed qkv rows [0, T) for n_seq sequences at cu (minus cu_base).
int launch_attention(const __half* qkv, int64_t T, int qkv_width, const int* cu, int cu_base, int n_seq, int max_len,
                     int n_q_heads, int n_kv_heads, int window, __half* out, int* status, cudaStream_t st,
                     int head_dim = glp::kFaD) {
  if (T <= 0 || n_seq <= 0 || max_len <= 0) return GLP_OK;
  if (head_dim == glp::kF5D) {  // 512-wide heads: two CTAs per (block, head), one O half each
    CUtensorMap mq, mkv, mo;
    GLP_TRY(make_map16(&mq, qkv, T, qkv_width, qkv_width, glp::kF5BQ, true));
    GLP_TRY(make_map16(&mkv, qkv, T, qkv_width, qkv_width, glp::kF5BKV, true));
    GLP_TRY(make_map16(&mo, out, T, static_cast<int64_t>(n_q_heads) * glp::kF5D,
                       static_cast<int64_t>(n_q_heads) * glp::kF5D, glp::kFaOutBoxRows, true));
    glp::FaParams fp{};
    fp.cu_seqlens = cu;
    fp.cu_base = cu_base;
    fp.n_seq = n_seq;
    fp.q_blocks = (max_len + glp::kF5BQ - 1) / glp::kF5BQ;
    fp.n_q_heads = n_q_heads;
    fp.n_kv_heads = n_kv_heads;
    fp.window = window;
    fp.out = out;
    fp.ld_out = n_q_heads * glp::kF5D;
    fp.status = status;
    const int64_t items = static_cast<int64_t>(n_seq) * fp.q_blocks * n_q_heads * 2;
    const int grid = static_cast<int>(std::min<int64_t>(items, sm_count()));
    glp::flash_attn_d512_kernel<<<grid, glp::kFaThreads, glp::kF5Smem, st>>>(mq, mkv, mo, fp);
    GLP_CUDA(cudaGetLastError());
    return GLP_OK;
  }
  if (head_dim != glp::kFaD) return fail(GLP_ERR_UNSUPPORTED, "head_dim must be 256 or 512");
  // 256-wide heads: CTA pairs over 256-query blocks and 128-key tiles (GLP_ATTENTION=single:
  // the one-CTA kernel over 128-query blocks and 64-key tiles)
  const char* attn_env = std::getenv("GLP_ATTENTION");  // read per call (A/B measurements)
  const bool single = attn_env && std::strcmp(attn_env, "single") == 0;
  if (!single) {
    CUtensorMap mqv, mk;
    GLP_TRY(make_map16(&mqv, qkv, T, qkv_width, qkv_width, glp::kFpBQ, true));
    GLP_TRY(make_map16(&mk, qkv, T, qkv_width, qkv_width, 64, true));
    glp::FaParams fp{};
    fp.cu_seqlens = cu;
    fp.cu_base = cu_base;
    fp.n_seq = n_seq;
    fp.q_blocks = (max_len + 2 * glp::kFpBQ - 1) / (2 * glp::kFpBQ);
    fp.n_q_heads = n_q_heads;
    fp.n_kv_heads = n_kv_heads;
    fp.window = window;
    fp.out = out;
    fp.ld_out = n_q_heads * glp::kFaD;
    fp.status = status;
    const int64_t items = static_cast<int64_t>(n_seq) * fp.q_blocks * n_q_heads;
    const int pairs = static_cast<int>(std::min<int64_t>(items, std::max(1, sm_count() / 2)));
    glp::flash_attn_pair_kernel<<<2 * pairs, glp::kFpThreads, glp::kFpSmem, st>>>(mqv, mk, fp);
    GLP_CUDA(cudaGetLastError());
    return GLP_OK;
  }
  CUtensorMap mq, mkv, mo;
  GLP_TRY(make_map16(&mq, qkv, T, qkv_width, qkv_width, glp::kFaBQ, true));
  GLP_TRY(make_map16(&mkv, qkv, T, qkv_width, qkv_width, glp::kFaBKV, true));
  // output rows [T, Hq * 256]: bulk stores of 64 columns x 32 rows
  GLP_TRY(make_map16(&mo, out, T, static_cast<int64_t>(n_q_heads) * glp::kFaD,
                     static_cast<int64_t>(n_q_heads) * glp::kFaD, glp::kFaOutBoxRows, true));
  glp::FaParams fp{};
  fp.cu_seqlens = cu;
  fp.cu_base = cu_base;
  fp.n_seq = n_seq;
  fp.q_blocks = (max_len + glp::kFaBQ - 1) / glp::kFaBQ;
  fp.n_q_heads = n_q_heads;
  fp.n_kv_heads = n_kv_heads;
  fp.window = window;
  fp.out = out;
  fp.ld_out = n_q_heads * glp::kFaD;
  fp.status = status;
  const int64_t items = static_cast<int64_t>(n_seq) * fp.q_blocks * n_q_heads;
  const int grid = static_cast<int>(std::min<int64_t>(items, sm_count()));  // persistent CTAs
  glp::flash_attn_tc_kernel<<<grid, glp::kFaThreads, glp::kFaSmem, st>>>(mq, mkv, mo, fp);
  GLP_CUDA(cudaGetLastError());
  return GLP_OK;
}

// ------------------------------------------------------------------------------ per-device kernel setup
std::mutex g_attr_mu;
std::array<bool, 64> g_attr_done{};

int ensure_kernel_attrs() {
  int dev = 0;
  GLP_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (dev < 0 || dev >= 64) return fail(GLP_ERR_INVALID_ARG, "device index out of range");
  if (g_attr_done[dev]) return GLP_OK;
  const int s256 = static_cast<int>(glp::GemmCfg<256>::SMEM), s128 = static_cast<int>(glp::GemmCfg<128>::SMEM);
  const cudaFuncAttribute A = cudaFuncAttributeMaxDynamicSharedMemorySize;
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<256, glp::kEpiStore16, __half>, A, s256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<256, glp::kEpiF32, __half>, A, s256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<256, glp::kEpiQkv, __half>, A, s256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<256, glp::kEpiGeglu, __half>, A, s256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<128, glp::kEpiStore16, __half>, A, s128));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<128, glp::kEpiF32, __half>, A, s128));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<256, glp::kEpiMulGeglu, __half>, A, s256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<128, glp::kEpiMulGeglu, __half>, A, s128));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<256, glp::kEpiStore16, __nv_bfloat16>, A, s256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<256, glp::kEpiF32, __nv_bfloat16>, A, s256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<128, glp::kEpiStore16, __nv_bfloat16>, A, s128));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_tc_kernel<128, glp::kEpiF32, __nv_bfloat16>, A, s128));
  const int sp = static_cast<int>(glp::GemmPairCfg::SMEM);
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_pair_kernel<glp::kEpiStore16, __half>, A, sp));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_pair_kernel<glp::kEpiF32, __half>, A, sp));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_pair_kernel<glp::kEpiQkv, __half>, A, sp));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_pair_kernel<glp::kEpiGeglu, __half>, A, sp));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_pair_kernel<glp::kEpiMulGeglu, __half>, A, sp));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_pair_kernel<glp::kEpiStore16, __nv_bfloat16>, A, sp));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_pair_kernel<glp::kEpiF32, __nv_bfloat16>, A, sp));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_rownorm_kernel<__half, 2>, A, static_cast<int>(glp::GemmRowCfgT<2>::SMEM)));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_rownorm_kernel<__half, 3>, A, static_cast<int>(glp::GemmRowCfgT<3>::SMEM)));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_rownorm_kernel<__half, 4>, A, static_cast<int>(glp::GemmRowCfgT<4>::SMEM)));
  GLP_CUDA(cudaFuncSetAttribute(glp::flash_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(glp::kFaSmem)));
  GLP_CUDA(cudaFuncSetAttribute(glp::flash_attn_d512_kernel, A, static_cast<int>(glp::kF5Smem)));
  GLP_CUDA(cudaFuncSetAttribute(glp::flash_attn_pair_kernel, A, static_cast<int>(glp::kFpSmem)));
  const int q256 = static_cast<int>(glp::Q8PairCfg<256>::SMEM), q128 = static_cast<int>(glp::Q8PairCfg<128>::SMEM);
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_q8_pair_kernel<glp::kEpiStore16, __nv_bfloat16, 256>, A, q256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_q8_pair_kernel<glp::kEpiStore16, __nv_bfloat16, 128>, A, q128));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_q8_pair_kernel<glp::kEpiF32, __nv_bfloat16, 256>, A, q256));
  GLP_CUDA(cudaFuncSetAttribute(glp::gemm_q8_pair_kernel<glp::kEpiF32, __nv_bfloat16, 128>, A, q128));
  g_attr_done[dev] = true;
  return GLP_OK;
}

int sm_count() {
  static std::array<std::atomic<int>, 64> cached{};  // per device, read once
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && (n = cached[dev].load(std::memory_order_relaxed)) > 0) return n;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  n = n > 0 ? n : 148;
  if (dev >= 0 && dev < 64) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

int bn_for(int n) { return n % 256 == 0 ? 256 : 128; }

// The row kernels are compiled per hidden size: f(std::integral_constant<int, H>{}) for H a
// multiple of 256 up to glp::kMaxHidden.
template <class F>
int with_hidden(int H, F&& f) {
  switch (H) {
    case 256: return f(std::integral_constant<int, 256>{});
    case 512: return f(std::integral_constant<int, 512>{});
    case 768: return f(std::integral_constant<int, 768>{});
    case 1024: return f(std::integral_constant<int, 1024>{});
    case 1280: return f(std::integral_constant<int, 1280>{});
    case 1536: return f(std::integral_constant<int, 1536>{});
    case 1792: return f(std::integral_constant<int, 1792>{});
    case 2048: return f(std::integral_constant<int, 2048>{});
    default: return fail(GLP_ERR_UNSUPPORTED, "hidden size must be a multiple of 256 up to 2048");
  }
}
static_assert(glp::kMaxHidden == 2048, "with_hidden covers every supported hidden size");

// GEMM engine for 256-wide tiles: CTA pairs or one CTA per tile.
// Per kernel the pair is faster for the plain-store GEMMs (O 0.312 -> 0.269 ms, down 0.414 ->
// 0.372 ms per 262,144-token launch) and 3-6 % slower in cycles for the fused QKV and GeGLU
// epilogues; but under the 1 kW power cap the pairs' smaller L2 and shared-memory traffic lets
// the whole forward run at a higher clock (median 1,447-1,470 vs 1,402-1,410 MHz), and
// all-pairs gave the higher throughput: 6,141-6,191 vs 6,088-6,127 embeddings/s with pairs for
// the plain-store GEMMs only.  A GEMM of fewer 256-row tiles than one wave of pairs (a short
// launch chunk) runs on single CTAs instead: twice the tiles of half the size finish sooner
// (one 512-token sequence: 1.70 -> 1.62 ms).  GLP_GEMM=pair forces pairs for every 256-wide
// GEMM, GLP_GEMM=single single CTAs, GLP_GEMM=pair-store pairs for the plain-store epilogues only.
int gemm_engine_mode() {  // 0 single, 1 pair-store, 2 pairs for a full wave (default), 3 pairs
  static const int mode = [] {
    const char* e = std::getenv("GLP_GEMM");
    if (e && std::string(e) == "single") return 0;
    if (e && std::string(e) == "pair-store") return 1;
    if (e && std::string(e) == "pair") return 3;
    return 2;
  }();
  return mode;
}

bool use_pair_gemm(int epi) {
  const int mode = gemm_engine_mode();
  if (mode != 1) return mode >= 2;
  return epi == glp::kEpiStore16 || epi == glp::kEpiF32;
}

// pairs for this GEMM: the engine allows them and (by default) its 256-row tiles fill a wave
bool pair_gemm_for(int epi, int M, int n_tiles) {
  if (!use_pair_gemm(epi)) return false;
  if (gemm_engine_mode() != 2) return true;
  return static_cast<int64_t>((M + 255) / 256) * n_tiles >= sm_count() / 2;
}

// Post-norms fused into the O / down GEMMs (gemm_rownorm_kernel) for 512-, 768- and 1024-wide
// rows, for every launch chunk (GLP_FUSED_NORM=0: separate row kernels).  Not chosen by chunk
// size, although a single-wave chunk runs the row kernels faster (one 512-token sequence 1.70
// vs 1.81 ms): the two paths round differently, and a sequence's embedding stays bit-identical
// whatever batch it is embedded in only if every chunk takes the same path.
int fused_norm_mode() {  // 0 never, 2 always
  static const int mode = [] {
    const char* e = std::getenv("GLP_FUSED_NORM");
    return (e && std::string(e) == "0") ? 0 : 2;
  }();
  return mode;
}

// Row widths the clustered row-norm GEMM covers: 2, 3 or 4 CTA pairs of 256 columns.
bool rownorm_width(int n) { return n == 512 || n == 768 || n == 1024; }

// Clusters of 2 NP CTAs that fit the device at once (cached per device and NP): the persistent
// row-norm GEMM launches that many.
template <int NP>
int rownorm_clusters() {
  static std::mutex mu;
  static std::array<int, 64> cache{};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * NP * 16);
  cfg.blockDim = dim3(glp::kGemmThreads);
  cfg.dynamicSmemBytes = glp::GemmRowCfgT<NP>::SMEM;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, glp::gemm_rownorm_kernel<__half, NP>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = sm_count() / (2 * NP);
  }
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

template <int NP>
void launch_rownorm_np(const CUtensorMap& ma, const CUtensorMap& mb_pair, const CUtensorMap& mh, const CUtensorMap& mx,
                       const GemmParams& p, cudaStream_t st) {
  const int clusters = std::min(p.m_tiles, rownorm_clusters<NP>());
  glp::gemm_rownorm_kernel<__half, NP>
      <<<2 * NP * clusters, glp::kGemmThreads, glp::GemmRowCfgT<NP>::SMEM, st>>>(ma, mb_pair, mh, mx, p);
}

// y = A * B^T (N = 512, 768 or 1024: clusters of 2, 3 or 4 CTA pairs) fused with the post-norm
// + residual + next pre-norm: updates p.h in place and writes p.x_next.  `mb_pair` covers B
// with 128-row boxes, `mh` the residual rows [M, N] bf16 and `mx` the next pre-normed rows
// [M, N] f16, both with 32-row boxes.
int launch_rownorm_gemm(const CUtensorMap& ma, const CUtensorMap& mb_pair, const CUtensorMap& mh, const CUtensorMap& mx,
                        GemmParams p, cudaStream_t st) {
  if (p.M <= 0) return GLP_OK;
  if (!rownorm_width(p.N) || p.K % 64 || p.K <= 0)
    return fail(GLP_ERR_INVALID_ARG, "row-norm GEMM needs N in {512, 768, 1024}, K % 64 == 0");
  p.m_tiles = (p.M + 255) / 256;
  p.n_tiles = p.N / 256;
  p.k_blocks = p.K / 64;
  static const bool direct = [] {  // GLP_ROWNORM_DIRECT=1: the exact two-exchange scale everywhere
    const char* e = std::getenv("GLP_ROWNORM_DIRECT");
    return e && std::string(e) == "1";
  }();
  p.rownorm_direct = direct ? 1 : 0;
  switch (p.N) {
    case 512: launch_rownorm_np<2>(ma, mb_pair, mh, mx, p, st); break;
    case 768: launch_rownorm_np<3>(ma, mb_pair, mh, mx, p, st); break;
    default: launch_rownorm_np<4>(ma, mb_pair, mh, mx, p, st); break;
  }
  GLP_CUDA(cudaGetLastError());
  return GLP_OK;
}

// Launch C = A * B^T with the given epilogue; T is the 16-bit operand type.  `ma` covers
// A [M, K] (box rows 128), `mb` covers B [N, K] with box rows == bn; `mb_pair` (optional,
// box rows 128) lets 256-wide tiles run on CTA pairs.
// One launch of the CTA-pair GEMM; with `dependent` as a programmatic dependent launch (its
// prologue overlaps the previous kernel, its producer waits for that kernel's writes).
template <int EPI, typename T>
cudaError_t launch_pair_gemm(dim3 grid, size_t smem, cudaStream_t st, bool dependent, const CUtensorMap& ma,
                             const CUtensorMap& mb, const CUtensorMap& mc, const GemmParams& p) {
  if (!dependent) {
    glp::gemm_pair_kernel<EPI, T><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, mc, p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(glp::kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, glp::gemm_pair_kernel<EPI, T>, ma, mb, mc, p);
}

template <typename T>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, int bn, int epi, GemmParams p, cudaStream_t st,
                const CUtensorMap* mb_pair = nullptr, const CUtensorMap* mc = nullptr, bool dependent = false) {
  p.m_tiles = (p.M + 127) / 128;
  p.n_tiles = p.N / bn;
  p.k_blocks = p.K / 64;
  if (p.M <= 0) return GLP_OK;
  if (p.K % 64 || p.K <= 0 || p.N % 128) return fail(GLP_ERR_INVALID_ARG, "GEMM needs K % 64 == 0 and N % 128 == 0");
  const bool f16 = std::is_same<T, __half>::value;
  // plain stores with N % 256 == 128 may still take 256-wide pair tiles: the last one's second
  // half lies past N (zero-filled B rows, nothing stored), which beats 128-wide tiles' 1.5x
  // operand bytes per MMA once the tiles fill the device
  const bool store_epi = epi == glp::kEpiStore16 || epi == glp::kEpiF32;
  const int pair_n_tiles = store_epi ? (p.N + 255) / 256 : p.N / 256;
  if ((bn == 256 || (store_epi && p.N % 256)) && mb_pair && (store_epi || p.N % 256 == 0) &&
      pair_gemm_for(epi, p.M, pair_n_tiles)) {
    p.n_tiles = pair_n_tiles;
    if ((epi == glp::kEpiQkv || epi == glp::kEpiGeglu || epi == glp::kEpiMulGeglu) && !f16)
      return fail(GLP_ERR_INVALID_ARG, "fused epilogues run on f16 operands");
    p.m_tiles = (p.M + 255) / 256;  // 256-row pair tiles
    const int pairs = std::min(p.m_tiles * p.n_tiles, sm_count() / 2);
    const size_t smem = glp::GemmPairCfg::SMEM;
    const dim3 grid(static_cast<unsigned>(2 * pairs));
    switch (epi) {
      case glp::kEpiStore16: GLP_CUDA((launch_pair_gemm<glp::kEpiStore16, T>(grid, smem, st, dependent, ma, *mb_pair, ma, p))); break;
      case glp::kEpiF32: GLP_CUDA((launch_pair_gemm<glp::kEpiF32, T>(grid, smem, st, dependent, ma, *mb_pair, ma, p))); break;
      case glp::kEpiQkv:
        if (!mc) return fail(GLP_ERR_INVALID_ARG, "the QKV epilogue needs the output's tensor map");
        glp::gemm_pair_kernel<glp::kEpiQkv, __half><<<grid, glp::kGemmThreads, smem, st>>>(ma, *mb_pair, *mc, p);
        break;
      case glp::kEpiGeglu: glp::gemm_pair_kernel<glp::kEpiGeglu, __half><<<grid, glp::kGemmThreads, smem, st>>>(ma, *mb_pair, ma, p); break;
      case glp::kEpiMulGeglu:
        glp::gemm_pair_kernel<glp::kEpiMulGeglu, __half><<<grid, glp::kGemmThreads, smem, st>>>(ma, *mb_pair, ma, p);
        break;
      default: return fail(GLP_ERR_INVALID_ARG, "bad epilogue");
    }
    GLP_CUDA(cudaGetLastError());
    return GLP_OK;
  }
  if (p.N % bn) return fail(GLP_ERR_INVALID_ARG, "GEMM needs N % tile == 0");
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = std::min(tiles, sm_count());
  if (bn == 256) {
    const size_t smem = glp::GemmCfg<256>::SMEM;
    switch (epi) {
      case glp::kEpiStore16: glp::gemm_tc_kernel<256, glp::kEpiStore16, T><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p); break;
      case glp::kEpiF32: glp::gemm_tc_kernel<256, glp::kEpiF32, T><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p); break;
      case glp::kEpiQkv:
        if (!f16) return fail(GLP_ERR_INVALID_ARG, "fused epilogues run on f16 operands");
        glp::gemm_tc_kernel<256, glp::kEpiQkv, __half><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p);
        break;
      case glp::kEpiGeglu:
        if (!f16) return fail(GLP_ERR_INVALID_ARG, "fused epilogues run on f16 operands");
        glp::gemm_tc_kernel<256, glp::kEpiGeglu, __half><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p);
        break;
      case glp::kEpiMulGeglu:
        if (!f16) return fail(GLP_ERR_INVALID_ARG, "fused epilogues run on f16 operands");
        glp::gemm_tc_kernel<256, glp::kEpiMulGeglu, __half><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p);
        break;
      default: return fail(GLP_ERR_INVALID_ARG, "bad epilogue");
    }
  } else {
    const size_t smem = glp::GemmCfg<128>::SMEM;
    switch (epi) {
      case glp::kEpiStore16: glp::gemm_tc_kernel<128, glp::kEpiStore16, T><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p); break;
      case glp::kEpiF32: glp::gemm_tc_kernel<128, glp::kEpiF32, T><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p); break;
      case glp::kEpiMulGeglu:
        if (!f16) return fail(GLP_ERR_INVALID_ARG, "fused epilogues run on f16 operands");
        glp::gemm_tc_kernel<128, glp::kEpiMulGeglu, __half><<<grid, glp::kGemmThreads, smem, st>>>(ma, mb, p);
        break;
      default: return fail(GLP_ERR_INVALID_ARG, "fused epilogues need 256-wide tiles");
    }
  }
  GLP_CUDA(cudaGetLastError());
  return GLP_OK;
}

// ------------------------------------------------------------------------------ Q8_0 GEMM on raw rows
// Rows per TMA group row for raw Q8_0 rows of K elements: the smallest G in {1, 2, 4} with
// G * (34 K / 32) a multiple of 16 bytes (a TMA row stride); 0 when K % 64 != 0.
int q8_raw_group(int K) {
  if (K <= 0 || K % 64) return 0;
  const int64_t pitch = static_cast<int64_t>(K) / 32 * 34;
  for (int g = 1; g <= 4; g *= 2)
    if ((g * pitch) % 16 == 0) return g;
  return 0;
}

// The raw rows W [N, 34 K / 32 bytes] as the byte tensor {G P, N / G}, boxes of 80 bytes x
// box_rows group rows (see gemm_q8_pair_kernel).
int make_map_q8_raw(CUtensorMap* m, const void* base, int N, int K, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GLP_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (driver too old?)");
  const int G = q8_raw_group(K);
  if (!G || N % G) return fail(GLP_ERR_INVALID_ARG, "Q8_0 GEMM needs K % 64 == 0");
  if (reinterpret_cast<uintptr_t>(base) & 15) return fail(GLP_ERR_INVALID_ARG, "Q8_0 weight must be 16-byte aligned");
  const MapKey key{base, N, K, 0, box_rows, 2};
  if (g_maps.get(key, m)) return GLP_OK;
  const uint64_t row = static_cast<uint64_t>(G) * (K / 32) * 34;
  const cuuint64_t dims[2] = {row, static_cast<cuuint64_t>(N / G)};
  const cuuint64_t strides[1] = {row};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(glp::kQ8RawBoxBytes), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GLP_ERR_CUDA, "cuTensorMapEncodeTiled (raw Q8_0) failed: " + std::to_string(r));
  g_maps.put(key, *m);
  return GLP_OK;
}

// Pair-tile width for an M x N Q8_0 GEMM: 256 columns, or 128 when that finishes in fewer
// waves of the device's pairs (each 128-wide tile costs about 0.55 of a 256-wide one).
int q8_tile_n(int M, int N) {
  const int64_t pairs = std::max(1, sm_count() / 2);
  const int64_t m_tiles = (M + 255) / 256;
  double best = 1e30;
  int bn = 128;
  for (int cand : {256, 128}) {
    if (N % cand) continue;
    const int64_t tiles = m_tiles * (N / cand);
    const double cost = static_cast<double>((tiles + pairs - 1) / pairs) * (cand == 256 ? 1.0 : 0.55);
    if (cost < best) {
      best = cost;
      bn = cand;
    }
  }
  return bn;
}

// C = A * dequant(W)^T with W as raw Q8_0 rows in device memory: one launch of the pair
// kernel that streams the raw bytes and dequantises them in shared memory.
int launch_q8_gemm(const CUtensorMap& ma, const void* w_raw, bool f32_out, GemmParams p, cudaStream_t st) {
  if (p.M <= 0) return GLP_OK;
  if (p.N <= 0 || p.N % 128 || p.K <= 0 || p.K % 64) return fail(GLP_ERR_INVALID_ARG, "Q8_0 GEMM needs N % 128 == 0, K % 64 == 0");
  const int bn = q8_tile_n(p.M, p.N);
  p.raw_group = q8_raw_group(p.K);
  p.raw_pitch = p.K / 32 * 34;
  p.m_tiles = (p.M + 255) / 256;
  p.n_tiles = p.N / bn;
  p.k_blocks = p.K / 64;
  CUtensorMap mw;
  GLP_TRY(make_map_q8_raw(&mw, w_raw, p.N, p.K, bn / 2 / p.raw_group));
  const int pairs = std::min(p.m_tiles * p.n_tiles, std::max(1, sm_count() / 2));
  const dim3 grid(static_cast<unsigned>(2 * pairs));
  if (bn == 256) {
    const size_t smem = glp::Q8PairCfg<256>::SMEM;
    if (f32_out)
      glp::gemm_q8_pair_kernel<glp::kEpiF32, __nv_bfloat16, 256><<<grid, glp::kQ8Threads, smem, st>>>(ma, mw, p);
    else
      glp::gemm_q8_pair_kernel<glp::kEpiStore16, __nv_bfloat16, 256><<<grid, glp::kQ8Threads, smem, st>>>(ma, mw, p);
  } else {
    const size_t smem = glp::Q8PairCfg<128>::SMEM;
    if (f32_out)
      glp::gemm_q8_pair_kernel<glp::kEpiF32, __nv_bfloat16, 128><<<grid, glp::kQ8Threads, smem, st>>>(ma, mw, p);
    else
      glp::gemm_q8_pair_kernel<glp::kEpiStore16, __nv_bfloat16, 128><<<grid, glp::kQ8Threads, smem, st>>>(ma, mw, p);
  }
  GLP_CUDA(cudaGetLastError());
  return GLP_OK;
}

// ------------------------------------------------------------------------------ model config
struct Config {
  int n_layers = 0, hidden = 0, ffn = 0, n_heads = 0, n_kv = 0, head_dim = 0, vocab = 0;
  int emb_out = 768, max_pos = 262144, window = 512;
  double eps = 1e-6, theta_swa = 1e4, theta_full = 1e6;
  std::vector<bool> sliding;
  std::vector<int> kv;  // KV heads per layer (config.rs:141-160: head_count_kv[i], global layers may differ)
  std::vector<int> hd;  // head_dim per layer: key_length_swa on sliding layers, key_length on global ones
  uint32_t linear_type = glp::kGgmlQ8_0;
  int ple_dim = 0;  // per-layer-embedding width D; 0 = no PLE tensors (model.rs:257-275)
};

int parse_config(const glp::GgufFile& g, Config* c) {
  const std::string a = "gemma-embedding2.";
  uint32_t u = 0;
  if (!g.get_u32(a + "block_count", &u)) return fail(GLP_ERR_FORMAT, "Missing gemma-embedding2.block_count");
  c->n_layers = static_cast<int>(u);
  if (!g.get_u32(a + "embedding_length", &u)) return fail(GLP_ERR_FORMAT, "Missing gemma-embedding2.embedding_length");
  c->hidden = static_cast<int>(u);
  if (!g.get_u32(a + "feed_forward_length", &u))
    return fail(GLP_ERR_FORMAT, "Missing gemma-embedding2.feed_forward_length");
  c->ffn = static_cast<int>(u);
  if (!g.get_u32(a + "attention.head_count", &u))
    return fail(GLP_ERR_FORMAT, "Missing gemma-embedding2.attention.head_count");
  c->n_heads = static_cast<int>(u);
  uint32_t hd_swa = 256, hd_full = 512;
  g.get_u32(a + "attention.key_length_swa", &hd_swa);
  g.get_u32(a + "attention.key_length", &hd_full);
  if (g.get_u32(a + "embedding_length_out", &u)) c->emb_out = static_cast<int>(u);
  if (g.get_u32(a + "context_length", &u)) c->max_pos = static_cast<int>(u);
  g.get_f64(a + "attention.layer_norm_rms_epsilon", &c->eps);
  g.get_f64(a + "rope.freq_base_swa", &c->theta_swa);
  g.get_f64(a + "rope.freq_base", &c->theta_full);
  const glp::GgufValue* toks = g.find("tokenizer.ggml.tokens");
  c->vocab = toks && toks->type == 9 ? static_cast<int>(toks->arr_len) : 262144;
  const glp::GgufValue* pat = g.find(a + "attention.sliding_window_pattern");
  c->sliding.resize(c->n_layers);
  for (int i = 0; i < c->n_layers; ++i) {
    if (pat && pat->type == 9) {
      if (pat->arr_type != 7 || i >= static_cast<int>(pat->arr.size()))
        return fail(GLP_ERR_FORMAT, "Invalid boolean in sliding_window_pattern");
      c->sliding[i] = pat->arr[i] != 0;
    } else {
      c->sliding[i] = (i + 1) % 6 != 0;
    }
  }
  // config.rs:141-160: element 0 of head_count_kv (default 2) for the sliding layers, element
  // i (default 1) for global layer i; an element that is not an integer takes the default
  const std::string kv_key = a + "attention.head_count_kv";
  c->n_kv = g.get_array_u32(kv_key, 0, &u) ? static_cast<int>(u) : 2;
  c->kv.assign(c->n_layers, c->n_kv);
  c->hd.assign(c->n_layers, static_cast<int>(hd_swa));
  for (int i = 0; i < c->n_layers; ++i) {
    int kvi = c->n_kv;
    if (!c->sliding[i]) kvi = g.get_array_u32(kv_key, static_cast<size_t>(i), &u) ? static_cast<int>(u) : 1;
    const int hd = c->sliding[i] ? static_cast<int>(hd_swa) : static_cast<int>(hd_full);
    // sliding layers run 256-wide heads; global layers 256 or 512 (EmbeddingGemma 2's 512,
    // config.rs:141-160, with the 512-wide RoPE of model.rs:279)
    if (hd != 256 && !(hd == 512 && !c->sliding[i]))
      return fail(GLP_ERR_UNSUPPORTED, "head_dim must be 256 (512 is supported on global layers)");
    c->hd[i] = hd;
    if (kvi <= 0 || c->n_heads % kvi)
      return fail(GLP_ERR_FORMAT, "head_count must be a multiple of head_count_kv");
    c->kv[i] = kvi;
  }
  c->head_dim = static_cast<int>(hd_swa);
  if (c->hidden <= 0 || c->hidden % 256 || c->hidden > glp::kMaxHidden)
    return fail(GLP_ERR_UNSUPPORTED, "hidden size must be a multiple of 256 up to 2048");
  if (c->head_dim != 256) return fail(GLP_ERR_UNSUPPORTED, "head_dim must be 256");
  if (c->n_kv <= 0 || c->n_heads % c->n_kv) return fail(GLP_ERR_FORMAT, "head_count must be a multiple of head_count_kv");
  if (c->ffn % 128) return fail(GLP_ERR_UNSUPPORTED, "feed_forward_length must be a multiple of 128");
  if ((c->n_heads * c->head_dim) % 64) return fail(GLP_ERR_UNSUPPORTED, "attention width must be a multiple of 64");
  if (g.tensor("per_layer_model_proj.weight")) {
    // config.rs:100-102: embedding_length_per_layer_input, default 512
    c->ple_dim = g.get_u32(a + "embedding_length_per_layer_input", &u) ? static_cast<int>(u) : 512;
    if (c->ple_dim <= 0 || c->ple_dim % 128)
      return fail(GLP_ERR_UNSUPPORTED, "embedding_length_per_layer_input must be a multiple of 128");
  }
  return GLP_OK;
}

// Check every tensor the forward needs (names as in model.rs:251-473) before any device
// work, so a malformed file fails without allocating.
int validate_tensors(const glp::GgufFile& g, const Config& c) {
  const int64_t H = c.hidden, F = c.ffn;
  auto need = [&](const std::string& name, std::vector<int64_t> ne, bool matrix) -> int {
    const glp::GgufTensor* t = g.tensor(name);
    if (!t) return fail(GLP_ERR_FORMAT, "missing tensor " + name);
    if (t->ne != ne) return fail(GLP_ERR_FORMAT, "bad shape for " + name);
    if (matrix && t->type != glp::kGgmlQ8_0 && t->type != glp::kGgmlBF16)
      return fail(GLP_ERR_UNSUPPORTED, name + " must be Q8_0 or BF16");
    if (!matrix && t->type != glp::kGgmlF32 && t->type != glp::kGgmlF16 && t->type != glp::kGgmlBF16)
      return fail(GLP_ERR_UNSUPPORTED, name + " must be F32, F16 or BF16");
    return GLP_OK;
  };
  const glp::GgufTensor* te = g.tensor("token_embd.weight");
  if (!te) return fail(GLP_ERR_FORMAT, "missing tensor token_embd.weight");
  if (te->ne.size() != 2 || te->ne[0] != H || te->ne[1] < c.vocab)
    return fail(GLP_ERR_FORMAT, "bad shape for token_embd.weight");
  if (te->type != glp::kGgmlQ8_0 && te->type != glp::kGgmlBF16)
    return fail(GLP_ERR_UNSUPPORTED, "token_embd.weight must be Q8_0 or BF16");
  // per-layer embeddings (model.rs:257-275, 418-453): all of them or none
  const int64_t PD = c.ple_dim;
  if (PD) {
    GLP_TRY(need("per_layer_model_proj.weight", {H, c.n_layers * PD}, true));
    GLP_TRY(need("per_layer_proj_norm.weight", {PD}, false));
  }
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    const int64_t D = c.hd[l];
    if (PD) {
      GLP_TRY(need(p + "inp_gate.weight", {H, PD}, true));
      GLP_TRY(need(p + "proj.weight", {PD, H}, true));
      GLP_TRY(need(p + "post_norm.weight", {H}, false));
      const glp::GgufTensor* s = g.tensor(p + "layer_output_scale.weight");
      if (!s) return fail(GLP_ERR_FORMAT, "missing tensor " + p + "layer_output_scale.weight");
      if (s->type != glp::kGgmlF32 || s->numel() != 1) return fail(GLP_ERR_FORMAT, "bad layer_output_scale");
    } else if (g.tensor(p + "proj.weight") || g.tensor(p + "inp_gate.weight")) {
      return fail(GLP_ERR_FORMAT, "missing tensor per_layer_model_proj.weight");
    }
    GLP_TRY(need(p + "attn_norm.weight", {H}, false));
    GLP_TRY(need(p + "attn_q_norm.weight", {D}, false));
    GLP_TRY(need(p + "attn_k_norm.weight", {D}, false));
    GLP_TRY(need(p + "post_attention_norm.weight", {H}, false));
    GLP_TRY(need(p + "ffn_norm.weight", {H}, false));
    GLP_TRY(need(p + "post_ffw_norm.weight", {H}, false));
    GLP_TRY(need(p + "attn_q.weight", {H, c.n_heads * D}, true));
    GLP_TRY(need(p + "attn_k.weight", {H, c.kv[l] * D}, true));
    GLP_TRY(need(p + "attn_v.weight", {H, c.kv[l] * D}, true));
    GLP_TRY(need(p + "attn_output.weight", {c.n_heads * D, H}, true));
    GLP_TRY(need(p + "ffn_gate.weight", {H, F}, true));
    GLP_TRY(need(p + "ffn_up.weight", {H, F}, true));
    GLP_TRY(need(p + "ffn_down.weight", {F, H}, true));
  }
  GLP_TRY(need("output_norm.weight", {H}, false));
  int64_t prev = H;
  int stages = 0;
  for (int j = 0;; ++j) {
    const glp::GgufTensor* t = g.tensor("dense." + std::to_string(j) + ".weight");
    if (!t) break;
    if (t->ne.size() != 2 || t->ne[0] != prev) return fail(GLP_ERR_FORMAT, "bad shape for dense head stage " + std::to_string(j));
    GLP_TRY(need("dense." + std::to_string(j) + ".weight", {prev, t->ne[1]}, true));
    if (t->ne[1] % 128) return fail(GLP_ERR_UNSUPPORTED, "dense head dims must be multiples of 128");
    prev = t->ne[1];
    ++stages;
  }
  if (stages == 0) {
    const glp::GgufTensor* t = g.tensor("output.weight");
    if (!t) return fail(GLP_ERR_FORMAT, "missing tensor output.weight");
    if (t->ne.size() != 2) return fail(GLP_ERR_FORMAT, "bad shape for output.weight");
    GLP_TRY(need("output.weight", {H, t->ne[1]}, true));
    if (t->ne[1] % 128) return fail(GLP_ERR_UNSUPPORTED, "output.weight rows must be a multiple of 128");
    prev = t->ne[1];
  }
  if (prev != c.emb_out) return fail(GLP_ERR_FORMAT, "head output dim != embedding_length_out");
  return GLP_OK;
}

// ------------------------------------------------------------------------------ device state
struct LayerW {
  __half *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;  // f16 weights
  float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *post_attn = nullptr, *ffn_norm = nullptr,
        *post_ffw = nullptr;
  float layer_scalar = 1.0f;
  bool sliding = true;
  int kv = 1, qkv_w = 0;  // KV heads and q|k|v width of this layer
  int hd = 256;           // head_dim of this layer (512 on EmbeddingGemma 2's global layers)
  CUtensorMap m_qkv, m_o, m_gu, m_down;
  CUtensorMap p_qkv, p_o, p_gu, p_down;  // the same weights, 128-row boxes for CTA pairs
  // per-layer-embedding block (ple.rs:96-145): gate [D, H], projection [H, D], post-norm
  __half *ple_gate = nullptr, *ple_proj = nullptr;
  float* ple_post = nullptr;
  CUtensorMap m_pg, m_pp, p_pg, p_pp;
};

struct HeadW {
  __half* w = nullptr;
  int n = 0, k = 0, bn = 256;
  CUtensorMap map, map_pair;
};

struct Device {
  int dev = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  std::vector<void*> allocs;
  // device memory this device's context holds (bytes requested from cudaMalloc, including the
  // host-API staging buffers) and the caller's limit on it (0 = none)
  int64_t bytes = 0, limit_bytes = 0;
  void* table = nullptr;
  uint32_t table_type = glp::kGgmlQ8_0;
  std::vector<LayerW> layers;
  float* out_norm = nullptr;
  std::vector<HeadW> head;
  // per-layer embeddings: projection [L * D, H] and its norm gain [D]
  __half* ple_w = nullptr;
  float* ple_norm = nullptr;
  CUtensorMap m_plew, p_plew;
  float2 *cs_swa = nullptr, *cs_full = nullptr;  // RoPE tables (sliding / global layers)
  float2* cs_full512 = nullptr;                   // global layers with 512-wide heads
  int64_t cap_tokens = 0;
  int cap_seqs = 0;
  __nv_bfloat16* h = nullptr;  // residual stream
  float* xf = nullptr;          // final normalised rows (pooling input)
  __half* x = nullptr;
  __half* qkv = nullptr;
  __half* attn = nullptr;
  __half* y = nullptr;
  __half* a = nullptr;
  int* pos = nullptr;
  __half* pooled = nullptr;
  float* pool_part = nullptr;  // per-segment sums of sequences longer than one pooling segment
  __half* mid = nullptr;
  float* emb = nullptr;
  __half* ple = nullptr;     // per-layer inputs [T, L, D] (PLE models)
  __half* ple_g = nullptr;   // the PLE block's gate activations [T, D]
  int* status = nullptr;
  // host-API staging (device + pinned host), grown on demand
  int* d_ids = nullptr;
  int* d_cu = nullptr;
  float* d_out = nullptr;
  int* h_ids = nullptr;
  int* h_cu = nullptr;
  float* h_out = nullptr;
  int64_t stage_tokens = 0, stage_seqs = 0, stage_out = 0;
  // profiling: event pairs around launches (when enabled) + launch counters (always)
  bool prof_on = false;
  std::vector<std::array<cudaEvent_t, 2>> prof_ev;
  std::vector<int> prof_kind;
  size_t prof_used = 0;
  std::array<int64_t, GLP_PROFILE_KINDS> prof_launch{};
  std::array<double, GLP_PROFILE_KINDS> prof_flops{}, prof_bytes{};
  // instantiated CUDA graphs of launch chunks, keyed by everything that reaches a kernel
  // parameter (see run_packed); each keeps the launch counters its capture added, which every
  // replay adds again
  struct ChunkGraph {
    std::array<int64_t, 8> key{};
    cudaGraphExec_t exec = nullptr;
    std::array<int64_t, GLP_PROFILE_KINDS> launches{};
    std::array<double, GLP_PROFILE_KINDS> flops{}, bytes{};
    uint64_t last_use = 0;
  };
  std::vector<ChunkGraph> graphs;
  uint64_t graph_clock = 0;

  // Reserve n bytes against the limit (GLP_ERR_OOM beyond it); release() gives them back.
  int reserve(size_t n) {
    if (limit_bytes > 0 && bytes + static_cast<int64_t>(n) > limit_bytes)
      return fail(GLP_ERR_OOM, "device memory limit of " + std::to_string(limit_bytes >> 20) +
                                   " MiB reached on device " + std::to_string(dev));
    bytes += static_cast<int64_t>(n);
    return GLP_OK;
  }
  int raw_malloc(void** v, size_t n) {
    GLP_TRY(reserve(n));
    const cudaError_t e = cudaMalloc(v, n);
    if (e != cudaSuccess) {
      bytes -= static_cast<int64_t>(n);
      *v = nullptr;
      return fail(e == cudaErrorMemoryAllocation ? GLP_ERR_OOM : GLP_ERR_CUDA,
                  std::string("cudaMalloc: ") + cudaGetErrorString(e));
    }
    return GLP_OK;
  }
  void raw_free(void* v, size_t n) {
    if (!v) return;
    cudaFree(v);
    bytes -= static_cast<int64_t>(n);
  }
  template <class T>
  int alloc(T** p, size_t count) {
    void* v = nullptr;
    GLP_TRY(raw_malloc(&v, std::max<size_t>(count, 1) * sizeof(T)));
    allocs.push_back(v);
    *p = static_cast<T*>(v);
    return GLP_OK;
  }
  void release() {
    cudaSetDevice(dev);
    if (stream) cudaStreamSynchronize(stream);
    for (void* p : allocs) cudaFree(p);
    allocs.clear();
    if (d_ids) cudaFree(d_ids);
    if (d_cu) cudaFree(d_cu);
    if (d_out) cudaFree(d_out);
    bytes = 0;
    if (h_ids) cudaFreeHost(h_ids);
    if (h_cu) cudaFreeHost(h_cu);
    if (h_out) cudaFreeHost(h_out);
    d_ids = d_cu = nullptr;
    d_out = nullptr;
    h_ids = h_cu = nullptr;
    h_out = nullptr;
    for (auto& e : prof_ev) {
      cudaEventDestroy(e[0]);
      cudaEventDestroy(e[1]);
    }
    prof_ev.clear();
    for (auto& g : graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    graphs.clear();
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (stream) cudaStreamDestroy(stream);
    stream = nullptr;
    ev0 = ev1 = nullptr;
  }
};

enum ProfKind : int {
  kProfEmbed = 0,
  kProfGemmQkv,
  kProfAttention,
  kProfGemmO,
  kProfPostNorm,
  kProfGemmGateUp,
  kProfGemmDown,
  kProfPool,
  kProfHeadGemm,
  kProfL2,
  kProfMisc,
  kProfKernelApi,
  kProfPleGemm,  // per-layer-embedding projections (PLE models only)
  kProfPleRows,  // per-layer-embedding input norm
};
const char* const kProfNames[GLP_PROFILE_KINDS] = {
    "embed_gather_norm", "gemm_qkv_norm_rope", "flash_attention", "gemm_o", "post_norm_residual",
    "gemm_gate_up_geglu", "gemm_down", "mean_pool", "gemm_head", "l2_mrl", "positions", "kernel_api",
    "ple_gemm", "ple_rows"};

// Bracket one kernel launch: counts it and, when profiling is on, records an event pair on
// the launching stream.  Returns the launch's status.
template <class F>
int prof_launch(Device& d, cudaStream_t st, int kind, double flops, double bytes, F&& launch) {
  if (d.prof_on) {
    if (d.prof_used == d.prof_ev.size()) {
      std::array<cudaEvent_t, 2> e{};
      GLP_CUDA(cudaEventCreate(&e[0]));
      GLP_CUDA(cudaEventCreate(&e[1]));
      d.prof_ev.push_back(e);
      d.prof_kind.push_back(0);
    }
    GLP_CUDA(cudaEventRecord(d.prof_ev[d.prof_used][0], st));
  }
  const int rc = launch();
  if (rc != GLP_OK) return rc;
  d.prof_launch[kind] += 1;
  d.prof_flops[kind] += flops;
  d.prof_bytes[kind] += bytes;
  if (d.prof_on) {
    GLP_CUDA(cudaEventRecord(d.prof_ev[d.prof_used][1], st));
    d.prof_kind[d.prof_used] = kind;
    ++d.prof_used;
  }
  return GLP_OK;
}

// Visible (query, key) pairs of one sequence under the attention mask (|i-j| <= w when
// w > 0): the attention kernel's algorithmic work is 4 * head_dim * heads * pairs FLOPs.
double visible_pairs(int64_t len, int w) {
  if (w <= 0 || len <= w + 1) return static_cast<double>(len) * len;
  // full square minus the two corners where |i - j| > w
  const double excl = static_cast<double>(len - w - 1) * (len - w) ;
  return static_cast<double>(len) * len - excl;
}

}  // namespace

struct glp_ctx {
  Config cfg;
  int64_t plan_bytes = 0;  // device memory each device's setup requests (device_plan_bytes)
  std::vector<std::unique_ptr<Device>> devs;
};

namespace {

// ------------------------------------------------------------------------------ upload
int upload_gain(Device& d, const glp::GgufFile& g, const std::string& name, int n, float** out) {
  const glp::GgufTensor* t = g.tensor(name);
  if (!t) return fail(GLP_ERR_FORMAT, "missing tensor " + name);
  if (t->ne.size() != 1 || t->ne[0] != n) return fail(GLP_ERR_FORMAT, "bad shape for " + name);
  std::vector<float> v(n);
  for (int i = 0; i < n; ++i) {
    if (t->type == glp::kGgmlF32) {
      std::memcpy(&v[i], t->data + 4 * i, 4);
    } else if (t->type == glp::kGgmlF16) {
      uint16_t hbits;
      std::memcpy(&hbits, t->data + 2 * i, 2);
      __half_raw hr;
      hr.x = hbits;
      v[i] = __half2float(__half(hr));
    } else if (t->type == glp::kGgmlBF16) {
      uint16_t b;
      std::memcpy(&b, t->data + 2 * i, 2);
      const uint32_t bits = static_cast<uint32_t>(b) << 16;
      std::memcpy(&v[i], &bits, 4);
    } else {
      return fail(GLP_ERR_UNSUPPORTED, "unsupported dtype for " + name);
    }
  }
  GLP_TRY(d.alloc(out, n));
  GLP_CUDA(cudaMemcpy(*out, v.data(), n * sizeof(float), cudaMemcpyHostToDevice));
  return GLP_OK;
}

// Upload linear `name` [n, k] into rows of dst (bf16 [*, k]) with the row mapping of
// q8_0_dequant_bf16_rows_kernel.  Uses a device staging buffer for the raw bytes.
int upload_linear(Device& d, const glp::GgufFile& g, const std::string& name, int n, int k, __half* dst,
                  int row_base, int group, int group_stride, void* staging, size_t staging_bytes) {
  const glp::GgufTensor* t = g.tensor(name);
  if (!t) return fail(GLP_ERR_FORMAT, "missing tensor " + name);
  if (t->ne.size() != 2 || t->ne[0] != k || t->ne[1] != n) return fail(GLP_ERR_FORMAT, "bad shape for " + name);
  if (t->nbytes > staging_bytes) return fail(GLP_ERR_FORMAT, "tensor too large: " + name);
  GLP_CUDA(cudaMemcpy(staging, t->data, t->nbytes, cudaMemcpyHostToDevice));
  if (t->type == glp::kGgmlQ8_0) {
    const int64_t nb = static_cast<int64_t>(n) * (k / 32);
    glp::q8_0_dequant_rows_kernel<__half><<<static_cast<unsigned>((nb + 255) / 256), 256>>>(
        static_cast<const uint8_t*>(staging), n, k, dst, row_base, group, group_stride);
  } else if (t->type == glp::kGgmlBF16) {
    const int64_t nc = static_cast<int64_t>(n) * (k / 2);
    glp::bf16_rows_convert_kernel<__half><<<static_cast<unsigned>((nc + 255) / 256), 256>>>(
        static_cast<const __nv_bfloat16*>(staging), n, k, dst, row_base, group, group_stride);
  } else {
    return fail(GLP_ERR_UNSUPPORTED, "linear " + name + " must be Q8_0 or BF16");
  }
  GLP_CUDA(cudaGetLastError());
  GLP_CUDA(cudaDeviceSynchronize());
  return GLP_OK;
}

// RoPE tables exactly as rope.rs:14-87: inv_freq_i = f32(1 / theta^(2i/d)) in f64, then
// freqs = f32(pos) * inv_freq (f32), cos/sin in f32.  Only the first half is stored (the
// reference table is cat(freqs, freqs)), frequency-major [half][max_pos] so that the GEMM
// epilogue's 32 lanes (consecutive rows = consecutive positions) read one coalesced line.
// RoPE table (rope.rs:14-76 values) with cos and sin of two consecutive frequencies side by
// side, frequency-pair-major: as float4, cs4[(i / 2) * max_pos + p] = {cos(p f_i), sin(p f_i),
// cos(p f_i+1), sin(p f_i+1)} for even i, so the QKV epilogue's lanes (consecutive rows =
// consecutive positions) read two frequencies per 16-byte load and a warp one coalesced 512 B.
// position_major: cs[p * half + i] instead (the 512-wide row kernel reads a lane's 8
// consecutive frequencies of one position).
int upload_rope(Device& d, double theta, int d_head, int max_pos, float2** cs, bool position_major = false) {
  const int half = d_head / 2;
  std::vector<float> inv(half);
  std::vector<float2> c(static_cast<size_t>(max_pos) * half);
  for (int i = 0; i < half; ++i) inv[i] = static_cast<float>(1.0 / std::pow(theta, (2.0 * i) / d_head));
  for (int i = 0; i < half; ++i)
    for (int p = 0; p < max_pos; ++p) {
      const float f = static_cast<float>(p) * inv[i];
      const size_t at = position_major ? static_cast<size_t>(p) * half + i
                                       : (static_cast<size_t>(i >> 1) * max_pos + p) * 2 + (i & 1);
      c[at] = make_float2(std::cos(f), std::sin(f));
    }
  GLP_TRY(d.alloc(cs, c.size()));
  GLP_CUDA(cudaMemcpy(*cs, c.data(), c.size() * sizeof(float2), cudaMemcpyHostToDevice));
  return GLP_OK;
}

// Device staging for one linear's raw bytes while the weights upload: the largest linear.
size_t load_staging_bytes(const glp::GgufFile& g, const Config& c) {
  size_t n = 0;
  for (const auto* nm : {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"}) {
    const glp::GgufTensor* t = g.tensor(std::string("blk.0.") + nm + ".weight");
    if (t) n = std::max(n, t->nbytes);
  }
  for (int j = 0;; ++j) {
    const glp::GgufTensor* t = g.tensor("dense." + std::to_string(j) + ".weight");
    if (!t) break;
    n = std::max(n, t->nbytes);
  }
  if (const glp::GgufTensor* t = g.tensor("output.weight")) n = std::max(n, t->nbytes);
  if (const glp::GgufTensor* t = g.tensor("per_layer_model_proj.weight")) n = std::max(n, t->nbytes);
  for (const auto* nm : {"inp_gate", "proj"})
    if (const glp::GgufTensor* t = g.tensor(std::string("blk.0.") + nm + ".weight")) n = std::max(n, t->nbytes);
  return std::max(n, static_cast<size_t>(4) * c.ffn * std::max(c.hidden, c.ffn));
}

// Device memory setup_device requests per device (weights, RoPE tables, one launch chunk's
// activations), without the load staging.  Computed from the file and the configuration
// alone, so glp_open can hold it against the caller's limit before touching a device.
int64_t device_plan_bytes(const glp::GgufFile& g, const Config& c, int64_t cap_tokens, int cap_seqs) {
  const int64_t H = c.hidden, F = c.ffn;
  const int64_t T = cap_tokens, S = cap_seqs, PD = c.ple_dim;
  int64_t AW = 0;  // the widest layer's attention width
  bool d512 = false;
  for (int l = 0; l < c.n_layers; ++l) {
    AW = std::max<int64_t>(AW, static_cast<int64_t>(c.n_heads) * c.hd[l]);
    d512 = d512 || c.hd[l] == 512;
  }
  auto b = [](int64_t count, int64_t elem) { return std::max<int64_t>(count, 1) * elem; };
  int64_t n = b(static_cast<int64_t>(g.tensor("token_embd.weight")->nbytes), 1);
  int64_t qkv_max = 0;
  for (int l = 0; l < c.n_layers; ++l) {
    const int64_t D = c.hd[l], W = (c.n_heads + 2 * c.kv[l]) * D;
    qkv_max = std::max(qkv_max, W);
    n += 4 * b(H, 4) + 2 * b(D, 4);                                            // norm gains
    n += b(W * H, 2) + b(H * c.n_heads * D, 2) + b(2 * F * H, 2) + b(H * F, 2);  // f16 linears
    if (PD) n += b(H, 4) + b(PD * H, 2) + b(H * PD, 2);                  // PLE block
  }
  if (PD) n += b(PD, 4) + b(c.n_layers * PD * H, 2);
  n += b(H, 4);  // output_norm
  int64_t prev = H, max_head = H;
  for (int j = 0;; ++j) {
    const glp::GgufTensor* t = g.tensor("dense." + std::to_string(j) + ".weight");
    if (!t) break;
    n += b(t->ne[1] * prev, 2);
    prev = t->ne[1];
    max_head = std::max(max_head, prev);
  }
  if (!g.tensor("dense.0.weight")) {
    const glp::GgufTensor* t = g.tensor("output.weight");
    n += b(t->ne[1] * H, 2);
    max_head = std::max(max_head, t->ne[1]);
  }
  n += 2 * b(static_cast<int64_t>(c.max_pos) * (c.head_dim / 2), 8);  // RoPE tables (256-wide heads)
  if (d512) n += b(static_cast<int64_t>(c.max_pos) * 256, 8);       // global RoPE over 512 dims
  n += b(T * H, 2) + b(T * H, 4) + b(T * H, 2) + b(T * qkv_max, 2) + b(T * AW, 2) + b(T * H, 2) + b(T * F, 2);
  if (PD) n += b(T * c.n_layers * PD, 2) + b(T * PD, 2);
  n += b(T, 4) + b(S * max_head, 2) + b((T / glp::kPoolSeg + S + 1) * H, 4) + b(S * max_head, 2) +
       b(S * max_head, 4) + b(1, 4);
  return n;
}

int setup_device(Device& d, const Config& c, const glp::GgufFile& g, int64_t cap_tokens, int cap_seqs) {
  GLP_CUDA(cudaSetDevice(d.dev));
  GLP_TRY(ensure_kernel_attrs());
  GLP_CUDA(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking));
  GLP_CUDA(cudaEventCreate(&d.ev0));
  GLP_CUDA(cudaEventCreate(&d.ev1));
  const int H = c.hidden, F = c.ffn, D = c.head_dim;
  int QKV = 0, AW = 0;  // the widest layer's q|k|v and attention widths (the activation buffers)
  bool d512 = false;
  for (int l = 0; l < c.n_layers; ++l) {
    QKV = std::max(QKV, (c.n_heads + 2 * c.kv[l]) * c.hd[l]);
    AW = std::max(AW, c.n_heads * c.hd[l]);
    d512 = d512 || c.hd[l] == 512;
  }

  // token table: kept as raw Q8_0 (or bf16) rows, gathered per token
  const glp::GgufTensor* te = g.tensor("token_embd.weight");
  if (!te) return fail(GLP_ERR_FORMAT, "missing tensor token_embd.weight");
  if (te->ne.size() != 2 || te->ne[0] != H) return fail(GLP_ERR_FORMAT, "bad shape for token_embd.weight");
  if (te->ne[1] < c.vocab) return fail(GLP_ERR_FORMAT, "token_embd.weight has fewer rows than the vocabulary");
  if (te->type != glp::kGgmlQ8_0 && te->type != glp::kGgmlBF16)
    return fail(GLP_ERR_UNSUPPORTED, "token_embd.weight must be Q8_0 or BF16");
  d.table_type = te->type;
  uint8_t* table = nullptr;
  GLP_TRY(d.alloc(&table, te->nbytes));
  GLP_CUDA(cudaMemcpy(table, te->data, te->nbytes, cudaMemcpyHostToDevice));
  d.table = table;

  // staging for raw linear bytes: the largest linear (freed when the upload is done)
  const size_t staging_bytes = load_staging_bytes(g, c);
  void* staging = nullptr;
  GLP_TRY(d.raw_malloc(&staging, staging_bytes));
  struct Free {
    Device& d;
    void* p;
    size_t n;
    ~Free() { d.raw_free(p, n); }
  } free_staging{d, staging, staging_bytes};

  d.layers.resize(c.n_layers);
  for (int l = 0; l < c.n_layers; ++l) {
    LayerW& L = d.layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    L.sliding = c.sliding[l];
    L.hd = c.hd[l];
    const int DL = L.hd, AWL = c.n_heads * DL;  // this layer's head and attention widths
    GLP_TRY(upload_gain(d, g, p + "attn_norm.weight", H, &L.attn_norm));
    GLP_TRY(upload_gain(d, g, p + "attn_q_norm.weight", DL, &L.q_norm));
    GLP_TRY(upload_gain(d, g, p + "attn_k_norm.weight", DL, &L.k_norm));
    GLP_TRY(upload_gain(d, g, p + "post_attention_norm.weight", H, &L.post_attn));
    GLP_TRY(upload_gain(d, g, p + "ffn_norm.weight", H, &L.ffn_norm));
    GLP_TRY(upload_gain(d, g, p + "post_ffw_norm.weight", H, &L.post_ffw));
    if (const glp::GgufTensor* s = g.tensor(p + "layer_output_scale.weight")) {
      if (s->type != glp::kGgmlF32 || s->numel() != 1) return fail(GLP_ERR_FORMAT, "bad layer_output_scale");
      std::memcpy(&L.layer_scalar, s->data, 4);
    }
    L.kv = c.kv[l];
    L.qkv_w = (c.n_heads + 2 * L.kv) * DL;
    GLP_TRY(d.alloc(&L.qkv, static_cast<size_t>(L.qkv_w) * H));
    GLP_TRY(d.alloc(&L.o, static_cast<size_t>(H) * AWL));
    GLP_TRY(d.alloc(&L.gu, static_cast<size_t>(2 * F) * H));
    GLP_TRY(d.alloc(&L.down, static_cast<size_t>(H) * F));
    GLP_TRY(upload_linear(d, g, p + "attn_q.weight", c.n_heads * DL, H, L.qkv, 0, 0, 0, staging, staging_bytes));
    GLP_TRY(upload_linear(d, g, p + "attn_k.weight", L.kv * DL, H, L.qkv, c.n_heads * DL, 0, 0, staging, staging_bytes));
    GLP_TRY(upload_linear(d, g, p + "attn_v.weight", L.kv * DL, H, L.qkv, (c.n_heads + L.kv) * DL, 0, 0, staging,
                          staging_bytes));
    GLP_TRY(upload_linear(d, g, p + "attn_output.weight", H, AWL, L.o, 0, 0, 0, staging, staging_bytes));
    GLP_TRY(upload_linear(d, g, p + "ffn_gate.weight", F, H, L.gu, 0, 128, 256, staging, staging_bytes));
    GLP_TRY(upload_linear(d, g, p + "ffn_up.weight", F, H, L.gu, 128, 128, 256, staging, staging_bytes));
    GLP_TRY(upload_linear(d, g, p + "ffn_down.weight", H, F, L.down, 0, 0, 0, staging, staging_bytes));
    GLP_TRY(make_map16(&L.m_qkv, L.qkv, L.qkv_w, H, H, 256, true));
    GLP_TRY(make_map16(&L.m_o, L.o, H, AWL, AWL, bn_for(H), true));
    GLP_TRY(make_map16(&L.m_gu, L.gu, 2 * F, H, H, 256, true));
    GLP_TRY(make_map16(&L.m_down, L.down, H, F, F, bn_for(H), true));
    GLP_TRY(make_map16(&L.p_qkv, L.qkv, L.qkv_w, H, H, 128, true));
    GLP_TRY(make_map16(&L.p_o, L.o, H, AWL, AWL, 128, true));
    GLP_TRY(make_map16(&L.p_gu, L.gu, 2 * F, H, H, 128, true));
    GLP_TRY(make_map16(&L.p_down, L.down, H, F, F, 128, true));
    if (c.ple_dim) {
      const int PD = c.ple_dim;
      GLP_TRY(upload_gain(d, g, p + "post_norm.weight", H, &L.ple_post));
      GLP_TRY(d.alloc(&L.ple_gate, static_cast<size_t>(PD) * H));
      GLP_TRY(d.alloc(&L.ple_proj, static_cast<size_t>(H) * PD));
      GLP_TRY(upload_linear(d, g, p + "inp_gate.weight", PD, H, L.ple_gate, 0, 0, 0, staging, staging_bytes));
      GLP_TRY(upload_linear(d, g, p + "proj.weight", H, PD, L.ple_proj, 0, 0, 0, staging, staging_bytes));
      GLP_TRY(make_map16(&L.m_pg, L.ple_gate, PD, H, H, bn_for(PD), true));
      GLP_TRY(make_map16(&L.p_pg, L.ple_gate, PD, H, H, 128, true));
      GLP_TRY(make_map16(&L.m_pp, L.ple_proj, H, PD, PD, bn_for(H), true));
      GLP_TRY(make_map16(&L.p_pp, L.ple_proj, H, PD, PD, 128, true));
    }
  }
  if (c.ple_dim) {
    const int LD = c.n_layers * c.ple_dim;
    GLP_TRY(upload_gain(d, g, "per_layer_proj_norm.weight", c.ple_dim, &d.ple_norm));
    GLP_TRY(d.alloc(&d.ple_w, static_cast<size_t>(LD) * H));
    GLP_TRY(upload_linear(d, g, "per_layer_model_proj.weight", LD, H, d.ple_w, 0, 0, 0, staging, staging_bytes));
    GLP_TRY(make_map16(&d.m_plew, d.ple_w, LD, H, H, bn_for(LD), true));
    GLP_TRY(make_map16(&d.p_plew, d.ple_w, LD, H, H, 128, true));
  }
  GLP_TRY(upload_gain(d, g, "output_norm.weight", H, &d.out_norm));
  // dense head: dense.0 .. dense.N (BASELINE two-stage 768->3072->768), else output.weight
  int prev = H;
  for (int j = 0;; ++j) {
    const std::string nm = "dense." + std::to_string(j) + ".weight";
    const glp::GgufTensor* t = g.tensor(nm);
    if (!t) break;
    HeadW hw;
    hw.n = static_cast<int>(t->ne.size() == 2 ? t->ne[1] : 0);
    hw.k = prev;
    if (hw.n % 128 || hw.k % 64) return fail(GLP_ERR_UNSUPPORTED, "dense head dims must be multiples of 128");
    hw.bn = bn_for(hw.n);
    GLP_TRY(d.alloc(&hw.w, static_cast<size_t>(hw.n) * hw.k));
    GLP_TRY(upload_linear(d, g, nm, hw.n, hw.k, hw.w, 0, 0, 0, staging, staging_bytes));
    GLP_TRY(make_map16(&hw.map, hw.w, hw.n, hw.k, hw.k, hw.bn, true));
    GLP_TRY(make_map16(&hw.map_pair, hw.w, hw.n, hw.k, hw.k, 128, true));
    d.head.push_back(hw);
    prev = hw.n;
  }
  if (d.head.empty()) {
    const glp::GgufTensor* t = g.tensor("output.weight");
    if (!t) return fail(GLP_ERR_FORMAT, "missing tensor output.weight");
    HeadW hw;
    hw.n = static_cast<int>(t->ne.size() == 2 ? t->ne[1] : 0);
    hw.k = H;
    if (hw.n % 128) return fail(GLP_ERR_UNSUPPORTED, "output.weight rows must be a multiple of 128");
    hw.bn = bn_for(hw.n);
    GLP_TRY(d.alloc(&hw.w, static_cast<size_t>(hw.n) * hw.k));
    GLP_TRY(upload_linear(d, g, "output.weight", hw.n, hw.k, hw.w, 0, 0, 0, staging, staging_bytes));
    GLP_TRY(make_map16(&hw.map, hw.w, hw.n, hw.k, hw.k, hw.bn, true));
    GLP_TRY(make_map16(&hw.map_pair, hw.w, hw.n, hw.k, hw.k, 128, true));
    d.head.push_back(hw);
  }
  if (d.head.back().n != c.emb_out) return fail(GLP_ERR_FORMAT, "head output dim != embedding_length_out");
  GLP_TRY(upload_rope(d, c.theta_swa, D, c.max_pos, &d.cs_swa));
  GLP_TRY(upload_rope(d, c.theta_full, D, c.max_pos, &d.cs_full));
  if (d512) GLP_TRY(upload_rope(d, c.theta_full, 512, c.max_pos, &d.cs_full512, true));

  // activations for one launch chunk
  d.cap_tokens = cap_tokens;
  d.cap_seqs = cap_seqs;
  int max_head = H;
  for (auto& hw : d.head) max_head = std::max(max_head, hw.n);
  GLP_TRY(d.alloc(&d.h, static_cast<size_t>(cap_tokens) * H));
  GLP_TRY(d.alloc(&d.xf, static_cast<size_t>(cap_tokens) * H));
  GLP_TRY(d.alloc(&d.x, static_cast<size_t>(cap_tokens) * H));
  GLP_TRY(d.alloc(&d.qkv, static_cast<size_t>(cap_tokens) * QKV));
  GLP_TRY(d.alloc(&d.attn, static_cast<size_t>(cap_tokens) * AW));
  GLP_TRY(d.alloc(&d.y, static_cast<size_t>(cap_tokens) * H));
  GLP_TRY(d.alloc(&d.a, static_cast<size_t>(cap_tokens) * F));
  if (c.ple_dim) {
    GLP_TRY(d.alloc(&d.ple, static_cast<size_t>(cap_tokens) * c.n_layers * c.ple_dim));
    GLP_TRY(d.alloc(&d.ple_g, static_cast<size_t>(cap_tokens) * c.ple_dim));
  }
  GLP_TRY(d.alloc(&d.pos, static_cast<size_t>(cap_tokens)));
  GLP_TRY(d.alloc(&d.pooled, static_cast<size_t>(cap_seqs) * max_head));  // also a head stage's output
  GLP_TRY(d.alloc(&d.pool_part, (static_cast<size_t>(cap_tokens) / glp::kPoolSeg + cap_seqs + 1) * H));
  GLP_TRY(d.alloc(&d.mid, static_cast<size_t>(cap_seqs) * max_head));
  GLP_TRY(d.alloc(&d.emb, static_cast<size_t>(cap_seqs) * max_head));
  GLP_TRY(d.alloc(&d.status, 1));
  GLP_CUDA(cudaMemset(d.status, 0, sizeof(int)));
  GLP_CUDA(cudaDeviceSynchronize());
  return GLP_OK;
}

// ------------------------------------------------------------------------------ forward
// One launch chunk: sequences [s0, s1) of the packed input; tokens are rows 0..T-1 of the
// activation buffers (global packed index = row + base).  h_cu (host offsets of the chunk's
// sequences) only feeds the profiler's algorithmic work counts.
int run_chunk(const Config& c, Device& d, const int* d_ids_chunk, const int* d_cu_chunk, const int* h_cu_chunk,
              int base, int n_seq, int T, int max_len, int out_dim, float* d_out, cudaStream_t st) {
  const int H = c.hidden, F = c.ffn;
  // layer 0's q|k|v and attention widths (layers of other widths re-encode their maps)
  const int QKV = d.layers.empty() ? 0 : d.layers[0].qkv_w;
  const int AW = d.layers.empty() ? 0 : c.n_heads * d.layers[0].hd;
  const float eps = static_cast<float>(c.eps);
  const double Td = T;
  auto gemm_flops = [&](double m, double n, double k) { return 2.0 * m * n * k; };
  auto gemm_bytes = [&](double m, double n, double k, double out_elem) { return 2.0 * m * k + 2.0 * n * k + out_elem * m * n; };
  if (T > 0) {
    GLP_TRY(prof_launch(d, st, kProfMisc, 0.0, 8.0 * Td, [&] {
      glp::positions_kernel<<<n_seq, 256, 0, st>>>(d_cu_chunk, base, n_seq, d.pos);
      GLP_CUDA(cudaGetLastError());
      return GLP_OK;
    }));
    const unsigned rows_grid = static_cast<unsigned>((T + 7) / 8);
    const float scale = static_cast<float>(std::sqrt(static_cast<double>(H)));
    // per-layer embeddings: the embedding rows x0 (f16, staged in y until layer 0's O
    // projection) feed the projection to [T, L * D]
    const int PD = c.ple_dim, LD = c.n_layers * c.ple_dim;
    const bool ple = PD != 0;
    const double row_in = d.table_type == glp::kGgmlQ8_0 ? H / 32 * 34.0 : 2.0 * H;
    GLP_TRY(prof_launch(d, st, kProfEmbed, 0.0, Td * (4.0 + row_in + 4.0 * H), [&] {
      return with_hidden(H, [&](auto hc) {
        constexpr int kH = decltype(hc)::value;
        if (d.table_type == glp::kGgmlQ8_0)
          glp::embed_gather_norm_kernel<kH><<<rows_grid, 256, 0, st>>>(static_cast<const uint8_t*>(d.table),
                                                                       d_ids_chunk, T, scale, d.layers[0].attn_norm,
                                                                       eps, d.h, d.x, ple ? d.y : nullptr);
        else
          glp::embed_gather_norm_bf16_kernel<kH><<<rows_grid, 256, 0, st>>>(
              static_cast<const __nv_bfloat16*>(d.table), d_ids_chunk, T, scale, d.layers[0].attn_norm, eps, d.h,
              d.x, ple ? d.y : nullptr);
        GLP_CUDA(cudaGetLastError());
        return GLP_OK;
      });
    }));

    CUtensorMap m_x, m_attn, m_a, m_qkv_out;
    GLP_TRY(make_map16(&m_x, d.x, T, H, H, 128, true));
    CUtensorMap m_pg;  // the PLE block's gate activations (the projection's A operand)
    if (ple) {
      CUtensorMap m_x0;
      GLP_TRY(make_map16(&m_x0, d.y, T, H, H, 128, true));
      GLP_TRY(make_map16(&m_pg, d.ple_g, T, PD, PD, 128, true));
      GemmParams pp{};
      pp.M = T;
      pp.N = LD;
      pp.K = H;
      pp.C = d.ple;
      pp.ldc = LD;
      pp.status = d.status;
      GLP_TRY(prof_launch(d, st, kProfPleGemm, gemm_flops(Td, LD, H), gemm_bytes(Td, LD, H, 2.0), [&] {
        return launch_gemm<__half>(m_x0, d.m_plew, bn_for(LD), glp::kEpiStore16, pp, st, &d.p_plew);
      }));
      const int64_t rows = static_cast<int64_t>(T) * c.n_layers;
      GLP_TRY(prof_launch(d, st, kProfPleRows, 0.0, 4.0 * rows * PD, [&] {
        glp::ple_norm_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(
            d.ple, rows, PD, static_cast<float>(std::pow(static_cast<double>(H), -0.5)), d.ple_norm, eps);
        GLP_CUDA(cudaGetLastError());
        return GLP_OK;
      }));
    }
    GLP_TRY(make_map16(&m_qkv_out, d.qkv, T, QKV, QKV, 32, true));  // the QKV epilogue's bulk stores
    CUtensorMap m_qkv_out2;  // the same for layers of another KV-head count (re-encoded when that width changes)
    int qkv_w2 = 0;
    GLP_TRY(make_map16(&m_attn, d.attn, T, AW, AW, 128, true));
    CUtensorMap m_attn2;  // the attention output of layers of another width
    int aw2 = 0;
    GLP_TRY(make_map16(&m_a, d.a, T, F, F, 128, true));
    double pairs_local = 0, pairs_global = 0;
    for (int b = 0; b < n_seq; ++b) {
      const int64_t len = h_cu_chunk[b + 1] - h_cu_chunk[b];
      pairs_local += visible_pairs(len, c.window);
      pairs_global += visible_pairs(len, 0);
    }

    const double post_bytes = Td * (2.0 * H + 4.0 * H + 2.0 * H);  // y + h in/out + x (16-bit)
    const double fused_bytes = Td * (4.0 * H + 2.0 * H);              // h in/out + x, no y
    // the row-norm GEMM covers 512-, 768- and 1024-wide rows (2-4 CTA pairs per cluster) and
    // needs the CTA-pair weight maps; other widths run the GEMM then post_norm_residual_kernel
    const bool fused = fused_norm_mode() != 0 && rownorm_width(H) && use_pair_gemm(glp::kEpiStore16);
    CUtensorMap m_h, m_xo;  // residual rows (loads and stores) and next pre-normed rows, 32-row boxes
    if (fused) GLP_TRY(make_map16(&m_h, d.h, T, H, H, 32, false));
    if (fused) GLP_TRY(make_map16(&m_xo, d.x, T, H, H, 32, true));
    for (int l = 0; l < c.n_layers; ++l) {
      LayerW& L = d.layers[l];
      GemmParams p{};
      p.M = T;
      p.K = H;
      p.status = d.status;
      // QKV projection + per-head RMSNorm + RoPE -> f16 qkv
      const int W = L.qkv_w;
      const CUtensorMap* m_out = &m_qkv_out;
      if (W != QKV) {
        if (W != qkv_w2) {
          GLP_TRY(make_map16(&m_qkv_out2, d.qkv, T, W, W, 32, true));
          qkv_w2 = W;
        }
        m_out = &m_qkv_out2;
      }
      p.N = W;
      p.C = d.qkv;
      p.ldc = W;
      p.q_gain = L.q_norm;
      p.k_gain = L.k_norm;
      p.rope_cs = L.sliding ? d.cs_swa : d.cs_full;
      p.pos = d.pos;
      p.rope_stride = c.max_pos;
      p.n_q_heads = c.n_heads;
      p.n_kv_heads = L.kv;
      p.eps = eps;
      const int DL = L.hd, AWL = c.n_heads * DL;
      if (DL == 256) {
        GLP_TRY(prof_launch(d, st, kProfGemmQkv, gemm_flops(Td, W, H), gemm_bytes(Td, W, H, 2.0),
                            [&] { return launch_gemm<__half>(m_x, L.m_qkv, 256, glp::kEpiQkv, p, st, &L.p_qkv, m_out); }));
      } else {
        // 512-wide heads span two 256-column tiles: the GEMM stores, then a row kernel applies
        // the per-head norms and the 512-wide RoPE (model.rs:279)
        GLP_TRY(prof_launch(d, st, kProfGemmQkv, gemm_flops(Td, W, H), gemm_bytes(Td, W, H, 2.0),
                            [&] { return launch_gemm<__half>(m_x, L.m_qkv, 256, glp::kEpiStore16, p, st, &L.p_qkv); }));
        const int64_t head_rows = static_cast<int64_t>(T) * (c.n_heads + 2 * L.kv);
        GLP_TRY(prof_launch(d, st, kProfGemmQkv, 0.0, 4.0 * Td * W, [&] {
          glp::qkv_norm_rope512_kernel<<<static_cast<unsigned>((head_rows + 7) / 8), 256, 0, st>>>(
              d.qkv, T, c.n_heads, L.kv, L.q_norm, L.k_norm, d.cs_full512, c.max_pos, d.pos, eps);
          GLP_CUDA(cudaGetLastError());
          return GLP_OK;
        }));
      }
      // attention
      const double pairs = L.sliding ? pairs_local : pairs_global;
      const double attn_bytes = 2.0 * Td * W + 2.0 * Td * AWL;
      GLP_TRY(prof_launch(d, st, kProfAttention, 4.0 * DL * c.n_heads * pairs, attn_bytes, [&] {
        return launch_attention(d.qkv, T, W, d_cu_chunk, base, n_seq, max_len, c.n_heads, L.kv,
                                L.sliding ? c.window : 0, d.attn, d.status, st, DL);
      }));
      const CUtensorMap* m_att = &m_attn;
      if (AWL != AW) {
        if (AWL != aw2) {
          GLP_TRY(make_map16(&m_attn2, d.attn, T, AWL, AWL, 128, true));
          aw2 = AWL;
        }
        m_att = &m_attn2;
      }
      // O projection
      GemmParams po{};
      po.M = T;
      po.N = H;
      po.K = AWL;
      po.C = d.y;
      po.ldc = H;
      po.status = d.status;
      if (fused) {
        po.h = d.h;
        po.x_next = d.x;
        po.w_post = L.post_attn;
        po.w_next = L.ffn_norm;
        po.layer_scalar = 1.0f;
        po.eps = eps;
        GLP_TRY(prof_launch(d, st, kProfGemmO, gemm_flops(Td, H, AWL), gemm_bytes(Td, H, AWL, 0.0) + fused_bytes,
                            [&] { return launch_rownorm_gemm(*m_att, L.p_o, m_h, m_xo, po, st); }));
      } else {
        GLP_TRY(prof_launch(d, st, kProfGemmO, gemm_flops(Td, H, AWL), gemm_bytes(Td, H, AWL, 2.0),
                            [&] { return launch_gemm<__half>(*m_att, L.m_o, bn_for(H), glp::kEpiStore16, po, st, &L.p_o); }));
        GLP_TRY(prof_launch(d, st, kProfPostNorm, 0.0, post_bytes, [&] {
          return with_hidden(H, [&](auto hc) {
            glp::post_norm_residual_kernel<decltype(hc)::value, glp::kPostNext>
                <<<rows_grid, 256, 0, st>>>(d.y, d.h, L.post_attn, 1.0f, L.ffn_norm, eps, T, d.x, nullptr);
            GLP_CUDA(cudaGetLastError());
            return GLP_OK;
          });
        }));
      }
      // gate|up + GeGLU
      GemmParams pg{};
      pg.M = T;
      pg.N = 2 * F;
      pg.K = H;
      pg.C = d.a;
      pg.ldc = F;
      pg.status = d.status;
      GLP_TRY(prof_launch(d, st, kProfGemmGateUp, gemm_flops(Td, 2.0 * F, H),
                          2.0 * Td * H + 2.0 * 2.0 * F * H + 2.0 * Td * F,
                          [&] { return launch_gemm<__half>(m_x, L.m_gu, 256, glp::kEpiGeglu, pg, st, &L.p_gu); }));
      // down projection
      GemmParams pd{};
      pd.M = T;
      pd.N = H;
      pd.K = F;
      pd.C = d.y;
      pd.ldc = H;
      pd.status = d.status;
      const bool last = l + 1 == c.n_layers;
      if (fused && !last && !ple) {
        pd.h = d.h;
        pd.x_next = d.x;
        pd.w_post = L.post_ffw;
        pd.w_next = d.layers[l + 1].attn_norm;
        pd.layer_scalar = L.layer_scalar;
        pd.eps = eps;
        GLP_TRY(prof_launch(d, st, kProfGemmDown, gemm_flops(Td, H, F), gemm_bytes(Td, H, F, 0.0) + fused_bytes,
                            [&] { return launch_rownorm_gemm(m_a, L.p_down, m_h, m_xo, pd, st); }));
        continue;
      }
      GLP_TRY(prof_launch(d, st, kProfGemmDown, gemm_flops(Td, H, F), gemm_bytes(Td, H, F, 2.0),
                          [&] { return launch_gemm<__half>(m_a, L.m_down, bn_for(H), glp::kEpiStore16, pd, st, &L.p_down); }));
      if (ple) {
        // ple.rs:118-145 after the FFN block: h2 = h + RMSNorm(y) w (kept raw in x for the
        // gate), g = geglu(gate(h2), P_l) in the gate GEMM's epilogue, y = proj(g), then the
        // post-norm, residual add and layer scalar of the shared tail below
        GLP_TRY(prof_launch(d, st, kProfPostNorm, 0.0, post_bytes, [&] {
          return with_hidden(H, [&](auto hc) {
            glp::post_norm_residual_kernel<decltype(hc)::value, glp::kPostRaw>
                <<<rows_grid, 256, 0, st>>>(d.y, d.h, L.post_ffw, 1.0f, nullptr, eps, T, d.x, nullptr);
            GLP_CUDA(cudaGetLastError());
            return GLP_OK;
          });
        }));
        // gate GEMM with the GeGLU against this layer's per-layer inputs in its epilogue
        GemmParams pg2{};
        pg2.M = T;
        pg2.N = PD;
        pg2.K = H;
        pg2.C = d.ple_g;
        pg2.ldc = PD;
        pg2.mul = d.ple + static_cast<size_t>(l) * PD;
        pg2.ld_mul = LD;
        pg2.status = d.status;
        GLP_TRY(prof_launch(d, st, kProfPleGemm, gemm_flops(Td, PD, H), gemm_bytes(Td, PD, H, 4.0), [&] {
          return launch_gemm<__half>(m_x, L.m_pg, bn_for(PD), glp::kEpiMulGeglu, pg2, st, &L.p_pg);
        }));
        GemmParams pp2{};
        pp2.M = T;
        pp2.N = H;
        pp2.K = PD;
        pp2.C = d.y;
        pp2.ldc = H;
        pp2.status = d.status;
        GLP_TRY(prof_launch(d, st, kProfPleGemm, gemm_flops(Td, H, PD), gemm_bytes(Td, H, PD, 2.0), [&] {
          return launch_gemm<__half>(m_pg, L.m_pp, bn_for(H), glp::kEpiStore16, pp2, st, &L.p_pp);
        }));
      }
      const float* w_tail = ple ? L.ple_post : L.post_ffw;
      GLP_TRY(prof_launch(d, st, kProfPostNorm, 0.0, last ? Td * 8.0 * H : post_bytes, [&] {
        return with_hidden(H, [&](auto hc) {
          constexpr int kH = decltype(hc)::value;
          if (!last)
            glp::post_norm_residual_kernel<kH, glp::kPostNext><<<rows_grid, 256, 0, st>>>(
                d.y, d.h, w_tail, L.layer_scalar, d.layers[l + 1].attn_norm, eps, T, d.x, nullptr);
          else
            glp::post_norm_residual_kernel<kH, glp::kPostFinal><<<rows_grid, 256, 0, st>>>(
                d.y, d.h, w_tail, L.layer_scalar, d.out_norm, eps, T, nullptr, d.xf);
          GLP_CUDA(cudaGetLastError());
          return GLP_OK;
        });
      }));
    }
  }
  // masked mean of the final-normed rows, then the dense head on the pooled vectors
  GLP_TRY(prof_launch(d, st, kProfPool, 0.0, 4.0 * Td * H + 2.0 * n_seq * H, [&] {
    const int segs = std::max(1, (max_len + glp::kPoolSeg - 1) / glp::kPoolSeg);
    const unsigned pool_threads = static_cast<unsigned>(H / 4);
    glp::mean_pool_kernel<<<dim3(static_cast<unsigned>(n_seq), static_cast<unsigned>(segs)), pool_threads, 0, st>>>(
        d.xf, d_cu_chunk, base, n_seq, H, d.pooled, nullptr, d.pool_part);
    if (segs > 1)
      glp::mean_pool_finish_kernel<<<n_seq, pool_threads, 0, st>>>(d_cu_chunk, base, n_seq, H, d.pool_part, d.pooled,
                                                                    nullptr);
    GLP_CUDA(cudaGetLastError());
    return GLP_OK;
  }));
  const __half* cur = d.pooled;
  int cur_k = H;
  for (size_t j = 0; j < d.head.size(); ++j) {
    HeadW& hw = d.head[j];
    const bool last = j + 1 == d.head.size();
    CUtensorMap m_in;
    GLP_TRY(make_map16(&m_in, cur, n_seq, cur_k, cur_k, 128, true));
    GemmParams ph{};
    ph.M = n_seq;
    ph.N = hw.n;
    ph.K = hw.k;
    ph.C = last ? static_cast<void*>(d.emb) : static_cast<void*>(j % 2 ? d.pooled : d.mid);
    ph.ldc = hw.n;
    ph.status = d.status;
    GLP_TRY(prof_launch(d, st, kProfHeadGemm, gemm_flops(n_seq, hw.n, hw.k),
                        gemm_bytes(n_seq, hw.n, hw.k, last ? 4.0 : 2.0),
                        [&] { return launch_gemm<__half>(m_in, hw.map, hw.bn, last ? glp::kEpiF32 : glp::kEpiStore16, ph, st, &hw.map_pair); }));
    cur = static_cast<const __half*>(ph.C);
    cur_k = hw.n;
  }
  GLP_TRY(prof_launch(d, st, kProfL2, 0.0, 4.0 * n_seq * (c.emb_out + out_dim), [&] {
    glp::l2_mrl_kernel<<<static_cast<unsigned>((n_seq + 7) / 8), 256, 0, st>>>(d.emb, n_seq, c.emb_out, out_dim, d_out);
    GLP_CUDA(cudaGetLastError());
    return GLP_OK;
  }));
  return GLP_OK;
}

// Small launch chunks are bound by launch latency (one 512-token sequence: 174 launches for about
// a millisecond of GPU work), so each chunk shape runs as an instantiated CUDA graph: captured
// from run_chunk on its first use, replayed afterwards.  The key holds every value that reaches
// a kernel parameter (the activation buffers, tensor maps and status word are fixed per device;
// token ids and sequence offsets are read from device memory at run time).  Not used while the
// per-kernel profiler records events, or with GLP_GRAPHS=0.
bool use_graphs() {
  static const bool on = [] {
    const char* e = std::getenv("GLP_GRAPHS");
    return !(e && std::string(e) == "0");
  }();
  return on;
}

constexpr size_t kMaxChunkGraphs = 16;

int run_chunk_graph(const Config& c, Device& d, const int* d_ids_chunk, const int* d_cu_chunk, const int* h_cu_chunk,
                    int base, int n_seq, int T, int max_len, int out_dim, float* d_out, cudaStream_t st) {
  // the legacy default stream cannot be captured, and a stream the caller is capturing
  // already records these launches into the caller's graph
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  const bool capturable = st != nullptr && st != cudaStreamLegacy && st != cudaStreamPerThread &&
                          cudaStreamIsCapturing(st, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone;
  if (!use_graphs() || d.prof_on || !capturable)
    return run_chunk(c, d, d_ids_chunk, d_cu_chunk, h_cu_chunk, base, n_seq, T, max_len, out_dim, d_out, st);
  const std::array<int64_t, 8> key{base, n_seq, T, max_len, out_dim, reinterpret_cast<int64_t>(d_ids_chunk),
                                   reinterpret_cast<int64_t>(d_cu_chunk), reinterpret_cast<int64_t>(d_out)};
  ++d.graph_clock;
  for (auto& g : d.graphs) {
    if (g.key != key) continue;
    GLP_CUDA(cudaGraphLaunch(g.exec, st));
    for (int k = 0; k < GLP_PROFILE_KINDS; ++k) {
      d.prof_launch[k] += g.launches[k];
      d.prof_flops[k] += g.flops[k];
      d.prof_bytes[k] += g.bytes[k];
    }
    g.last_use = d.graph_clock;
    return GLP_OK;
  }
  Device::ChunkGraph g;
  g.key = key;
  g.launches = d.prof_launch;
  g.flops = d.prof_flops;
  g.bytes = d.prof_bytes;
  GLP_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  const int rc = run_chunk(c, d, d_ids_chunk, d_cu_chunk, h_cu_chunk, base, n_seq, T, max_len, out_dim, d_out, st);
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(st, &graph);  // always ends the capture
  if (rc != GLP_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (ce != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return fail(GLP_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
  }
  const cudaError_t ie = cudaGraphInstantiate(&g.exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) return fail(GLP_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ie));
  for (int k = 0; k < GLP_PROFILE_KINDS; ++k) {  // what this chunk added to the counters
    g.launches[k] = d.prof_launch[k] - g.launches[k];
    g.flops[k] = d.prof_flops[k] - g.flops[k];
    g.bytes[k] = d.prof_bytes[k] - g.bytes[k];
  }
  g.last_use = d.graph_clock;
  GLP_CUDA(cudaGraphLaunch(g.exec, st));
  if (d.graphs.size() >= kMaxChunkGraphs) {  // evict the least recently used (after its launches)
    auto lru = std::min_element(d.graphs.begin(), d.graphs.end(),
                                [](const Device::ChunkGraph& x, const Device::ChunkGraph& y) { return x.last_use < y.last_use; });
    GLP_CUDA(cudaStreamSynchronize(st));
    cudaGraphExecDestroy(lru->exec);
    d.graphs.erase(lru);
  }
  d.graphs.push_back(g);
  return GLP_OK;
}

// Run all sequences of a packed input on one device, cutting launch chunks by token count.
int run_packed(const Config& c, Device& d, const int* d_ids, const int* d_cu, const int* h_cu, int n_seq, int out_dim,
               float* d_out, cudaStream_t st) {
  // d_ids[h_cu[b] .. h_cu[b+1]) are the tokens of sequence b (offsets index d_ids)
  int s0 = 0;
  while (s0 < n_seq) {
    int s1 = s0;
    int max_len = 0;
    while (s1 < n_seq && s1 - s0 < d.cap_seqs &&
           static_cast<int64_t>(h_cu[s1 + 1]) - h_cu[s0] <= d.cap_tokens) {
      max_len = std::max(max_len, h_cu[s1 + 1] - h_cu[s1]);
      ++s1;
    }
    if (s1 == s0) return fail(GLP_ERR_INVALID_ARG, "sequence longer than the launch chunk (max_batch_tokens)");
    const int base = h_cu[s0];
    const int T = h_cu[s1] - base;
    GLP_TRY(run_chunk_graph(c, d, d_ids + base, d_cu + s0, h_cu + s0, base, s1 - s0, T, max_len, out_dim,
                            d_out + static_cast<size_t>(s0) * out_dim, st));
    s0 = s1;
  }
  return GLP_OK;
}

int grow_staging(Device& d, int64_t tokens, int64_t seqs, int64_t outs) {
  if (tokens > d.stage_tokens) {
    d.raw_free(d.d_ids, std::max<int64_t>(d.stage_tokens, 1) * sizeof(int));
    if (d.h_ids) cudaFreeHost(d.h_ids);
    d.d_ids = nullptr;
    d.h_ids = nullptr;
    d.stage_tokens = 0;
    void* v = nullptr;
    GLP_TRY(d.raw_malloc(&v, std::max<int64_t>(tokens, 1) * sizeof(int)));
    d.d_ids = static_cast<int*>(v);
    GLP_CUDA(cudaHostAlloc(&d.h_ids, std::max<int64_t>(tokens, 1) * sizeof(int), cudaHostAllocDefault));
    d.stage_tokens = tokens;
  }
  if (seqs > d.stage_seqs) {
    d.raw_free(d.d_cu, (d.stage_seqs + 1) * sizeof(int));
    if (d.h_cu) cudaFreeHost(d.h_cu);
    d.d_cu = nullptr;
    d.h_cu = nullptr;
    d.stage_seqs = 0;
    void* v = nullptr;
    GLP_TRY(d.raw_malloc(&v, (seqs + 1) * sizeof(int)));
    d.d_cu = static_cast<int*>(v);
    GLP_CUDA(cudaHostAlloc(&d.h_cu, (seqs + 1) * sizeof(int), cudaHostAllocDefault));
    d.stage_seqs = seqs;
  }
  if (outs > d.stage_out) {
    d.raw_free(d.d_out, std::max<int64_t>(d.stage_out, 1) * sizeof(float));
    if (d.h_out) cudaFreeHost(d.h_out);
    d.d_out = nullptr;
    d.h_out = nullptr;
    d.stage_out = 0;
    void* v = nullptr;
    GLP_TRY(d.raw_malloc(&v, std::max<int64_t>(outs, 1) * sizeof(float)));
    d.d_out = static_cast<float*>(v);
    GLP_CUDA(cudaHostAlloc(&d.h_out, std::max<int64_t>(outs, 1) * sizeof(float), cudaHostAllocDefault));
    d.stage_out = outs;
  }
  return GLP_OK;
}

const char* status_text(int code) {
  switch (code) {
    case glp::kErrNone: return "no device error";
    case glp::kErrTimeoutProducer: return "a TMA producer's wait for a free pipeline stage timed out";
    case glp::kErrTimeoutMma: return "the MMA issuer's wait for operands or a free accumulator timed out";
    case glp::kErrTimeoutEpilogue: return "an epilogue wait (accumulator, row exchange or load) timed out";
    case glp::kErrTimeoutDrain: return "the wait for the last MMAs to retire timed out";
    case glp::kErrBadArgs: return "a kernel found its shared memory misaligned and did no work";
    case glp::kErrTimeoutSelfTest: return "the self-test's wait on a barrier nobody arrives at ran out, as intended";
    default: return "unknown device status code";
  }
}

int check_status(Device& d) {
  int st = 0;
  GLP_CUDA(cudaMemcpy(&st, d.status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st != 0) {
    cudaMemset(d.status, 0, sizeof(int));
    return fail(GLP_ERR_DEVICE, "device pipeline wait timed out (status " + std::to_string(st) + ": " +
                                    status_text(st) + ")");
  }
  return GLP_OK;
}

// Host-API shard on one device: pack, H2D, forward, D2H (all on the device's stream).  The
// embeddings stay in the device's pinned staging buffer (d.h_out); the caller copies them out
// once every shard has succeeded, so a failed call leaves the caller's buffer untouched.
int run_shard(const Config& c, Device& d, const int32_t* ids, const int32_t* lengths, int s0, int s1, int max_len,
              int out_dim, float* ms) {
  GLP_CUDA(cudaSetDevice(d.dev));
  const int n = s1 - s0;
  int64_t tokens = 0;
  for (int i = s0; i < s1; ++i) tokens += lengths[i];
  GLP_TRY(grow_staging(d, tokens, n, static_cast<int64_t>(n) * out_dim));
  int64_t off = 0;
  d.h_cu[0] = 0;
  for (int i = 0; i < n; ++i) {
    const int len = lengths[s0 + i];
    std::memcpy(d.h_ids + off, ids + static_cast<int64_t>(s0 + i) * max_len, len * sizeof(int));
    off += len;
    d.h_cu[i + 1] = static_cast<int>(off);
  }
  cudaStream_t st = d.stream;
  GLP_CUDA(cudaEventRecord(d.ev0, st));
  GLP_CUDA(cudaMemcpyAsync(d.d_ids, d.h_ids, tokens * sizeof(int), cudaMemcpyHostToDevice, st));
  GLP_CUDA(cudaMemcpyAsync(d.d_cu, d.h_cu, (n + 1) * sizeof(int), cudaMemcpyHostToDevice, st));
  GLP_TRY(run_packed(c, d, d.d_ids, d.d_cu, d.h_cu, n, out_dim, d.d_out, st));
  GLP_CUDA(cudaMemcpyAsync(d.h_out, d.d_out, static_cast<size_t>(n) * out_dim * sizeof(float), cudaMemcpyDeviceToHost,
                           st));
  GLP_CUDA(cudaEventRecord(d.ev1, st));
  GLP_CUDA(cudaStreamSynchronize(st));
  GLP_TRY(check_status(d));
  if (ms) cudaEventElapsedTime(ms, d.ev0, d.ev1);
  return GLP_OK;
}

// Contiguous shards [bounds[i], bounds[i+1]) of n_seq sequences for nd workers, balanced by
// token count (total = sum of lengths).
std::vector<int> shard_bounds(const int32_t* lengths, int n_seq, int nd, int64_t total) {
  std::vector<int> bounds(nd + 1, n_seq);
  bounds[0] = 0;
  int64_t acc = 0;
  int k = 1;
  for (int i = 0; i < n_seq && k < nd; ++i) {
    acc += lengths[i];
    while (k < nd && acc * nd >= total * k) bounds[k++] = i + 1;
  }
  for (; k < nd; ++k) bounds[k] = n_seq;
  return bounds;
}

// work(i) for every worker i in [0, nd): one host thread each (the calling thread alone when
// nd == 1, or for the workers no thread could be created for); the caller's current device is
// restored afterwards.
template <class Work>
void run_shards(int nd, Work&& work, bool cuda_workers = true) {
  int prev = 0;
  if (cuda_workers) cudaGetDevice(&prev);
  if (nd == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    int spawned = 0;
    try {
      for (; spawned < nd; ++spawned) th.emplace_back(work, spawned);
    } catch (const std::exception&) {  // no more threads: the calling thread runs the other shards
      for (int i = spawned; i < nd; ++i) work(i);
    }
    for (auto& t : th) t.join();
  }
  if (cuda_workers) cudaSetDevice(prev);
}

// ------------------------------------------------------------------------------ kernel-level scratch
struct Scratch {
  std::mutex mu;
  std::array<__nv_bfloat16*, 64> w{};
  std::array<size_t, 64> cap{};
  std::array<int*, 64> status{};
  std::array<__half*, 64> gu{};  // glp_gate_up_geglu's interleaved weight
  std::array<size_t, 64> gu_cap{};
  struct Rope {
    int dev;
    double theta;
    int max_pos;
    float2* cs;
  };
  std::vector<Rope> rope;  // glp_qkv_norm_rope's tables, kept per (device, theta, max_pos)
};
Scratch g_scratch;

// RoPE table of head_dim 256 for (theta, max_pos) on the current device, built once (the
// values of rope.rs:14-76, the layout of upload_rope) and kept until the process exits.
int kernel_rope_table(int dev, double theta, int max_pos, const float2** out) {
  std::lock_guard<std::mutex> lk(g_scratch.mu);
  for (const auto& r : g_scratch.rope)
    if (r.dev == dev && r.theta == theta && r.max_pos == max_pos) {
      *out = r.cs;
      return GLP_OK;
    }
  constexpr int kHalf = 128;
  std::vector<float> inv(kHalf);
  for (int i = 0; i < kHalf; ++i) inv[i] = static_cast<float>(1.0 / std::pow(theta, (2.0 * i) / 256.0));
  std::vector<float2> c(static_cast<size_t>(max_pos) * kHalf);
  for (int i = 0; i < kHalf; ++i)
    for (int p = 0; p < max_pos; ++p) {
      const float f = static_cast<float>(p) * inv[i];
      c[(static_cast<size_t>(i >> 1) * max_pos + p) * 2 + (i & 1)] = make_float2(std::cos(f), std::sin(f));
    }
  float2* cs = nullptr;
  GLP_CUDA(cudaMalloc(&cs, c.size() * sizeof(float2)));
  const cudaError_t e = cudaMemcpy(cs, c.data(), c.size() * sizeof(float2), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(cs);
    return fail(GLP_ERR_CUDA, std::string("RoPE table upload: ") + cudaGetErrorString(e));
  }
  g_scratch.rope.push_back({dev, theta, max_pos, cs});
  *out = cs;
  return GLP_OK;
}

int device_status_word(int dev, int** out) {
  std::lock_guard<std::mutex> lk(g_scratch.mu);
  if (!g_scratch.status[dev]) {
    GLP_CUDA(cudaMalloc(&g_scratch.status[dev], sizeof(int)));
    GLP_CUDA(cudaMemset(g_scratch.status[dev], 0, sizeof(int)));
  }
  *out = g_scratch.status[dev];
  return GLP_OK;
}

int run_bf16_gemm(const __nv_bfloat16* w, int N, int K, const void* x, int M, void* y, int y_is_f32, cudaStream_t st,
                  bool dependent = false) {
  if (N <= 0 || K <= 0 || M < 0 || N % 128 || K % 64)
    return fail(GLP_ERR_INVALID_ARG, "GEMM needs N % 128 == 0, K % 64 == 0, M >= 0");
  if (!w || !x || !y) return fail(GLP_ERR_INVALID_ARG, "null pointer");
  GLP_TRY(ensure_kernel_attrs());
  int dev = 0;
  GLP_CUDA(cudaGetDevice(&dev));
  int* status = nullptr;
  GLP_TRY(device_status_word(dev, &status));
  if (M == 0) return GLP_OK;
  const int bn = bn_for(N);
  CUtensorMap ma, mb, mbp;
  GLP_TRY(make_map16(&ma, x, M, K, K, 128, false));
  GLP_TRY(make_map16(&mb, w, N, K, K, bn, false));
  GLP_TRY(make_map16(&mbp, w, N, K, K, 128, false));
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = y;
  p.ldc = N;
  p.status = status;
  return launch_gemm<__nv_bfloat16>(ma, mb, bn, y_is_f32 ? glp::kEpiF32 : glp::kEpiStore16, p, st, &mbp, nullptr,
                                    dependent);
}

}  // namespace

// ------------------------------------------------------------------------------ bounded-wait self-test
// One thread waits, with the kernels' bounded wait, on an mbarrier that nobody arrives at: the
// wait must run out after limit_ns and record kErrTimeoutSelfTest in the status word, and the
// kernel returns normally (no trap, no fault), so the context stays usable.
__global__ void wait_selftest_kernel(uint64_t limit_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    glp::mbar_init(&bar, 1);
    abort_flag = 0;
    glp::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !glp::mbar_wait(&bar, 0, &abort_flag, limit_ns)) glp::record_error(status, glp::kErrTimeoutSelfTest);
}

// ------------------------------------------------------------------------------ no-allocation GEMM
// glp_q8_0_gemm_noalloc keeps its dequantised weight in this file-scope device array instead
// of memory the library allocates: every GPU that loads the library holds the array (6 MiB
// of bf16) until the process exits, and every call on a device shares it.
constexpr int64_t kNoAllocMaxWeightElems = 3 * 1024 * 1024;  // N * K limit of the entry point
static __device__ __align__(256) __nv_bfloat16 g_noalloc_weight[kNoAllocMaxWeightElems];
static __device__ int g_noalloc_status;

namespace {

struct NoAllocDevicePtrs {
  std::mutex mu;
  std::array<__nv_bfloat16*, 64> weight{};
  std::array<int*, 64> status{};
};
NoAllocDevicePtrs g_noalloc_ptrs;

// Device addresses of the file-scope scratch on the current device, looked up once per device
// with that device current (the host-side names are only stand-ins for them).
int noalloc_pointers(int dev, __nv_bfloat16** weight, int** status) {
  std::lock_guard<std::mutex> lk(g_noalloc_ptrs.mu);
  if (!g_noalloc_ptrs.weight[dev]) {
    void* w = nullptr;
    void* s = nullptr;
    GLP_CUDA(cudaGetSymbolAddress(&w, g_noalloc_weight));
    GLP_CUDA(cudaGetSymbolAddress(&s, g_noalloc_status));
    g_noalloc_ptrs.weight[dev] = static_cast<__nv_bfloat16*>(w);
    g_noalloc_ptrs.status[dev] = static_cast<int*>(s);
  }
  *weight = g_noalloc_ptrs.weight[dev];
  *status = g_noalloc_ptrs.status[dev];
  return GLP_OK;
}

}  // namespace

// ================================================================================= C ABI
namespace glp {
// for the engine (engine.cpp): set the calling thread's glp_last_error() message
void set_last_error(const std::string& msg) { t_err = msg; }
}  // namespace glp

extern "C" {

const char* glp_last_error(void) { return t_err.c_str(); }

int glp_open(const char* gguf_path, const int* device_ids, int n_devices, const glp_options* opt, glp_ctx** out) {
  if (!out) return fail(GLP_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  if (!gguf_path) return fail(GLP_ERR_INVALID_ARG, "gguf_path is NULL");
  if (n_devices < 0 || n_devices > GLP_MAX_DEVICES) return fail(GLP_ERR_INVALID_ARG, "bad device count");
  glp::GgufFile g;
  std::string err;
  if (!g.open(gguf_path, &err)) return fail(err.rfind("cannot open", 0) == 0 ? GLP_ERR_IO : GLP_ERR_FORMAT, err);
  auto ctx = std::make_unique<glp_ctx>();
  GLP_TRY(parse_config(g, &ctx->cfg));
  GLP_TRY(validate_tensors(g, ctx->cfg));
  if (const glp::GgufTensor* q = g.tensor("blk.0.attn_q.weight")) ctx->cfg.linear_type = q->type;
  int64_t cap_tokens = opt && opt->max_batch_tokens > 0 ? opt->max_batch_tokens : 262144;
  cap_tokens = std::max<int64_t>(cap_tokens, ctx->cfg.max_pos);
  const int cap_seqs = opt && opt->max_batch_seqs > 0 ? opt->max_batch_seqs : 4096;
  // the caller's device-memory limit, checked against the plan before any device is touched
  ctx->plan_bytes = device_plan_bytes(g, ctx->cfg, cap_tokens, cap_seqs);
  const int64_t limit = opt && opt->device_memory_limit_mib > 0 ? static_cast<int64_t>(opt->device_memory_limit_mib) << 20 : 0;
  const int64_t peak = ctx->plan_bytes + static_cast<int64_t>(load_staging_bytes(g, ctx->cfg));
  if (limit > 0 && peak > limit)
    return fail(GLP_ERR_OOM, "the model needs " + std::to_string((peak + (1 << 20) - 1) >> 20) +
                                 " MiB of device memory per device (weights, RoPE tables and one launch chunk of " +
                                 std::to_string(cap_tokens) + " tokens), above the limit of " +
                                 std::to_string(opt->device_memory_limit_mib) + " MiB");
  std::vector<int> ids;
  if (n_devices == 0 || !device_ids) {
    int cur = 0;
    GLP_CUDA(cudaGetDevice(&cur));
    ids.push_back(cur);
  } else {
    ids.assign(device_ids, device_ids + n_devices);
  }
  int ndev_avail = 0;
  GLP_CUDA(cudaGetDeviceCount(&ndev_avail));
  for (int id : ids)
    if (id < 0 || id >= ndev_avail) return fail(GLP_ERR_INVALID_ARG, "device id out of range");
  int prev = 0;
  cudaGetDevice(&prev);
  for (int id : ids) {
    auto d = std::make_unique<Device>();
    d->dev = id;
    d->limit_bytes = limit;
    const int rc = setup_device(*d, ctx->cfg, g, cap_tokens, cap_seqs);
    if (rc != GLP_OK) {
      const std::string keep = t_err;
      d->release();
      for (auto& e : ctx->devs) e->release();
      cudaSetDevice(prev);
      t_err = keep;
      return rc;
    }
    if (d->bytes != ctx->plan_bytes) {  // the plan the limit is checked against must be exact
      const std::string msg = "device memory plan " + std::to_string(ctx->plan_bytes) + " B differs from the " +
                              std::to_string(d->bytes) + " B allocated";
      d->release();
      for (auto& e : ctx->devs) e->release();
      cudaSetDevice(prev);
      return fail(GLP_ERR_CUDA, msg);
    }
    ctx->devs.push_back(std::move(d));
  }
  cudaSetDevice(prev);
  *out = ctx.release();
  return GLP_OK;
}

void glp_close(glp_ctx* ctx) {
  if (!ctx) return;
  int prev = 0;
  cudaGetDevice(&prev);
  for (auto& d : ctx->devs) d->release();
  cudaSetDevice(prev);
  delete ctx;
}

int glp_model_info(const glp_ctx* ctx, glp_model_info_t* info) {
  if (!ctx || !info) return fail(GLP_ERR_INVALID_ARG, "NULL argument");
  const Config& c = ctx->cfg;
  info->n_layers = c.n_layers;
  info->hidden = c.hidden;
  info->ffn = c.ffn;
  info->n_heads = c.n_heads;
  info->n_kv_heads = c.n_kv;
  info->head_dim = c.head_dim;
  info->vocab = c.vocab;
  info->embedding_dim = c.emb_out;
  info->max_position = c.max_pos;
  info->sliding_window = c.window;
  info->weight_type = static_cast<int>(c.linear_type);
  info->n_devices = static_cast<int>(ctx->devs.size());
  info->device_bytes = ctx->devs.empty() ? ctx->plan_bytes : ctx->devs[0]->bytes;
  return GLP_OK;
}

int glp_embed_tokens(glp_ctx* ctx, const int32_t* ids, const int32_t* lengths, int n_seq, int max_len, int out_dim,
                     float* out, glp_timing* timing) {
  if (!ctx) return fail(GLP_ERR_INVALID_ARG, "ctx is NULL");
  const Config& c = ctx->cfg;
  if (n_seq < 0 || max_len < 0) return fail(GLP_ERR_INVALID_ARG, "negative batch shape");
  if (n_seq > 0 && (!ids || !lengths || !out)) return fail(GLP_ERR_INVALID_ARG, "NULL buffer");
  if (out_dim <= 0 || out_dim > c.emb_out)
    return fail(GLP_ERR_INVALID_ARG, "out_dim must be in (0, " + std::to_string(c.emb_out) + "]");
  if (max_len > c.max_pos)
    return fail(GLP_ERR_CONTEXT_LIMIT, "Input sequence length (" + std::to_string(max_len) +
                                           ") exceeds model max_position_embeddings (" + std::to_string(c.max_pos) + ")");
  int64_t total = 0;
  for (int i = 0; i < n_seq; ++i) {
    if (lengths[i] < 0 || lengths[i] > max_len) return fail(GLP_ERR_INVALID_ARG, "length out of [0, max_len]");
    const int32_t* row = ids + static_cast<int64_t>(i) * max_len;
    for (int j = 0; j < lengths[i]; ++j)
      if (row[j] < 0 || row[j] >= c.vocab)
        return fail(GLP_ERR_INVALID_ARG, "token id " + std::to_string(row[j]) + " outside the vocabulary");
    total += lengths[i];
  }
  const int nd = static_cast<int>(ctx->devs.size());
  if (timing) {
    timing->n_devices = nd;
    for (int i = 0; i < GLP_MAX_DEVICES; ++i) timing->device_ms[i] = 0.f;
  }
  if (n_seq == 0) return GLP_OK;
  const std::vector<int> bounds = shard_bounds(lengths, n_seq, nd, total);
  std::vector<int> rcs(nd, GLP_OK);
  std::vector<std::string> errs(nd);
  std::vector<float> ms(nd, 0.f);
  run_shards(nd, [&](int i) {
    if (bounds[i] >= bounds[i + 1]) return;
    rcs[i] = run_shard(c, *ctx->devs[i], ids, lengths, bounds[i], bounds[i + 1], max_len, out_dim, &ms[i]);
    if (rcs[i] != GLP_OK) errs[i] = t_err;
  });
  for (int i = 0; i < nd; ++i) {
    if (timing && i < GLP_MAX_DEVICES) timing->device_ms[i] = ms[i];
    if (rcs[i] != GLP_OK) return fail(rcs[i], "device " + std::to_string(ctx->devs[i]->dev) + ": " + errs[i]);
  }
  // every shard succeeded: only now do the embeddings reach the caller's buffer
  for (int i = 0; i < nd; ++i)
    if (bounds[i] < bounds[i + 1])
      std::memcpy(out + static_cast<size_t>(bounds[i]) * out_dim, ctx->devs[i]->h_out,
                  static_cast<size_t>(bounds[i + 1] - bounds[i]) * out_dim * sizeof(float));
  return GLP_OK;
}

int glp_embed_tokens_sharded(const glp_batch_fn* fns, void* const* users, int n_executors, int embedding_dim,
                             const int32_t* ids, const int32_t* lengths, int n_seq, int max_len, int out_dim,
                             float* out) {
  if (!fns || n_executors <= 0 || n_executors > GLP_MAX_DEVICES) return fail(GLP_ERR_INVALID_ARG, "bad executor list");
  for (int i = 0; i < n_executors; ++i)
    if (!fns[i]) return fail(GLP_ERR_INVALID_ARG, "NULL executor");
  if (n_seq < 0 || max_len < 0) return fail(GLP_ERR_INVALID_ARG, "negative batch shape");
  if (n_seq > 0 && (!ids || !lengths || !out)) return fail(GLP_ERR_INVALID_ARG, "NULL buffer");
  if (out_dim <= 0 || out_dim > embedding_dim)
    return fail(GLP_ERR_INVALID_ARG, "out_dim must be in (0, " + std::to_string(embedding_dim) + "]");
  int64_t total = 0;
  for (int i = 0; i < n_seq; ++i) {
    if (lengths[i] < 0 || lengths[i] > max_len) return fail(GLP_ERR_INVALID_ARG, "length out of [0, max_len]");
    total += lengths[i];
  }
  if (n_seq == 0) return GLP_OK;
  const int nd = n_executors;
  const std::vector<int> bounds = shard_bounds(lengths, n_seq, nd, total);
  std::vector<int> rcs(nd, GLP_OK);
  std::vector<std::string> errs(nd);
  std::vector<std::vector<float>> part(nd);
  run_shards(
      nd,
      [&](int i) {
        const int s0 = bounds[i], s1 = bounds[i + 1];
        if (s0 >= s1) return;
        try {
          part[i].assign(static_cast<size_t>(s1 - s0) * out_dim, 0.f);
        } catch (const std::exception&) {
          rcs[i] = GLP_ERR_OOM;
          errs[i] = "out of host memory";
          return;
        }
        t_err.clear();
        rcs[i] = fns[i](users ? users[i] : nullptr, ids + static_cast<int64_t>(s0) * max_len, lengths + s0, s1 - s0,
                        max_len, out_dim, part[i].data());
        if (rcs[i] != GLP_OK) errs[i] = t_err.empty() ? "executor failed with status " + std::to_string(rcs[i]) : t_err;
      },
      false);
  for (int i = 0; i < nd; ++i)
    if (rcs[i] != GLP_OK) return fail(rcs[i], "executor " + std::to_string(i) + ": " + errs[i]);
  for (int i = 0; i < nd; ++i)
    if (bounds[i] < bounds[i + 1]) std::memcpy(out + static_cast<size_t>(bounds[i]) * out_dim, part[i].data(),
                                               part[i].size() * sizeof(float));
  return GLP_OK;
}

int glp_embed_packed_device(glp_ctx* ctx, int dev_index, const int32_t* d_ids, const int32_t* d_cu_seqlens,
                            const int32_t* h_cu_seqlens, int n_seq, int out_dim, float* d_out, void* stream) {
  if (!ctx) return fail(GLP_ERR_INVALID_ARG, "ctx is NULL");
  if (dev_index < 0 || dev_index >= static_cast<int>(ctx->devs.size())) return fail(GLP_ERR_INVALID_ARG, "bad dev_index");
  const Config& c = ctx->cfg;
  if (n_seq < 0 || (n_seq > 0 && (!d_ids || !d_cu_seqlens || !h_cu_seqlens || !d_out)))
    return fail(GLP_ERR_INVALID_ARG, "NULL buffer");
  if (out_dim <= 0 || out_dim > c.emb_out) return fail(GLP_ERR_INVALID_ARG, "bad out_dim");
  for (int i = 0; i < n_seq; ++i) {
    const int len = h_cu_seqlens[i + 1] - h_cu_seqlens[i];
    if (len < 0) return fail(GLP_ERR_INVALID_ARG, "cu_seqlens must be non-decreasing");
    if (len > c.max_pos)
      return fail(GLP_ERR_CONTEXT_LIMIT, "Input sequence length (" + std::to_string(len) +
                                             ") exceeds model max_position_embeddings (" + std::to_string(c.max_pos) + ")");
  }
  Device& d = *ctx->devs[dev_index];
  int prev = 0;
  cudaGetDevice(&prev);
  GLP_CUDA(cudaSetDevice(d.dev));
  const int rc = run_packed(c, d, d_ids, d_cu_seqlens, h_cu_seqlens, n_seq, out_dim, d_out,
                            static_cast<cudaStream_t>(stream));
  cudaSetDevice(prev);
  return rc;
}

int glp_device_status(glp_ctx* ctx, int dev_index, int* status) {
  if (!ctx || !status || dev_index < 0 || dev_index >= static_cast<int>(ctx->devs.size()))
    return fail(GLP_ERR_INVALID_ARG, "bad argument");
  Device& d = *ctx->devs[dev_index];
  int prev = 0;
  cudaGetDevice(&prev);
  GLP_CUDA(cudaSetDevice(d.dev));
  const cudaError_t e = cudaMemcpy(status, d.status, sizeof(int), cudaMemcpyDeviceToHost);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(GLP_ERR_CUDA, cudaGetErrorString(e));
  return GLP_OK;
}

int glp_profile_enable(glp_ctx* ctx, int dev_index, int enable) {
  if (!ctx || dev_index < 0 || dev_index >= static_cast<int>(ctx->devs.size()))
    return fail(GLP_ERR_INVALID_ARG, "bad argument");
  Device& d = *ctx->devs[dev_index];
  d.prof_on = enable != 0;
  d.prof_used = 0;
  d.prof_launch.fill(0);
  d.prof_flops.fill(0.0);
  d.prof_bytes.fill(0.0);
  return GLP_OK;
}

int glp_profile_read(glp_ctx* ctx, int dev_index, glp_profile* out) {
  if (!ctx || !out || dev_index < 0 || dev_index >= static_cast<int>(ctx->devs.size()))
    return fail(GLP_ERR_INVALID_ARG, "bad argument");
  Device& d = *ctx->devs[dev_index];
  int prev = 0;
  cudaGetDevice(&prev);
  GLP_CUDA(cudaSetDevice(d.dev));
  std::memset(out, 0, sizeof(*out));
  out->n_kinds = GLP_PROFILE_KINDS;
  for (int k = 0; k < GLP_PROFILE_KINDS; ++k) {
    out->names[k] = kProfNames[k];
    out->launches[k] = d.prof_launch[k];
    out->flops[k] = d.prof_flops[k];
    out->bytes[k] = d.prof_bytes[k];
    out->total_launches += d.prof_launch[k];
  }
  for (size_t i = 0; i < d.prof_used; ++i) {
    float ms = 0.f;
    GLP_CUDA(cudaEventSynchronize(d.prof_ev[i][1]));
    GLP_CUDA(cudaEventElapsedTime(&ms, d.prof_ev[i][0], d.prof_ev[i][1]));
    out->total_ms[d.prof_kind[i]] += ms;
  }
  d.prof_used = 0;
  d.prof_launch.fill(0);
  d.prof_flops.fill(0.0);
  d.prof_bytes.fill(0.0);
  cudaSetDevice(prev);
  return GLP_OK;
}

int glp_q8_0_dequant(const void* d_blocks, int64_t n_blocks, float* d_out, void* stream) {
  if (n_blocks < 0 || (n_blocks > 0 && (!d_blocks || !d_out))) return fail(GLP_ERR_INVALID_ARG, "bad argument");
  if (reinterpret_cast<uintptr_t>(d_out) & 15) return fail(GLP_ERR_INVALID_ARG, "output must be 16-byte aligned");
  if (n_blocks == 0) return GLP_OK;
  glp::q8_0_dequant_f32_kernel<<<static_cast<unsigned>((n_blocks + 255) / 256), 256, 0,
                                  static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t*>(d_blocks), n_blocks,
                                                                      d_out);
  GLP_CUDA(cudaGetLastError());
  return GLP_OK;
}

int glp_q8_0_gemm(const void* d_q8_w, int N, int K, const void* d_x_bf16, int M, void* d_y, int y_is_f32,
                  void* stream) {
  if (N <= 0 || K <= 0 || N % 128 || K % 64 || M < 0)
    return fail(GLP_ERR_INVALID_ARG, "Q8_0 GEMM needs N % 128 == 0, K % 64 == 0, M >= 0");
  if (!d_q8_w || !d_x_bf16 || !d_y) return fail(GLP_ERR_INVALID_ARG, "null pointer");
  int dev = 0;
  GLP_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(GLP_ERR_INVALID_ARG, "device index out of range");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Two routes, chosen by measurement (B200, bf16 out): up to M = 8192 rows one launch of the
  // kernel that streams the raw rows and dequantises them in shared memory (768 x 768 at
  // M = 512: 13.7 vs 25 us; at M = 4096: 16.7 vs 24 us); above it the weight is dequantised
  // into library scratch and the bf16 CTA-pair GEMM runs (M = 131072: 124 vs 170 us; the
  // fused kernel's tensor pipe waits on the dequantisation warps there).  A weight that is not
  // 16-byte aligned (a row slice of a fused weight) always takes the second route.
  // GLP_Q8_GEMM=fused or =two-pass forces one route (for A/B measurements; read on every call).
  const int route = [] {
    const char* e = std::getenv("GLP_Q8_GEMM");
    if (e && std::strcmp(e, "two-pass") == 0) return 2;
    if (e && std::strcmp(e, "fused") == 0) return 1;
    return 0;
  }();
  constexpr int kFusedMaxM = 8192;
  const bool fused = !(reinterpret_cast<uintptr_t>(d_q8_w) & 15) && (route == 1 || (route == 0 && M <= kFusedMaxM));
  if (fused) {
    GLP_TRY(ensure_kernel_attrs());
    int* status = nullptr;
    GLP_TRY(device_status_word(dev, &status));
    if (M == 0) return GLP_OK;
    CUtensorMap ma;
    GLP_TRY(make_map16(&ma, d_x_bf16, M, K, K, 128, false));
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.C = d_y;
    p.ldc = N;
    p.status = status;
    return launch_q8_gemm(ma, d_q8_w, y_is_f32 != 0, p, st);
  }
  __nv_bfloat16* w = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_scratch.mu);
    const size_t need = static_cast<size_t>(N) * K;
    if (g_scratch.cap[dev] < need) {
      if (g_scratch.w[dev]) {
        cudaStreamSynchronize(st);
        cudaFree(g_scratch.w[dev]);
        g_scratch.w[dev] = nullptr;
        g_scratch.cap[dev] = 0;
      }
      GLP_CUDA(cudaMalloc(&g_scratch.w[dev], need * sizeof(__nv_bfloat16)));
      g_scratch.cap[dev] = need;
    }
    w = g_scratch.w[dev];
  }
  const int64_t nb = static_cast<int64_t>(N) * (K / 32);
  glp::q8_0_dequant_rows_kernel<__nv_bfloat16><<<static_cast<unsigned>((nb + 255) / 256), 256, 0, st>>>(
      static_cast<const uint8_t*>(d_q8_w), N, K, w, 0, 0, 0);
  GLP_CUDA(cudaGetLastError());
  // the GEMM as the dequantisation's dependent launch: its prologue overlaps that kernel
  return run_bf16_gemm(w, N, K, d_x_bf16, M, d_y, y_is_f32, st, true);
}

int glp_bf16_gemm(const void* d_w_bf16, int N, int K, const void* d_x_bf16, int M, void* d_y, int y_is_f32,
                  void* stream) {
  return run_bf16_gemm(static_cast<const __nv_bfloat16*>(d_w_bf16), N, K, d_x_bf16, M, d_y, y_is_f32,
                       static_cast<cudaStream_t>(stream));
}

int glp_flash_attention(const void* d_qkv, const int32_t* d_cu_seqlens, int n_seq, int max_len, int n_q_heads,
                        int n_kv_heads, int head_dim, int window, void* d_out, void* stream) {
  if (head_dim != glp::kFaD && head_dim != glp::kF5D) return fail(GLP_ERR_UNSUPPORTED, "head_dim must be 256 or 512");
  if (n_seq < 0 || max_len < 0 || n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads)
    return fail(GLP_ERR_INVALID_ARG, "bad attention shape");
  if (n_seq == 0 || max_len == 0) return GLP_OK;
  if (!d_qkv || !d_cu_seqlens || !d_out) return fail(GLP_ERR_INVALID_ARG, "null pointer");
  GLP_TRY(ensure_kernel_attrs());
  int dev = 0;
  GLP_CUDA(cudaGetDevice(&dev));
  int* status = nullptr;
  GLP_TRY(device_status_word(dev, &status));
  const int ld = (n_q_heads + 2 * n_kv_heads) * head_dim;
  int total = 0;
  GLP_CUDA(cudaMemcpy(&total, d_cu_seqlens + n_seq, sizeof(int), cudaMemcpyDeviceToHost));
  return launch_attention(static_cast<const __half*>(d_qkv), total, ld, d_cu_seqlens, 0, n_seq, max_len, n_q_heads,
                          n_kv_heads, window, static_cast<__half*>(d_out), status,
                          static_cast<cudaStream_t>(stream), head_dim);
}

// Variant of glp_q8_0_gemm for callers that cannot allocate device memory: the dequantised
// weight goes into the library's file-scope scratch array instead of a cudaMalloc'd buffer,
// and the call itself allocates nothing.  N * K must not exceed kNoAllocMaxWeightElems.
int glp_q8_0_gemm_noalloc(const void* d_q8_w, int N, int K, const void* d_x_bf16, int M, void* d_y, int y_is_f32,
                          void* stream) {
  if (N <= 0 || K <= 0 || N % 128 || K % 64 || M < 0)
    return fail(GLP_ERR_INVALID_ARG, "Q8_0 GEMM needs N % 128 == 0, K % 64 == 0, M >= 0");
  if (static_cast<int64_t>(N) * K > kNoAllocMaxWeightElems)
    return fail(GLP_ERR_INVALID_ARG, "glp_q8_0_gemm_noalloc: weight of " + std::to_string(static_cast<int64_t>(N) * K) +
                                         " elements exceeds the no-allocation scratch limit of " +
                                         std::to_string(kNoAllocMaxWeightElems) + " (N * K)");
  if (!d_q8_w || !d_x_bf16 || !d_y) return fail(GLP_ERR_INVALID_ARG, "null pointer");
  int dev = 0;
  GLP_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(GLP_ERR_INVALID_ARG, "device index out of range");
  __nv_bfloat16* w = nullptr;
  int* status = nullptr;
  GLP_TRY(noalloc_pointers(dev, &w, &status));
  GLP_TRY(ensure_kernel_attrs());
  if (M == 0) return GLP_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t nb = static_cast<int64_t>(N) * (K / 32);
  glp::q8_0_dequant_rows_kernel<__nv_bfloat16><<<static_cast<unsigned>((nb + 255) / 256), 256, 0, st>>>(
      static_cast<const uint8_t*>(d_q8_w), N, K, w, 0, 0, 0);
  GLP_CUDA(cudaGetLastError());
  const int bn = bn_for(N);
  // tensor maps are host-side descriptors: building them allocates no device memory; with the
  // 128-row map the GEMM runs the same kernel (CTA pairs or single CTAs) as glp_q8_0_gemm
  CUtensorMap ma, mb, mbp;
  GLP_TRY(make_map16(&ma, d_x_bf16, M, K, K, 128, false));
  GLP_TRY(make_map16(&mb, w, N, K, K, bn, false));
  GLP_TRY(make_map16(&mbp, w, N, K, K, 128, false));
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = d_y;
  p.ldc = N;
  p.status = status;
  return launch_gemm<__nv_bfloat16>(ma, mb, bn, y_is_f32 ? glp::kEpiF32 : glp::kEpiStore16, p, st, &mbp);
}

const char* glp_status_text(int status) { return status_text(status); }

int glp_kernel_status(int device, int* status) {
  if (!status) return fail(GLP_ERR_INVALID_ARG, "status is NULL");
  *status = 0;
  int n = 0;
  GLP_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n || device >= 64) return fail(GLP_ERR_INVALID_ARG, "device index out of range");
  int prev = 0;
  cudaGetDevice(&prev);
  GLP_CUDA(cudaSetDevice(device));
  int code = 0;
  const cudaError_t se = cudaDeviceSynchronize();
  int* word = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_scratch.mu);
    word = g_scratch.status[device];
  }
  cudaError_t e = se;
  if (e == cudaSuccess && word) {
    int v = 0;
    e = cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && v != 0) e = cudaMemset(word, 0, sizeof(int));
    if (v != 0) code = v;
  }
  bool noalloc_used = false;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_ptrs.mu);
    noalloc_used = g_noalloc_ptrs.status[device] != nullptr;
  }
  if (e == cudaSuccess && noalloc_used) {  // symbol copies: nothing is allocated
    int v = 0;
    e = cudaMemcpyFromSymbol(&v, g_noalloc_status, sizeof(int));
    if (e == cudaSuccess && v != 0) {
      const int zero = 0;
      e = cudaMemcpyToSymbol(g_noalloc_status, &zero, sizeof(int));
      if (code == 0) code = v;
    }
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(GLP_ERR_CUDA, std::string("reading the kernel status: ") + cudaGetErrorString(e));
  *status = code;
  if (code != 0)
    return fail(GLP_ERR_DEVICE, "device status " + std::to_string(code) + ": " + status_text(code));
  return GLP_OK;
}

int glp_selftest_wait_timeout(int device, int limit_us) {
  if (limit_us <= 0 || limit_us > 2000000) return fail(GLP_ERR_INVALID_ARG, "limit_us must be in (0, 2000000]");
  int n = 0;
  GLP_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n || device >= 64) return fail(GLP_ERR_INVALID_ARG, "device index out of range");
  int prev = 0;
  cudaGetDevice(&prev);
  GLP_CUDA(cudaSetDevice(device));
  int* status = nullptr;
  int rc = device_status_word(device, &status);
  if (rc == GLP_OK) {
    wait_selftest_kernel<<<1, 32>>>(static_cast<uint64_t>(limit_us) * 1000ull, status);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) rc = fail(GLP_ERR_CUDA, std::string("self-test kernel: ") + cudaGetErrorString(e));
  }
  cudaSetDevice(prev);
  return rc;
}

int glp_gate_up_geglu(const void* d_w_gate, const void* d_w_up, int F, int K, const void* d_x, int M, void* d_out,
                      void* stream) {
  if (F <= 0 || K <= 0 || M < 0 || F % 128 || K % 64)
    return fail(GLP_ERR_INVALID_ARG, "gate/up GEMM needs F % 128 == 0, K % 64 == 0, M >= 0");
  if (!d_w_gate || !d_w_up || !d_x || !d_out) return fail(GLP_ERR_INVALID_ARG, "null pointer");
  GLP_TRY(ensure_kernel_attrs());
  int dev = 0;
  GLP_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(GLP_ERR_INVALID_ARG, "device index out of range");
  int* status = nullptr;
  GLP_TRY(device_status_word(dev, &status));
  if (M == 0) return GLP_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __half* gu = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_scratch.mu);
    const size_t need = static_cast<size_t>(2) * F * K;
    if (g_scratch.gu_cap[dev] < need) {
      if (g_scratch.gu[dev]) {
        cudaDeviceSynchronize();
        cudaFree(g_scratch.gu[dev]);
        g_scratch.gu[dev] = nullptr;
        g_scratch.gu_cap[dev] = 0;
      }
      GLP_CUDA(cudaMalloc(&g_scratch.gu[dev], need * sizeof(__half)));
      g_scratch.gu_cap[dev] = need;
    }
    gu = g_scratch.gu[dev];
  }
  // the model path's layout: tile t of 256 rows = [gate rows 128t.. | up rows 128t..]
  const size_t blk = static_cast<size_t>(128) * K * sizeof(__half);
  GLP_CUDA(cudaMemcpy2DAsync(gu, 2 * blk, d_w_gate, blk, blk, F / 128, cudaMemcpyDeviceToDevice, st));
  GLP_CUDA(cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(gu) + blk, 2 * blk, d_w_up, blk, blk, F / 128,
                             cudaMemcpyDeviceToDevice, st));
  CUtensorMap ma, mb, mbp;
  GLP_TRY(make_map16(&ma, d_x, M, K, K, 128, true));
  GLP_TRY(make_map16(&mb, gu, 2 * F, K, K, 256, true));
  GLP_TRY(make_map16(&mbp, gu, 2 * F, K, K, 128, true));
  GemmParams p{};
  p.M = M;
  p.N = 2 * F;
  p.K = K;
  p.C = d_out;
  p.ldc = F;
  p.status = status;
  return launch_gemm<__half>(ma, mb, 256, glp::kEpiGeglu, p, st, &mbp);
}

int glp_qkv_norm_rope(const void* d_w_qkv, int n_q_heads, int n_kv_heads, int K, const void* d_x, int M,
                      const float* d_q_gain, const float* d_k_gain, const int32_t* d_pos, double theta, int max_pos,
                      float eps, void* d_out, void* stream) {
  if (n_q_heads <= 0 || n_kv_heads <= 0 || K <= 0 || K % 64 || M < 0 || max_pos <= 0 || !(theta > 0.0))
    return fail(GLP_ERR_INVALID_ARG, "QKV GEMM needs heads > 0, K % 64 == 0, M >= 0, max_pos > 0, theta > 0");
  if (!d_w_qkv || !d_x || !d_q_gain || !d_k_gain || !d_pos || !d_out) return fail(GLP_ERR_INVALID_ARG, "null pointer");
  if ((reinterpret_cast<uintptr_t>(d_q_gain) | reinterpret_cast<uintptr_t>(d_k_gain)) & 15)
    return fail(GLP_ERR_INVALID_ARG, "gains must be 16-byte aligned");
  GLP_TRY(ensure_kernel_attrs());
  int dev = 0;
  GLP_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(GLP_ERR_INVALID_ARG, "device index out of range");
  int* status = nullptr;
  GLP_TRY(device_status_word(dev, &status));
  if (M == 0) return GLP_OK;
  const float2* cs = nullptr;
  GLP_TRY(kernel_rope_table(dev, theta, max_pos, &cs));
  const int W = (n_q_heads + 2 * n_kv_heads) * glp::kFaD;
  CUtensorMap ma, mb, mbp, mc;
  GLP_TRY(make_map16(&ma, d_x, M, K, K, 128, true));
  GLP_TRY(make_map16(&mb, d_w_qkv, W, K, K, 256, true));
  GLP_TRY(make_map16(&mbp, d_w_qkv, W, K, K, 128, true));
  GLP_TRY(make_map16(&mc, d_out, M, W, W, 32, true));
  GemmParams p{};
  p.M = M;
  p.N = W;
  p.K = K;
  p.C = d_out;
  p.ldc = W;
  p.q_gain = d_q_gain;
  p.k_gain = d_k_gain;
  p.rope_cs = cs;
  p.pos = d_pos;
  p.rope_stride = max_pos;
  p.n_q_heads = n_q_heads;
  p.n_kv_heads = n_kv_heads;
  p.eps = eps;
  p.status = status;
  return launch_gemm<__half>(ma, mb, 256, glp::kEpiQkv, p, static_cast<cudaStream_t>(stream), &mbp, &mc);
}

}  // extern "C"
