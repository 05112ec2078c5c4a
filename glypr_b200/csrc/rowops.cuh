// Memory-bound row kernels (one warp per token row, 128-bit vector accesses, warp-shuffle
// reductions) and the Q8_0 dequantisation kernels.
//
// Residual stream h is bf16 [T, H] (the hidden-state type of the reference's Metal path; f32
// arithmetic on every update); the GEMM inputs x are f16 [T, H] (every GEMM input is a
// normalised row or a convex combination of normalised rows, so f16's range suffices and its
// 11-bit mantissa keeps the dequantised weights and activations close to exact).
#pragma once
#include "common.cuh"

namespace glp {

// The row kernels are compiled per hidden size H: a multiple of 256 up to kMaxHidden (the
// BASELINE model has H = 768).
constexpr int kMaxHidden = 2048;

// ---------------------------------------------------------------------------- Q8_0
// Exact dequantisation f32(d) * q (the product of an int8 and an fp16 value is exact in
// f32, so this is bit-identical to any correct dequantiser).  One thread per 32-block.
__global__ void q8_0_dequant_f32_kernel(const uint8_t* __restrict__ blocks, int64_t n_blocks,
                                        float* __restrict__ out) {
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= n_blocks) return;
  const uint8_t* src = blocks + b * 34;
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(src[0] | (src[1] << 8))));
  float4* dst = reinterpret_cast<float4*>(out + b * 32);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int8_t* s = reinterpret_cast<const int8_t*>(src + 2 + 4 * q);
    dst[q] = make_float4(s[0] * d, s[1] * d, s[2] * d, s[3] * d);
  }
}

// Dequantise a Q8_0 matrix [N, K] into 16-bit rows of a destination matrix.  Row n goes to
//   dst_row = group ? (n / group) * group_stride + row_base + n % group : row_base + n
// which builds the fused QKV weight (row_base offsets) and the gate/up interleave
// (group = 128, group_stride = 256, row_base = 0 for gate and 128 for up).
template <typename T>
__global__ void q8_0_dequant_rows_kernel(const uint8_t* __restrict__ blocks, int n, int k, T* __restrict__ dst,
                                         int row_base, int group, int group_stride) {
  griddep_launch();  // a GEMM launched after this one as its dependent may start its prologue
  const int nb = k / 32;
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= static_cast<int64_t>(n) * nb) return;
  const int row = static_cast<int>(b / nb), blk = static_cast<int>(b % nb);
  const int drow = group ? (row / group) * group_stride + row_base + row % group : row_base + row;
  const uint8_t* src = blocks + b * 34;
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(src[0] | (src[1] << 8))));
  uint4* out = reinterpret_cast<uint4*>(dst + static_cast<size_t>(drow) * k + blk * 32);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int8_t* s = reinterpret_cast<const int8_t*>(src + 2 + 8 * q);
    uint4 u;
    u.x = Half16<T>::pack(s[0] * d, s[1] * d);
    u.y = Half16<T>::pack(s[2] * d, s[3] * d);
    u.z = Half16<T>::pack(s[4] * d, s[5] * d);
    u.w = Half16<T>::pack(s[6] * d, s[7] * d);
    out[q] = u;
  }
}

// bf16 [N, K] source (BF16 GGUF weights) converted into the same fused/interleaved layout.
template <typename T>
__global__ void bf16_rows_convert_kernel(const __nv_bfloat16* __restrict__ src, int n, int k, T* __restrict__ dst,
                                         int row_base, int group, int group_stride) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // 2-element pairs
  const int per_row = k / 2;
  if (i >= static_cast<int64_t>(n) * per_row) return;
  const int row = static_cast<int>(i / per_row), c = static_cast<int>(i % per_row);
  const int drow = group ? (row / group) * group_stride + row_base + row % group : row_base + row;
  const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(src + static_cast<size_t>(row) * k)[c];
  const float2 f = __bfloat1622float2(v);
  reinterpret_cast<uint32_t*>(dst + static_cast<size_t>(drow) * k)[c] = Half16<T>::pack(f.x, f.y);
}

// ---------------------------------------------------------------------------- helpers
__device__ __forceinline__ void load_f32x8(const float* p, float* v) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void store_f32x8(float* p, const float* v) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <typename T>
__device__ __forceinline__ void store16x8(T* p, const float* v) {
  uint4 u;
  u.x = Half16<T>::pack(v[0], v[1]);
  u.y = Half16<T>::pack(v[2], v[3]);
  u.z = Half16<T>::pack(v[4], v[5]);
  u.w = Half16<T>::pack(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ---------------------------------------------------------------------------- embedding
// h[t] = dequant(E[id_t]) * f32(sqrt(H))   (model.rs:252-255, 507-508)
// x[t] = f16(RMSNorm(h[t]) * w)             (first layer's attn_norm, norm.rs:22-63)
// x_raw[t] = f16(h[t] in f32), when given    (the per-layer-embedding projection's input)
// One warp per token; lane l covers elements l, l+32, ... (coalesced byte reads of the
// 34-byte blocks).
template <int H>
__global__ void embed_gather_norm_kernel(const uint8_t* __restrict__ table, const int* __restrict__ ids,
                                         int n_tokens, float scale, const float* __restrict__ w, float eps,
                                         __nv_bfloat16* __restrict__ h, __half* __restrict__ x,
                                         __half* __restrict__ x_raw) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= n_tokens) return;
  const uint8_t* row = table + static_cast<size_t>(ids[t]) * (H / 32) * 34;
  float v[H / 32];
  float ss = 0.f;
#pragma unroll
  for (int b = 0; b < H / 32; ++b) {
    const uint8_t* blk = row + b * 34;
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
    const float q = static_cast<float>(static_cast<int8_t>(blk[2 + lane]));
    v[b] = (q * d) * scale;
    ss = fmaf(v[b], v[b], ss);
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(H) + eps);
  __nv_bfloat16* hr = h + static_cast<size_t>(t) * H;
  __half* xr = x + static_cast<size_t>(t) * H;
#pragma unroll
  for (int b = 0; b < H / 32; ++b) {
    const int e = b * 32 + lane;
    hr[e] = __float2bfloat16_rn(v[b]);
    xr[e] = __float2half_rn(v[b] * inv * __ldg(w + e));
    if (x_raw) x_raw[static_cast<size_t>(t) * H + e] = __float2half_rn(v[b]);
  }
}

// Same gather for a bf16 token table (BF16 GGUF).
template <int H>
__global__ void embed_gather_norm_bf16_kernel(const __nv_bfloat16* __restrict__ table, const int* __restrict__ ids,
                                              int n_tokens, float scale, const float* __restrict__ w, float eps,
                                              __nv_bfloat16* __restrict__ h, __half* __restrict__ x,
                                              __half* __restrict__ x_raw) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= n_tokens) return;
  const __nv_bfloat16* row = table + static_cast<size_t>(ids[t]) * H;
  float v[H / 32];
  float ss = 0.f;
#pragma unroll
  for (int b = 0; b < H / 32; ++b) {
    v[b] = __bfloat162float(row[b * 32 + lane]) * scale;
    ss = fmaf(v[b], v[b], ss);
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(H) + eps);
  __nv_bfloat16* hr = h + static_cast<size_t>(t) * H;
  __half* xr = x + static_cast<size_t>(t) * H;
#pragma unroll
  for (int b = 0; b < H / 32; ++b) {
    const int e = b * 32 + lane;
    hr[e] = __float2bfloat16_rn(v[b]);
    xr[e] = __float2half_rn(v[b] * inv * __ldg(w + e));
    if (x_raw) x_raw[static_cast<size_t>(t) * H + e] = __float2half_rn(v[b]);
  }
}

// ---------------------------------------------------------------------------- post-norm
// h <- (h + RMSNorm(y) * w_post) * layer_scalar            (norm.rs:65-94, layer.rs:20-50)
// then, by MODE:
//   kPostNext : the next pre-norm x = f16(RMSNorm(h) * w_next), h updated (bf16)
//   kPostFinal: the final norm RMSNorm(h) * w_next written to xf in f32 (output_norm, model.rs:576)
//   kPostRaw  : x = f16(h) without a norm, h updated (the per-layer-embedding block's gate
//               input is the un-normalised residual, ple.rs:130)
// All arithmetic in f32.  One warp per row; lane owns elements [c*256 + lane*8, +8).  Up to
// H = 768 capped at 64 registers (4 blocks of 8 rows per SM) for more rows in flight (H = 768:
// 5.26 -> 5.56 TB/s); wider rows keep 2 blocks per SM (1 above 1536, no spills).
constexpr int kPostNext = 0, kPostFinal = 1, kPostRaw = 2;

template <int H, int MODE>
__global__ void __launch_bounds__(256, H <= 768 ? 4 : (H <= 1536 ? 2 : 1)) post_norm_residual_kernel(const __half* __restrict__ y, __nv_bfloat16* __restrict__ h,
                                          const float* __restrict__ w_post, float layer_scalar,
                                          const float* __restrict__ w_next, float eps, int n_tokens,
                                          __half* __restrict__ x, float* __restrict__ xf) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  constexpr int kVec = H / 256;  // 8-element chunks per lane
  if (t >= n_tokens) return;
  const __half* yr = y + static_cast<size_t>(t) * H;
  __nv_bfloat16* hr = h + static_cast<size_t>(t) * H;
  // raw 16-bit rows (12 + 12 registers): converted where used, so 4 blocks fit an SM
  uint4 yu[kVec], hu[kVec];
#pragma unroll
  for (int c = 0; c < kVec; ++c) {
    yu[c] = *reinterpret_cast<const uint4*>(yr + c * 256 + lane * 8);
    hu[c] = *reinterpret_cast<const uint4*>(hr + c * 256 + lane * 8);
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kVec; ++c) {
    const __half* e = reinterpret_cast<const __half*>(&yu[c]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __half2float(e[j]);
      ss = fmaf(v, v, ss);
    }
  }
  ss = warp_sum(ss);
  const float inv_y = 1.0f / sqrtf(ss / static_cast<float>(H) + eps);
  float ss2 = 0.f;
  float hv[kVec][8];
#pragma unroll
  for (int c = 0; c < kVec; ++c) {
    const int e0 = c * 256 + lane * 8;
    float wv[8];
    load_f32x8(w_post + e0, wv);
    const __half* ye = reinterpret_cast<const __half*>(&yu[c]);
    const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hu[c]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      hv[c][j] = (__bfloat162float(he[j]) + __half2float(ye[j]) * inv_y * wv[j]) * layer_scalar;
      ss2 = fmaf(hv[c][j], hv[c][j], ss2);
    }
  }
  if constexpr (MODE == kPostRaw) {
#pragma unroll
    for (int c = 0; c < kVec; ++c) {
      const int e0 = c * 256 + lane * 8;
      store16x8<__nv_bfloat16>(hr + e0, hv[c]);
      store16x8<__half>(x + static_cast<size_t>(t) * H + e0, hv[c]);
    }
    return;
  }
  ss2 = warp_sum(ss2);
  const float inv_h = 1.0f / sqrtf(ss2 / static_cast<float>(H) + eps);
#pragma unroll
  for (int c = 0; c < kVec; ++c) {
    const int e0 = c * 256 + lane * 8;
    float wv[8], o[8];
    load_f32x8(w_next + e0, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = hv[c][j] * inv_h * wv[j];
    if constexpr (MODE == kPostFinal) {
      store_f32x8(xf + static_cast<size_t>(t) * H + e0, o);
    } else {
      store16x8<__nv_bfloat16>(hr + e0, hv[c]);
      store16x8<__half>(x + static_cast<size_t>(t) * H + e0, o);
    }
  }
}

// ---------------------------------------------------------------------------- positions
// pos[t] = position of token t inside its sequence (RoPE positions restart at 0 for every
// right-padded sequence, rope.rs:53-76).  Block per sequence.
__global__ void positions_kernel(const int* __restrict__ cu_seqlens, int cu_base, int n_seq, int* __restrict__ pos) {
  const int b = blockIdx.x;
  if (b >= n_seq) return;
  const int t0 = cu_seqlens[b] - cu_base, t1 = cu_seqlens[b + 1] - cu_base;
  for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x) pos[t] = t - t0;
}

// ---------------------------------------------------------------------------- pooling
// pooled[b] = sum_{t in seq b} xf[t] / max(len_b, 1e-9)   (model.rs:671-680), f32, fixed
// summation order (deterministic, independent of the other sequences of the batch).
// Block (sequence b, segment s) sums tokens [512 s, 512 s + 512) of the sequence in order,
// H / 4 threads x 4 columns.  A sequence of at most 512 tokens is one segment and is finished in
// place; longer ones leave per-segment sums in `part` at slot floor(t0 / 512) + b + s (t0 = the
// sequence's first token in the chunk: distinct for every (b, s), below T / 512 + n_seq), and
// mean_pool_finish_kernel adds them in segment order.
constexpr int kPoolSeg = 512;

__device__ __forceinline__ void pool_write(float4 acc, float cnt, int b, int c, int H, __half* pooled16,
                                           float* pooled_f32) {
  acc.x /= cnt;
  acc.y /= cnt;
  acc.z /= cnt;
  acc.w /= cnt;
  if (pooled_f32) *reinterpret_cast<float4*>(pooled_f32 + static_cast<size_t>(b) * H + c) = acc;
  uint2 pk;
  pk.x = pack_f16(acc.x, acc.y);
  pk.y = pack_f16(acc.z, acc.w);
  *reinterpret_cast<uint2*>(pooled16 + static_cast<size_t>(b) * H + c) = pk;
}

__global__ void mean_pool_kernel(const float* __restrict__ xf, const int* __restrict__ cu_seqlens, int cu_base,
                                 int n_seq, int H, __half* __restrict__ pooled16, float* __restrict__ pooled_f32,
                                 float* __restrict__ part) {
  const int b = blockIdx.x, sg = blockIdx.y;
  if (b >= n_seq) return;
  const int t0 = cu_seqlens[b] - cu_base, t1 = cu_seqlens[b + 1] - cu_base;
  const int n_segs = max(1, (t1 - t0 + kPoolSeg - 1) / kPoolSeg);
  if (sg >= n_segs) return;
  const int c = threadIdx.x * 4;
  if (c >= H) return;
  const int s0 = t0 + sg * kPoolSeg, s1 = min(t1, s0 + kPoolSeg);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int t = s0; t < s1; ++t) {
    const float4 v = *reinterpret_cast<const float4*>(xf + static_cast<size_t>(t) * H + c);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  if (n_segs == 1) {
    pool_write(acc, fmaxf(static_cast<float>(t1 - t0), 1e-9f), b, c, H, pooled16, pooled_f32);
  } else {
    const size_t slot = static_cast<size_t>(t0 / kPoolSeg + b + sg);
    *reinterpret_cast<float4*>(part + slot * H + c) = acc;
  }
}

__global__ void mean_pool_finish_kernel(const int* __restrict__ cu_seqlens, int cu_base, int n_seq, int H,
                                        const float* __restrict__ part, __half* __restrict__ pooled16,
                                        float* __restrict__ pooled_f32) {
  const int b = blockIdx.x;
  if (b >= n_seq) return;
  const int t0 = cu_seqlens[b] - cu_base, t1 = cu_seqlens[b + 1] - cu_base;
  const int n_segs = max(1, (t1 - t0 + kPoolSeg - 1) / kPoolSeg);
  if (n_segs == 1) return;  // finished by mean_pool_kernel
  const int c = threadIdx.x * 4;
  if (c >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int sg = 0; sg < n_segs; ++sg) {
    const float4 v = *reinterpret_cast<const float4*>(part + static_cast<size_t>(t0 / kPoolSeg + b + sg) * H + c);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  pool_write(acc, static_cast<float>(t1 - t0), b, c, H, pooled16, pooled_f32);
}

// L2-normalise (clamp 1e-12) then MRL: the first out_dim values renormalised
// (model.rs:682-698).  One warp per sequence; e is f32 [n_seq, dim].
__global__ void l2_mrl_kernel(const float* __restrict__ e, int n_seq, int dim, int out_dim,
                              float* __restrict__ out) {
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= n_seq) return;
  const float* r = e + static_cast<size_t>(b) * dim;
  float ss = 0.f;
  for (int j = lane; j < dim; j += 32) ss = fmaf(r[j], r[j], ss);
  ss = warp_sum(ss);
  const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
  float* o = out + static_cast<size_t>(b) * out_dim;
  if (out_dim >= dim) {
    for (int j = lane; j < dim; j += 32) o[j] = r[j] * inv;
    return;
  }
  float s2 = 0.f;
  for (int j = lane; j < out_dim; j += 32) {
    const float v = r[j] * inv;
    s2 = fmaf(v, v, s2);
  }
  s2 = warp_sum(s2);
  const float inv2 = 1.0f / fmaxf(sqrtf(s2), 1e-12f);
  for (int j = lane; j < out_dim; j += 32) o[j] = (r[j] * inv) * inv2;
}

}  // namespace glp

namespace glp {

// ---------------------------------------------------------------------------- 512-wide heads
// Per-head RMSNorm + NeoX RoPE of the QKV GEMM's output for layers with head_dim 512 (the
// 256-wide heads have it fused into the GEMM epilogue): qkv [T, (Hq + 2 Hkv) * 512] f16 in
// place.  One warp per (token, head): lane l holds dims 8l .. 8l + 7 of the lower half and
// 256 + 8l .. of the upper half, i.e. its 8 RoPE pairs (i, i + 256).  Query heads take
// q_gain, key heads k_gain (both then rotated with the position-major table cs [pos][256] of
// {cos, sin}, rope.rs:14-106 values: a lane's 8 frequencies are 64 contiguous bytes), value
// heads are normalised without a gain (attention/mod.rs:166-188, model.rs:371-373).
__global__ void qkv_norm_rope512_kernel(__half* __restrict__ qkv, int64_t T, int n_q_heads, int n_kv_heads,
                                        const float* __restrict__ q_gain, const float* __restrict__ k_gain,
                                        const float2* __restrict__ cs, int rope_stride, const int* __restrict__ pos,
                                        float eps) {
  const int heads = n_q_heads + 2 * n_kv_heads;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wid >= T * heads) return;
  const int lane = threadIdx.x & 31;
  const int64_t t = wid / heads;
  const int h = static_cast<int>(wid - t * heads);
  __half* row = qkv + t * static_cast<int64_t>(heads) * 512 + static_cast<int64_t>(h) * 512;
  uint4 lo4 = reinterpret_cast<const uint4*>(row)[lane];
  uint4 hi4 = reinterpret_cast<const uint4*>(row + 256)[lane];
  const __half* lo = reinterpret_cast<const __half*>(&lo4);
  const __half* hi = reinterpret_cast<const __half*>(&hi4);
  float x1[8], x2[8];
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    x1[e] = __half2float(lo[e]);
    x2[e] = __half2float(hi[e]);
    ss = fmaf(x1[e], x1[e], ss);
    ss = fmaf(x2[e], x2[e], ss);
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / 512.0f + eps);
  const bool is_q = h < n_q_heads, is_k = !is_q && h < n_q_heads + n_kv_heads;
  const float* gain = is_q ? q_gain : (is_k ? k_gain : nullptr);
  const int p = (is_q || is_k) ? min(max(pos[t], 0), rope_stride - 1) : 0;
  uint32_t olo[4], ohi[4];
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    float a[2], b[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = 8 * lane + e + u;
      float v1 = x1[e + u] * inv, v2 = x2[e + u] * inv;
      if (gain) {
        v1 *= __ldg(gain + i);
        v2 *= __ldg(gain + 256 + i);
      }
      if (is_q || is_k) {  // x cos + rotate_half(x) sin, rotate_half = cat(-x2, x1)
        const float2 c = __ldg(cs + static_cast<size_t>(p) * 256 + i);
        a[u] = v1 * c.x + (-v2) * c.y;
        b[u] = v2 * c.x + v1 * c.y;
      } else {
        a[u] = v1;
        b[u] = v2;
      }
    }
    olo[e / 2] = pack_f16(a[0], a[1]);
    ohi[e / 2] = pack_f16(b[0], b[1]);
  }
  reinterpret_cast<uint4*>(row)[lane] = make_uint4(olo[0], olo[1], olo[2], olo[3]);
  reinterpret_cast<uint4*>(row + 256)[lane] = make_uint4(ohi[0], ohi[1], ohi[2], ohi[3]);
}

}  // namespace glp
