// Per-layer-embedding (PLE) row kernels: the normalised per-layer inputs and the PLE block's
// GeGLU (crates/glypr-core/src/ple.rs:48-145).  The projections around them are the Q8_0
// GEMMs of gemm.cuh.
#pragma once
#include "gemm.cuh"    // geglu_f: the MLP's GeGLU, which the PLE block reuses (cpu_simd::cpu_geglu)
#include "rowops.cuh"  // warp_sum, 8-element vector loads and stores

namespace glp {

// P[r] = f16(RMSNorm(f32(P[r]) * scale) * w) in place for every row r of D values, where the
// rows are the [T, L, D] reshape of the projection [T, L * D] (ple.rs:48-93; scale = f32(H^-0.5)).
// One warp per row, 8 elements per lane per step (D % 8 == 0); the sum of squares is taken
// in a first pass and the row re-read (from L1) in the second.
__global__ void ple_norm_kernel(__half* __restrict__ p, int64_t n_rows, int D, float scale,
                                const float* __restrict__ w, float eps) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= n_rows) return;
  __half* row = p + r * D;
  float ss = 0.f;
  for (int e0 = lane * 8; e0 < D; e0 += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + e0);
    const __half* e = reinterpret_cast<const __half*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __half2float(e[j]) * scale;
      ss = fmaf(v, v, ss);
    }
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
  for (int e0 = lane * 8; e0 < D; e0 += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + e0);
    const __half* e = reinterpret_cast<const __half*>(&u);
    float wv[8], o[8];
    load_f32x8(w + e0, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = (__half2float(e[j]) * scale) * inv * wv[j];
    store16x8<__half>(row + e0, o);
  }
}

// g[t, j] = f16(geglu(g[t, j], P[t, layer, j])) in place: the PLE block's gate output times the
// layer's slice of the per-layer inputs (ple.rs:118-136).  8 elements per thread (D % 8 == 0,
// so a group never crosses a row).
__global__ void ple_geglu_kernel(__half* __restrict__ g, const __half* __restrict__ p, int64_t n_tokens, int D,
                                 int layer, int n_layers) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= n_tokens * D) return;
  const int64_t t = i / D;
  const int64_t j = i - t * D;
  const uint4 gu = *reinterpret_cast<const uint4*>(g + i);
  const uint4 pu = *reinterpret_cast<const uint4*>(p + (t * n_layers + layer) * D + j);
  const __half* ge = reinterpret_cast<const __half*>(&gu);
  const __half* pe = reinterpret_cast<const __half*>(&pu);
  float o[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) o[k] = geglu_f(__half2float(ge[k]), __half2float(pe[k]));
  store16x8<__half>(g + i, o);
}

}  // namespace glp
