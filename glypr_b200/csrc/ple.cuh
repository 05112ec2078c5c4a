// Per-layer-embedding (PLE) row kernel: the normalised per-layer inputs
// (crates/glypr-core/src/ple.rs:48-93).  The projections around it are the Q8_0 GEMMs of
// gemm.cuh; the PLE block's GeGLU runs in its gate GEMM's epilogue (kEpiMulGeglu).
#pragma once
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

}  // namespace glp
