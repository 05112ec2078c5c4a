// Bidirectional GQA flash attention, head_dim 256, f16 operands, f32 online softmax.
//
// Semantics (reference): scores = q . k with scale 1.0 (attention/standard.rs:62,
// metal_flash.rs:329); a key j is visible from query i iff j < len(seq) and, on sliding
// layers, |i - j| <= W (model.rs:634-638, chunked.rs:14-50); softmax in f32; query head h
// reads kv head h / (Hq / Hkv) (repeat_kv, attention/mod.rs:22-31).  Padding is handled
// analytically from the packed sequence offsets (no mask tensors).
//
// v1 engine: warp-level mma.sync m16n8k16 (f16 -> f32).  CTA = 128 query rows of one
// (sequence, head), 8 warps x 16 rows; K/V tiles of 64 keys double-buffered with cp.async
// in an XOR-swizzled shared-memory layout (conflict-free ldmatrix).  KV tiles entirely
// outside the window are skipped.
#pragma once
#include "common.cuh"

namespace glp {

constexpr int kAttnD = 256;
constexpr int kAttnBQ = 128;
constexpr int kAttnBKV = 64;
constexpr int kAttnThreads = 256;
constexpr size_t kAttnSmem = (kAttnBQ + 4 * kAttnBKV) * kAttnD * 2 + 128;  // Q + 2x(K,V)

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;  // 0 -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// byte offset of 16-byte chunk `c` of row `r` in a [rows][256] f16 tile (512 B rows)
__device__ __forceinline__ uint32_t attn_swz(int r, int c) {
  return static_cast<uint32_t>(r * 512 + ((c ^ (r & 7)) << 4));
}

// Load `rows` rows (tokens base_tok + r, valid when r < n_valid) of one 256-wide head slice.
__device__ __forceinline__ void attn_load_tile(uint32_t sdst, const __half* qkv, int ld, int col0,
                                               int base_tok, int n_valid, int rows) {
  const int chunks = rows * 32;
  for (int i = threadIdx.x; i < chunks; i += kAttnThreads) {
    const int r = i >> 5, c = i & 31;
    const bool v = r < n_valid;
    const __half* src = qkv + static_cast<size_t>(base_tok + (v ? r : 0)) * ld + col0 + c * 8;
    cp_async16(sdst + attn_swz(r, c), src, v);
  }
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attn_fwd_kernel(const __half* __restrict__ qkv, int ld_qkv, const int* __restrict__ cu_seqlens,
                          int cu_base, int n_q_heads, int n_kv_heads, int window,
                          __half* __restrict__ out, int ld_out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + kAttnBQ * 512;
  const uint32_t sV0 = sK0 + 2 * kAttnBKV * 512;

  const int b = blockIdx.z, head = blockIdx.y;
  const int tok0 = cu_seqlens[b] - cu_base;  // row of the sequence's first token
  const int len = cu_seqlens[b + 1] - cu_seqlens[b];
  const int q0 = blockIdx.x * kAttnBQ;
  if (q0 >= len) return;
  const int kvh = head / (n_q_heads / n_kv_heads);
  const int qcol = head * kAttnD;
  const int kcol = (n_q_heads + kvh) * kAttnD;
  const int vcol = (n_q_heads + n_kv_heads + kvh) * kAttnD;

  int kv_lo = 0, kv_hi = len;
  if (window > 0) {
    kv_lo = max(0, q0 - window);
    kv_hi = min(len, q0 + kAttnBQ + window);
  }
  const int t_lo = kv_lo / kAttnBKV;
  const int t_hi = (kv_hi + kAttnBKV - 1) / kAttnBKV;

  // Q tile + first K/V tile
  attn_load_tile(sQ, qkv, ld_qkv, qcol, tok0 + q0, len - q0, kAttnBQ);
  attn_load_tile(sK0, qkv, ld_qkv, kcol, tok0 + t_lo * kAttnBKV, len - t_lo * kAttnBKV, kAttnBKV);
  attn_load_tile(sV0, qkv, ld_qkv, vcol, tok0 + t_lo * kAttnBKV, len - t_lo * kAttnBKV, kAttnBKV);
  cp_async_commit();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qrow_w = warp * 16;  // this warp's first row inside the Q tile
  const int i0 = q0 + qrow_w + (lane >> 2);  // sequence positions of this thread's two rows
  const int i1 = i0 + 8;

  float o[32][4];
#pragma unroll
  for (int n = 0; n < 32; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  constexpr float kLog2e = 1.4426950408889634f;

  for (int t = t_lo; t < t_hi; ++t) {
    const int stage = (t - t_lo) & 1;
    if (t + 1 < t_hi) {
      const int ns = stage ^ 1;
      const int kb = (t + 1) * kAttnBKV;
      attn_load_tile(sK0 + ns * kAttnBKV * 512, qkv, ld_qkv, kcol, tok0 + kb, len - kb, kAttnBKV);
      attn_load_tile(sV0 + ns * kAttnBKV * 512, qkv, ld_qkv, vcol, tok0 + kb, len - kb, kAttnBKV);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + stage * kAttnBKV * 512;
    const uint32_t sV = sV0 + stage * kAttnBKV * 512;

    // ---- S = Q K^T (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < 16; ++kk) {
      uint32_t a[4];
      {
        const int r = qrow_w + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = 2 * kk + (lane >> 4);
        ldsm_x4(sQ + attn_swz(r, c), a);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bk[4];
        const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(sK + attn_swz(r, c), bk);
        mma_f16_16816(s[2 * np], a, bk[0], bk[1]);
        mma_f16_16816(s[2 * np + 1], a, bk[2], bk[3]);
      }
    }

    // ---- mask (padding keys, window) + online softmax
    const int jb = t * kAttnBKV + 2 * (lane & 3);
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = jb + n * 8 + e;
        bool v0 = j < len, v1 = j < len;
        if (window > 0) {
          v0 = v0 && abs(i0 - j) <= window;
          v1 = v1 && abs(i1 - j) <= window;
        }
        if (!v0) s[n][e] = -INFINITY;
        if (!v1) s[n][2 + e] = -INFINITY;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float mu0 = mn0 == -INFINITY ? 0.f : mn0;  // fully masked so far: keep zeros
    const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
    const float alpha0 = exp2f((m0 - mu0) * kLog2e);
    const float alpha1 = exp2f((m1 - mu1) * kLog2e);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = exp2f((s[n][0] - mu0) * kLog2e);
      s[n][1] = exp2f((s[n][1] - mu0) * kLog2e);
      s[n][2] = exp2f((s[n][2] - mu1) * kLog2e);
      s[n][3] = exp2f((s[n][3] - mu1) * kLog2e);
      rs0 += s[n][0] + s[n][1];
      rs1 += s[n][2] + s[n][3];
    }
    l0 = l0 * alpha0 + rs0;
    l1 = l1 * alpha1 + rs1;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      o[n][0] *= alpha0;
      o[n][1] *= alpha0;
      o[n][2] *= alpha1;
      o[n][3] *= alpha1;
    }

    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_f16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_f16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_f16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_f16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int dp = 0; dp < 16; ++dp) {
        uint32_t bv[4];
        const int c = 2 * dp + (lane >> 4);
        ldsm_x4_t(sV + attn_swz(r, c), bv);
        mma_f16_16816(o[2 * dp], a, bv[0], bv[1]);
        mma_f16_16816(o[2 * dp + 1], a, bv[2], bv[3]);
      }
    }
    __syncthreads();  // this stage is overwritten by the load issued next iteration
  }

  // ---- normalise and store (f16, the O-projection input)
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float r0 = l0 > 0.f ? 1.0f / l0 : 0.f;
  const float r1 = l1 > 0.f ? 1.0f / l1 : 0.f;
  const int dcol = qcol + 2 * (lane & 3);
  if (i0 < len) {
    __half* dst = out + static_cast<size_t>(tok0 + i0) * ld_out + dcol;
#pragma unroll
    for (int n = 0; n < 32; ++n)
      *reinterpret_cast<uint32_t*>(dst + n * 8) = pack_f16(o[n][0] * r0, o[n][1] * r0);
  }
  if (i1 < len) {
    __half* dst = out + static_cast<size_t>(tok0 + i1) * ld_out + dcol;
#pragma unroll
    for (int n = 0; n < 32; ++n)
      *reinterpret_cast<uint32_t*>(dst + n * 8) = pack_f16(o[n][2] * r1, o[n][3] * r1);
  }
}

}  // namespace glp
