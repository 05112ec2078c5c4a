// Persistent tcgen05 GEMM for sm_100a:  C[M, N] = A[M, K] * B[N, K]^T
//
//   A  activations, 16-bit T (f16 or bf16), row-major (K contiguous) -> TMA, 128B swizzle
//   B  weights (dequantised Q8_0 / converted BF16) as T, row-major [N,K] -> TMA, 128B swizzle
//   accumulator f32 in tensor memory (TMEM), two buffers of BN columns
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = MMA issuer (+ TMEM owner),
// warps 2..9 = epilogue: warp w reads TMEM lanes 32*(w%4)..+31 (one output row per thread)
// and converts half of the tile's columns ((w-2)/4 selects the half), so every lane
// quadrant has two warps converting while the next tile accumulates.
// Tiles are 128 x BN, K is consumed 64 elements (one 128-byte swizzle row) per stage.
// Tile order is M-major over N so consecutive CTAs share the same A rows (read from HBM
// once, then from L2) while the weights stay L2-resident.
//
// Epilogues (fused so the activations make one trip through HBM):
//   kEpiStore16 store T
//   kEpiF32     store f32
//   kEpiQkv     per-head RMSNorm (q/k with gain, v without), NeoX RoPE on q/k, store f16.
//               One 256-column tile == one head (attention/mod.rs:166-188, rope.rs:90-106).
//   kEpiGeglu   B rows interleaved [gate 128 | up 128] per tile; out = gelu_tanh(g)*u as T
//               (cpu_simd/geglu.rs:6-18, with its +-10 clamp).
//   kEpiMulGeglu  out = gelu_tanh(acc) * U[row, col] as f16, U an f16 matrix in HBM (the
//               per-layer-embedding block's gate times the layer's per-layer inputs,
//               ple.rs:118-136).
#pragma once
#include "common.cuh"

namespace glp {

enum EpiKind : int { kEpiStore16 = 0, kEpiF32 = 1, kEpiQkv = 2, kEpiGeglu = 3, kEpiMulGeglu = 4 };

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  void* C;      // output base
  int ldc;      // output row stride in elements
  // kEpiQkv
  const float* q_gain;    // [head_dim]
  const float* k_gain;    // [head_dim]
  const float2* rope_cs;  // {cos, sin} of two frequencies per position: [head_dim/4, rope_stride] float4
  const int* pos;         // [M] position of each row inside its sequence
  int rope_stride;        // positions per frequency row (the model's context length)
  int n_q_heads, n_kv_heads;
  float eps;
  int* status;  // device status word (error codes above)
  // gemm_rownorm_kernel: residual rows (updated in place), next pre-normed rows, norm gains
  __nv_bfloat16* h;
  __half* x_next;
  const float* w_post;
  const float* w_next;
  float layer_scalar;
  int rownorm_direct;  // 1: always the exact two-exchange row scale (testing)
  // kEpiMulGeglu: the second GeGLU operand U (row stride ld_mul elements)
  const __half* mul;
  int ld_mul;
  // gemm_q8_pair_kernel: bytes per raw Q8_0 row (34 K / 32) and the rows per TMA group row
  int raw_pitch, raw_group;
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // double-buffered accumulator
  // after the stages: 512 B of barriers/flags, the epilogue pairs' row-sum exchange, then one
  // 32-row x 128-byte output staging tile per epilogue warp
  static constexpr uint32_t RED_OFFSET = 512;
  static constexpr uint32_t RED_BYTES = 2 * 2 * 128 * 4;
  static constexpr uint32_t STAGE_OFFSET = STAGES * (A_BYTES + B_BYTES) + RED_OFFSET + RED_BYTES;
  static constexpr uint32_t STAGE_BYTES = 8 * 32 * 128;
  // the dynamic shared-memory base is declared 1024-aligned (checked at run time)
  static constexpr size_t SMEM = STAGE_OFFSET + STAGE_BYTES;
};

// gelu_tanh(g) * u with the reference's clamp (cpu_simd/geglu.rs:6-18), branch-free so the
// 32 elements of a chunk interleave.  Uses the identity 0.5 * (1 + tanh(z)) = 1 / (1 + e^-2z);
// for g <= -10 the exponential may overflow to inf, giving -0 before the clamp selects 0.
__device__ __forceinline__ float geglu_f(float g, float u) {
  const float z = 0.7978846f * fmaf(0.044715f * g, g * g, g);
  float a = __fdividef(g, 1.0f + __expf(-2.0f * z)) * u;
  a = g >= 10.0f ? g * u : a;
  return g <= -10.0f ? 0.0f : a;
}

// The same on two (g, u) pairs at once, on the packed f32x2 pipe: with
// c0 = -2 sqrt(2/pi) log2(e) and c1 = 0.044715 c0, e^(-2z) = 2^(g (c0 + c1 g^2)), so an output
// is g u / (1 + 2^x) -- three packed FMA-pipe instructions and one exp2 per pair of lanes up to
// the reciprocal, against ~7 scalar instructions per element (the GeGLU epilogue's arithmetic
// set the pace of the whole gate/up GEMM).  Same clamps as geglu_f.
__device__ __forceinline__ float geglu_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float geglu_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void geglu_f2(float g0, float g1, float u0, float u1, float& o0, float& o1) {
  constexpr float kC0 = -2.3022082f, kC1 = -0.10294324f;
  const uint64_t g = f2(g0, g1);
  const uint64_t x = f2_mul(f2_fma(f2_mul(g, g), f2(kC1, kC1), f2(kC0, kC0)), g);
  float x0, x1;
  f2_split(x, x0, x1);
  float d0, d1;
  f2_split(f2_add(f2(geglu_ex2(x0), geglu_ex2(x1)), f2(1.0f, 1.0f)), d0, d1);
  f2_split(f2_mul(f2_mul(g, f2(u0, u1)), f2(geglu_rcp(d0), geglu_rcp(d1))), o0, o1);
  o0 = g0 >= 10.0f ? g0 * u0 : o0;
  o1 = g1 >= 10.0f ? g1 * u1 : o1;
  o0 = g0 <= -10.0f ? 0.0f : o0;
  o1 = g1 <= -10.0f ? 0.0f : o1;
}

// 8 frequency pairs (i, i + 128), i = f0 .. f0 + 7, of one head row: RMS scale, gain, NeoX
// RoPE; f16 pairs of the lower (x1) and upper (x2) halves into plo / phi.
__device__ __forceinline__ void epi_qkv_chunk8(int f0, float inv, const float* gain, bool rope,
                                               const uint32_t (&lo)[8], const uint32_t (&hi)[8],
                                               const float (&cv)[8], const float (&sv)[8], uint32_t (&plo)[4],
                                               uint32_t (&phi)[4]) {
  float g1[8], g2[8];
  if (gain) {
    const float4* ga = reinterpret_cast<const float4*>(gain + f0);
    const float4* gb = reinterpret_cast<const float4*>(gain + 128 + f0);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float4 a = __ldg(ga + q), b = __ldg(gb + q);
      g1[4 * q] = a.x, g1[4 * q + 1] = a.y, g1[4 * q + 2] = a.z, g1[4 * q + 3] = a.w;
      g2[4 * q] = b.x, g2[4 * q + 1] = b.y, g2[4 * q + 2] = b.z, g2[4 * q + 3] = b.w;
    }
  }
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    float a[2], b[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float x1 = u2f(lo[j + e]) * inv;
      float x2 = u2f(hi[j + e]) * inv;
      if (gain) {
        x1 *= g1[j + e];
        x2 *= g2[j + e];
      }
      if (rope) {  // x*cos + rotate_half(x)*sin, rotate_half = cat(-x2, x1)
        a[e] = x1 * cv[j + e] + (-x2) * sv[j + e];
        b[e] = x2 * cv[j + e] + x1 * sv[j + e];
      } else {
        a[e] = x1;
        b[e] = x2;
      }
    }
    plo[j / 2] = pack_f16(a[0], a[1]);
    phi[j / 2] = pack_f16(b[0], b[1]);
  }
}

// One accumulator tile -> global, by the two epilogue warps of one TMEM lane quadrant: `half`
// selects which half of the tile's columns this warp converts; `stage` is the warp's
// 32 x 128 B staging tile and `row0` the tile row of its lane 0.  `red` is the pair's
// shared-memory exchange for the QKV row sums, synchronised through the pair's rendezvous
// barrier `xbar` (phase bit `xph`).  Returns false if that rendezvous timed out.
template <int BN, int EPI, typename T>
__device__ __forceinline__ bool gemm_epilogue_tile(const GemmParams& p, uint32_t tacc, int m_blk, int n_blk,
                                                   int row_in_tile, int half, float* red, uint64_t* xbar,
                                                   uint32_t& xph, volatile int* abort_flag, uint8_t* stage,
                                                   const CUtensorMap* tmc = nullptr) {
  const int row = m_blk * 128 + row_in_tile;
  const int wrow0 = row - (threadIdx.x & 31);  // first row of this warp's 32
  const int rows_valid = min(32, p.M - wrow0);
  if constexpr (EPI == kEpiStore16 || EPI == kEpiF32 || EPI == kEpiMulGeglu) {
    // this warp's BN/2 columns in slices of 128 bytes per row: 64 16-bit or 32 f32 columns
    constexpr int ELT = EPI == kEpiF32 ? 4 : 2;
    constexpr int SLICE = 128 / ELT;
    constexpr int NSL = BN / 2 / SLICE;
    const int col0 = n_blk * BN + half * (BN / 2);
    // a last tile past N (N a multiple of 128 but not of BN: the B rows there are the TMA's
    // zero fill) stores nothing from this warp's half
    if (col0 >= p.N) return true;
    const size_t ld_bytes = static_cast<size_t>(p.ldc) * ELT;
    uint8_t* dst0 = reinterpret_cast<uint8_t*>(p.C) + (static_cast<size_t>(wrow0) * p.ldc + col0) * ELT;
    const uint32_t tbase = tacc + half * (BN / 2);
#pragma unroll 1
    for (int sl = 0; sl < NSL; ++sl) {
      uint32_t w[32];
      if constexpr (EPI == kEpiF32) {
        tmem_ld32(tbase + sl * 32, w);
        tmem_ld_wait_tied(w);
      } else {
        uint32_t ra[32], rb[32];
        tmem_ld32(tbase + sl * 64, ra);
        tmem_ld32(tbase + sl * 64 + 32, rb);
        tmem_ld_wait_tied(ra);
        tmem_ld_wait_tied(rb);
        if constexpr (EPI == kEpiMulGeglu) {
          // this lane's row of U under the slice: 64 f16 = 128 contiguous bytes (rows past M
          // are not read; their outputs are clipped by the flush)
          uint4 uu[8];
          const int r = wrow0 + static_cast<int>(threadIdx.x & 31);
          const uint4* src = reinterpret_cast<const uint4*>(p.mul + static_cast<size_t>(r) * p.ld_mul + col0 + sl * 64);
#pragma unroll
          for (int i = 0; i < 8; ++i) uu[i] = r < p.M ? src[i] : make_uint4(0u, 0u, 0u, 0u);
          const __half* ue = reinterpret_cast<const __half*>(uu);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            w[j] = Half16<T>::pack(geglu_f(u2f(ra[2 * j]), __half2float(ue[2 * j])),
                                   geglu_f(u2f(ra[2 * j + 1]), __half2float(ue[2 * j + 1])));
            w[16 + j] = Half16<T>::pack(geglu_f(u2f(rb[2 * j]), __half2float(ue[32 + 2 * j])),
                                        geglu_f(u2f(rb[2 * j + 1]), __half2float(ue[32 + 2 * j + 1])));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            w[j] = Half16<T>::pack(u2f(ra[2 * j]), u2f(ra[2 * j + 1]));
            w[16 + j] = Half16<T>::pack(u2f(rb[2 * j]), u2f(rb[2 * j + 1]));
          }
        }
      }
      stage_words32(stage, w);
      flush_rows128(stage, dst0 + sl * 128, ld_bytes, rows_valid);
    }
  } else if constexpr (EPI == kEpiGeglu) {
    static_assert(BN == 256, "GeGLU tiles pair 128 gate with 128 up columns");
    const int c0 = half * 64;  // this warp's 64 outputs: gate columns c0.., up columns 128 + c0..
    uint32_t w[32];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {  // 32 outputs per round, read as two 32-column loads
      uint32_t g[32], u[32];
      tmem_ld32(tacc + c0 + hh * 32, g);
      tmem_ld32(tacc + 128 + c0 + hh * 32, u);
      tmem_ld_wait_tied(g);
      tmem_ld_wait_tied(u);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float o0, o1;
        geglu_f2(u2f(g[2 * j]), u2f(g[2 * j + 1]), u2f(u[2 * j]), u2f(u[2 * j + 1]), o0, o1);
        w[hh * 16 + j] = Half16<T>::pack(o0, o1);
      }
    }
    stage_words32(stage, w);
    uint8_t* dst0 = reinterpret_cast<uint8_t*>(p.C) +
                    (static_cast<size_t>(wrow0) * p.ldc + n_blk * 128 + c0) * sizeof(T);
    flush_rows128(stage, dst0, static_cast<size_t>(p.ldc) * sizeof(T), rows_valid);
  } else {  // kEpiQkv: this warp owns frequency pairs (i, i + 128), i in [64 half, 64 half + 64)
    static_assert(BN == 256, "QKV tiles are one 256-wide head");
    const bool live = row < p.M;
    const bool is_q = n_blk < p.n_q_heads;
    const bool is_k = !is_q && n_blk < p.n_q_heads + p.n_kv_heads;
    const float* gain = is_q ? p.q_gain : (is_k ? p.k_gain : nullptr);
    const bool rope = is_q || is_k;
    // positions outside the table read its last row instead of past its end
    const int pos = live ? min(max(p.pos[row], 0), p.rope_stride - 1) : 0;
    // frequency-pair-major {cos, sin} table: lanes (consecutive rows) read consecutive
    // positions, one 16-byte load per two frequencies
    const float4* tab = reinterpret_cast<const float4*>(p.rope_cs) + pos;
    const size_t fstride = static_cast<size_t>(p.rope_stride);
    const int f0 = half * 64;  // this warp's frequencies [f0, f0 + 64), 8 chunks of 8
    float cva[8], sva[8], cvb[8], svb[8];
    auto load_tab = [&](int k, float (&cv)[8], float (&sv)[8]) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float4 t = __ldg(tab + static_cast<size_t>((f0 + 8 * k + j) >> 1) * fstride);
        cv[j] = t.x;
        sv[j] = t.y;
        cv[j + 1] = t.z;
        sv[j + 1] = t.w;
      }
    };
    if (rope) load_tab(0, cva, sva);  // in flight during pass 1
    if (tmc) {  // the previous tile's bulk stores have read the staging tile
      if ((threadIdx.x & 31) == 0) bulk_wait_read_all();
      __syncwarp();
    }
    // pass 1: this warp's half of the head's sum of squares (cpu_simd/rmsnorm.rs:13-21)
    float ss = 0.f;
    {
      uint32_t ra[32], rb[32];
      tmem_ld32(tacc + f0, ra);
      tmem_ld32(tacc + f0 + 32, rb);
      tmem_ld_wait_tied(ra);
      tmem_ld_wait_tied(rb);
#pragma unroll
      for (int j = 0; j < 32; ++j) ss = fmaf(u2f(ra[j]), u2f(ra[j]), ss);
#pragma unroll
      for (int j = 0; j < 32; ++j) ss = fmaf(u2f(rb[j]), u2f(rb[j]), ss);
      tmem_ld32(tacc + 128 + f0, ra);
      tmem_ld32(tacc + 128 + f0 + 32, rb);
      tmem_ld_wait_tied(ra);
      tmem_ld_wait_tied(rb);
#pragma unroll
      for (int j = 0; j < 32; ++j) ss = fmaf(u2f(ra[j]), u2f(ra[j]), ss);
#pragma unroll
      for (int j = 0; j < 32; ++j) ss = fmaf(u2f(rb[j]), u2f(rb[j]), ss);
    }
    red[half * 128 + row_in_tile] = ss;
    if (!pair_rendezvous(xbar, xph, abort_flag)) return false;
    ss += red[(half ^ 1) * 128 + row_in_tile];
    const float inv = 1.0f / sqrtf(ss / 256.0f + p.eps);
    // pass 2: 8 chunks of 8 frequency pairs; the next chunk's table values are in flight.
    // The lower halves go straight into the staging tile; the upper halves are parked in
    // accumulator columns this warp has already consumed (chunk k's 4 words at columns
    // f0 + 4k, which chunks <= k have read) and staged after the lower slice is out.
    // The next chunk's accumulator columns are loaded while this chunk is converted (none of
    // the parked columns is read again).
    const uint32_t park = tacc + f0;
    uint32_t loA[8], hiA[8], loB[8], hiB[8];
    auto issue = [&](int k, uint32_t (&lo)[8], uint32_t (&hi)[8]) {
      tmem_ld8(tacc + f0 + 8 * k, lo);
      tmem_ld8(tacc + 128 + f0 + 8 * k, hi);
    };
    auto finish = [&](int k, const uint32_t (&lo)[8], const uint32_t (&hi)[8], const float (&cv)[8],
                      const float (&sv)[8]) {
      uint32_t plo[4], phi[4];
      epi_qkv_chunk8(f0 + 8 * k, inv, gain, rope, lo, hi, cv, sv, plo, phi);
      stage_chunk(stage, k, make_uint4(plo[0], plo[1], plo[2], plo[3]));
      tmem_st4(park + 4 * k, phi);
    };
    issue(0, loA, hiA);
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      if (rope) load_tab(k + 1, cvb, svb);
      tmem_ld_wait_tied8(loA, hiA);
      issue(k + 1, loB, hiB);
      finish(k, loA, hiA, cva, sva);
      if (rope && k + 2 < 8) load_tab(k + 2, cva, sva);
      tmem_ld_wait_tied8(loB, hiB);
      if (k + 2 < 8) issue(k + 2, loA, hiA);
      finish(k + 1, loB, hiB, cvb, svb);
    }
    if (tmc) {  // bulk tensor stores (rows past M clipped); the staging tile is 1024-byte aligned
      const int col = n_blk * 256 + f0;
      fence_proxy_async_smem();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) {
        tma_store_2d(tmc, stage, col, wrow0);
        bulk_commit();
      }
      uint32_t w[32];
      tmem_st_wait();
      tmem_ld32(park, w);
      tmem_ld_wait_tied(w);
      if ((threadIdx.x & 31) == 0) bulk_wait_read_all();
      __syncwarp();
      stage_words32(stage, w);
      fence_proxy_async_smem();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) {
        tma_store_2d(tmc, stage, col + 128, wrow0);
        bulk_commit();
      }
    } else {
      const size_t ld_bytes = static_cast<size_t>(p.ldc) * 2;
      uint8_t* dst0 = reinterpret_cast<uint8_t*>(p.C) +
                      (static_cast<size_t>(wrow0) * p.ldc + static_cast<size_t>(n_blk) * 256 + f0) * 2;
      flush_rows128(stage, dst0, ld_bytes, rows_valid);
      uint32_t w[32];
      tmem_st_wait();
      tmem_ld32(park, w);
      tmem_ld_wait_tied(w);
      stage_words32(stage, w);
      flush_rows128(stage, dst0 + 256, ld_bytes, rows_valid);
    }
  }
  return true;
}

constexpr int kGemmThreads = 320;

template <int BN, int EPI, typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the swizzled operand tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* xbar = drain + 1;  // [4] per-quadrant rendezvous of the two epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [2 accumulator buffers][2 halves][128 rows]
  float* red = reinterpret_cast<float*>(sB + STAGES * Cfg::B_BYTES + Cfg::RED_OFFSET);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(drain, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 2);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      griddep_wait();  // (see gemm_pair_kernel)
      int s = 0;
      uint32_t ph = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const int m_blk = tile / p.n_tiles, n_blk = tile % p.n_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            record_error(p.status, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], Cfg::A_BYTES + Cfg::B_BYTES);
          tma_load_2d(sA + s * Cfg::A_BYTES, &tmA, &full[s], kb * Cfg::BK, m_blk * Cfg::BM);
          tma_load_2d(sB + s * Cfg::B_BYTES, &tmB, &full[s], kb * Cfg::BK, n_blk * BN);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = idesc_f16(128, BN, Half16<T>::kIsBf16);
      int s = 0;
      uint32_t ph = 0;
      int ab = 0;
      uint32_t aph = 0;
      bool issued = false;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        if (!mbar_wait(&tempty[ab], aph ^ 1, abort_flag)) {
          record_error(p.status, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * BN);
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            record_error(p.status, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_kmajor_sw128(smem_u32(sA + s * Cfg::A_BYTES));
          const uint64_t bdesc = desc_kmajor_sw128(smem_u32(sB + s * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            // +32 bytes along K inside the 128-byte swizzle row (descriptor address is >>4)
            umma_f16_ss(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[ab]);
        ab ^= 1;
        if (ab == 0) aph ^= 1;
      }
      if (issued) {
        // make sure every MMA has retired before TMEM is released
        umma_commit(drain);
        if (!mbar_wait(drain, 0, abort_flag) && !*abort_flag) record_error(p.status, kErrTimeoutDrain);
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue warps
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quad * 32 + lane;
    uint8_t* stage = smem + Cfg::STAGE_OFFSET + (warp - 2) * (32 * 128);
    uint32_t xph = 0;
    int ab = 0;
    uint32_t aph = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_blk = tile / p.n_tiles, n_blk = tile % p.n_tiles;
      bool ok = mbar_wait(&tfull[ab], aph, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) {
          record_error(p.status, kErrTimeoutEpilogue);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(ab * BN);
      if (!gemm_epilogue_tile<BN, EPI, T>(p, tacc, m_blk, n_blk, row_in_tile, half, red + ab * 256, &xbar[quad],
                                           xph, abort_flag, stage)) {
        if (lane == 0) {
          record_error(p.status, kErrTimeoutEpilogue);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[ab]);
      ab ^= 1;
      if (ab == 0) aph ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- CTA-pair GEMM
// The same GEMM on pairs of SMs (cluster of 2, tcgen05.mma.cta_group::2): a pair computes a
// 256 x 256 tile, each CTA loading its 128 rows of A and 128 of the 256 B rows per K step and
// holding its 128 accumulator rows.  Per SM and K step that is 32 KB instead of the 48 KB of a
// 128 x 256 tile of its own, so the same 192 KB of stages cover 6 K steps of load latency
// instead of 4.  Roles per CTA as above; the MMA warp of the leader (rank 0) issues for both,
// signals both CTAs' empty / tfull barriers (one commit per destination CTA), and waits on
// tempty barriers that the epilogue warps of both CTAs release (the peer's through one
// forwarded arrive: a cluster-scope release by every epilogue warp would make each of them
// wait for its output stores, which measured 1.8x slower epilogues).  The loads of both CTAs
// complete on the leader's full barriers (its producer expects the bytes of both).
struct GemmPairCfg {
  static constexpr int BM = 128;  // rows per CTA (256 per pair)
  static constexpr int BN = 256;  // columns per pair tile; each CTA loads 128 rows of B
  static constexpr int BK = 64;
  static constexpr int STAGES = 6;
  static constexpr uint32_t A_BYTES = 128 * BK * 2;
  static constexpr uint32_t B_BYTES = 128 * BK * 2;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr uint32_t RED_OFFSET = 512;
  static constexpr uint32_t RED_BYTES = 2 * 2 * 128 * 4;
  // 1024-byte aligned: the QKV epilogue's staging tiles are the sources of 128B-swizzled bulk stores
  static constexpr uint32_t STAGE_OFFSET = (STAGES * (A_BYTES + B_BYTES) + RED_OFFSET + RED_BYTES + 1023) / 1024 * 1024;
  static constexpr uint32_t STAGE_BYTES = 8 * 32 * 128;
  static constexpr size_t SMEM = STAGE_OFFSET + STAGE_BYTES;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

// p.m_tiles counts 256-row pair tiles here.  tmC: the output as 32-row x 64-column boxes, for the
// QKV epilogue's bulk stores (unused by the other epilogues).
template <int EPI, typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using Cfg = GemmPairCfg;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // (the same for both CTAs of the pair, so both leave before any cluster-wide step)
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);  // used in the leader
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  // accumulator buffer released: in the leader 8 local epilogue warps + 1 arrive forwarded from
  // the peer; in the peer its 8 epilogue warps (forwarded by its warp 1)
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* xbar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(sB + STAGES * Cfg::B_BYTES + Cfg::RED_OFFSET);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int n_pairs = static_cast<int>(n_clusters_x());
  const int num_tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], leader ? 9 : 8);
    }
    mbar_init(drain, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 2);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {  // the same warp in both CTAs allocates the pair's tensor memory
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // barriers of both CTAs initialised and tensor memory allocated before anyone uses them
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      // Everything this kernel reads or writes in global memory follows the producer's
      // loads, so this one wait orders it after the previous kernel under a dependent launch.
      griddep_wait();
      int s = 0;
      uint32_t ph = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs) {
        const int m_blk = tile / p.n_tiles, n_blk = tile % p.n_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            record_error(p.status, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
          const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
          tma_load_2d_pair(sA + s * Cfg::A_BYTES, &tmA, fbar, kb * Cfg::BK, m_blk * 256 + static_cast<int>(rank) * 128);
          tma_load_2d_pair(sB + s * Cfg::B_BYTES, &tmB, fbar, kb * Cfg::BK, n_blk * 256 + static_cast<int>(rank) * 128);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      constexpr uint32_t idesc = idesc_f16(256, Cfg::BN, Half16<T>::kIsBf16);
      int s = 0;
      uint32_t ph = 0;
      int ab = 0;
      uint32_t aph = 0;
      bool issued = false;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs) {
        if (!mbar_wait(&tempty[ab], aph ^ 1, abort_flag)) {
          record_error(p.status, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * Cfg::BN);
        bool ok = true;
        // Few MMAs queue ahead of the pipe, so this thread issues at the pipe's pace, and a wait
        // on the next stage after the step's last MMA -- ~200 cycles even for a phase that
        // completed long ago -- idles the pipe once per K step.  Halfway through each step the
        // next stage's barrier is probed (non-blocking); when it has completed, the next step
        // starts without waiting.
        bool ready = false;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ready && !mbar_wait(&full[s], ph, abort_flag)) {
            record_error(p.status, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_kmajor_sw128(smem_u32(sA + s * Cfg::A_BYTES));
          const uint64_t bdesc = desc_kmajor_sw128(smem_u32(sB + s * Cfg::B_BYTES));
          const int s1 = s + 1 == STAGES ? 0 : s + 1;
          const uint32_t ph1 = s + 1 == STAGES ? ph ^ 1u : ph;
#pragma unroll
          for (int k = 0; k < Cfg::BK / 16; ++k) {
            umma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
            if (k == 1) ready = kb + 1 < p.k_blocks && mbar_test_wait(&full[s1], ph1);
          }
          issued = true;
          umma_commit_pair_both(smem_u32(&empty[s]));  // the stage in both CTAs
          s = s1;
          ph = ph1;
        }
        if (!ok) break;
        umma_commit_pair_both(smem_u32(&tfull[ab]));
        ab ^= 1;
        if (ab == 0) aph ^= 1;
      }
      if (issued) {
        // every MMA (which writes both CTAs' tensor memory) retires before the pair leaves
        umma_commit_pair(smem_u32(drain));
        if (!mbar_wait(drain, 0, abort_flag) && !*abort_flag) record_error(p.status, kErrTimeoutDrain);
      }
    } else if (lane == 0) {
      // ------------------------------------------------------------ release forwarder (peer)
      // The peer's epilogue warps release an accumulator buffer on a barrier of their own CTA
      // (a CTA-scope arrive does not wait for their output stores); this thread carries that
      // as one cluster-scope arrive to the leader, whose MMA waits for both CTAs.
      const uint32_t lead_tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
      int ab = 0;
      uint32_t aph = 0;
      for (int tile = pair; tile < num_tiles; tile += n_pairs) {
        if (!mbar_wait(&tempty[ab], aph, abort_flag)) {
          record_error(p.status, kErrTimeoutEpilogue);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        tc_fence_before();
        mbar_arrive_cluster(lead_tempty0 + static_cast<uint32_t>(ab * sizeof(uint64_t)));
        ab ^= 1;
        if (ab == 0) aph ^= 1;
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue warps (both CTAs)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quad * 32 + lane;
    uint8_t* stage = smem + Cfg::STAGE_OFFSET + (warp - 2) * (32 * 128);
    uint32_t xph = 0;
    int ab = 0;
    uint32_t aph = 0;
    for (int tile = pair; tile < num_tiles; tile += n_pairs) {
      const int m_blk = tile / p.n_tiles, n_blk = tile % p.n_tiles;
      bool ok = mbar_wait(&tfull[ab], aph, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) {
          record_error(p.status, kErrTimeoutEpilogue);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t tacc =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(ab * Cfg::BN);
      // this CTA's 128 rows are 128-row block 2 m_blk + rank
      if (!gemm_epilogue_tile<256, EPI, T>(p, tacc, 2 * m_blk + static_cast<int>(rank), n_blk, row_in_tile, half,
                                           red + ab * 256, &xbar[quad], xph, abort_flag, stage,
                                           EPI == kEpiQkv ? &tmC : nullptr)) {
        if (lane == 0) {
          record_error(p.status, kErrTimeoutEpilogue);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[ab]);  // this CTA's barrier (the peer's is forwarded)
      ab ^= 1;
      if (ab == 0) aph ^= 1;
    }
    if (EPI == kEpiQkv && lane == 0) bulk_wait_all();  // this warp's bulk stores are complete
  }

  // neither CTA leaves (or frees tensor memory) while the other may still touch its shared
  // memory, barriers or tensor memory
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- row-norm GEMM
// y = A * B^T with N == 256 NP (NP 256-column blocks: 512, 768 or 1024 columns), fused with the
// post-norm + residual + next pre-norm that follows the O and down projections (norm.rs:22-94, layer.rs:20-50):
//   s  = rsqrt(mean(y^2) + eps),  hv = (h + y * s * w_post) * lambda,  h <- bf16(hv),
//   x  = f16(hv * rsqrt(mean(hv^2) + eps) * w_next)
// so y never goes to HBM and the row pass over h happens in the GEMM's shadow.
// A cluster of 2 NP CTAs = NP CTA pairs: pair j computes columns [256 j, 256 j + 256) of a
// 256-row tile exactly as gemm_pair_kernel does (cta_group::2, leader = the even rank), so the
// NP CTAs with the same in-pair rank hold the same 128 rows' N columns.  Both row scales
// come from one exchange per tile: with u = y * w_post, sum(hv^2) = lambda^2 (sum h^2 +
// 2 s sum(h u) + s^2 sum u^2), so every CTA sends the four partial sums (y^2, h^2, h u, u^2) of
// its columns to the other NP - 1 (st.async into their slots, counted on their exchange
// mbarrier) and each adds the NP in pair order: all of them derive bit-identical scales.
// When the expansion cancels for a row (sum hv^2 below 2^-8 of its positive terms, where its
// rounding would show), that row's quad of 32 rows in the NP CTAs -- deciding on identical
// totals -- takes a second exchange of the directly summed hv^2, which that row then uses
// (GemmParams::rownorm_direct selects it for every row).
// The residual rows are fetched by TMA into each epilogue warp's two 4 KB boxes (64 columns
// each, one mbarrier per box); the output rows are staged through the same boxes and leave by
// coalesced 16-byte stores (x, then h, rows past M not stored), and each box is refilled with
// the next tile's rows right after, so the loads overlap the rest of the epilogue.  Epilogue
// warp (quad q, half c) owns rows 32q..32q+31 and the 128 columns 128c.. of its CTA's 256; the
// row arithmetic runs on packed f32x2 pairs.
template <int NP>
struct GemmRowCfgT {
  static constexpr int STAGES = NP <= 3 ? 4 : 3;  // 8-CTA clusters' larger exchange slots take a stage
  static constexpr uint32_t A_BYTES = 128 * 64 * 2;
  static constexpr uint32_t B_BYTES = 128 * 64 * 2;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t HBUF_OFFSET = STAGES * (A_BYTES + B_BYTES);  // 1024-aligned
  static constexpr uint32_t HBUF_WARP = 2 * 32 * 128;                     // two 32-row x 128-B boxes
  static constexpr uint32_t BAR_OFFSET = HBUF_OFFSET + 8 * HBUF_WARP;
  static constexpr uint32_t RED4_OFFSET = BAR_OFFSET + 512;   // float4 [acc buf][half][row]
  static constexpr uint32_t RED1_OFFSET = RED4_OFFSET + 2 * 2 * 128 * 16;  // float [buf][half][row]
  static constexpr uint32_t XV_OFFSET = RED1_OFFSET + 2 * 2 * 128 * 4;     // float4 [buf][pair][row]
  static constexpr uint32_t XT_OFFSET = XV_OFFSET + 2 * NP * 128 * 16;     // float [buf][pair][row]
  static constexpr uint32_t XS_OFFSET = XT_OFFSET + 2 * NP * 128 * 4;      // float [buf][pair][half][row]
  static constexpr uint32_t W_OFFSET = XS_OFFSET + 2 * NP * 2 * 128 * 4;   // float [post | next][256]
  static constexpr size_t SMEM = W_OFFSET + 2 * 256 * 4;
  // bytes each CTA receives per exchange from the other NP - 1: sums (half-0 warps, 16 B a
  // row) and arrival tokens (half-1 warps, 4 B a row); a quad's direct exchange: 4 B from both
  // of the quad's warps
  static constexpr uint32_t XCH_TX = (NP - 1) * (128 * 16 + 128 * 4);
  static constexpr uint32_t XS_TX = (NP - 1) * (2 * 32 * 4);
  static_assert(NP >= 2 && NP <= 4, "clusters of 4, 6 or 8 CTAs");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, float4 v, uint32_t cluster_mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   cluster_addr),
               "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
               "r"(__float_as_uint(v.w)), "r"(cluster_mbar)
               : "memory");
}

// p.m_tiles counts 256-row tiles; p.N == 256 NP; p.C is unused (outputs go to p.h and p.x_next).
template <typename T, int NP>
__global__ void __cluster_dims__(2 * NP, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_rownorm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmX,
                        const GemmParams p) {
  using Cfg = GemmRowCfgT<NP>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the same in every CTA: all leave before any cluster step
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFFSET);  // used in the pair leader
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;  // leader: 8 local + 1 forwarded from the peer; peer: 8 local
  uint64_t* drain = tempty + 2;
  uint64_t* xbar = drain + 1;    // [4] rendezvous of a quad's two column halves
  uint64_t* xf0 = xbar + 4;      // [2] per accumulator buffer: the tile's sums exchange
  uint64_t* xf1 = xf0 + 2;       // [2][4] per buffer and quad: the direct exchange (rare)
  uint64_t* hbar = xf1 + 8;      // [8][2] residual-row loads, per epilogue warp and box
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(hbar + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t prank = rank & 1u;            // which 128 rows of the pair tile
  const uint32_t lead = rank & ~1u;            // the pair's leader
  const int pj = static_cast<int>(rank >> 1);  // column block
  const bool leader = prank == 0;
  const int cl = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(n_clusters_x());

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], leader ? 9 : 8);
      mbar_init(&xf0[b], 1);
      for (int q = 0; q < 4; ++q) mbar_init(&xf1[b * 4 + q], 1);
    }
    mbar_init(drain, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 2);
    for (int w = 0; w < 16; ++w) mbar_init(&hbar[w], 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmH);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (every CTA)
      int s = 0;
      uint32_t ph = 0;
      for (int mt = cl; mt < p.m_tiles && !*abort_flag; mt += ncl) {
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            record_error(p.status, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
          const uint32_t fbar = mapa_shared(smem_u32(&full[s]), lead);
          tma_load_2d_pair(sA + s * Cfg::A_BYTES, &tmA, fbar, kb * 64, mt * 256 + static_cast<int>(prank) * 128);
          tma_load_2d_pair(sB + s * Cfg::B_BYTES, &tmB, fbar, kb * 64, pj * 256 + static_cast<int>(prank) * 128);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (pair leaders)
      constexpr uint32_t idesc = idesc_f16(256, 256, Half16<T>::kIsBf16);
      const uint16_t pair_mask = static_cast<uint16_t>(3u << rank);  // this leader (even rank) and its peer
      int s = 0;
      uint32_t ph = 0;
      int ab = 0;
      uint32_t aph = 0;
      bool issued = false;
      for (int mt = cl; mt < p.m_tiles && !*abort_flag; mt += ncl) {
        if (!mbar_wait(&tempty[ab], aph ^ 1, abort_flag)) {
          record_error(p.status, kErrTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * 256);
        bool ok = true;
        bool ready = false;  // the mid-step probe of the next stage (as in gemm_pair_kernel)
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ready && !mbar_wait(&full[s], ph, abort_flag)) {
            record_error(p.status, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_kmajor_sw128(smem_u32(sA + s * Cfg::A_BYTES));
          const uint64_t bdesc = desc_kmajor_sw128(smem_u32(sB + s * Cfg::B_BYTES));
          const int s1 = s + 1 == STAGES ? 0 : s + 1;
          const uint32_t ph1 = s + 1 == STAGES ? ph ^ 1u : ph;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
            if (k == 1) ready = kb + 1 < p.k_blocks && mbar_test_wait(&full[s1], ph1);
          }
          issued = true;
          umma_commit_pair_mask(smem_u32(&empty[s]), pair_mask);  // the stage in both CTAs of the pair
          s = s1;
          ph = ph1;
        }
        if (!ok) break;
        umma_commit_pair_mask(smem_u32(&tfull[ab]), pair_mask);
        ab ^= 1;
        if (ab == 0) aph ^= 1;
      }
      if (issued) {
        umma_commit_pair(smem_u32(drain));
        if (!mbar_wait(drain, 0, abort_flag) && !*abort_flag) record_error(p.status, kErrTimeoutDrain);
      }
    } else if (lane == 0) {
      // ------------------------------------------------------------ release forwarder (peers)
      const uint32_t lead_tempty0 = mapa_shared(smem_u32(&tempty[0]), lead);
      int ab = 0;
      uint32_t aph = 0;
      for (int mt = cl; mt < p.m_tiles; mt += ncl) {
        if (!mbar_wait(&tempty[ab], aph, abort_flag)) {
          record_error(p.status, kErrTimeoutEpilogue);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        tc_fence_before();
        mbar_arrive_cluster(lead_tempty0 + static_cast<uint32_t>(ab * sizeof(uint64_t)));
        ab ^= 1;
        if (ab == 0) aph ^= 1;
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue warps
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int half = ew >> 2;
    const int row_in_tile = quad * 32 + lane;
    const int col0 = pj * 256 + half * 128;  // this warp's first column of the row
    uint8_t* hb = smem + Cfg::HBUF_OFFSET + ew * Cfg::HBUF_WARP;
    float4* red4 = reinterpret_cast<float4*>(smem + Cfg::RED4_OFFSET);
    float* red1 = reinterpret_cast<float*>(smem + Cfg::RED1_OFFSET);
    float4* xv = reinterpret_cast<float4*>(smem + Cfg::XV_OFFSET);
    float* xt = reinterpret_cast<float*>(smem + Cfg::XT_OFFSET);
    float* xs = reinterpret_cast<float*>(smem + Cfg::XS_OFFSET);
    float* wsm = reinterpret_cast<float*>(smem + Cfg::W_OFFSET);
    {  // this CTA's 256 columns of both gains, once per launch (the 8 epilogue warps)
      const int t = threadIdx.x - 64;
      wsm[t] = p.w_post[pj * 256 + t];
      wsm[256 + t] = p.w_next[pj * 256 + t];
      asm volatile("bar.sync 1, 256;" ::: "memory");
    }
    const float* wp = wsm + half * 128;
    const float* wn = wsm + 256 + half * 128;
    const float inv_n = 1.0f / static_cast<float>(p.N);
    const float lam = p.layer_scalar;
    // this warp's 32 rows x 64 columns (box g) of the residual of tile mt
    auto prefetch_box = [&](int mt, int g) {
      if (lane == 0) {
        const int r0 = mt * 256 + static_cast<int>(prank) * 128 + quad * 32;
        mbar_arrive_expect_tx(&hbar[2 * ew + g], 4096);
        tma_load_2d(hb + g * 4096, &tmH, &hbar[2 * ew + g], col0 + 64 * g, r0);
      }
    };
    // the residual chunk k (8 columns) of box g for this lane's row
    auto h_chunk = [&](int g, int k) {
      return *reinterpret_cast<const uint4*>(hb + g * 4096 + lane * 128 + ((k ^ (lane & 7)) << 4));
    };
    uint32_t xph = 0, xf1ph = 0;
    int ab = 0;
    uint32_t aph = 0, hph = 0;
    bool h_pending = false, aborted = false, direct_armed = false;
    if (cl < p.m_tiles) {
      prefetch_box(cl, 0);
      prefetch_box(cl, 1);
      h_pending = true;
    }
    for (int mt = cl; mt < p.m_tiles; mt += ncl) {
      if (ew == 0 && lane == 0) mbar_arrive_expect_tx(&xf0[ab], Cfg::XCH_TX);
      direct_armed = false;
      bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[ab], aph, abort_flag));
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&hbar[2 * ew], hph, abort_flag));
      const uint32_t tacc =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(ab * 256 + half * 128);
      float s = 0.f, inv_h = 0.f;
      if (ok) {
        tc_fence_after();
        // pass A: partial sums of y^2, h^2, h u, u^2 over this warp's 128 columns
        uint64_t Y2 = 0, H2 = 0, HU = 0, U2 = 0;  // packed pairs of partial sums
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {  // 32 columns: box q / 2, chunks 4 (q % 2) ..
          uint32_t a[32];
          tmem_ld32(tacc + 32 * q, a);
          if (q == 2) {  // the second box (fetched last) is needed from here on
            if (!__all_sync(0xffffffffu, mbar_wait(&hbar[2 * ew + 1], hph, abort_flag))) ok = false;
          }
          tmem_ld_wait_tied(a);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint4 hq = h_chunk(q >> 1, 4 * (q & 1) + k);
            const uint32_t hw4[4] = {hq.x, hq.y, hq.z, hq.w};
            const float4 w0 = *reinterpret_cast<const float4*>(wp + 32 * q + 8 * k);
            const float4 w1 = *reinterpret_cast<const float4*>(wp + 32 * q + 8 * k + 4);
            const uint64_t wv[4] = {f2(w0.x, w0.y), f2(w0.z, w0.w), f2(w1.x, w1.y), f2(w1.z, w1.w)};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint64_t y = f2(u2f(a[8 * k + 2 * j]), u2f(a[8 * k + 2 * j + 1]));
              const uint64_t h = f2(__uint_as_float(hw4[j] << 16), __uint_as_float(hw4[j] & 0xffff0000u));
              const uint64_t u = f2_mul(y, wv[j]);
              Y2 = f2_fma(y, y, Y2);
              H2 = f2_fma(h, h, H2);
              HU = f2_fma(h, u, HU);
              U2 = f2_fma(u, u, U2);
            }
          }
        }
        hph ^= 1;
        h_pending = false;
        float y2, h2, hu, u2, t0, t1;
        f2_split(Y2, t0, t1);
        y2 = t0 + t1;
        f2_split(H2, t0, t1);
        h2 = t0 + t1;
        f2_split(HU, t0, t1);
        hu = t0 + t1;
        f2_split(U2, t0, t1);
        u2 = t0 + t1;
        // exchange: quad halves -> this CTA's sums -> the other NP - 1 CTAs holding these rows
        red4[(ab * 2 + half) * 128 + row_in_tile] = make_float4(y2, h2, hu, u2);
        if (ok) ok = pair_rendezvous(&xbar[quad], xph, abort_flag);
        if (ok) {
          const float4 r0 = red4[(ab * 2) * 128 + row_in_tile], r1 = red4[(ab * 2 + 1) * 128 + row_in_tile];
          const float4 mine = make_float4(r0.x + r1.x, r0.y + r1.y, r0.z + r1.z, r0.w + r1.w);
          const uint32_t bar = smem_u32(&xf0[ab]);
#pragma unroll
          for (int k = 1; k < NP; ++k) {
            const uint32_t dst = static_cast<uint32_t>(((pj + k) % NP) * 2) + prank;
            if (half == 0)
              st_async_v4(mapa_shared(smem_u32(xv + (ab * NP + pj) * 128 + row_in_tile), dst), mine,
                          mapa_shared(bar, dst));
            else
              st_async_b32(mapa_shared(smem_u32(xt + (ab * NP + pj) * 128 + row_in_tile), dst), 0u,
                           mapa_shared(bar, dst));
          }
          ok = __all_sync(0xffffffffu, mbar_wait_cluster(&xf0[ab], aph, abort_flag));
          if (ok) {
            float4 tot = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < NP; ++j) {
              const float4 v = j == pj ? mine : xv[(ab * NP + j) * 128 + row_in_tile];
              tot.x += v.x;
              tot.y += v.y;
              tot.z += v.z;
              tot.w += v.w;
            }
            s = 1.0f / sqrtf(tot.x * inv_n + p.eps);
            const float pos = fmaf(s * s, tot.w, tot.y);
            float ss2 = lam * lam * fmaf(s, fmaf(s, tot.w, 2.0f * tot.z), tot.y);
            // identical totals (and rows) in the NP CTAs, so all of them decide alike; each
            // row keeps its own choice, so a row's result never depends on its neighbours
            const bool live = mt * 256 + static_cast<int>(prank) * 128 + row_in_tile < p.M;
            const bool direct = live && (p.rownorm_direct || !(ss2 > pos * lam * lam * 0.00390625f));
            // (the same vote in both warps of the quad and in the NP CTAs)
            if (__any_sync(0xffffffffu, direct)) {
              // exact sum of hv^2 for the quad's rows, second exchange on the quad's barrier
              uint64_t* qbar = &xf1[ab * 4 + quad];
              if (half == 0 && lane == 0) mbar_arrive_expect_tx(qbar, Cfg::XS_TX);
              direct_armed = true;
              float sq = 0.f;
#pragma unroll 1
              for (int q = 0; q < 4; ++q) {
                uint32_t a[32];
                tmem_ld32(tacc + 32 * q, a);
                tmem_ld_wait_tied(a);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const uint4 hq = h_chunk(q >> 1, 4 * (q & 1) + k);
                  const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hq);
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                    const float hv = (__bfloat162float(he[j]) + u2f(a[8 * k + j]) * s * wp[32 * q + 8 * k + j]) * lam;
                    sq = fmaf(hv, hv, sq);
                  }
                }
              }
              red1[(ab * 2 + half) * 128 + row_in_tile] = sq;
              ok = pair_rendezvous(&xbar[quad], xph, abort_flag);
              if (ok) {
                const float m1 = red1[(ab * 2) * 128 + row_in_tile] + red1[(ab * 2 + 1) * 128 + row_in_tile];
                const uint32_t bar1 = smem_u32(qbar);
#pragma unroll
                for (int k = 1; k < NP; ++k) {
                  const uint32_t dst = static_cast<uint32_t>(((pj + k) % NP) * 2) + prank;
                  st_async_b32(mapa_shared(smem_u32(xs + ((ab * NP + pj) * 2 + half) * 128 + row_in_tile), dst),
                               __float_as_uint(m1), mapa_shared(bar1, dst));
                }
                const uint32_t par = (xf1ph >> (ab * 4 + quad)) & 1u;
                ok = __all_sync(0xffffffffu, mbar_wait_cluster(qbar, par, abort_flag));
                if (ok) {
                  xf1ph ^= 1u << (ab * 4 + quad);
                  direct_armed = false;
                  float sd = 0.f;
#pragma unroll
                  for (int j = 0; j < NP; ++j) sd += j == pj ? m1 : xs[((ab * NP + j) * 2) * 128 + row_in_tile];
                  if (direct) ss2 = sd;
                }
              }
            }
            inv_h = 1.0f / sqrtf(ss2 * inv_n + p.eps);
          }
        }
      }
      if (ok) {
        // pass C: hv, x = hv * inv_h * w_next (f16) and h = bf16(hv), 64 columns (one box) at a
        // time; each box is read into registers before the outputs are staged over it
        const int wrow0 = mt * 256 + static_cast<int>(prank) * 128 + quad * 32;
        const uint64_t sl2 = f2(s * lam, s * lam), lam2 = f2(lam, lam), inv2 = f2(inv_h, inv_h);
#pragma unroll 1
        for (int g = 0; g < 2; ++g) {
          uint32_t hw[32];
          uint8_t* box = hb + g * 4096;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {  // 32 columns per TMEM load
            uint32_t a[32];
            tmem_ld32(tacc + 64 * g + 32 * hh, a);
            tmem_ld_wait_tied(a);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int k = 4 * hh + kk;
              const uint4 hq = h_chunk(g, k);
              const uint32_t hw4[4] = {hq.x, hq.y, hq.z, hq.w};
              const float* pw = wp + 64 * g + 8 * k;
              const float* nw = wn + 64 * g + 8 * k;
              const float4 p0 = *reinterpret_cast<const float4*>(pw), p1 = *reinterpret_cast<const float4*>(pw + 4);
              const float4 n0 = *reinterpret_cast<const float4*>(nw), n1 = *reinterpret_cast<const float4*>(nw + 4);
              const uint64_t pv[4] = {f2(p0.x, p0.y), f2(p0.z, p0.w), f2(p1.x, p1.y), f2(p1.z, p1.w)};
              const uint64_t nv[4] = {f2(n0.x, n0.y), f2(n0.z, n0.w), f2(n1.x, n1.y), f2(n1.z, n1.w)};
              uint32_t xw[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint64_t y = f2(u2f(a[8 * kk + 2 * j]), u2f(a[8 * kk + 2 * j + 1]));
                const uint64_t h = f2(__uint_as_float(hw4[j] << 16), __uint_as_float(hw4[j] & 0xffff0000u));
                // hv = (h + y s w) lam = h lam + y (s lam) w;  x = hv (inv_h w_next)
                const uint64_t hv = f2_fma(f2_mul(y, sl2), pv[j], f2_mul(h, lam2));
                const uint64_t xv = f2_mul(hv, f2_mul(inv2, nv[j]));
                float v0, v1;
                f2_split(xv, v0, v1);
                xw[j] = pack_f16(v0, v1);
                f2_split(hv, v0, v1);
                hw[4 * k + j] = pack_bf16(v0, v1);
              }
              stage_chunk(box, k, make_uint4(xw[0], xw[1], xw[2], xw[3]));
            }
          }
          // x, then h, leave through the box by coalesced 16-byte stores (4 rows x 128 bytes per
          // instruction; rows past M are not stored).  Bulk tensor stores from the box were 20 %
          // slower in all: each store's read of the box queued behind the main loop's operand
          // loads in the TMA unit, and the box could be restaged only once it had been read,
          // four waits per tile.
          const int rows_valid = min(32, p.M - wrow0);
          const size_t ldb = static_cast<size_t>(p.N) * 2;
          const size_t off = (static_cast<size_t>(wrow0) * p.N + col0 + 64 * g) * 2;
          flush_rows128(box, reinterpret_cast<uint8_t*>(p.x_next) + off, ldb, rows_valid);
          stage_words32(box, hw);
          flush_rows128(box, reinterpret_cast<uint8_t*>(p.h) + off, ldb, rows_valid);
          if (mt + ncl < p.m_tiles) {  // the next tile's residual rows into the box
            fence_proxy_async_smem();  // this warp's reads of the box before the TMA refill
            __syncwarp();
            prefetch_box(mt + ncl, g);
            h_pending = true;
          }
        }
      }
      if (!ok) {
        if (lane == 0) {
          record_error(p.status, kErrTimeoutEpilogue);
          *abort_flag = 1;
        }
        aborted = true;
        break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[ab]);
      ab ^= 1;
      if (ab == 0) aph ^= 1;
    }
    if (aborted) {
      // After a failed wait the other CTAs may still deliver this tile's sums (they cannot get
      // further: each exchange needs this CTA's sums first); let those land.
      int never = 0;
      mbar_wait_cluster(&xf0[ab], aph, &never);
      if (direct_armed) mbar_wait_cluster(&xf1[ab * 4 + quad], (xf1ph >> (ab * 4 + quad)) & 1u, &never);
    }
    if (lane == 0) bulk_wait_all();  // this warp's output stores are complete
    if (h_pending) {  // no load may still be writing this CTA's shared memory when it leaves
      int never = 0;
      mbar_wait(&hbar[2 * ew], hph, &never);
      mbar_wait(&hbar[2 * ew + 1], hph, &never);
    }
  }

  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace glp
