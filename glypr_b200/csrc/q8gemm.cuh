// Q8_0 GEMM with the weights streamed as raw GGUF blocks: C[M, N] = A[M, K] * dequant(W[N, K])^T
//
//   W   raw Q8_0 rows (ggml block_q8_0 = {f16 d; int8 qs[32]}, K/32 blocks = P = 34 K / 32 bytes
//       per row), exactly the bytes LinearOp::MetalQ8_0 keeps on the device (linear.rs:55-64)
//       and fused_metal_q8_0_matmul reads (metal_kernels/mod.rs:1271-1394, q8_0_mm_impl in
//       fused_ops.metal:650-758, which dequantises a tile in threadgroup memory before its MMA)
//   A   activations, 16-bit T (bf16 for the Q8_0 x bf16 entry point), row-major -> TMA, 128B swizzle
//   accumulator f32 in tensor memory, CTA pairs (cta_group::2): a pair owns 256 rows x BNP columns
//
// The raw rows travel by TMA into shared memory and a group of dequantisation warps turns each
// K step's bytes into the K-major 128-byte-swizzled 16-bit tile the tensor core reads, so the
// weight crosses HBM/L2 as 1.0625 bytes per element and is never written back dequantised.
//
// TMA view of the raw rows.  A tiled TMA copy needs a 16-byte aligned start (x) and row stride;
// P is a multiple of 16 only when K % 256 == 0 (K = 1152 gives P = 1224).  So the rows are seen
// in groups of G (1, 2 or 4: the smallest with G P % 16 == 0) as a 2-D byte tensor
// {G P, N / G}: row r = G j + i is group row j, bytes [i P, i P + P).  One K step (64 elements =
// 2 blocks = 68 bytes) of sub-row i starts at x = i P + 68 kb, a multiple of 4; the copy starts
// at x0 = x & ~15 and takes 80 bytes, which hold the 68 at offset x - x0 in {0, 4, 8, 12}.
//
// Roles (448 threads): warp 0 TMA producer (A through the pair's leader barrier, raw W on this
// CTA's own barrier), warp 1 MMA issuer (leader) / release forwarder (peer), warps 2-9 epilogue
// (gemm_epilogue_tile), warps 10-13 dequantisation.  Rings: SR stages of {A tile, raw W}, SD
// stages of dequantised W.  A raw stage is free when the MMA has consumed its A tile (commit)
// and the four dequant warps have read its bytes; a dequantised stage is filled by the dequant
// warps of both CTAs and freed by the MMA's commit.  The leader's MMA learns that a stage is
// ready from its own dequant warps' arrivals and from one 4-byte st.async token per peer warp
// counted on the same barrier: a remote mbarrier.arrive.release.cluster per warp and K step
// stalled each peer warp about a microsecond (measured: 2.1x the kernel time), while st.async
// does not block the warp and its completion carries the release.
#pragma once
#include "gemm.cuh"

namespace glp {

constexpr int kQ8DequantWarps = 8;
constexpr int kQ8Threads = 320 + 32 * kQ8DequantWarps;
constexpr int kQ8DequantWarp0 = 10;
constexpr int kQ8RawBoxBytes = 80;  // x width of one raw box row (68 bytes needed + up to 12 of lead-in)

template <int BNP>
struct Q8PairCfg {
  static constexpr int B_ROWS = BNP / 2;  // rows of W per CTA
#ifndef GLP_Q8_SR256
#define GLP_Q8_SR256 5
#define GLP_Q8_SD256 3
#endif
  static constexpr int SR = BNP == 256 ? GLP_Q8_SR256 : 6;
  static constexpr int SD = BNP == 256 ? GLP_Q8_SD256 : 4;
  static constexpr uint32_t A_BYTES = 128 * 64 * 2;
  static constexpr uint32_t RAW_BYTES = B_ROWS * kQ8RawBoxBytes;  // G boxes of B_ROWS / G rows
  static constexpr uint32_t DEQ_BYTES = B_ROWS * 128;
  static constexpr uint32_t TMEM_COLS = 2 * BNP;
  static constexpr uint32_t RAW_OFFSET = SR * A_BYTES;
  static constexpr uint32_t DEQ_OFFSET = (RAW_OFFSET + SR * RAW_BYTES + 1023) / 1024 * 1024;
  static constexpr uint32_t BAR_OFFSET = DEQ_OFFSET + SD * DEQ_BYTES;
  static constexpr uint32_t STAGE_OFFSET = (BAR_OFFSET + 1024 + 1023) / 1024 * 1024;
  static constexpr uint32_t STAGE_BYTES = 8 * 32 * 128;
  static constexpr size_t SMEM = STAGE_OFFSET + STAGE_BYTES;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert((3 * SR + 2 * SD + 2 + 2 + 1 + 4) * 8 + 8 <= 512, "barriers before the token slots");
  static_assert(512 + SD * 4 * 4 <= 1024, "token slots");
};

// Eight int8 weights (lo, hi: bytes 0-3, 4-7) times the block scale d, rounded once to T:
// the value f32(d) * q of q8_0_dequant_rows_kernel, bit for bit.
template <typename T>
__device__ __forceinline__ uint4 q8_scale8(uint32_t lo, uint32_t hi, uint16_t d16);

template <>
__device__ __forceinline__ uint4 q8_scale8<__nv_bfloat16>(uint32_t lo, uint32_t hi, uint16_t d16) {
  // int8 -> f32 without I2F: bias each byte to b + 128 and place it in the mantissa of 2^23,
  // then subtract 2^23 + 128 (exact); q * d is exact in f32 and rounds once to bf16
  const float d = __half2float(__ushort_as_half(d16));
  const uint64_t dd = f2(d, d);
  const uint64_t bias = f2(8388736.0f, 8388736.0f);
  const uint32_t ul = lo ^ 0x80808080u, uh = hi ^ 0x80808080u;
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t u = j < 2 ? ul : uh;
    const int b0 = (j & 1) * 2;
    const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u + b0));
    const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u + b0 + 1));
    float v0, v1;
    f2_split(f2_mul(f2_sub(f2(f0, f1), bias), dd), v0, v1);
    out[j] = pack_bf16(v0, v1);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

template <>
__device__ __forceinline__ uint4 q8_scale8<__half>(uint32_t lo, uint32_t hi, uint16_t d16) {
  // int8 -> f16 exactly: bias to b + 128, place it in the mantissa of 1024 (0x6400), subtract
  // 1152; the f16 product q * d is correctly rounded, i.e. f16(f32(d) * q)
  const uint32_t dd = static_cast<uint32_t>(d16) * 0x10001u;
  const uint32_t ul = lo ^ 0x80808080u, uh = hi ^ 0x80808080u;
  const uint32_t m1152 = 0x64806480u;  // {1152, 1152}
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t u = j < 2 ? ul : uh;
    const uint32_t h = __byte_perm(u, 0x64646464u, (j & 1) ? 0x4342u : 0x4140u);
    uint32_t q, r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(q) : "r"(h), "r"(m1152));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(q), "r"(dd));
    out[j] = r;
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// p.m_tiles counts 256-row pair tiles, p.n_tiles BNP-column tiles; p.raw_pitch = P,
// p.raw_group = G.  tmA: A [M, K] (64 x 128 boxes, 128B swizzle); tmW: the raw rows as bytes
// {G P, N / G} (80 x B_ROWS / G boxes, no swizzle).
template <int EPI, typename T, int BNP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kQ8Threads, 1)
    gemm_q8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                        const GemmParams p) {
  using Cfg = Q8PairCfg<BNP>;
  constexpr int SR = Cfg::SR, SD = Cfg::SD;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the same in both CTAs: both leave before any cluster step
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sA = smem;
  uint8_t* sRaw = smem + Cfg::RAW_OFFSET;
  uint8_t* sDeq = smem + Cfg::DEQ_OFFSET;
  uint64_t* afull = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFFSET);  // used in the leader
  uint64_t* rfull = afull + SR;
  uint64_t* empty = rfull + SR;   // MMA commit (A consumed) + the 4 dequant warps (raw consumed)
  uint64_t* dfull = empty + SR;   // used in the leader: its 4 dequant warps + the peer's 4 tokens
  uint64_t* dempty = dfull + SD;  // MMA commit
  uint64_t* tfull = dempty + SD;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* xbar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* tokens = reinterpret_cast<uint32_t*>(smem + Cfg::BAR_OFFSET + 512);  // [SD][4], leader only

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int n_pairs = static_cast<int>(n_clusters_x());
  const int num_tiles = p.m_tiles * p.n_tiles;
  const int G = p.raw_group;
  const int P = p.raw_pitch;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SR; ++s) {
      mbar_init(&afull[s], 1);
      mbar_init(&rfull[s], 1);
      mbar_init(&empty[s], 1 + kQ8DequantWarps);
    }
    for (int d = 0; d < SD; ++d) {
      mbar_init(&dfull[d], kQ8DequantWarps);
      mbar_init(&dempty[d], 1);
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
    tma_prefetch_desc(&tmW);
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
      // ------------------------------------------------------------ TMA producer (both CTAs)
      const int box_rows = Cfg::B_ROWS / G;
      const uint32_t box_bytes = static_cast<uint32_t>(box_rows) * kQ8RawBoxBytes;
      int s = 0;
      uint32_t ph = 0;
      for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs) {
        const int m_blk = tile / p.n_tiles, n_blk = tile % p.n_tiles;
        const int grow0 = (n_blk * BNP + static_cast<int>(rank) * Cfg::B_ROWS) / G;  // first group row
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            record_error(p.status, kErrTimeoutProducer);
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&afull[s], 2 * Cfg::A_BYTES);
          tma_load_2d_pair(sA + s * Cfg::A_BYTES, &tmA, mapa_shared(smem_u32(&afull[s]), 0), kb * 64,
                           m_blk * 256 + static_cast<int>(rank) * 128);
          mbar_arrive_expect_tx(&rfull[s], Cfg::RAW_BYTES);
          uint8_t* dst = sRaw + s * Cfg::RAW_BYTES;
          for (int i = 0; i < G; ++i)
            tma_load_2d(dst + i * box_bytes, &tmW, &rfull[s], (i * P + 68 * kb) & ~15, grow0);
          if (++s == SR) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      constexpr uint32_t idesc = idesc_f16(256, BNP, Half16<T>::kIsBf16);
      int s = 0, d = 0;
      uint32_t ph = 0, dph = 0;
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
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * BNP);
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&afull[s], ph, abort_flag) || !mbar_wait_cluster(&dfull[d], dph, abort_flag)) {
            record_error(p.status, kErrTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = desc_kmajor_sw128(smem_u32(sA + s * Cfg::A_BYTES));
          const uint64_t bdesc = desc_kmajor_sw128(smem_u32(sDeq + d * Cfg::DEQ_BYTES));
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          issued = true;
          umma_commit_pair(smem_u32(&empty[s]));
          umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
          umma_commit_pair(smem_u32(&dempty[d]));
          umma_commit_pair(mapa_shared(smem_u32(&dempty[d]), 1));
          if (++s == SR) {
            s = 0;
            ph ^= 1;
          }
          if (++d == SD) {
            d = 0;
            dph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull[ab]));
        umma_commit_pair(mapa_shared(smem_u32(&tfull[ab]), 1));
        ab ^= 1;
        if (ab == 0) aph ^= 1;
      }
      if (issued) {
        umma_commit_pair(smem_u32(drain));
        if (!mbar_wait(drain, 0, abort_flag) && !*abort_flag) record_error(p.status, kErrTimeoutDrain);
      }
    } else if (lane == 0) {
      // ------------------------------------------------------------ release forwarder (peer)
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
  } else if (warp >= kQ8DequantWarp0) {
    // -------------------------------------------------------------- dequantisation warps
    // Per K step this warp turns rows [dw R, dw R + R) of the CTA's B_ROWS (R = B_ROWS / warps),
    // 8 rows x 4 quarters per pass: lane = (row, quarter).  Quarter q holds elements 16 q ..
    // 16 q + 15 of the step, i.e. half q % 2 of block q / 2 -- chunks 2 q and 2 q + 1 of 8
    // elements, which land in the 128B-swizzled row at 16-byte positions c ^ (row & 7), as a
    // TMA load would have put them.
    constexpr int R = Cfg::B_ROWS / kQ8DequantWarps;
    static_assert(R % 8 == 0, "dequant passes of 8 rows");
    const int dw = warp - kQ8DequantWarp0;
    const int qt = lane & 3;
    const int blk = qt >> 1;
    const int c0 = 2 * qt;  // first of the quarter's two chunks
    const int lg = G >> 1;  // log2 G for G in {1, 2, 4}
    const uint32_t box_bytes = static_cast<uint32_t>(Cfg::B_ROWS >> lg) * kQ8RawBoxBytes;
    const uint32_t lead_dfull0 = mapa_shared(smem_u32(&dfull[0]), 0);
    // the peer's "stage ready" token: 4 bytes stored into the leader's slot [d][dw] with the
    // byte count completing on the leader's dfull[d] (st.async: the issuing warp does not wait
    // for it, and its completion releases this CTA's earlier writes at cluster scope)
    const uint32_t lead_tok0 = mapa_shared(smem_u32(tokens), 0) + static_cast<uint32_t>(dw) * 4u;
    // this lane's rows are r0 + 8 it: all in sub-row i = r0 % G (R and 8 are multiples of G),
    // group rows (r0 >> lg) + (8 it >> lg)
    const int r0 = dw * R + (lane >> 2);
    const int i_sub = r0 & (G - 1);
    const uint32_t lane_off = static_cast<uint32_t>(i_sub) * box_bytes + static_cast<uint32_t>(r0 >> lg) * kQ8RawBoxBytes +
                              34u * blk;
    int s = 0, d = 0;
    uint32_t ph = 0, dph = 0;
    for (int tile = pair; tile < num_tiles && !*abort_flag; tile += n_pairs) {
      bool ok = true;
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        ok = mbar_wait(&rfull[s], ph, abort_flag) && mbar_wait(&dempty[d], dph ^ 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        // bytes before the step's 68 in this lane's box rows
        const uint32_t lead = static_cast<uint32_t>(i_sub * P + 68 * kb) & 15u;
        const uint32_t base = s * Cfg::RAW_BYTES + lane_off + lead;  // byte offset of the block in sRaw
        uint8_t* deq = sDeq + d * Cfg::DEQ_BYTES;
        const uint32_t qa0 = base + 2 + 16 * (qt & 1);  // the quarter's 16 int8 (2-byte aligned), first row
        const uint32_t sh = (qa0 & 3u) * 8u;
        const uint32_t* qw0 = reinterpret_cast<const uint32_t*>(sRaw + (qa0 & ~3u));
        const uint32_t* dw0 = reinterpret_cast<const uint32_t*>(sRaw + (base & ~3u));  // word with the f16 scale
        const bool d_hi = (base & 2u) != 0;
        constexpr int NIT = R / 8;
        // all of this lane's loads first (one shared-memory latency for the whole step), then
        // the conversions and stores
        uint32_t w[NIT][5], dv[NIT];
#pragma unroll
        for (int it = 0; it < NIT; ++it) {
          const int off = ((8 * it) >> lg) * (kQ8RawBoxBytes / 4);
#pragma unroll
          for (int j = 0; j < 4; ++j) w[it][j] = qw0[off + j];
          w[it][4] = sh ? qw0[off + 4] : 0u;
          dv[it] = dw0[off];
        }
#pragma unroll
        for (int it = 0; it < NIT; ++it) {
          uint32_t q[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) q[j] = __funnelshift_r(w[it][j], w[it][j + 1], sh);
          const uint16_t d16 = static_cast<uint16_t>(d_hi ? (dv[it] >> 16) : (dv[it] & 0xffffu));
          const int r = r0 + 8 * it;
          uint8_t* row = deq + r * 128;
          *reinterpret_cast<uint4*>(row + ((c0 ^ (r & 7)) << 4)) = q8_scale8<T>(q[0], q[1], d16);
          *reinterpret_cast<uint4*>(row + (((c0 + 1) ^ (r & 7)) << 4)) = q8_scale8<T>(q[2], q[3], d16);
        }
        fence_proxy_async_smem();  // the tensor core reads these tiles through the async proxy
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty[s]);  // this CTA's raw stage is read
          if (leader)  // ready here, and expect the peer warp's 4-byte token
            mbar_arrive_expect_tx(&dfull[d], 4);
          else
            st_async_b32(lead_tok0 + static_cast<uint32_t>(d * kQ8DequantWarps * 4), 1u,
                         lead_dfull0 + static_cast<uint32_t>(d * sizeof(uint64_t)));
        }
        if (++s == SR) {
          s = 0;
          ph ^= 1;
        }
        if (++d == SD) {
          d = 0;
          dph ^= 1;
        }
      }
      if (!ok) {
        if (lane == 0) {
          record_error(p.status, kErrTimeoutProducer);
          *abort_flag = 1;
        }
        break;
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
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(ab * BNP);
      if (!gemm_epilogue_tile<BNP, EPI, T>(p, tacc, 2 * m_blk + static_cast<int>(rank), n_blk, row_in_tile, half,
                                           nullptr, &xbar[quad], xph, abort_flag, stage)) {
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
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace glp
