// Bidirectional GQA flash attention on the 5th-generation tensor cores (tcgen05), head_dim
// 256, f16 operands, f32 accumulation in tensor memory, f32 softmax.
//
// Semantics (reference): scores = q . k with scale 1.0 (attention/standard.rs:62,
// metal_flash.rs:329); a key j is visible from query i iff j < len(seq) and, on sliding
// layers, |i - j| <= W (model.rs:634-638, chunked.rs:14-50); softmax in f32; query head h
// reads kv head h / (Hq / Hkv) (repeat_kv, attention/mod.rs:22-31).  Padding is handled
// analytically from the packed sequence offsets (no mask tensors).
//
// Persistent kernel: one CTA per SM loops over work items (sequence, 128-row query block,
// head), ordered so that the CTAs running at the same time share sequences (K/V stay in L2).
// Tensor memory and the mbarriers are set up once; every ring below is indexed by a running
// KV-tile counter g that continues across items.  352 threads:
//   warp 0      TMA producer of Q and K: Q of the item (4 boxes of 64 dims x 128 rows) once
//               the previous item's Q has been copied out of the buffer, then the K tiles of
//               64 keys into a 2-stage ring (a stage frees as soon as S_j is computed)
//   warp 10     TMA producer of the V tiles (2-stage ring, a stage frees once P_j V_j is
//               computed).  K and V have separate producers so that a K load never queues
//               behind a wait for a V stage: S_{j+2} needs K_{j+2} about one softmax tile
//               after S_j frees its stage, which is little more than an L2 round trip.
//   warp 1      TMEM owner + single-thread MMA issuer.  Both MMAs read their A operand from
//               tensor memory, so shared-memory bandwidth goes to K and V only:
//                 Q  -> TMEM      (16 tcgen05.cp of 128 rows x 16 dims, once per item)
//                 S_j = Q K_j^T   (M=128, N=64, K=256; Q in TMEM, K K-major in SMEM) -> S[g%2]
//                 O  += P_j V_j   (M=128, N=256, K=64; P in TMEM over S[g%2], V MN-major)
//               S_{j+1} is issued before waiting for P_j, and the next item's Q and S_0 are
//               in flight while the previous item's O is drained.
//   warps 2..9  softmax / correction / epilogue: the two warps of a TMEM lane quadrant
//               share its 32 query rows (one row per thread) and split the 64 key columns
//               of S_j (and later the 256 columns of O) in halves.
//
// Softmax of one tile, per thread (one row, 32 keys):
//   * mask (boundary tiles only), row maximum of the 32 scores (three-input max), log2 domain;
//   * publish that maximum to the partner warp (one mbarrier arrive, double-buffered
//     exchange slots) and, without waiting, exponentiate against the running reference max
//     (or against its own maximum if that alone exceeds the reference by more than 2^12);
//   * then collect the partner's maximum: the joint row maximum decides the new reference
//     (lazy rescaling: the reference moves only when the row maximum exceeds it by more than
//     2^12, and the stale reference is exact for the final O / l); in the rare case that the
//     speculative reference was not the final one the 32 exponentials are multiplied by the
//     correction, and O (in TMEM) and l by the reference change;
//   * 2^x: MUFU.EX2 for most pairs, a degree-4 polynomial on the FMA pipe for the pairs in
//     kFaPolyPairs (the special-function unit is the bottleneck otherwise);
//   * P (f16 pairs) into tensor memory over the first 32 columns of its own S slot (both
//     halves have read S_j before either writes P_j: the write follows the exchange); only
//     then is the next tile's S waited for and read.
// At the item's end O / l is converted to f16 and staged through shared memory (4 KB per
// warp): bulk tensor stores for 32-row slices inside the sequence, coalesced stores row by
// row for the slice that crosses its end.
// TMEM columns: S[0] 0-63, S[1] 64-127 (P_j in the first 32 of its slot), Q 128-255, O 256-511.
// Every mbarrier wait is bounded (see common.cuh) and reports through the status word.
#pragma once
#include "common.cuh"

namespace glp {

constexpr int kFaBQ = 128;
constexpr int kFaBKV = 64;
constexpr int kFaD = 256;
constexpr uint32_t kFaQBytes = kFaBQ * kFaD * 2;         // 64 KB (4 chunks of 16 KB)
constexpr uint32_t kFaKVChunk = kFaBKV * 128;            // 8 KB: 64 keys x 64 dims
constexpr uint32_t kFaKVBytes = 4 * kFaKVChunk;          // 32 KB per K or V tile
constexpr uint32_t kFaStageBytes = 8 * 4096;            // output staging, 4 KB per epilogue warp
constexpr uint32_t kFaBarBytes = 256;
constexpr uint32_t kFaXchBytes = 2 * 2 * 128 * 4;        // [2 slots][2 halves][128 rows] f32
// the dynamic shared-memory base is declared 1024-aligned (checked at run time)
constexpr size_t kFaSmem = kFaQBytes + 4 * kFaKVBytes + kFaStageBytes + kFaBarBytes + kFaXchBytes;
constexpr int kFaThreads = 352;
constexpr int kFaOutBoxRows = 32;                        // rows of one output bulk store
constexpr uint32_t kFaTmemQ = 128;                       // TMEM column of Q (128 columns)
constexpr uint32_t kFaTmemO = 256;                       // TMEM column of O (256 columns)
constexpr float kFaRescaleLog2 = 12.0f;                  // lazy-rescale threshold (P <= 4096)
// Of the 16 exponential pairs per thread and tile, the ones evaluated by the polynomial
// (bit e = pair e): 6 of 16, which balances the special-function unit against the issue slots.
constexpr uint32_t kFaPolyPairs = (1u << 1) | (1u << 4) | (1u << 6) | (1u << 9) | (1u << 11) | (1u << 14);

struct FaParams {
  const int* cu_seqlens;
  int cu_base;
  int n_seq;
  int q_blocks;  // ceil(max_len / 128)
  int n_q_heads, n_kv_heads;
  int window;
  __half* out;
  int ld_out;
  int* status;
};

struct FaItem {
  bool valid;
  int tok0, len, q0, qcol, kcol, vcol, t_lo, n_tiles;
};

__device__ __forceinline__ FaItem fa_item(const FaParams& p, int item) {
  FaItem w;
  const int per_seq = p.q_blocks * p.n_q_heads;
  const int b = item / per_seq;
  const int r = item - b * per_seq;
  const int qb = r / p.n_q_heads;
  const int head = r - qb * p.n_q_heads;
  const int seq0 = __ldg(p.cu_seqlens + b);
  w.tok0 = seq0 - p.cu_base;
  w.len = __ldg(p.cu_seqlens + b + 1) - seq0;
  w.q0 = qb * kFaBQ;
  w.valid = w.q0 < w.len;
  const int kvh = head / (p.n_q_heads / p.n_kv_heads);
  w.qcol = head * kFaD;
  w.kcol = (p.n_q_heads + kvh) * kFaD;
  w.vcol = (p.n_q_heads + p.n_kv_heads + kvh) * kFaD;
  int kv_lo = 0, kv_hi = w.len;
  if (p.window > 0) {
    kv_lo = max(0, w.q0 - p.window);
    kv_hi = min(w.len, w.q0 + kFaBQ + p.window);
  }
  w.t_lo = kv_lo / kFaBKV;
  w.n_tiles = (kv_hi + kFaBKV - 1) / kFaBKV - w.t_lo;
  return w;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for both lanes of a pair, x <= 64, on the FMA pipe: x = j + f with j = round(x)
// (1.5 * 2^23 added and subtracted), 2^f on |f| <= 1/2 by a degree-4 polynomial fitted here
// (weighted least squares towards minimax relative error, c0 fixed at 1 so integers are
// exact; max relative error 2.9e-6, far below f16 rounding of P), and 2^j added to the
// exponent field.  x is clamped at -125 (result ~2^-125, zero once P is rounded to f16).
__device__ __forceinline__ uint64_t exp2_poly_pair(uint64_t x) {
  float a, b;
  f2_split(x, a, b);
  a = fmaxf(a, -125.f);
  b = fmaxf(b, -125.f);
  const uint64_t xc = f2(a, b);
  const uint64_t magic = f2(12582912.f, 12582912.f);
  const uint64_t t = f2_add(xc, magic);
  const uint64_t f = f2_sub(xc, f2_sub(t, magic));
  uint64_t q = f2_fma(f2(0.009582829661667347f, 0.009582829661667347f), f, f2(0.05590638890862465f, 0.05590638890862465f));
  q = f2_fma(q, f, f2(0.24024099111557007f, 0.24024099111557007f));
  q = f2_fma(q, f, f2(0.6931241750717163f, 0.6931241750717163f));
  q = f2_fma(q, f, f2(1.0f, 1.0f));
  float qa, qb, ta, tb;
  f2_split(q, qa, qb);
  f2_split(t, ta, tb);
  // the low mantissa bits of t hold j (two's complement); << 23 moves them into the exponent
  const float ra = __uint_as_float(__float_as_uint(qa) + (__float_as_uint(ta) << 23));
  const float rb = __uint_as_float(__float_as_uint(qb) + (__float_as_uint(tb) << 23));
  return f2(ra, rb);
}

__device__ __forceinline__ float max32(const float (&v)[32]) {
  float m[11];
#pragma unroll
  for (int k = 0; k < 10; ++k) m[k] = fmax3(v[3 * k], v[3 * k + 1], v[3 * k + 2]);
  m[10] = fmaxf(v[30], v[31]);
  const float a = fmax3(m[0], m[1], m[2]), b = fmax3(m[3], m[4], m[5]), c = fmax3(m[6], m[7], m[8]);
  return fmax3(fmax3(a, b, c), m[9], m[10]);
}

__global__ void __launch_bounds__(kFaThreads, 1)
    flash_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                         const __grid_constant__ CUtensorMap tmO, const FaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the swizzled operand tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kFaQBytes;            // [2][4][64 x 128 B]
  uint8_t* sV = sK + 2 * kFaKVBytes;       // [2][4][64 x 128 B]
  uint8_t* sStage = sV + 2 * kFaKVBytes;   // [8 warps][32 x 128 B]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sStage + kFaStageBytes);
  uint64_t* q_full = bar;
  uint64_t* q_empty = bar + 1;   // Q SMEM buffer free once Q is copied into TMEM
  uint64_t* k_full = bar + 2;    // [2]
  uint64_t* k_empty = bar + 4;   // [2]  K stage free once S_j is computed
  uint64_t* v_full = bar + 6;    // [2]
  uint64_t* v_empty = bar + 8;   // [2]  V stage free once P_j V_j is computed
  uint64_t* s_full = bar + 10;   // [2]
  uint64_t* p_full = bar + 12;   // [2]
  uint64_t* pv_done = bar + 14;  // [2]
  uint64_t* o_free = bar + 16;   // O drained by the epilogue warps
  uint64_t* drain = bar + 17;
  uint64_t* xbar = bar + 18;     // [4] per-quadrant exchange barrier of the two softmax warps
  uint64_t* q_tfree = bar + 22;  // Q columns of TMEM free once the item's last S is computed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bar) + kFaBarBytes);  // [2][2][128]

  const int n_items = p.n_seq * p.q_blocks * p.n_q_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_free, 8);
    mbar_init(drain, 1);
    mbar_init(q_tfree, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 2);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ Q / K producer
      int it = 0;
      uint32_t g = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const FaItem w = fa_item(p, item);
        if (!w.valid) continue;
        if (!mbar_wait(q_empty, (it & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, kFaQBytes);
        for (int c = 0; c < 4; ++c)
          tma_load_2d(sQ + c * (kFaBQ * 128), &tmQ, q_full, w.qcol + 64 * c, w.tok0 + w.q0);
        for (int j = 0; j < w.n_tiles; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = ((g >> 1) & 1) ^ 1;
          const int row = w.tok0 + (w.t_lo + j) * kFaBKV;
          if (!mbar_wait(&k_empty[st], ph, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], kFaKVBytes);
          for (int c = 0; c < 4; ++c)
            tma_load_2d(sK + st * kFaKVBytes + c * kFaKVChunk, &tmKV, &k_full[st], w.kcol + 64 * c, row);
        }
        ++it;
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutProducer);
        *abort_flag = 1;
      }
    }
  } else if (warp == 10) {
    if (lane == 0) {
      // ------------------------------------------------------------------ V producer
      uint32_t g = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const FaItem w = fa_item(p, item);
        if (!w.valid) continue;
        for (int j = 0; j < w.n_tiles; ++j, ++g) {
          const int st = g & 1;
          const int row = w.tok0 + (w.t_lo + j) * kFaBKV;
          if (!mbar_wait(&v_empty[st], ((g >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], kFaKVBytes);
          for (int c = 0; c < 4; ++c)
            tma_load_2d(sV + st * kFaKVBytes + c * kFaKVChunk, &tmKV, &v_full[st], w.vcol + 64 * c, row);
        }
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutProducer);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = idesc_f16(128, kFaBKV, 0);
      constexpr uint32_t idesc_pv = idesc_f16(128, kFaD, 0) | (1u << 16);  // B (V) MN-major
      auto issue_s = [&](uint32_t gx) -> bool {
        const int st = gx & 1;
        if (!mbar_wait(&k_full[st], (gx >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(st * kFaBKV);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint64_t kd = desc_kmajor_sw128(smem_u32(sK + st * kFaKVBytes + c * kFaKVChunk));
#pragma unroll
          for (int k = 0; k < 4; ++k)  // 16 dims = 8 TMEM columns of Q per K step
            umma_f16_ts(d, tmem + kFaTmemQ + (4 * c + k) * 8, kd + 2 * k, idesc_s, (c | k) != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        return true;
      };
      int it = 0;
      uint32_t g = 0;
      bool ok = true;
      bool issued = false;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const FaItem w = fa_item(p, item);
        if (!w.valid) continue;
        // the previous item's S MMAs have read the Q columns; this item's Q has landed
        if ((it >= 1 && !mbar_wait(q_tfree, (it - 1) & 1, abort_flag)) || !mbar_wait(q_full, it & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issued = true;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint64_t qd = desc_kmajor_sw128(smem_u32(sQ + c * (kFaBQ * 128)));
#pragma unroll
          for (int k = 0; k < 4; ++k) tmem_cp_128x256b(tmem + kFaTmemQ + (4 * c + k) * 8, qd + 2 * k);
        }
        umma_commit(q_empty);  // Q SMEM buffer free once the copies have read it
        if (!issue_s(g)) {
          ok = false;
          break;
        }
        for (int j = 0; j < w.n_tiles; ++j) {
          const uint32_t gj = g + j;
          const int st = gj & 1;
          if (j + 1 < w.n_tiles) {
            if (!issue_s(gj + 1)) {
              ok = false;
              break;
            }
          } else {
            umma_commit(q_tfree);  // every S of this item has been issued
          }
          if (!mbar_wait(&p_full[st], (gj >> 1) & 1, abort_flag) ||
              !mbar_wait(&v_full[st], (gj >> 1) & 1, abort_flag) ||
              (j == 0 && it >= 1 && !mbar_wait(o_free, (it - 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // V rows k*16..k*16+15 of this stage: 16 keys x 128 B further per K step; P: 16 keys
            // = 8 TMEM columns per K step
            const uint64_t vd =
                desc_mnmajor_sw128(smem_u32(sV + st * kFaKVBytes + k * 16 * 128), kFaKVChunk, 1024);
            umma_f16_ts(tmem + kFaTmemO, tmem + st * kFaBKV + k * 8, vd, idesc_pv, (j | k) != 0 ? 1u : 0u);
          }
          umma_commit(&pv_done[st]);
          umma_commit(&v_empty[st]);
        }
        g += w.n_tiles;
        ++it;
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutMma);
        *abort_flag = 1;
      }
      if (issued) {
        // let every issued MMA retire before tensor memory is released
        umma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < GLP_WAIT_TIMEOUT_NS) {
        }
      }
    }
  } else {
    // -------------------------------------------------------------------- softmax + epilogue
    // (warps 2..9)
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // which 32 key columns of S / 128 columns of O
    const int r = quad * 32 + lane;    // query row inside the tile == TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr float kLog2e = 1.4426950408889634f;
    // Per-row value exchange with the partner warp: publish() writes this half's value into
    // the current slot and arrives; collect() waits for the partner's arrival and reads its
    // value.  Two slots alternate, so one arrival per exchange suffices: a warp rewrites a
    // slot only after the next exchange's barrier phase, which needs the partner's arrival,
    // which follows the partner's read of that slot.
    uint32_t xph = 0, xslot = 0;
    auto publish = [&](float v) {
      xch[xslot * 256 + half * 128 + r] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[quad]);
    };
    auto collect = [&](float* other) -> bool {
      const bool wt = mbar_wait(&xbar[quad], xph, abort_flag);
      xph ^= 1u;
      if (!__all_sync(0xffffffffu, wt)) return false;
      *other = xch[xslot * 256 + (half ^ 1) * 128 + r];
      xslot ^= 1u;
      return true;
    };
    // staging tile of this warp's output slices (32 rows x 128 B)
    uint8_t* stage = sStage + (warp - 2) * (kFaOutBoxRows * 128);
    bool stores_pending = false;
    uint32_t g = 0;
    bool ok = true;
    uint32_t sr[32];
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
      const FaItem w = fa_item(p, item);
      if (!w.valid) continue;
      const int i = w.q0 + r;  // position inside the sequence
      float m_ref = -INFINITY, l = 0.f;
      {
        const int st = g & 1;
        const bool wt = mbar_wait(&s_full[st], (g >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, wt)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_ld32(lane_base + st * kFaBKV + half * 32, sr);
        tmem_ld_wait_tied(sr);
      }
      for (int j = 0; j < w.n_tiles; ++j) {
        const uint32_t gj = g + j;
        const int st = gj & 1;
        const int kb = (w.t_lo + j) * kFaBKV + half * 32;  // first key of this warp's columns
        // masking is needed only on tiles that reach past the sequence or the window edge
        // (the same for every row of the item and both halves: warp-uniform)
        const int kt = (w.t_lo + j) * kFaBKV;
        const bool full_tile =
            kt + kFaBKV <= w.len &&
            (p.window <= 0 || (kt >= w.q0 + kFaBQ - 1 - p.window && kt + kFaBKV - 1 <= w.q0 + p.window));
        float sv[32];
        if (full_tile) {
#pragma unroll
          for (int e = 0; e < 32; ++e) sv[e] = u2f(sr[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int kj = kb + e;
            bool valid = kj < w.len;
            if (p.window > 0) valid = valid && abs(i - kj) <= p.window;
            sv[e] = valid ? u2f(sr[e]) : -INFINITY;
          }
        }
        const float mine = max32(sv) * kLog2e;  // this half's row maximum, log2 domain
        publish(mine);
        // speculative reference: the running one unless this half alone needs a rescale
        const float mu_s = mine > m_ref + kFaRescaleLog2 ? mine : m_ref;
        const float mu = mu_s == -INFINITY ? 0.f : mu_s;
        const uint64_t l2e = f2(kLog2e, kLog2e), nmu = f2(-mu, -mu);
        uint64_t ev[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint64_t x = f2_fma(f2(sv[2 * e], sv[2 * e + 1]), l2e, nmu);
          if ((kFaPolyPairs >> e) & 1u) {
            ev[e] = exp2_poly_pair(x);
          } else {
            float a, b;
            f2_split(x, a, b);
            ev[e] = f2(fast_exp2(a), fast_exp2(b));
          }
        }
        float other;
        if (!collect(&other)) {
          ok = false;
          break;
        }
        const float joint = fmaxf(mine, other);
        const float m_new = joint > m_ref + kFaRescaleLog2 ? joint : m_ref;
        // O and l: rescale when the reference moves (nothing accumulated while it was -inf)
        const float factor = (m_ref == -INFINITY || m_new == m_ref) ? 1.f : fast_exp2(m_ref - m_new);
        // this half's exponentials: correction when the speculative reference was not m_new
        const float corr = mu_s == m_new ? 1.f : fminf(fast_exp2(mu - m_new), 1.f);
        m_ref = m_new;
        if (__any_sync(0xffffffffu, corr != 1.f)) {
          const uint64_t c2 = f2(corr, corr);
#pragma unroll
          for (int e = 0; e < 16; ++e) ev[e] = f2_mul(ev[e], c2);
        }
        uint32_t pk[16];
        uint64_t acc[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float a, b;
          f2_split(ev[e], a, b);
          pk[e] = pack_f16(a, b);
          acc[e & 3] = f2_add(acc[e & 3], ev[e]);
        }
        {
          float s0, s1;
          f2_split(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), s0, s1);
          l = l * factor + (s0 + s1);  // this half's partial row sum
        }
        // O may be rescaled only after P_{j-1} V_{j-1} has landed.  (P_j's columns are free:
        // S_j, written after P_{j-2} V_{j-2} had read them, has completed.)  Both warps of a
        // pair take the same branch (same rows, same factors).
        if (j >= 1 && __any_sync(0xffffffffu, factor != 1.0f)) {
          const bool wt = mbar_wait(&pv_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, wt)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // this half's 128 O columns, two 32-column chunks in flight per round (the stores
          // complete at the wait that follows the P store below)
          const uint64_t f2x = f2(factor, factor);
#pragma unroll 1
          for (int c = 0; c < 4; c += 2) {
            uint32_t oa[32], ob[32];
            const uint32_t ta = lane_base + kFaTmemO + half * 128 + c * 32;
            tmem_ld32(ta, oa);
            tmem_ld32(ta + 32, ob);
            tmem_ld_wait_tied(oa);
            tmem_ld_wait_tied(ob);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float a, b;
              f2_split(f2_mul(f2(u2f(oa[e]), u2f(oa[e + 1])), f2x), a, b);
              oa[e] = __float_as_uint(a);
              oa[e + 1] = __float_as_uint(b);
              f2_split(f2_mul(f2(u2f(ob[e]), u2f(ob[e + 1])), f2x), a, b);
              ob[e] = __float_as_uint(a);
              ob[e + 1] = __float_as_uint(b);
            }
            tmem_st32(ta, oa);
            tmem_st32(ta + 32, ob);
          }
        }
        // P row r, this half's 32 keys: 16 columns of f16 pairs over the S slot
        tmem_st16(lane_base + st * kFaBKV + half * 16, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[st]);
        // then the next tile's scores (S_{j+1} is queued behind P_{j-1} V_{j-1}: waiting for it
        // before publishing P_j would chain the tensor core and the softmax)
        if (j + 1 < w.n_tiles) {
          const uint32_t gn = gj + 1;
          const bool wt = mbar_wait(&s_full[gn & 1], (gn >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, wt)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_ld32(lane_base + (gn & 1) * kFaBKV + half * 32, sr);
          tmem_ld_wait_tied(sr);
        }
      }
      if (!ok) break;
      // ---- drain O of this item (the next item's Q load and S_0 are already in flight)
      const uint32_t gl = g + w.n_tiles - 1;
      const bool wt = mbar_wait(&pv_done[gl & 1], (gl >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, wt)) {
        ok = false;
        break;
      }
      tc_fence_after();
      publish(l);
      float l_other;
      if (!collect(&l_other)) {
        ok = false;
        break;
      }
      const float lt = l + l_other;
      const float inv = lt > 0.f ? 1.0f / lt : 0.f;
      const uint64_t inv2 = f2(inv, inv);
      // this warp's 32 rows: all inside the sequence -> bulk tensor stores, else row by row
      const int row0 = w.q0 + quad * kFaOutBoxRows;
      const bool bulk = row0 + kFaOutBoxRows <= w.len;
      const uint32_t ob_base = lane_base + kFaTmemO + half * 128;
#pragma unroll 1
      for (int k = 0; k < 2; ++k) {  // two slices of 64 output columns
        uint32_t oa[32], ob[32];
        tmem_ld32(ob_base + k * 64, oa);
        tmem_ld32(ob_base + k * 64 + 32, ob);
        if (stores_pending) {  // the previous slice's bulk store has read the staging tile
          if (lane == 0) bulk_wait_read_all();
          stores_pending = false;
        }
        __syncwarp();
        tmem_ld_wait_tied(oa);
        tmem_ld_wait_tied(ob);
        // row `lane` of the 32 x 128 B staging tile, 16-byte chunks swizzled (chunk ^ (row & 7))
        uint8_t* srow = stage + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* o = c < 4 ? &oa[8 * c] : &ob[8 * (c - 4)];
          uint32_t h[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float a, b;
            f2_split(f2_mul(f2(u2f(o[2 * q]), u2f(o[2 * q + 1])), inv2), a, b);
            h[q] = pack_f16(a, b);
          }
          *reinterpret_cast<uint4*>(srow + ((c ^ (lane & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
        }
        const int col = w.qcol + half * 128 + k * 64;
        if (bulk) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmO, stage, col, w.tok0 + row0);
            bulk_commit();
          }
          stores_pending = true;
        } else {
          __syncwarp();
          // 4 rows of 128 B per instruction: lane -> (row rr + lane / 8, chunk lane % 8)
#pragma unroll 1
          for (int rr = 0; rr < kFaOutBoxRows; rr += 4) {
            const int row = rr + (lane >> 3), c = lane & 7;
            const uint4 v = *reinterpret_cast<const uint4*>(stage + row * 128 + ((c ^ (row & 7)) << 4));
            if (row0 + row < w.len)
              *reinterpret_cast<uint4*>(p.out + static_cast<size_t>(w.tok0 + row0 + row) * p.ld_out + col + c * 8) = v;
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      g += w.n_tiles;
    }
    if (lane == 0) {
      bulk_wait_all();  // output rows written before the CTA exits
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutEpilogue);
        *abort_flag = 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace glp
