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
// KV-tile counter g that continues across items.  320 threads:
//   warp 0      TMA producer: Q of the item (4 boxes of 64 dims x 128 rows) once the
//               previous item's last S has read the Q buffer, then K and V tiles of 64 keys
//               into two separate 2-stage rings (a K stage frees as soon as S_j is computed)
//   warp 1      TMEM owner + single-thread MMA issuer:
//                 S_j = Q K_j^T   (M=128, N=64, K=256; A and B K-major)   -> TMEM S[g%2]
//                 O  += P_j V_j   (M=128, N=256, K=64;  P K-major in SMEM, V MN-major)
//               S_{j+1} is issued before waiting for P_j, and the next item's Q and S_0 are
//               in flight while the previous item's O is drained.
//   warps 2..9  softmax / correction / epilogue: the two warps of a TMEM lane quadrant
//               share its 32 query rows (one row per thread) and split the 64 key columns
//               of S_j (and later the 256 columns of O) in halves; row maxima and row sums
//               are exchanged through shared memory with a bounded mbarrier rendezvous.  Mask
//               (boundary tiles only), online max in the log2 domain with lazy rescaling (O
//               is rescaled in TMEM only when the running max grows by more than 2^8; the
//               stale max is exact for the final O / l), write P_j (f16) into a 128B-swizzled
//               K-major SMEM tile; at the item's end O / l -> f16.
// TMEM: S[0] cols 0-63, S[1] cols 64-127, O cols 256-511.
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
constexpr uint32_t kFaPBytes = kFaBQ * kFaBKV * 2;       // 16 KB
constexpr uint32_t kFaBarBytes = 256;
constexpr uint32_t kFaXchBytes = 2 * 128 * 4;            // [2 halves][128 rows] f32 exchange
// the dynamic shared-memory base is declared 1024-aligned (checked at run time)
constexpr size_t kFaSmem = kFaQBytes + 4 * kFaKVBytes + 2 * kFaPBytes + kFaBarBytes + kFaXchBytes;
constexpr int kFaThreads = 320;
constexpr float kFaRescaleLog2 = 8.0f;                   // lazy-rescale threshold (factor 256)

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

__device__ __forceinline__ void fa_store_o32(__half* dst, const uint32_t (&o)[32], float inv) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    d4[q] = make_uint4(pack_f16(u2f(o[8 * q]) * inv, u2f(o[8 * q + 1]) * inv),
                       pack_f16(u2f(o[8 * q + 2]) * inv, u2f(o[8 * q + 3]) * inv),
                       pack_f16(u2f(o[8 * q + 4]) * inv, u2f(o[8 * q + 5]) * inv),
                       pack_f16(u2f(o[8 * q + 6]) * inv, u2f(o[8 * q + 7]) * inv));
}

__global__ void __launch_bounds__(kFaThreads, 1)
    flash_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                         const FaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the swizzled operand tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kFaQBytes;            // [2][4][64 x 128 B]
  uint8_t* sV = sK + 2 * kFaKVBytes;       // [2][4][64 x 128 B]
  uint8_t* sP = sV + 2 * kFaKVBytes;       // [2][128 x 128 B]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + 2 * kFaPBytes);
  uint64_t* q_full = bar;
  uint64_t* q_empty = bar + 1;   // Q buffer free once the item's last S is computed
  uint64_t* k_full = bar + 2;    // [2]
  uint64_t* k_empty = bar + 4;   // [2]  K stage free once S_j is computed
  uint64_t* v_full = bar + 6;    // [2]
  uint64_t* v_empty = bar + 8;   // [2]  V stage free once P_j V_j is computed
  uint64_t* s_full = bar + 10;   // [2]
  uint64_t* p_full = bar + 12;   // [2]
  uint64_t* pv_done = bar + 14;  // [2]
  uint64_t* o_free = bar + 16;   // O drained by the epilogue warps
  uint64_t* drain = bar + 17;
  uint64_t* xbar = bar + 18;     // [4] per-quadrant rendezvous of the two softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bar) + kFaBarBytes);  // [2][128]

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
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 2);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
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
      // ------------------------------------------------------------------ producer
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
          if (!mbar_wait(&v_empty[st], ph, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], kFaKVBytes);
          for (int c = 0; c < 4; ++c)
            tma_load_2d(sV + st * kFaKVBytes + c * kFaKVChunk, &tmKV, &v_full[st], w.vcol + 64 * c, row);
        }
        ++it;
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
          const uint64_t qd = desc_kmajor_sw128(smem_u32(sQ + c * (kFaBQ * 128)));
          const uint64_t kd = desc_kmajor_sw128(smem_u32(sK + st * kFaKVBytes + c * kFaKVChunk));
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16_ss(d, qd + 2 * k, kd + 2 * k, idesc_s, (c | k) != 0 ? 1u : 0u);
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
        if (!mbar_wait(q_full, it & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (!issue_s(g)) {
          ok = false;
          break;
        }
        issued = true;
        for (int j = 0; j < w.n_tiles; ++j) {
          const uint32_t gj = g + j;
          const int st = gj & 1;
          if (j + 1 < w.n_tiles) {
            if (!issue_s(gj + 1)) {
              ok = false;
              break;
            }
          } else {
            umma_commit(q_empty);  // every S of this item has been issued
          }
          if (!mbar_wait(&p_full[st], (gj >> 1) & 1, abort_flag) ||
              !mbar_wait(&v_full[st], (gj >> 1) & 1, abort_flag) ||
              (j == 0 && it >= 1 && !mbar_wait(o_free, (it - 1) & 1, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t pd = desc_kmajor_sw128(smem_u32(sP + st * kFaPBytes));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // V rows k*16..k*16+15 of this stage: 16 keys x 128 B further per K step
            const uint64_t vd =
                desc_mnmajor_sw128(smem_u32(sV + st * kFaKVBytes + k * 16 * 128), kFaKVChunk, 1024);
            umma_f16_ss(tmem + 256, pd + 2 * k, vd, idesc_pv, (j | k) != 0 ? 1u : 0u);
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
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // which 32 key columns of S / 128 columns of O
    const int r = quad * 32 + lane;    // query row inside the tile == TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr float kLog2e = 1.4426950408889634f;
    // exchange a per-row value with the partner warp (two rendezvous: the buffer is
    // reusable as soon as the call returns); false on timeout / abort
    uint32_t xph = 0;
    auto exchange = [&](float v, float* other) -> bool {
      xch[half * 128 + r] = v;
      if (!pair_rendezvous(&xbar[quad], xph, abort_flag)) return false;
      *other = xch[(half ^ 1) * 128 + r];
      return pair_rendezvous(&xbar[quad], xph, abort_flag);
    };
    uint32_t g = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
      const FaItem w = fa_item(p, item);
      if (!w.valid) continue;
      const int i = w.q0 + r;  // position inside the sequence
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < w.n_tiles; ++j) {
        const uint32_t gj = g + j;
        const int st = gj & 1;
        bool wt = mbar_wait(&s_full[st], (gj >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, wt)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[32];
        tmem_ld32(lane_base + st * kFaBKV + half * 32, sr);
        tmem_ld_wait_tied(sr);
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
        float mx[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) mx[q] = fmaxf(fmaxf(sv[4 * q], sv[4 * q + 1]), fmaxf(sv[4 * q + 2], sv[4 * q + 3]));
        float tmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        float tmax_other;
        if (!exchange(tmax, &tmax_other)) {
          ok = false;
          break;
        }
        tmax = fmaxf(tmax, tmax_other) * kLog2e;  // row max over all 64 keys, log2 domain
        float factor = 1.0f;
        if (m_ref == -INFINITY) {
          m_ref = tmax;
        } else if (tmax > m_ref + kFaRescaleLog2) {
          factor = fast_exp2(m_ref - tmax);
          m_ref = tmax;
        }
        const float mu = m_ref == -INFINITY ? 0.f : m_ref;
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = fast_exp2(fmaf(sv[2 * e], kLog2e, -mu));
          const float c = fast_exp2(fmaf(sv[2 * e + 1], kLog2e, -mu));
          rs[e & 3] += a + c;
          pk[e] = pack_f16(a, c);
        }
        l = l * factor + ((rs[0] + rs[1]) + (rs[2] + rs[3]));  // this half's partial row sum
        // O may be rescaled only after P_{j-1} V_{j-1} has landed; P buffer (g % 2) is free once
        // P_{j-2} V_{j-2} has (for j < 2 the previous item's drain already waited for it).
        // Both warps of a pair take the same branch (same rows, same factors).
        if (j >= 1 && __any_sync(0xffffffffu, factor != 1.0f)) {
          wt = mbar_wait(&pv_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, wt)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            const uint32_t ta = lane_base + 256 + half * 128 + c * 32;
            tmem_ld32(ta, o);
            tmem_ld_wait_tied(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(u2f(o[e]) * factor);
            tmem_st32(ta, o);
          }
          tmem_st_wait();
        } else if (j >= 2) {
          wt = mbar_wait(&pv_done[gj & 1], ((gj - 2) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, wt)) {
            ok = false;
            break;
          }
        }
        // P row r, this half's 4 chunks of 8 keys, 128B-swizzled (chunk ^ (row & 7))
        uint8_t* prow = sP + st * kFaPBytes + r * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int chunk = half * 4 + c;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[st]);
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
      float l_other;
      if (!exchange(l, &l_other)) {
        ok = false;
        break;
      }
      const float lt = l + l_other;
      const float inv = lt > 0.f ? 1.0f / lt : 0.f;
      const bool live = i < w.len;
      __half* dst = p.out + static_cast<size_t>(w.tok0 + i) * p.ld_out + w.qcol + half * 128;
      const uint32_t ob_base = lane_base + 256 + half * 128;
      uint32_t oa[32], ob[32];
      tmem_ld32(ob_base, oa);
      tmem_ld_wait_tied(oa);
#pragma unroll 1
      for (int c = 0; c < 4; c += 2) {
        tmem_ld32(ob_base + (c + 1) * 32, ob);
        if (live) fa_store_o32(dst + c * 32, oa, inv);
        tmem_ld_wait_tied(ob);
        if (c + 2 < 4) tmem_ld32(ob_base + (c + 2) * 32, oa);
        if (live) fa_store_o32(dst + (c + 1) * 32, ob, inv);
        if (c + 2 < 4) tmem_ld_wait_tied(oa);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      g += w.n_tiles;
    }
    if (!ok && lane == 0) {
      if (!*abort_flag) record_error(p.status, kErrTimeoutEpilogue);
      *abort_flag = 1;
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
