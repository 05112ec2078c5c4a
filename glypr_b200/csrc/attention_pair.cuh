// Bidirectional GQA flash attention, head_dim 256, on CTA pairs (tcgen05.mma.cta_group::2).
//
// Semantics as flash_attn_tc_kernel (scale 1.0, standard.rs:62; key j visible iff j < len and,
// with a window, |i - j| <= W, model.rs:634-638; f32 softmax; query head h reads KV head
// h / (Hq / Hkv), attention/mod.rs:22-31).
//
// Why pairs: with one CTA per 128-query block the S = Q K^T MMAs are M=128, N=64 and issue at
// about 30 % of the tensor rate, and 128-key tiles do not fit one CTA (double-buffered 128-key K
// and V tiles alone are 256 KB).  A pair owns 256 queries of one (sequence, head): every MMA is
// M=256, each CTA holds half of every K tile (64 of its 128 keys) and half of every V tile (128
// of its 256 dims), so S tiles of 128 keys fit: S_j = Q K_j^T is M=256, N=128, K=256
// (16 MMAs, both operands in shared memory) and O += P_j V_j is M=256, N=256, K=128 (8 MMAs, P
// from tensor memory, V MN-major).
//
// Per CTA (480 threads): shared memory Q 128 rows x 256 dims (64 KB), a ring of four 32 KB
// operand slots that the MMAs consume in issue order (K_0, then per tile j K_{j+1} when there is
// one, and V_j; a K slot is 64 keys x 256 dims, a V slot 128 keys x 128 dims), and 16 KB of
// output staging.  Tensor memory: S[0] 0-127, S[1] 128-255 (P_j as f16 pairs in the first 64
// columns of its slot), O 256-511 (this CTA's 128 rows).
//   warp 0     TMA producer of the K / V ring (pair loads completing on the leader's barriers)
//   warp 10    TMA producer of Q: the next item's Q loads as soon as the item's last S completes
//              (L2 prefetches of the next item's Q and first K / V tiles measured 2.5 % slower:
//              they added a quarter to the DRAM reads and did not shorten the loads)
//   warp 1     leader: MMA issuer (one multicast commit reaches both CTAs' barriers); peer: idle
//   warps 2-9  softmax for this CTA's 128 rows: the two warps of a lane quadrant take 64 of the
//              128 keys of a tile (and 128 of the 256 O columns when rescaling), exchange row
//              maxima, rescale O lazily (the reference moves only past 2^12), write P over
//              their slot, and at the end of an item hand 1/l of each row to the drain warps
//   warps 11-14 drain: one per lane quadrant, O of the finished item to global memory while the
//              softmax warps start the next item
// The leader's MMA learns that P_j (or a drained O) is ready from its own warps' arrivals and
// from one 4-byte st.async token per peer warp counted on the same barrier (a remote
// mbarrier.arrive.release.cluster per warp and tile would stall the peer's warps).  It waits on
// those barriers with the plain (CTA-scope) try_wait, as CUTLASS's pair GEMMs do for barriers
// their peer arrives on.
#pragma once
#include "attention_tc.cuh"

namespace glp {

constexpr int kFpBQ = 128;                         // query rows per CTA (256 per pair)
constexpr int kFpBKV = 128;                        // keys per tile (64 per CTA for K)
constexpr uint32_t kFpQChunk = 128 * 128;          // 16 KB: 128 rows x 64 dims
constexpr uint32_t kFpQBytes = 4 * kFpQChunk;      // 64 KB
constexpr uint32_t kFpKChunk = 64 * 128;           // 8 KB: 64 keys x 64 dims
constexpr uint32_t kFpKBytes = 4 * kFpKChunk;      // 32 KB: this CTA's 64 keys x 256 dims
constexpr uint32_t kFpVChunk = 128 * 128;          // 16 KB: 128 keys x 64 dims
constexpr uint32_t kFpVBytes = 2 * kFpVChunk;      // 32 KB: 128 keys x this CTA's 128 dims
constexpr uint32_t kFpSlotBytes = 32768;           // one ring slot: a K or a V tile half
// 2^x pairs of a softmax round taken by the FMA-pipe polynomial instead of MUFU ex2: none.  The
// one-CTA kernel's split (6 of 16) measured 3 % slower here (0.424 vs 0.412 ms on 512 x
// 512-token sequences; 4 of 16: 0.419, 8: 0.432) -- these softmax warps are bound by issue
// slots, not by the special-function unit.
constexpr uint32_t kFpPolyPairs = 0;
constexpr int kFpSlots = 4;
constexpr uint32_t kFpStageBytes = 4 * 4096;       // output staging: 32 rows x 128 B per drain warp
constexpr int kFpThreads = 480;                    // 15 warps (roles below)
static_assert(kFpKBytes == kFpSlotBytes && kFpVBytes == kFpSlotBytes, "K and V tile halves share the ring");
constexpr uint32_t kFpBarBytes = 512;              // barriers, then the token slots
constexpr uint32_t kFpXchBytes = 2 * 2 * 128 * 4 + 2 * 128 * 4;  // row maxima / sums, then 1/l per row [2][128]
constexpr size_t kFpSmem = kFpQBytes + kFpSlots * kFpSlotBytes + kFpStageBytes + kFpBarBytes + kFpXchBytes;
static_assert(kFpSmem <= 232448, "shared memory per CTA");
constexpr uint32_t kFpTmemO = 256;

struct FpItem {
  bool valid;
  int tok0, len, qp0, q0, qcol, kcol, vcol, t_lo, n_tiles;
};

// p.q_blocks counts 256-query pair blocks here.  An item's two cu_seqlens entries are loaded
// one item ahead (fp_bounds) and only used the next time round (fp_item): anything computed
// from a load right after issuing it would stall the role for the load's ~1k cycles at every
// item boundary.
__device__ __forceinline__ void fp_bounds(const FaParams& p, int item, int& s0, int& s1) {
  const int b = item / (p.q_blocks * p.n_q_heads);
  s0 = __ldg(p.cu_seqlens + b);
  s1 = __ldg(p.cu_seqlens + b + 1);
}

__device__ __forceinline__ FpItem fp_item(const FaParams& p, int item, uint32_t rank, int seq0, int seq1) {
  FpItem w;
  const int per_seq = p.q_blocks * p.n_q_heads;
  const int b = item / per_seq;
  const int r = item - b * per_seq;
  const int pb = r / p.n_q_heads;
  const int head = r - pb * p.n_q_heads;
  w.tok0 = seq0 - p.cu_base;
  w.len = seq1 - seq0;
  w.qp0 = pb * 2 * kFpBQ;
  w.q0 = w.qp0 + static_cast<int>(rank) * kFpBQ;
  w.valid = w.qp0 < w.len;  // the same for both CTAs of the pair
  const int kvh = head / (p.n_q_heads / p.n_kv_heads);
  w.qcol = head * kFaD;
  w.kcol = (p.n_q_heads + kvh) * kFaD;
  w.vcol = (p.n_q_heads + p.n_kv_heads + kvh) * kFaD;
  int kv_lo = 0, kv_hi = w.len;
  if (p.window > 0) {
    kv_lo = max(0, w.qp0 - p.window);
    kv_hi = min(w.len, w.qp0 + 2 * kFpBQ + p.window);
  }
  w.t_lo = kv_lo / kFpBKV;
  w.n_tiles = (kv_hi + kFpBKV - 1) / kFpBKV - w.t_lo;
  return w;
}

// tmQV: qkv with 64 x 128 boxes (Q rows and V keys), tmK: qkv with 64 x 64 boxes (K keys).
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kFpThreads, 1)
    flash_attn_pair_kernel(const __grid_constant__ CUtensorMap tmQV, const __grid_constant__ CUtensorMap tmK,
                           const FaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // the same in both CTAs: both leave before any cluster step
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* sQ = smem_raw;
  uint8_t* sRing = sQ + kFpQBytes;  // [5] K slot: [4][64 x 128 B]; V slot: [2][128 x 128 B]
  uint8_t* sStage = sRing + kFpSlots * kFpSlotBytes;  // [8 warps][32 x 128 B]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sStage + kFpStageBytes);
  uint64_t* q_full = bar;            // leader: both CTAs' Q
  uint64_t* q_empty = bar + 1;       // Q buffer free (the item's last S has completed)
  uint64_t* ring_full = bar + 2;     // [4] leader: both CTAs' halves of the slot
  uint64_t* ring_empty = bar + 6;    // [4]
  uint64_t* s_full = bar + 10;       // [2]
  uint64_t* p_full = bar + 12;       // [2] leader: 8 local arrivals + 8 peer tokens
  uint64_t* pv_done = bar + 14;      // [2]
  uint64_t* o_free = bar + 16;       // leader: O drained in both CTAs (8 local + 8 peer tokens)
  uint64_t* drain = bar + 17;
  uint64_t* xbar = bar + 18;         // [4]
  uint64_t* l_ready = bar + 22;      // [2] per item parity: 1/l of every row written (4 softmax warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* tokens = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(bar) + 256);  // [3][8]: p[0], p[1], o
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bar) + kFpBarBytes);  // [2][2][128]
  float* inv_l = xch + 2 * 2 * 128;  // [2][128]: 1 / l per row, by item parity

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id_x());
  const int n_pairs = static_cast<int>(n_clusters_x());
  const int n_items = p.n_seq * p.q_blocks * p.n_q_heads;
  // each pair takes a contiguous run of items: the (query block, head) items of a sequence
  // follow one another, so its K / V tiles come from HBM for the first of them and from L2
  // for the rest (with items dealt round-robin, six pairs fetched the same tiles at once and
  // every one of them waited on HBM)
  const int item_lo = static_cast<int>(static_cast<int64_t>(pair) * n_items / n_pairs);
  const int item_hi = static_cast<int>(static_cast<int64_t>(pair + 1) * n_items / n_pairs);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < kFpSlots; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(o_free, 4);
    mbar_init(&l_ready[0], 4);
    mbar_init(&l_ready[1], 4);
    mbar_init(drain, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 2);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQV);
    tma_prefetch_desc(&tmK);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ K / V ring producer
      // slot order per item: K_0, then per tile j: K_{j+1} (if any), V_j -- the MMA order
      uint32_t r = 0;
      bool ok = true;
      auto fill = [&](bool is_k, const FpItem& w, int j) -> bool {
        const int slot = static_cast<int>(r % kFpSlots);
        if (!mbar_wait(&ring_empty[slot], ((r / kFpSlots) & 1) ^ 1, abort_flag)) return false;
        if (leader) mbar_arrive_expect_tx(&ring_full[slot], 2 * kFpSlotBytes);
        const uint32_t fb = mapa_shared(smem_u32(&ring_full[slot]), 0);
        uint8_t* dst = sRing + slot * kFpSlotBytes;
        const int key0 = w.tok0 + (w.t_lo + j) * kFpBKV;
        if (is_k) {
          for (int c = 0; c < 4; ++c)
            tma_load_2d_pair(dst + c * kFpKChunk, &tmK, fb, w.kcol + 64 * c, key0 + static_cast<int>(rank) * 64);
        } else {
          for (int c = 0; c < 2; ++c)
            tma_load_2d_pair(dst + c * kFpVChunk, &tmQV, fb, w.vcol + static_cast<int>(rank) * 128 + 64 * c, key0);
        }
        ++r;
        return true;
      };
      int nb0, nb1;
      if (item_lo < item_hi) fp_bounds(p, item_lo, nb0, nb1);
      for (int item = item_lo; ok && item < item_hi; ++item) {
        const FpItem w = fp_item(p, item, rank, nb0, nb1);
        if (item + 1 < item_hi) fp_bounds(p, item + 1, nb0, nb1);  // in flight during this item
        if (!w.valid) continue;
        ok = fill(true, w, 0);
        for (int j = 0; ok && j < w.n_tiles; ++j) {
          if (j + 1 < w.n_tiles) ok = fill(true, w, j + 1);
          if (ok) ok = fill(false, w, j);
        }
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutProducer);
        *abort_flag = 1;
      }
    }
  } else if (warp == 10) {
    if (lane == 0) {
      // ------------------------------------------------------------------ Q producer
      int it = 0;
      bool ok = true;
      int nb0, nb1;
      if (item_lo < item_hi) fp_bounds(p, item_lo, nb0, nb1);
      for (int item = item_lo; ok && item < item_hi; ++item) {
        const FpItem w = fp_item(p, item, rank, nb0, nb1);
        if (item + 1 < item_hi) fp_bounds(p, item + 1, nb0, nb1);  // in flight during this item
        if (!w.valid) continue;
        if (!mbar_wait(q_empty, (it & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        if (leader) mbar_arrive_expect_tx(q_full, 2 * kFpQBytes);
        const uint32_t qbar = mapa_shared(smem_u32(q_full), 0);
        for (int c = 0; c < 4; ++c) tma_load_2d_pair(sQ + c * kFpQChunk, &tmQV, qbar, w.qcol + 64 * c, w.tok0 + w.q0);
        ++it;
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutProducer);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------------ MMA issuer (leader)
      constexpr uint32_t idesc_s = idesc_f16(256, kFpBKV, 0);
      constexpr uint32_t idesc_pv = idesc_f16(256, kFaD, 0) | (1u << 16);  // B (V) MN-major
      auto commit_both = [&](uint64_t* b) { umma_commit_pair_both(smem_u32(b)); };
      uint32_t r = 0;  // ring position, in step with the producer
      auto take_slot = [&](int* slot) -> bool {
        *slot = static_cast<int>(r % kFpSlots);
        if (!mbar_wait(&ring_full[*slot], (r / kFpSlots) & 1, abort_flag)) return false;
        ++r;
        return true;
      };
      // S_gx = Q K^T into S slot gx & 1; `mid` runs after the first 8 of the 16 MMAs
      auto issue_s = [&](uint32_t gx, int slot, auto&& mid) {
        const uint32_t d = tmem + static_cast<uint32_t>((gx & 1) * kFpBKV);
        uint8_t* sK = sRing + slot * kFpSlotBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint64_t qd = desc_kmajor_sw128(smem_u32(sQ + c * kFpQChunk));
          const uint64_t kd = desc_kmajor_sw128(smem_u32(sK + c * kFpKChunk));
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16_pair(d, qd + 2 * k, kd + 2 * k, idesc_s, (c | k) != 0 ? 1u : 0u);
          if (c == 1) mid();
        }
      };
      // Per item: S_0 and S_1, then per tile j one run of MMAs: PV_j, S_{j+2} (into P_j's slot,
      // which PV_j has read by then: the pipe runs in order).  Only a few MMAs queue ahead of
      // the pipe, so this thread keeps pace with it, and a wait after a run -- even on a phase
      // that completed long ago costs ~200 cycles -- leaves the pipe idle.  So in the middle
      // of each run the thread probes (test_wait, non-blocking) the barriers the next run
      // needs; when all have completed, the run after it starts without waiting.
      int it = 0;
      uint32_t g = 0;
      bool ok = true;
      bool issued = false;
      int nb0, nb1;
      if (item_lo < item_hi) fp_bounds(p, item_lo, nb0, nb1);
      for (int item = item_lo; ok && item < item_hi; ++item) {
        const FpItem w = fp_item(p, item, rank, nb0, nb1);
        if (item + 1 < item_hi) fp_bounds(p, item + 1, nb0, nb1);  // in flight during this item
        if (!w.valid) continue;
        const int n = w.n_tiles;
        int ks0, ks1 = -1;
        if (!mbar_wait(q_full, it & 1, abort_flag) || !take_slot(&ks0) || (n > 1 && !take_slot(&ks1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        issued = true;
        auto nothing = [] {};
        issue_s(g, ks0, nothing);
        commit_both(&s_full[g & 1]);
        if (n > 1) {
          issue_s(g + 1, ks1, nothing);
          commit_both(&s_full[(g + 1) & 1]);
        }
        if (n <= 2) commit_both(q_empty);  // every S of this item issued: Q is free once they complete
        commit_both(&ring_empty[ks0]);
        if (n > 1) commit_both(&ring_empty[ks1]);
        bool ready = false;  // tile j's barriers found complete by the probe in the previous run
        for (int j = 0; j < n; ++j) {
          const uint32_t gj = g + j;
          const int st = gj & 1;
          int vslot, kslot = -1;
          if (ready) {
            vslot = static_cast<int>(r++ % kFpSlots);
            if (j + 2 < n) kslot = static_cast<int>(r++ % kFpSlots);
          } else if (!take_slot(&vslot) || (j + 2 < n && !take_slot(&kslot)) ||
                     !mbar_wait(&p_full[st], (gj >> 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          if (j == 0 && it >= 1 && !mbar_wait(o_free, (it - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // the probe for tile j + 1: its V slot, its K slot (S_{j+3}) and P_{j+1}
          ready = false;
          auto probe = [&] {
            if (j + 1 >= n) return;
            const uint32_t gn = gj + 1;
            ready = mbar_test_wait(&ring_full[r % kFpSlots], (r / kFpSlots) & 1) &&
                    (j + 3 >= n ||
                     mbar_test_wait(&ring_full[(r + 1) % kFpSlots], ((r + 1) / kFpSlots) & 1)) &&
                    mbar_test_wait(&p_full[gn & 1], (gn >> 1) & 1);
          };
          uint8_t* sV = sRing + vslot * kFpSlotBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k) {  // 16 keys per step: 16 rows of 128 B in V, 8 TMEM columns of P
            const uint64_t vd = desc_mnmajor_sw128(smem_u32(sV + k * 16 * 128), kFpVChunk, 1024);
            umma_f16_pair_ts(tmem + kFpTmemO, tmem + st * kFpBKV + k * 8, vd, idesc_pv, (j | k) != 0 ? 1u : 0u);
            if (k == 4 && kslot < 0) probe();
          }
          commit_both(&pv_done[st]);
          commit_both(&ring_empty[vslot]);  // released when PV_j completes: its refill starts a run earlier
          if (kslot >= 0) {
            issue_s(gj + 2, kslot, probe);
            commit_both(&s_full[st]);
            if (j + 3 == n) commit_both(q_empty);
            commit_both(&ring_empty[kslot]);
          }
          if (ready) tc_fence_after();
        }
        g += n;
        ++it;
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutMma);
        *abort_flag = 1;
      }
      if (issued) {
        umma_commit_pair(smem_u32(drain));
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < GLP_WAIT_TIMEOUT_NS) {
        }
      }
    }
  } else if (warp >= 2 && warp <= 9) {
    // -------------------------------------------------------------------- softmax + output
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // keys 64 half.. of a tile; O columns 128 half..
    const int ew = warp - 2;
    const int r = quad * 32 + lane;    // query row inside this CTA's 128 == TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr float kLog2e = 1.4426950408889634f;
    // readiness for the leader's MMA: local arrival there, a 4-byte token from the peer
    const uint32_t lead_p0 = mapa_shared(smem_u32(&p_full[0]), 0);
    const uint32_t tok0 = mapa_shared(smem_u32(tokens), 0) + static_cast<uint32_t>(ew) * 4u;
    auto signal = [&](uint64_t* local_bar, uint32_t lead_bar, uint32_t slot) {
      if (lane != 0) return;
      if (leader)
        mbar_arrive_expect_tx(local_bar, 4);
      else
        st_async_b32(tok0 + slot * 32u, 1u, lead_bar);
    };
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
    uint32_t g = 0;
    int it = 0;
    bool ok = true;
    uint32_t sa[32], sb[32];
    int nb0, nb1;
    if (item_lo < item_hi) fp_bounds(p, item_lo, nb0, nb1);
    for (int item = item_lo; ok && item < item_hi; ++item) {
      const FpItem w = fp_item(p, item, rank, nb0, nb1);
      if (item + 1 < item_hi) fp_bounds(p, item + 1, nb0, nb1);  // in flight during this item
      if (!w.valid) continue;
      const int i = w.q0 + r;
      float m_ref = -INFINITY, l = 0.f;
      {
        const int st = g & 1;
        const bool wt = mbar_wait(&s_full[st], (g >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, wt)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_ld32(lane_base + st * kFpBKV + half * 64, sa);
        tmem_ld32(lane_base + st * kFpBKV + half * 64 + 32, sb);
        tmem_ld_wait_tied(sa);
        tmem_ld_wait_tied(sb);
      }
      for (int j = 0; j < w.n_tiles; ++j) {
        const uint32_t gj = g + j;
        const int st = gj & 1;
        const int kt = (w.t_lo + j) * kFpBKV;
        const int kb = kt + half * 64;  // first key of this warp's 64
        const bool full_tile =
            kt + kFpBKV <= w.len &&
            (p.window <= 0 || (kt >= w.q0 + kFpBQ - 1 - p.window && kt + kFpBKV - 1 <= w.q0 + p.window));
        // masked keys become -inf in place (sa: keys kb .. kb + 31, sb: kb + 32 .. kb + 63)
        if (!full_tile) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int ka = kb + e, kc = kb + 32 + e;
            const bool va = ka < w.len && (p.window <= 0 || abs(i - ka) <= p.window);
            const bool vc = kc < w.len && (p.window <= 0 || abs(i - kc) <= p.window);
            sa[e] = va ? sa[e] : 0xff800000u;
            sb[e] = vc ? sb[e] : 0xff800000u;
          }
        }
        float mine;
        {
          float m[22];
#pragma unroll
          for (int k = 0; k < 10; ++k) {
            m[k] = fmax3(u2f(sa[3 * k]), u2f(sa[3 * k + 1]), u2f(sa[3 * k + 2]));
            m[11 + k] = fmax3(u2f(sb[3 * k]), u2f(sb[3 * k + 1]), u2f(sb[3 * k + 2]));
          }
          m[10] = fmaxf(u2f(sa[30]), u2f(sa[31]));
          m[21] = fmaxf(u2f(sb[30]), u2f(sb[31]));
          float t[8];
#pragma unroll
          for (int k = 0; k < 7; ++k) t[k] = fmax3(m[3 * k], m[3 * k + 1], m[3 * k + 2]);
          t[7] = m[21];
          mine = fmax3(fmax3(t[0], t[1], t[2]), fmax3(t[3], t[4], t[5]), fmaxf(t[6], t[7])) * kLog2e;
        }
        publish(mine);
        float other;
        if (!collect(&other)) {
          ok = false;
          break;
        }
        const float joint = fmaxf(mine, other);
        const float m_new = joint > m_ref + kFaRescaleLog2 ? joint : m_ref;
        const float factor = (m_ref == -INFINITY || m_new == m_ref) ? 1.f : fast_exp2(m_ref - m_new);
        // exponentials against the final reference directly.  The speculative form (against
        // this warp's own choice while the partner's maximum is in flight, scaled afterwards
        // where the joint choice differs) measured 10 % slower here: 0.60 vs 0.55 ms per
        // 262,144-token launch, the values held in f32 across the exchange and packed after it
        const float mref = m_new == -INFINITY ? 0.f : m_new;
        m_ref = m_new;
        // P row r, this warp's 64 keys in two rounds of 32: 16 columns of f16 pairs each, over
        // the first 64 columns of the S slot
        const uint64_t l2e = f2(kLog2e, kLog2e), nmu = f2(-mref, -mref);
        float lsum = 0.f;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t pk[16];
          uint64_t acc[2] = {0ull, 0ull};
          const uint32_t(&sx)[32] = h2 == 0 ? sa : sb;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const uint64_t x = f2_fma(f2(u2f(sx[2 * e]), u2f(sx[2 * e + 1])), l2e, nmu);
            uint64_t ev;
            if ((kFpPolyPairs >> e) & 1u) {
              ev = exp2_poly_pair(x);
            } else {
              float a, b;
              f2_split(x, a, b);
              ev = f2(fast_exp2(a), fast_exp2(b));
            }
            float a, b;
            f2_split(ev, a, b);
            pk[e] = pack_f16(a, b);
            acc[e & 1] = f2_add(acc[e & 1], ev);
          }
          float s0, s1;
          f2_split(f2_add(acc[0], acc[1]), s0, s1);
          lsum += s0 + s1;
          tmem_st16(lane_base + st * kFpBKV + half * 32 + h2 * 16, pk);
        }
        l = l * factor + lsum;
        // O may be rescaled only after P_{j-1} V_{j-1} has landed.  Done after the exponentials:
        // PV_{j-1} has mostly finished by then, where waiting for it first stalled this warp
        // ~1k cycles on most tiles when logits are spread wide (some row of the 32 almost always
        // moves its maximum past the lazy threshold)
        if (j >= 1 && __any_sync(0xffffffffu, factor != 1.0f)) {
          const bool wt = mbar_wait(&pv_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, wt)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t f2x = f2(factor, factor);
          // 128 columns as two loads of 64 in flight together (sa / sb are free by now)
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            const uint32_t ta = lane_base + kFpTmemO + half * 128 + c * 64;
            tmem_ld32(ta, sa);
            tmem_ld32(ta + 32, sb);
            tmem_ld_wait_tied(sa);
            tmem_ld_wait_tied(sb);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float a, b;
              f2_split(f2_mul(f2(u2f(sa[e]), u2f(sa[e + 1])), f2x), a, b);
              sa[e] = __float_as_uint(a);
              sa[e + 1] = __float_as_uint(b);
              f2_split(f2_mul(f2(u2f(sb[e]), u2f(sb[e + 1])), f2x), a, b);
              sb[e] = __float_as_uint(a);
              sb[e + 1] = __float_as_uint(b);
            }
            tmem_st32(ta, sa);
            tmem_st32(ta + 32, sb);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        signal(&p_full[st], lead_p0 + static_cast<uint32_t>(st * sizeof(uint64_t)), static_cast<uint32_t>(st));
        if (j + 1 < w.n_tiles) {
          const uint32_t gn = gj + 1;
          const bool wt = mbar_wait(&s_full[gn & 1], (gn >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, wt)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_ld32(lane_base + (gn & 1) * kFpBKV + half * 64, sa);
          tmem_ld32(lane_base + (gn & 1) * kFpBKV + half * 64 + 32, sb);
          tmem_ld_wait_tied(sa);
          tmem_ld_wait_tied(sb);
        }
      }
      if (!ok) break;
      // ---- the row sums to the drain warps (they store O once PV of the last tile lands);
      // this warp goes straight on to the next item's S_0
      publish(l);
      float l_other;
      if (!collect(&l_other)) {
        ok = false;
        break;
      }
      if (half == 0) {
        const float lt = l + l_other;
        inv_l[(it & 1) * 128 + r] = lt > 0.f ? 1.0f / lt : 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&l_ready[it & 1]);
      }
      g += w.n_tiles;
      ++it;
    }
    if (lane == 0 && !ok) {
      if (!*abort_flag) record_error(p.status, kErrTimeoutEpilogue);
      *abort_flag = 1;
    }
  } else if (warp >= 11 && warp <= 14) {
    // -------------------------------------------------------------------- drain of O
    // Warp (quad q) stores rows 32q.. of this CTA's 128: all 256 columns, 64 at a time, staged
    // (swizzled) in shared memory and written as 4 rows x 128 contiguous bytes per store.  The
    // SM writes to L2 at ~32 B/cycle, so the 64 KB of O per item take ~2k cycles: off the
    // softmax warps, they overlap the next item's S_0, S_1 and first softmax.  O's tensor memory
    // is released (o_free) once its last columns are in registers.
    const int quad = warp & 3;
    const int dw = warp - 11;
    const int r = quad * 32 + lane;
    const uint32_t ob_base = tmem + (static_cast<uint32_t>(quad * 32) << 16) + kFpTmemO;
    const uint32_t lead_o = mapa_shared(smem_u32(o_free), 0);
    const uint32_t tok = mapa_shared(smem_u32(tokens), 0) + 2u * 32u + static_cast<uint32_t>(dw) * 4u;
    uint8_t* stage = sStage + dw * 4096;
    uint32_t g = 0;
    int it = 0;
    bool ok = true;
    int nb0, nb1;
    if (item_lo < item_hi) fp_bounds(p, item_lo, nb0, nb1);
    for (int item = item_lo; ok && item < item_hi; ++item) {
      const FpItem w = fp_item(p, item, rank, nb0, nb1);
      if (item + 1 < item_hi) fp_bounds(p, item + 1, nb0, nb1);  // in flight during this item
      if (!w.valid) continue;
      const uint32_t gl = g + w.n_tiles - 1;
      const bool wt = mbar_wait(&l_ready[it & 1], (it >> 1) & 1, abort_flag) &&
                      mbar_wait(&pv_done[gl & 1], (gl >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, wt)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = inv_l[(it & 1) * 128 + r];
      const uint64_t inv2 = f2(inv, inv);
      const int row0 = w.q0 + quad * 32;
      const int rows = min(32, w.len - row0);  // rows of this warp inside the sequence
#pragma unroll 1
      for (int k = 0; k < 4; ++k) {  // four slices of 64 output columns
        uint32_t oa[32], ob[32];
        tmem_ld32(ob_base + k * 64, oa);
        tmem_ld32(ob_base + k * 64 + 32, ob);
        tmem_ld_wait_tied(oa);
        tmem_ld_wait_tied(ob);
        if (k == 3) {  // all of O read: the next item's PV may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              mbar_arrive_expect_tx(o_free, 4);
            else
              st_async_b32(tok, 1u, lead_o);
          }
        }
        if (rows <= 0) continue;  // every row of this warp lies past the sequence
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
        __syncwarp();
        const int col = w.qcol + k * 64 + (lane & 7) * 8;
#pragma unroll
        for (int rr = 0; rr < 32; rr += 4) {
          const int row = rr + (lane >> 3), c = lane & 7;
          const uint4 v = *reinterpret_cast<const uint4*>(stage + row * 128 + ((c ^ (row & 7)) << 4));
          if (row < rows) *reinterpret_cast<uint4*>(p.out + static_cast<size_t>(w.tok0 + row0 + row) * p.ld_out + col) = v;
        }
        __syncwarp();
      }
      g += w.n_tiles;
      ++it;
    }
    if (lane == 0 && !ok) {
      if (!*abort_flag) record_error(p.status, kErrTimeoutEpilogue);
      *abort_flag = 1;
    }
  }

  // neither CTA leaves (or frees tensor memory) while the other may still touch its shared
  // memory, barriers or tensor memory
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace glp
