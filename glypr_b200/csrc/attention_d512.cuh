// Bidirectional GQA flash attention for head_dim 512 (the global layers of EmbeddingGemma 2:
// config.rs:141-160 per-layer key_length, model.rs:279 global RoPE width 512), on tcgen05.
//
// Semantics as flash_attn_tc_kernel (scale 1.0, standard.rs:62; key j visible iff j < len and,
// with a window, |i - j| <= W, model.rs:634-638; f32 softmax; query head h reads KV head
// h / (Hq / Hkv)).  What changes with 512-wide heads is the budget: a 128 x 512 f32 O would need
// all 512 tensor-memory columns, so a work item is (sequence, 128-query block, head, O half):
// the two CTAs of a (block, head) each compute the full S = Q K^T over 512 dims and one
// 256-column half of O = P V.
//
// Per CTA (352 threads, one per SM, persistent over items):
//   shared memory  Q 128 rows x 512 dims (8 swizzled chunks of 64 dims, 128 KB; after the
//                  item's last S it doubles as the output staging), K tiles of 32 keys x 512
//                  dims (2 stages x 32 KB), V tiles of 32 keys x this half's 256 dims (2 x 16 KB)
//   tensor memory  S[0] columns 0-31, S[1] 32-63 (P_j as f16 pairs in the first 16 of its
//                  slot), O half 256-511
//   warp 0         TMA producer of Q (once per item, after the previous item's output left the
//                  staging area) and the K tiles
//   warp 10        TMA producer of the V tiles
//   warp 1         MMA issuer: S_j = Q K_j^T (M=128, N=32, 32 steps of K=16, both operands in
//                  shared memory); O += P_j V_j (M=128, N=256, K=32, P from tensor memory, V
//                  MN-major); S_{j+1} is issued before P_j is waited for
//   warps 2-9      softmax and output: the two warps of a lane quadrant take 16 of the 32 keys
//                  of a tile (and 128 of the 256 O columns), exchange row maxima through shared
//                  memory, rescale O lazily (the reference moves only when the row maximum
//                  exceeds it by more than 2^12) and write P over their S slot
// Every wait is bounded (common.cuh) and reports through the status word.
#pragma once
#include "attention_tc.cuh"

namespace glp {

constexpr int kF5BQ = 128;
constexpr int kF5BKV = 32;
constexpr int kF5D = 512;
constexpr uint32_t kF5QChunk = kF5BQ * 128;          // 16 KB: 128 rows x 64 dims
constexpr uint32_t kF5QBytes = 8 * kF5QChunk;        // 128 KB
constexpr uint32_t kF5KVChunk = kF5BKV * 128;        // 4 KB: 32 keys x 64 dims
constexpr uint32_t kF5KBytes = 8 * kF5KVChunk;       // 32 KB per K tile
constexpr uint32_t kF5VBytes = 4 * kF5KVChunk;       // 16 KB per V half tile
constexpr uint32_t kF5BarBytes = 256;
constexpr uint32_t kF5XchBytes = 2 * 2 * 128 * 4;
constexpr size_t kF5Smem = kF5QBytes + 2 * kF5KBytes + 2 * kF5VBytes + kF5BarBytes + kF5XchBytes;
static_assert(kF5Smem <= 232448, "shared memory per CTA");
constexpr uint32_t kF5TmemO = 256;

struct F5Item {
  bool valid;
  int tok0, len, q0, qcol, kcol, vcol, ocol, t_lo, n_tiles;
};

__device__ __forceinline__ F5Item f5_item(const FaParams& p, int item) {
  F5Item w;
  const int per_seq = p.q_blocks * p.n_q_heads * 2;
  const int b = item / per_seq;
  const int r = item - b * per_seq;
  const int qb = r / (p.n_q_heads * 2);
  const int rem = r - qb * p.n_q_heads * 2;
  const int head = rem >> 1, oh = rem & 1;
  const int seq0 = __ldg(p.cu_seqlens + b);
  w.tok0 = seq0 - p.cu_base;
  w.len = __ldg(p.cu_seqlens + b + 1) - seq0;
  w.q0 = qb * kF5BQ;
  w.valid = w.q0 < w.len;
  const int kvh = head / (p.n_q_heads / p.n_kv_heads);
  w.qcol = head * kF5D;
  w.kcol = (p.n_q_heads + kvh) * kF5D;
  w.vcol = (p.n_q_heads + p.n_kv_heads + kvh) * kF5D + oh * 256;
  w.ocol = head * kF5D + oh * 256;
  int kv_lo = 0, kv_hi = w.len;
  if (p.window > 0) {
    kv_lo = max(0, w.q0 - p.window);
    kv_hi = min(w.len, w.q0 + kF5BQ + p.window);
  }
  w.t_lo = kv_lo / kF5BKV;
  w.n_tiles = (kv_hi + kF5BKV - 1) / kF5BKV - w.t_lo;
  return w;
}

__device__ __forceinline__ float max16(const float (&v)[16]) {
  const float a = fmax3(v[0], v[1], v[2]), b = fmax3(v[3], v[4], v[5]), c = fmax3(v[6], v[7], v[8]);
  const float d = fmax3(v[9], v[10], v[11]), e = fmax3(v[12], v[13], v[14]);
  return fmax3(fmax3(a, b, c), fmax3(d, e, v[15]), -INFINITY);
}

// p.q_blocks = ceil(max_len / 128); tmQ: qkv with 64 x 128 boxes, tmKV: qkv with 64 x 32 boxes,
// tmO: the output [T, Hq * 512] with 64 x 32 boxes.
__global__ void __launch_bounds__(kFaThreads, 1)
    flash_attn_d512_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                           const __grid_constant__ CUtensorMap tmO, const FaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) record_error(p.status, kErrBadArgs);
    return;
  }
  uint8_t* sQ = smem_raw;
  uint8_t* sK = sQ + kF5QBytes;          // [2][8][32 x 128 B]
  uint8_t* sV = sK + 2 * kF5KBytes;      // [2][4][32 x 128 B]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sV + 2 * kF5VBytes);
  uint64_t* q_full = bar;
  uint64_t* q_free = bar + 1;    // Q / staging area free: the item's output left it (8 warps)
  uint64_t* k_full = bar + 2;    // [2]
  uint64_t* k_empty = bar + 4;   // [2]
  uint64_t* v_full = bar + 6;    // [2]
  uint64_t* v_empty = bar + 8;   // [2]
  uint64_t* s_full = bar + 10;   // [2]
  uint64_t* p_full = bar + 12;   // [2]
  uint64_t* pv_done = bar + 14;  // [2]
  uint64_t* drain = bar + 16;
  uint64_t* xbar = bar + 17;     // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 21);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bar) + kF5BarBytes);  // [2][2][128]

  const int n_items = p.n_seq * p.q_blocks * p.n_q_heads * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_free, 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
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
        const F5Item w = f5_item(p, item);
        if (!w.valid) continue;
        if (!mbar_wait(q_free, (it & 1) ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(q_full, kF5QBytes);
        for (int c = 0; c < 8; ++c) tma_load_2d(sQ + c * kF5QChunk, &tmQ, q_full, w.qcol + 64 * c, w.tok0 + w.q0);
        for (int j = 0; j < w.n_tiles; ++j, ++g) {
          const int st = g & 1;
          const int row = w.tok0 + (w.t_lo + j) * kF5BKV;
          if (!mbar_wait(&k_empty[st], ((g >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], kF5KBytes);
          for (int c = 0; c < 8; ++c)
            tma_load_2d(sK + st * kF5KBytes + c * kF5KVChunk, &tmKV, &k_full[st], w.kcol + 64 * c, row);
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
        const F5Item w = f5_item(p, item);
        if (!w.valid) continue;
        for (int j = 0; j < w.n_tiles; ++j, ++g) {
          const int st = g & 1;
          const int row = w.tok0 + (w.t_lo + j) * kF5BKV;
          if (!mbar_wait(&v_empty[st], ((g >> 1) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], kF5VBytes);
          for (int c = 0; c < 4; ++c)
            tma_load_2d(sV + st * kF5VBytes + c * kF5KVChunk, &tmKV, &v_full[st], w.vcol + 64 * c, row);
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
      constexpr uint32_t idesc_s = idesc_f16(128, kF5BKV, 0);
      constexpr uint32_t idesc_pv = idesc_f16(128, 256, 0) | (1u << 16);  // B (V) MN-major
      auto issue_s = [&](uint32_t gx) -> bool {
        const int st = gx & 1;
        if (!mbar_wait(&k_full[st], (gx >> 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(st * kF5BKV);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint64_t qd = desc_kmajor_sw128(smem_u32(sQ + c * kF5QChunk));
          const uint64_t kd = desc_kmajor_sw128(smem_u32(sK + st * kF5KBytes + c * kF5KVChunk));
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
        const F5Item w = f5_item(p, item);
        if (!w.valid) continue;
        if (!mbar_wait(q_full, it & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issued = true;
        if (!issue_s(g)) {
          ok = false;
          break;
        }
        for (int j = 0; j < w.n_tiles; ++j) {
          const uint32_t gj = g + j;
          const int st = gj & 1;
          if (j + 1 < w.n_tiles && !issue_s(gj + 1)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&p_full[st], (gj >> 1) & 1, abort_flag) || !mbar_wait(&v_full[st], (gj >> 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 2; ++k) {  // 16 keys per step: 16 rows of 128 B in V, 8 TMEM columns of P
            const uint64_t vd = desc_mnmajor_sw128(smem_u32(sV + st * kF5VBytes + k * 16 * 128), kF5KVChunk, 1024);
            umma_f16_ts(tmem + kF5TmemO, tmem + st * kF5BKV + k * 8, vd, idesc_pv, (j | k) != 0 ? 1u : 0u);
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
        umma_commit(drain);
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(drain, 0) && globaltimer() - t0 < GLP_WAIT_TIMEOUT_NS) {
        }
      }
    }
  } else {
    // -------------------------------------------------------------------- softmax + output
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // keys 16 half.. of a tile; O columns 128 half..
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr float kLog2e = 1.4426950408889634f;
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
    auto load_s = [&](uint32_t gx, uint32_t (&s)[16]) -> bool {
      const int st = gx & 1;
      const bool wt = mbar_wait(&s_full[st], (gx >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, wt)) return false;
      tc_fence_after();
      uint32_t a[8], b[8];
      tmem_ld8(lane_base + st * kF5BKV + half * 16, a);
      tmem_ld8(lane_base + st * kF5BKV + half * 16 + 8, b);
      tmem_ld_wait_tied8(a, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s[e] = a[e];
        s[8 + e] = b[e];
      }
      return true;
    };
    uint8_t* stage = sQ + (warp - 2) * (kFaOutBoxRows * 128);  // staging inside the Q area
    uint32_t g = 0;
    int it = 0;
    bool ok = true;
    uint32_t sr[16];
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
      const F5Item w = f5_item(p, item);
      if (!w.valid) continue;
      const int i = w.q0 + r;
      float m_ref = -INFINITY, l = 0.f;
      if (!load_s(g, sr)) {
        ok = false;
        break;
      }
      for (int j = 0; j < w.n_tiles; ++j) {
        const uint32_t gj = g + j;
        const int st = gj & 1;
        const int kt = (w.t_lo + j) * kF5BKV;
        const int kb = kt + half * 16;
        const bool full_tile =
            kt + kF5BKV <= w.len &&
            (p.window <= 0 || (kt >= w.q0 + kF5BQ - 1 - p.window && kt + kF5BKV - 1 <= w.q0 + p.window));
        float sv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          bool valid = true;
          if (!full_tile) {
            const int kj = kb + e;
            valid = kj < w.len && (p.window <= 0 || abs(i - kj) <= p.window);
          }
          sv[e] = valid ? u2f(sr[e]) : -INFINITY;
        }
        const float mine = max16(sv) * kLog2e;
        publish(mine);
        const float mu_s = mine > m_ref + kFaRescaleLog2 ? mine : m_ref;
        const float mu = mu_s == -INFINITY ? 0.f : mu_s;
        const uint64_t l2e = f2(kLog2e, kLog2e), nmu = f2(-mu, -mu);
        uint64_t ev[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint64_t x = f2_fma(f2(sv[2 * e], sv[2 * e + 1]), l2e, nmu);
          float a, b;
          f2_split(x, a, b);
          ev[e] = f2(fast_exp2(a), fast_exp2(b));
        }
        float other;
        if (!collect(&other)) {
          ok = false;
          break;
        }
        const float joint = fmaxf(mine, other);
        const float m_new = joint > m_ref + kFaRescaleLog2 ? joint : m_ref;
        const float factor = (m_ref == -INFINITY || m_new == m_ref) ? 1.f : fast_exp2(m_ref - m_new);
        const float corr = mu_s == m_new ? 1.f : fminf(fast_exp2(mu - m_new), 1.f);
        m_ref = m_new;
        if (__any_sync(0xffffffffu, corr != 1.f)) {
          const uint64_t c2 = f2(corr, corr);
#pragma unroll
          for (int e = 0; e < 8; ++e) ev[e] = f2_mul(ev[e], c2);
        }
        uint32_t pk[8];
        uint64_t acc[2] = {0ull, 0ull};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float a, b;
          f2_split(ev[e], a, b);
          pk[e] = pack_f16(a, b);
          acc[e & 1] = f2_add(acc[e & 1], ev[e]);
        }
        {
          float s0, s1;
          f2_split(f2_add(acc[0], acc[1]), s0, s1);
          l = l * factor + (s0 + s1);
        }
        // O is rescaled only after P_{j-1} V_{j-1} has landed (this half's 128 columns)
        if (j >= 1 && __any_sync(0xffffffffu, factor != 1.0f)) {
          const bool wt = mbar_wait(&pv_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, wt)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t f2x = f2(factor, factor);
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t oa[32];
            const uint32_t ta = lane_base + kF5TmemO + half * 128 + c * 32;
            tmem_ld32(ta, oa);
            tmem_ld_wait_tied(oa);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float a, b;
              f2_split(f2_mul(f2(u2f(oa[e]), u2f(oa[e + 1])), f2x), a, b);
              oa[e] = __float_as_uint(a);
              oa[e + 1] = __float_as_uint(b);
            }
            tmem_st32(ta, oa);
          }
        }
        // P row r, this half's 16 keys: 8 columns of f16 pairs over the S slot
        tmem_st8(lane_base + st * kF5BKV + half * 8, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[st]);
        if (j + 1 < w.n_tiles && !load_s(gj + 1, sr)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      // ---- output: every MMA of the item (its last S included) has completed once the last
      // P V has, so the Q area can take the staging tiles
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
      const int row0 = w.q0 + quad * kFaOutBoxRows;
      const bool bulk = row0 + kFaOutBoxRows <= w.len;
      const uint32_t ob_base = lane_base + kF5TmemO + half * 128;
#pragma unroll 1
      for (int k = 0; k < 2; ++k) {  // two slices of 64 output columns
        uint32_t oa[32], ob[32];
        tmem_ld32(ob_base + k * 64, oa);
        tmem_ld32(ob_base + k * 64 + 32, ob);
        if (k == 1 && lane == 0) bulk_wait_read_all();  // the first slice's store has read the tile
        __syncwarp();
        tmem_ld_wait_tied(oa);
        tmem_ld_wait_tied(ob);
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
        const int col = w.ocol + half * 128 + k * 64;
        if (bulk) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmO, stage, col, w.tok0 + row0);
            bulk_commit();
          }
        } else {
          __syncwarp();
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
      // the staging tile (part of the Q area) is read before the next item's Q may land
      if (lane == 0) bulk_wait_read_all();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_free);
      g += w.n_tiles;
      ++it;
    }
    if (lane == 0) {
      bulk_wait_all();
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
