// Bidirectional GQA flash attention on the 5th-generation tensor cores (tcgen05), head_dim
// 256, f16 operands, f32 accumulation in tensor memory, f32 softmax.
//
// Same semantics as attention.cuh (scale 1.0, standard.rs:62; key j visible iff j < len and,
// on sliding layers, |i - j| <= W, model.rs:634-638; GQA kv head = h / (Hq / Hkv)).
//
// CTA = 128 query rows of one (sequence, head); 192 threads:
//   warp 0      TMA producer: Q once (4 boxes of 64 dims x 128 rows), then K/V tiles of 64
//               keys into a 2-stage ring (4 boxes each)
//   warp 1      TMEM owner + single-thread MMA issuer:
//                 S_j = Q K_j^T   (M=128, N=64, K=256; A and B K-major)   -> TMEM S[j%2]
//                 O  += P_j V_j   (M=128, N=256, K=64;  P K-major in SMEM, V MN-major)
//               S_{j+1} is issued before waiting for P_j so the tensor core works while
//               the softmax warps run.
//   warps 2..5  softmax / correction / epilogue, one query row per thread (TMEM lane):
//               read S_j, mask, online max in the log2 domain with lazy rescaling (O is
//               rescaled in TMEM only when the running max grows by more than 2^8; the
//               stale max is exact for the final O / l), write P_j (f16) into a 128B-swizzled
//               K-major SMEM tile, and at the end O / l -> f16 (the O-projection's input).
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
constexpr size_t kFaSmem = 1024 + kFaQBytes + 4 * kFaKVBytes + 2 * kFaPBytes + 256;
constexpr float kFaRescaleLog2 = 8.0f;                   // lazy-rescale threshold (factor 256)

struct FaParams {
  const int* cu_seqlens;
  int cu_base;
  int n_q_heads, n_kv_heads;
  int window;
  __half* out;
  int ld_out;
  int* status;
};

__global__ void __launch_bounds__(192, 1)
    flash_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                         const FaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kFaQBytes;            // [2][4][64 x 128 B]
  uint8_t* sV = sK + 2 * kFaKVBytes;       // [2][4][64 x 128 B]
  uint8_t* sP = sV + 2 * kFaKVBytes;       // [2][128 x 128 B]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + 2 * kFaPBytes);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;   // [2]
  uint64_t* kv_empty = bar + 3;  // [2]
  uint64_t* s_full = bar + 5;    // [2]
  uint64_t* p_full = bar + 7;    // [2]
  uint64_t* pv_done = bar + 9;   // [2]
  uint64_t* drain = bar + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int b = blockIdx.z, head = blockIdx.y;
  const int seq0 = p.cu_seqlens[b];
  const int tok0 = seq0 - p.cu_base;
  const int len = p.cu_seqlens[b + 1] - seq0;
  const int q0 = blockIdx.x * kFaBQ;
  if (q0 >= len) return;  // whole CTA exits before any barrier or TMEM use
  const int kvh = head / (p.n_q_heads / p.n_kv_heads);
  const int qcol = head * kFaD;
  const int kcol = (p.n_q_heads + kvh) * kFaD;
  const int vcol = (p.n_q_heads + p.n_kv_heads + kvh) * kFaD;
  int kv_lo = 0, kv_hi = len;
  if (p.window > 0) {
    kv_lo = max(0, q0 - p.window);
    kv_hi = min(len, q0 + kFaBQ + p.window);
  }
  const int t_lo = kv_lo / kFaBKV;
  const int n_tiles = (kv_hi + kFaBKV - 1) / kFaBKV - t_lo;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
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
      mbar_arrive_expect_tx(q_full, kFaQBytes);
      for (int c = 0; c < 4; ++c) tma_load_2d(sQ + c * (kFaBQ * 128), &tmQ, q_full, qcol + 64 * c, tok0 + q0);
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, abort_flag)) {
          record_error(p.status, kErrTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        const int row = tok0 + (t_lo + j) * kFaBKV;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kFaKVBytes);
        for (int c = 0; c < 4; ++c) {
          tma_load_2d(sK + st * kFaKVBytes + c * kFaKVChunk, &tmKV, &kv_full[st], kcol + 64 * c, row);
          tma_load_2d(sV + st * kFaKVBytes + c * kFaKVChunk, &tmKV, &kv_full[st], vcol + 64 * c, row);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = idesc_f16(128, kFaBKV, 0);
      constexpr uint32_t idesc_pv = idesc_f16(128, kFaD, 0) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1, abort_flag)) return false;
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
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j & 1;
        if (j + 1 < n_tiles && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&p_full[st], (j >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t pd = desc_kmajor_sw128(smem_u32(sP + st * kFaPBytes));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          // V rows k*16..k*16+15 of this stage: 16 keys x 128 B further per K step
          const uint64_t vd = desc_mnmajor_sw128(smem_u32(sV + st * kFaKVBytes + k * 16 * 128), kFaKVChunk, 1024);
          umma_f16_ss(tmem + 256, pd + 2 * k, vd, idesc_pv, (j | k) != 0 ? 1u : 0u);
        }
        umma_commit(&pv_done[st]);
        umma_commit(&kv_empty[st]);
      }
      if (!ok) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutMma);
        *abort_flag = 1;
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
    const int r = quad * 32 + lane;  // query row inside the tile == TMEM lane
    const int i = q0 + r;            // position inside the sequence
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr float kLog2e = 1.4426950408889634f;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      bool w = mbar_wait(&s_full[st], (j >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, w)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s0[32], s1[32];
      tmem_ld32(lane_base + st * kFaBKV, s0);
      tmem_ld32(lane_base + st * kFaBKV + 32, s1);
      tmem_ld_wait();
      const int kb = (t_lo + j) * kFaBKV;
      float sv[64];
      float tmax = -INFINITY;
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const int kj = kb + e;
        bool valid = kj < len;
        if (p.window > 0) valid = valid && abs(i - kj) <= p.window;
        const float x = (e < 32 ? u2f(s0[e]) : u2f(s1[e - 32])) * kLog2e;
        sv[e] = valid ? x : -INFINITY;
        tmax = fmaxf(tmax, sv[e]);
      }
      float factor = 1.0f;
      if (m_ref == -INFINITY) {
        m_ref = tmax;
      } else if (tmax > m_ref + kFaRescaleLog2) {
        factor = exp2f(m_ref - tmax);
        m_ref = tmax;
      }
      const float mu = m_ref == -INFINITY ? 0.f : m_ref;
      float rs = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float a = exp2f(sv[2 * e] - mu), c = exp2f(sv[2 * e + 1] - mu);
        rs += a + c;
        pk[e] = pack_f16(a, c);
      }
      l = l * factor + rs;
      // PV_{j-1} must be complete before O is rescaled or P buffer (j % 2) is rewritten
      if (j >= 1) {
        w = mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, factor != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            uint32_t o[32];
            tmem_ld32(lane_base + 256 + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(u2f(o[e]) * factor);
            tmem_st32(lane_base + 256 + c * 32, o);
          }
          tmem_st_wait();
        }
      }
      // P row r: 8 chunks of 8 keys, 128B-swizzled (chunk ^ (row & 7))
      uint8_t* prow = sP + st * kFaPBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
    }
    if (ok) {
      const int jl = n_tiles - 1;
      const bool w = mbar_wait(&pv_done[jl & 1], (jl >> 1) & 1, abort_flag);
      ok = __all_sync(0xffffffffu, w);
    }
    if (!ok) {
      if (lane == 0) {
        if (!*abort_flag) record_error(p.status, kErrTimeoutEpilogue);
        *abort_flag = 1;
      }
    } else {
      tc_fence_after();
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __half* dst = p.out + static_cast<size_t>(tok0 + i) * p.ld_out + qcol;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + 256 + c * 32, o);
        tmem_ld_wait();
        if (i < len) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            d4[q] = make_uint4(pack_f16(u2f(o[8 * q]) * inv, u2f(o[8 * q + 1]) * inv),
                               pack_f16(u2f(o[8 * q + 2]) * inv, u2f(o[8 * q + 3]) * inv),
                               pack_f16(u2f(o[8 * q + 4]) * inv, u2f(o[8 * q + 5]) * inv),
                               pack_f16(u2f(o[8 * q + 6]) * inv, u2f(o[8 * q + 7]) * inv));
        }
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
