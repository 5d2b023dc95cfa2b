// Exact non-causal attention forward for MiniMax-H3 heads (head_dim 128, bf16 in,
// fp32 accumulate) on sm_100a.
//
// Replaces the attention op of the Ulysses runtime: the SDPA FLASH call at
// harness/sp_runtime.py:119-121 (and the unwired sm_80 kernel behind
// attn_sm80/attn_sm80.py:26-31). O = softmax(Q K^T * scale) V per head.
//
// CTA = one head x 256 query rows (two 128-row Q tiles), 12 warps:
//   warp 0      TMA producer: Q tiles once, then K_j / V_j tiles through a 4-stage ring
//   warp 1      MMA issuer (one thread): S_t = Q_t K_j^T (SS form), O_t += P_t V_j (TS form)
//   warp 2      TMEM allocator (512 columns)
//   warps 4-7   softmax warpgroup for Q tile 0; warps 8-11 for Q tile 1
// TMEM columns: S_0 [0,128) S_1 [128,256) O_0 [256,384) O_1 [384,512);
// P_t (bf16 pairs) overwrites the upper half of S_t, columns [64,128) of it.
// Each softmax thread owns one query row (TMEM lane), so row max / row sum are
// in-register. O is rescaled only when a row max grows by more than 2^8, which
// keeps P <= 256; every per-row decision depends on that row alone, so a row's
// result does not depend on which other rows or heads share the launch.
#include "h3_ptx.cuh"
#include "h3attn.h"

#include <cmath>
#include <cstdio>

namespace h3 {
namespace attn {

constexpr int kD = 128;
constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kRowsPerCta = 2 * kBlockM;
constexpr int kStages = 4;
constexpr uint32_t kHalfBytes = 128u * 64u * 2u;  // 128 rows x 64 bf16: one 128-B swizzle column block
constexpr uint32_t kTileBytes = 2u * kHalfBytes;  // 128 rows x 128 bf16
constexpr int kThreads = 384;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

enum Bar : int {
  kBarQFull = 0,
  kBarKVFull = 1,
  kBarKVEmpty = kBarKVFull + kStages,
  kBarSFull = kBarKVEmpty + kStages,
  kBarPFull = kBarSFull + 2,
  kBarODone = kBarPFull + 2,
  kBarDrain = kBarODone + 2,
  kNumBars = kBarDrain + 1
};

constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffKV = 2 * kTileBytes;
constexpr uint32_t kOffBars = kOffKV + kStages * kTileBytes;
constexpr uint32_t kSmemBytes = 1024 + kOffBars + kNumBars * 8 + 16;

__host__ __device__ constexpr uint32_t col_s(int t) { return uint32_t(t) * 128u; }
__host__ __device__ constexpr uint32_t col_p(int t) { return uint32_t(t) * 128u + 64u; }
__host__ __device__ constexpr uint32_t col_o(int t) { return 256u + uint32_t(t) * 128u; }

struct Params {
  int n_heads;
  int s_q;
  int s_kv;
  int n_kv_tiles;
  float scale_log2;
  __nv_bfloat16* o;
  long long o_rank_rows;
  long long o_rank_stride;
  long long o_head_stride;
  long long o_row_stride;
  int* status;
};

// S = Q K^T for one 128x128 tile pair; both operands K-major, SW128, two 64-column blocks.
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t a_base, uint32_t b_base) {
  constexpr uint32_t idesc = idesc_bf16_f32(128, 128, 0, 0);
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    const uint32_t off = uint32_t(kk >> 2) * kHalfBytes + uint32_t(kk & 3) * 32u;
    mma_ss(d_tmem, smem_desc_sw128(a_base + off, 16, 1024), smem_desc_sw128(b_base + off, 16, 1024), idesc,
           kk > 0 ? 1u : 0u);
  }
}

// O (+)= P V for one tile: P from TMEM (K = keys along columns, two bf16 per column),
// V MN-major in shared memory (d contiguous), two 64-wide d blocks 16 KB apart.
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_base, bool accumulate) {
  constexpr uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
  for (int kk = 0; kk < kBlockN / 16; ++kk) {
    mma_ts(d_tmem, p_tmem + uint32_t(kk) * 8u, smem_desc_sw128(v_base + uint32_t(kk) * 2048u, kHalfBytes, 1024),
           idesc, (accumulate || kk > 0) ? 1u : 0u);
  }
}

// Bounded wait that ignores the abort flag: used while draining copies/MMAs before exit.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int* status) {
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > H3_WAIT_LIMIT_NS) {
      atomicCAS(status, 0, kStatusTimeoutDrain);
      return;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int m0 = blockIdx.x * kRowsPerCta;
  const int n_kv = p.n_kv_tiles;

  if (threadIdx.x == 0) {
    mbar_init(bar(kBarQFull), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarKVFull + s), 1);
      mbar_init(bar(kBarKVEmpty + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kBarSFull + t), 1);
      mbar_init(bar(kBarPFull + t), 128);
      mbar_init(bar(kBarODone + t), 1);
    }
    mbar_init(bar(kBarDrain), 1);
    *abort_flag = (*reinterpret_cast<volatile int*>(p.status) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, p.status};
  const bool grid_aborted = *abort_flag != 0;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && !grid_aborted) {
      const uint32_t sq = sbase + kOffQ;
      const uint32_t skv = sbase + kOffKV;
      mbar_expect_tx(bar(kBarQFull), 2 * kTileBytes);
      for (int t = 0; t < 2; ++t)
        for (int hh = 0; hh < 2; ++hh)
          tma_load_3d(sq + t * kTileBytes + hh * kHalfBytes, &tmap_q, bar(kBarQFull), hh * 64, m0 + t * kBlockM,
                      head);
      int it = 0;
      for (int j = 0; j < n_kv; ++j) {
        bool ok = true;
        for (int kv = 0; kv < 2; ++kv, ++it) {
          const int st = it % kStages;
          const uint32_t ph = uint32_t(it / kStages) & 1u;
          if (!mbar_wait(bar(kBarKVEmpty + st), ph ^ 1u, ctx, kStatusTimeoutKV)) {
            ok = false;
            break;
          }
          const CUtensorMap* m = kv ? &tmap_v : &tmap_k;
          mbar_expect_tx(bar(kBarKVFull + st), kTileBytes);
          tma_load_3d(skv + st * kTileBytes, m, bar(kBarKVFull + st), 0, j * kBlockN, head);
          tma_load_3d(skv + st * kTileBytes + kHalfBytes, m, bar(kBarKVFull + st), 64, j * kBlockN, head);
        }
        if (!ok) break;
      }
      // Every issued copy must land before the CTA may exit.
      drain_wait(bar(kBarQFull), 0, p.status);
      for (int st = 0; st < kStages; ++st) {
        const int cnt = it / kStages + (st < it % kStages ? 1 : 0);
        if (cnt > 0) drain_wait(bar(kBarKVFull + st), uint32_t(cnt - 1) & 1u, p.status);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && !grid_aborted) {
      const uint32_t sq = sbase + kOffQ;
      const uint32_t skv = sbase + kOffKV;
      int it = 0;
      auto wait_full = [&](int st_it) -> bool {
        const int st = st_it % kStages;
        return mbar_wait(bar(kBarKVFull + st), uint32_t(st_it / kStages) & 1u, ctx, kStatusTimeoutKV);
      };
      bool ok = mbar_wait(bar(kBarQFull), 0, ctx, kStatusTimeoutQ);
      if (ok) ok = wait_full(it);
      if (ok) {
        tc_fence_after();
        const int st = it % kStages;
        issue_qk(tmem + col_s(0), sq, skv + st * kTileBytes);
        mma_commit(bar(kBarSFull + 0));
        issue_qk(tmem + col_s(1), sq + kTileBytes, skv + st * kTileBytes);
        mma_commit(bar(kBarSFull + 1));
        mma_commit(bar(kBarKVEmpty + st));
        ++it;
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int it_v = it++;
        if (!(ok = wait_full(it_v))) break;
        const int stv = it_v % kStages;
        const uint32_t ph = uint32_t(j) & 1u;
        if (!(ok = mbar_wait(bar(kBarPFull + 0), ph, ctx, kStatusTimeoutP))) break;
        tc_fence_after();
        issue_pv(tmem + col_o(0), tmem + col_p(0), skv + stv * kTileBytes, j > 0);
        mma_commit(bar(kBarODone + 0));
        int stk = -1;
        if (j + 1 < n_kv) {
          const int it_k = it++;
          if (!(ok = wait_full(it_k))) break;
          tc_fence_after();
          stk = it_k % kStages;
          issue_qk(tmem + col_s(0), sq, skv + stk * kTileBytes);
          mma_commit(bar(kBarSFull + 0));
        }
        if (!(ok = mbar_wait(bar(kBarPFull + 1), ph, ctx, kStatusTimeoutP))) break;
        tc_fence_after();
        issue_pv(tmem + col_o(1), tmem + col_p(1), skv + stv * kTileBytes, j > 0);
        mma_commit(bar(kBarODone + 1));
        mma_commit(bar(kBarKVEmpty + stv));
        if (stk >= 0) {
          issue_qk(tmem + col_s(1), sq + kTileBytes, skv + stk * kTileBytes);
          mma_commit(bar(kBarSFull + 1));
          mma_commit(bar(kBarKVEmpty + stk));
        }
      }
      // Every issued MMA must retire before TMEM is released.
      mma_commit(bar(kBarDrain));
      drain_wait(bar(kBarDrain), 0, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;  // Q tile
    const int quad = warp & 3;      // TMEM lane quadrant this warp may access
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + col_s(t);
    const uint32_t tP = tmem + lane_off + col_p(t);
    const uint32_t tO = tmem + lane_off + col_o(t);
    const float c = p.scale_log2;
    const int tail_valid = p.s_kv - (n_kv - 1) * kBlockN;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = !grid_aborted;
    for (int j = 0; ok && j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarSFull + t), uint32_t(j) & 1u, ctx, kStatusTimeoutS));
      if (!ok) break;
      tc_fence_after();
      uint32_t sa[64], sb[64];
      tmem_ld64_wait(tS, sa);
      tmem_ld64_wait(tS + 64, sb);
      float s[128];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        s[i] = __uint_as_float(sa[i]);
        s[64 + i] = __uint_as_float(sb[i]);
      }
      if (j == n_kv - 1 && tail_valid < kBlockN) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= tail_valid) s[i] = -INFINITY;
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int i = 4; i < 128; i += 4) {
        mx0 = fmaxf(mx0, s[i]);
        mx1 = fmaxf(mx1, s[i + 1]);
        mx2 = fmaxf(mx2, s[i + 2]);
        mx3 = fmaxf(mx3, s[i + 3]);
      }
      const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c);
      if (j == 0) {
        m_run = m_new;
      } else {
        const bool need = m_new > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          // O_t still holds the sum up to tile j-1: wait for that PV, then rescale in place.
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar(kBarODone + t), uint32_t(j - 1) & 1u, ctx, kStatusTimeoutO));
          if (!ok) break;
          tc_fence_after();
          const float f = need ? ex2_approx(m_run - m_new) : 1.0f;
          if (need) {
            l_run *= f;
            m_run = m_new;
          }
          // 16-column chunks keep this rare path within the register budget while s[] is live.
#pragma unroll 1
          for (int c16 = 0; c16 < 8; ++c16) {
            uint32_t o[16];
            tmem_ld16_wait(tO + c16 * 16, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
            tmem_st16(tO + c16 * 16, o);
          }
          tmem_st_wait();
        }
      }
      const float neg_m = -m_run;
      float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
      uint32_t pa[32], pb[32];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float e0 = ex2_approx(fmaf(s[2 * i], c, neg_m));
        const float e1 = ex2_approx(fmaf(s[2 * i + 1], c, neg_m));
        const float e2 = ex2_approx(fmaf(s[2 * i + 2], c, neg_m));
        const float e3 = ex2_approx(fmaf(s[2 * i + 3], c, neg_m));
        l0 += e0;
        l1 += e1;
        l2 += e2;
        l3 += e3;
        pa[i] = pack_bf16x2(e0, e1);
        pa[i + 1] = pack_bf16x2(e2, e3);
      }
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float e0 = ex2_approx(fmaf(s[64 + 2 * i], c, neg_m));
        const float e1 = ex2_approx(fmaf(s[64 + 2 * i + 1], c, neg_m));
        const float e2 = ex2_approx(fmaf(s[64 + 2 * i + 2], c, neg_m));
        const float e3 = ex2_approx(fmaf(s[64 + 2 * i + 3], c, neg_m));
        l0 += e0;
        l1 += e1;
        l2 += e2;
        l3 += e3;
        pb[i] = pack_bf16x2(e0, e1);
        pb[i + 1] = pack_bf16x2(e2, e3);
      }
      l_run += (l0 + l1) + (l2 + l3);
      tmem_st32(tP, pa);
      tmem_st32(tP + 32, pb);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(kBarPFull + t));
    }
    if (ok) {
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar(kBarODone + t), uint32_t(n_kv - 1) & 1u, ctx, kStatusTimeoutO));
    }
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / l_run;
      const int row = m0 + t * kBlockM + quad * 32 + lane;
      const bool valid = row < p.s_q;
      const long long rr = valid ? row : 0;
      __nv_bfloat16* dst = p.o + (rr / p.o_rank_rows) * p.o_rank_stride + (long long)head * p.o_head_stride +
                           (rr % p.o_rank_rows) * p.o_row_stride;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[32];
        tmem_ld32_wait(tO + c4 * 32, o);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
        if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c4 * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- tile known-answer kernels
// One 128x128x128 S = Q K^T through the same TMA / descriptor / tcgen05 path.
__global__ void __launch_bounds__(128, 1)
    kat_qk_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                  float* s_out, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t b_full = smem_u32(&bars[0]), b_done = smem_u32(&bars[1]);
  if (threadIdx.x == 0) {
    mbar_init(b_full, 1);
    mbar_init(b_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, status};
  if (threadIdx.x == 0) {
    mbar_expect_tx(b_full, 2 * kTileBytes);
    for (int hh = 0; hh < 2; ++hh) {
      tma_load_3d(sbase + hh * kHalfBytes, &tmap_q, b_full, hh * 64, 0, 0);
      tma_load_3d(sbase + kTileBytes + hh * kHalfBytes, &tmap_k, b_full, hh * 64, 0, 0);
    }
    if (mbar_wait(b_full, 0, ctx, kStatusTimeoutKat)) {
      tc_fence_after();
      issue_qk(tmem, sbase, sbase + kTileBytes);
    } else {
      drain_wait(b_full, 0, status);
    }
    mma_commit(b_done);
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait(b_done, 0, ctx, kStatusTimeoutKat));
  if (ok) {
    tc_fence_after();
    const int row = warp * 32 + lane;
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t r[32];
      tmem_ld32_wait(tmem + (uint32_t(warp * 32) << 16) + c4 * 32, r);
      for (int i = 0; i < 32; ++i) s_out[row * 128 + c4 * 32 + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// One O = P V tile: P [128 x 128] bf16 from global written into TMEM exactly as the
// softmax warps write it, V loaded by TMA, TS-form MMA, O read back as fp32.
__global__ void __launch_bounds__(128, 1)
    kat_pv_kernel(const __nv_bfloat16* p_in, const __grid_constant__ CUtensorMap tmap_v, float* o_out,
                  int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t b_full = smem_u32(&bars[0]), b_done = smem_u32(&bars[1]);
  if (threadIdx.x == 0) {
    mbar_init(b_full, 1);
    mbar_init(b_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, status};
  const uint32_t lane_off = uint32_t(warp * 32) << 16;
  {
    const int row = warp * 32 + lane;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p_in + row * 128);
    uint32_t pa[32], pb[32];
    for (int i = 0; i < 32; ++i) {
      pa[i] = src[i];
      pb[i] = src[32 + i];
    }
    tmem_st32(tmem + lane_off + 64, pa);
    tmem_st32(tmem + lane_off + 96, pb);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_expect_tx(b_full, kTileBytes);
    for (int hh = 0; hh < 2; ++hh) tma_load_3d(sbase + hh * kHalfBytes, &tmap_v, b_full, hh * 64, 0, 0);
    if (mbar_wait(b_full, 0, ctx, kStatusTimeoutKat)) {
      tc_fence_after();
      issue_pv(tmem + 128, tmem + 64, sbase, false);
    } else {
      drain_wait(b_full, 0, status);
    }
    mma_commit(b_done);
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait(b_done, 0, ctx, kStatusTimeoutKat));
  if (ok) {
    tc_fence_after();
    const int row = warp * 32 + lane;
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t r[32];
      tmem_ld32_wait(tmem + lane_off + 128 + c4 * 32, r);
      for (int i = 0; i < 32; ++i) o_out[row * 128 + c4 * 32 + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ---------------------------------------------------------------- host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) != cudaSuccess ||
      qres != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<EncodeTiledFn>(fn);
}

// [n_heads][rows][128] bf16 with element strides (row_stride, head_stride); box 64 x 128 x 1, SW128.
static int make_head_map(CUtensorMap* map, const void* base, long long rows, long long n_heads,
                         long long row_stride, long long head_stride) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return H3_ERR_DRIVER;
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)n_heads};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride * 2, (cuuint64_t)head_stride * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3_OK : H3_ERR_TENSOR_MAP;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace attn
}  // namespace h3

using namespace h3::attn;

extern "C" int h3_attn_fwd(const void* q, const void* k, const void* v, void* o, int64_t n_heads, int64_t s_q,
                           int64_t s_kv, int64_t q_head_stride, int64_t q_row_stride, int64_t kv_head_stride,
                           int64_t kv_row_stride, int64_t o_rank_rows, int64_t o_rank_stride, int64_t o_head_stride,
                           int64_t o_row_stride, float softmax_scale, int32_t* status, void* stream) {
  if (!q || !k || !v || !o || !status) return H3_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || (reinterpret_cast<uintptr_t>(status) & 3u))
    return H3_ERR_ALIGN;
  if (n_heads < 1 || n_heads > 65535 || s_q < 1 || s_kv < 1 || s_q > (1ll << 31) - 512 ||
      s_kv > (1ll << 31) - 512 || o_rank_rows < 1)
    return H3_ERR_SHAPE;
  if (q_row_stride < 128 || kv_row_stride < 128 || o_row_stride < 128 || (q_row_stride % 8) ||
      (kv_row_stride % 8) || (q_head_stride % 8) || (kv_head_stride % 8) || (o_row_stride % 8) ||
      (o_head_stride % 8) || (o_rank_stride % 8) || q_head_stride < 0 || kv_head_stride < 0 || o_head_stride < 0 ||
      o_rank_stride < 0)
    return H3_ERR_STRIDE;
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale)) return H3_ERR_SHAPE;
  if (n_heads > 1 && (q_head_stride == 0 || kv_head_stride == 0)) return H3_ERR_STRIDE;

  CUtensorMap tq, tk, tv;
  const long long qhs = n_heads > 1 ? q_head_stride : s_q * q_row_stride;
  const long long kvhs = n_heads > 1 ? kv_head_stride : s_kv * kv_row_stride;
  int rc;
  if ((rc = make_head_map(&tq, q, s_q, n_heads, q_row_stride, qhs)) != H3_OK) return rc;
  if ((rc = make_head_map(&tk, k, s_kv, n_heads, kv_row_stride, kvhs)) != H3_OK) return rc;
  if ((rc = make_head_map(&tv, v, s_kv, n_heads, kv_row_stride, kvhs)) != H3_OK) return rc;

  Params p;
  p.n_heads = (int)n_heads;
  p.s_q = (int)s_q;
  p.s_kv = (int)s_kv;
  p.n_kv_tiles = (int)((s_kv + kBlockN - 1) / kBlockN);
  p.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.o_rank_rows = o_rank_rows;
  p.o_rank_stride = o_rank_stride;
  p.o_head_stride = o_head_stride;
  p.o_row_stride = o_row_stride;
  p.status = status;

  if (cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
      cudaSuccess)
    return H3_ERR_LAUNCH;
  dim3 grid((unsigned)((s_q + kRowsPerCta - 1) / kRowsPerCta), (unsigned)n_heads);
  attn_fwd_kernel<<<grid, kThreads, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_tile_kat_qk(const void* q, const void* k, float* s_out, int32_t* status, void* stream) {
  if (!q || !k || !s_out || !status) return H3_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(s_out)) return H3_ERR_ALIGN;
  CUtensorMap tq, tk;
  int rc;
  if ((rc = make_head_map(&tq, q, 128, 1, 128, 128 * 128)) != H3_OK) return rc;
  if ((rc = make_head_map(&tk, k, 128, 1, 128, 128 * 128)) != H3_OK) return rc;
  const int smem = 1024 + 2 * kTileBytes + 64;
  if (cudaFuncSetAttribute(kat_qk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return H3_ERR_LAUNCH;
  kat_qk_kernel<<<1, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, s_out, status);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_tile_kat_pv(const void* p_in, const void* v, float* o_out, int32_t* status, void* stream) {
  if (!p_in || !v || !o_out || !status) return H3_ERR_NULL;
  if (!aligned16(p_in) || !aligned16(v) || !aligned16(o_out)) return H3_ERR_ALIGN;
  CUtensorMap tv;
  int rc;
  if ((rc = make_head_map(&tv, v, 128, 1, 128, 128 * 128)) != H3_OK) return rc;
  const int smem = 1024 + kTileBytes + 64;
  if (cudaFuncSetAttribute(kat_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return H3_ERR_LAUNCH;
  kat_pv_kernel<<<1, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(p_in), tv, o_out, status);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}
