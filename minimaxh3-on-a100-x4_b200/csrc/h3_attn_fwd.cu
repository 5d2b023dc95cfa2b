// Exact non-causal attention forward for MiniMax-H3 heads (head_dim 128, bf16 in,
// fp32 accumulate) on sm_100a.
//
// Replaces the attention op of the Ulysses runtime: the SDPA FLASH call at
// harness/sp_runtime.py:119-121 (and the unwired sm_80 kernel behind
// attn_sm80/attn_sm80.py:26-31). O = softmax(Q K^T * scale) V per head.
//
// CTA = one head x 256 query rows (two 128-row Q tiles), 12 warps:
//   warp 0      TMA producer: Q tiles once, then K_j / V_j tiles through a 5-stage ring
//   warp 1      MMA issuer (one thread): S_t = Q_t K_j^T (SS form), O_t += P_t V_j (TS form)
//   warp 2      TMEM allocator (512 columns)
//   warps 4-7   softmax warpgroup for Q tile 0; warps 8-11 for Q tile 1
// TMEM columns: S_0 [0,128) S_1 [128,256) O_0 [256,384) O_1 [384,512);
// P_t (bf16 pairs) overwrites the upper half of S_t, columns [64,128) of it.
// Each softmax thread owns one query row (TMEM lane), so row max / row sum are
// in-register. O is rescaled only when a row max grows by more than 2^8, which
// keeps P <= 256; every per-row decision depends on that row alone, so a row's
// result does not depend on which other rows or heads share the launch.
#include "h3_pair.cuh"
#include "h3attn.h"

#include <cmath>
#include <cstdio>

namespace h3 {
namespace attn {

constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kRowsPerCta = 2 * kBlockM;
constexpr int kStages = 5;  // K/V ring of whole tiles: the MMA thread waits for V_j and K_{j+1} a full iteration ahead
constexpr int kMaxRing = 2 * kStages;  // the pair form's ring of half tiles (same bytes)
// Ring stages are handed back through kRel release barriers used round robin: release r
// completes once S_1(r) is ready, i.e. once every MMA reading K_r and V_(r-1) has retired.
// A parity wait is safe while the producer trails by at most one phase of the barrier it
// waits on; it has loaded at most kRing - 1 items beyond the ones release e frees, and release
// e + kRel needs item 2(e + kRel), so kRel >= kMaxRing / 2 keeps every wait within one phase.
constexpr int kRel = kMaxRing / 2;
constexpr uint32_t kHalfBytes = 128u * 64u * 2u;  // 128 rows x 64 bf16: one 128-B swizzle column block
constexpr uint32_t kTileBytes = 2u * kHalfBytes;  // 128 rows x 128 bf16
constexpr int kThreads = 384;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Register budgets after the set-up: the producer / MMA / allocator warpgroup needs few, the two
// softmax warpgroups hold a 128-score row each. 128 * 72 + 256 * 216 = 384 * 168, the launch's total.
constexpr int kRegsLaunch = 168;
constexpr int kRegsControl = 72;
constexpr int kRegsSoftmax = 216;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kThreads * kRegsLaunch, "register split over budget");

enum Bar : int {
  kBarQFull = 0,
  kBarKVFull = 1,
  kBarRel = kBarKVFull + kMaxRing,    // ring releases, round robin (see kRel)
  kBarSFull = kBarRel + kRel,         // S_t ready (per Q tile)
  kBarPSplit = kBarSFull + 2,          // P_t chunks [0, kSplit) in TMEM
  kBarPLast = kBarPSplit + 2,          // all of P_t in TMEM
  kBarODone = kBarPLast + 2,           // the last P_t * V retired
  kBarDrain = kBarODone + 2,
  kBarTok = kBarDrain + 1,  // softmax ping-pong token, one per warpgroup
  kNumBars = kBarTok + 2
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
  long long* prof;  // phase timestamps of CTA (0, 0) when profiling, else nullptr
  int prof_iters;
  // attn_fwd_kernel only: per destination rank, the base of that rank's output (a peer's memory
  // over NVLink) replacing o + rank * o_rank_stride; nullptr otherwise
  const unsigned long long* o_peer;
};

// Phase profiler (the counterpart of the reference kernel's clock64 counters): the first
// thread of softmax warps 4 and 8 and the MMA thread of CTA (0, 0) record clock64() at
// fixed points of each KV iteration j < prof_iters into
//   prof[((role * prof_iters) + j) * 8 + point],  role 0/1 = softmax tile 0/1, role 2 = MMA.
template <bool kProf>
__device__ __forceinline__ void prof_mark(const Params& p, bool rec, int role, int j, int point) {
  if (kProf && rec && j < p.prof_iters) p.prof[((long long)role * p.prof_iters + j) * 8 + point] = clock64();
}

// Every 8-MMA group below is ONE asm block with the smem descriptors formed by immediate
// adds on the low word: the single MMA-issuing thread shares its SM sub-partition with two
// busy softmax warps, and the tensor pipe queue is shallow, so the instructions it spends
// per MMA directly become tensor-core idle time. Start addresses stay below 256 KB, so the
// low-word adds never carry out of the 14-bit start-address field.

// S = Q K^T for one 128x128 tile pair: both operands K-major, SW128, two 64-column blocks
// 16 KB apart; K steps of 16 elements advance 32 B inside a block.
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t a_base, uint32_t b_base) {
  constexpr uint32_t idesc = idesc_bf16_f32(128, 128, 0, 0);
  const uint64_t ad = smem_desc_sw128(a_base, 16, 1024), bd = smem_desc_sw128(b_base, 16, 1024);
  const uint32_t alo = uint32_t(ad), ahi = uint32_t(ad >> 32), blo = uint32_t(bd), bhi = uint32_t(bd >> 32);
#define H3_QK_STEP(OFF) \
  "add.u32 la, %1, " #OFF ";\n\t add.u32 lb, %3, " #OFF ";\n\t" \
  "mov.b64 da, {la, %2};\n\t mov.b64 db, {lb, %4};\n\t" \
  "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, pt;\n\t"
  asm volatile(
      "{\n\t.reg .pred pf, pt;\n\t.reg .b32 la, lb;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 pf, %0, %0;\n\t setp.eq.b32 pt, %0, %0;\n\t"
      "mov.b64 da, {%1, %2};\n\t mov.b64 db, {%3, %4};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, pf;\n\t"
      H3_QK_STEP(2) H3_QK_STEP(4) H3_QK_STEP(6) H3_QK_STEP(1024) H3_QK_STEP(1026) H3_QK_STEP(1028) H3_QK_STEP(1030)
      "}\n" ::"r"(d_tmem), "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc)
      : "memory");
#undef H3_QK_STEP
}

// Bounded wait that ignores the abort flag: used while draining copies/MMAs before exit.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int* status) {
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_sleep(bar, parity)) {
    if (globaltimer_ns() - t0 > H3_WAIT_LIMIT_NS) {
      atomicCAS(status, 0, kStatusTimeoutDrain);
      return;
    }
  }
}

// 2^x of one key pair of 32-key chunk `chunk`, pair `pair` (0..15) in it: on the FMA pipe when
// bit `pair` of kEmuMask and bit `chunk` of kEmuChunks are set, else on MUFU.
template <uint32_t kEmuMask, uint32_t kEmuChunks>
__device__ __forceinline__ void ex2_pair(float x0, float x1, int chunk, int pair, float& y0, float& y1) {
  if (((kEmuChunks >> chunk) & 1u) && ((kEmuMask >> pair) & 1u)) {
    ex2_poly2(x0, x1, y0, y1);
  } else {
    y0 = ex2_approx(x0);
    y1 = ex2_approx(x1);
  }
}

// O (+)= P V over K steps [kFirst, kFirst + kSteps) of one tile (16 keys per step): P from
// TMEM at 8 columns per step, V in shared memory 2 KB per step. One asm block per call.
template <int kFirst, int kSteps>
__device__ __forceinline__ void issue_pv_steps(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_base, bool accumulate) {
  static_assert(kFirst >= 0 && kSteps >= 0 && kFirst + kSteps <= 8, "8 K steps per tile");
  if constexpr (kSteps > 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
    // steps 0-3 sit in the first 64-key block of V's rows, 4-7 in the second (8 KB on); the two
    // 64-wide d blocks are 16 KB apart (LBO), 8-key groups 1 KB apart (SBO)
    const uint64_t bd = smem_desc_sw128(v_base + uint32_t(kFirst) * 2048u, kHalfBytes, 1024);
    const uint32_t blo = uint32_t(bd), bhi = uint32_t(bd >> 32);
    const uint32_t pa = p_tmem + uint32_t(kFirst) * 8u;
#define H3_PV_STEP(KK) \
  "add.u32 ta, %1, " #KK "*8;\n\t add.u32 lb, %2, " #KK "*128;\n\t mov.b64 db, {lb, %3};\n\t" \
  "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], db, %4, pt;\n\t"
#define H3_PV_HEAD \
  "{\n\t.reg .pred pf, pt;\n\t.reg .b32 ta, lb;\n\t.reg .b64 db;\n\t" \
  "setp.ne.b32 pf, %5, 0;\n\t setp.eq.b32 pt, %5, %5;\n\t mov.b64 db, {%2, %3};\n\t" \
  "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, pf;\n\t"
#define H3_PV_ARGS ::"r"(d_tmem), "r"(pa), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate ? 1u : 0u) : "memory"
    if constexpr (kSteps == 1) {
      asm volatile(H3_PV_HEAD "}\n" H3_PV_ARGS);
    } else if constexpr (kSteps == 2) {
      asm volatile(H3_PV_HEAD H3_PV_STEP(1) "}\n" H3_PV_ARGS);
    } else if constexpr (kSteps == 4) {
      asm volatile(H3_PV_HEAD H3_PV_STEP(1) H3_PV_STEP(2) H3_PV_STEP(3) "}\n" H3_PV_ARGS);
    } else if constexpr (kSteps == 6) {
      asm volatile(H3_PV_HEAD H3_PV_STEP(1) H3_PV_STEP(2) H3_PV_STEP(3) H3_PV_STEP(4) H3_PV_STEP(5) "}\n" H3_PV_ARGS);
    } else if constexpr (kSteps == 8) {
      asm volatile(H3_PV_HEAD H3_PV_STEP(1) H3_PV_STEP(2) H3_PV_STEP(3) H3_PV_STEP(4) H3_PV_STEP(5) H3_PV_STEP(6)
                       H3_PV_STEP(7) "}\n" H3_PV_ARGS);
    } else {
      static_assert(kSteps == 1 || kSteps == 2 || kSteps == 4 || kSteps == 6 || kSteps == 8, "step count");
    }
#undef H3_PV_ARGS
#undef H3_PV_HEAD
#undef H3_PV_STEP
  }
}

// One warp-specialised CTA (see the header). Per KV tile j and Q tile t:
//   MMA thread   waits P_t(j) chunks 0..kSplit-1 -> P_t V_j over their K steps; waits the
//                rest -> the remaining K steps -> S_t = Q_t K_{j+1}^T (overwrites P_t).
//   softmax t    waits S_t(j), loads its 128 scores, takes the row max over all 128 keys
//                (three-input max), rescales O_t when the max grew by more than 2^8, then
//                exponentiates in four 32-key chunks, storing each chunk's bf16 P into TMEM
//                and handing chunks [0, kSplit) over before computing the rest.
// So after the last exponential only (4 - kSplit) chunks of P V and one Q K^T stand between
// a tile's softmax and its next S. O_t is quiescent when S_t(j) is ready: the MMA thread
// issued every P_t V of iteration j-1 before S_t(j) = Q_t K_j^T, and its commit retires
// everything issued earlier.
// kPair: the CTA is one of a two-CTA cluster on two SMs whose tile t rows form one M = 256
// pair MMA (tcgen05 cta_group::2) issued by the even CTA's MMA thread: each SM stages half
// of every K tile (64 keys) and of every V tile (64 head-dimension columns) through a 10-stage
// ring of 16 KB halves, so a Q K^T MMA reads 6 KB of shared memory per SM instead of 8 KB and
// the per-SM K/V traffic halves. Commits reach both CTAs' barriers; the softmax warps of both
// CTAs hand P over on the even CTA's barriers (one arrival per warp).
// kEmuMask / kEmuChunks: which key pairs take the FMA-pipe exp2 (pair positions inside a
// 32-key chunk / chunks; zero: all on MUFU).
// kPingPong: the two softmax warpgroups take turns for their exponentials (a token passed
// through two mbarriers).
template <bool kPair, uint32_t kEmuMask, uint32_t kEmuChunks, int kSplit, bool kPingPong, bool kProf>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  static_assert(kSplit >= 1 && kSplit <= 4, "P hand-off after 1..4 of the 4 chunks");
  constexpr int kRing = kPair ? 2 * kStages : kStages;             // ring stages
  constexpr uint32_t kStage = kPair ? kTileBytes / 2 : kTileBytes;  // bytes per stage
  constexpr uint32_t kPCount = kPair ? 8 : 128;                     // P hand-off arrivals
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int head = blockIdx.y;
  // this CTA's rows: tile t covers [m0 + 128 t, m0 + 128 t + 128); a pair covers 512 rows
  const int m0 = kPair ? (blockIdx.x >> 1) * (2 * kRowsPerCta) + kRowsPerCta * int(rank) : blockIdx.x * kRowsPerCta;
  const int n_kv = p.n_kv_tiles;

  if (threadIdx.x == 0) {
    mbar_init(bar(kBarQFull), 1);
    for (int s = 0; s < kRing; ++s) mbar_init(bar(kBarKVFull + s), 1);
    for (int r = 0; r < kRel; ++r) mbar_init(bar(kBarRel + r), 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kBarSFull + t), 1);
      mbar_init(bar(kBarPSplit + t), kPCount);
      mbar_init(bar(kBarPLast + t), kPCount);
      mbar_init(bar(kBarODone + t), 1);
      mbar_init(bar(kBarTok + t), 128);
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
    if constexpr (kPair) {
      tmem_alloc_pair(smem_u32(tmem_slot), 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (kPair)
    cluster_sync_all();  // barriers and TMEM of both CTAs exist before anything remote touches them
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, p.status};
  const bool grid_aborted = *abort_flag != 0;
  if (warp < 4) {
    regs_dec<kRegsControl>();
    if (warp == 0) {
      // ------------------------------------------------------------ TMA producer
      // Ring order K_0, V_0, K_1, V_1, ...; in the pair form each CTA loads its halves and the
      // copies of both CTAs count on the even CTA's full barriers. The whole warp runs the loop
      // and agrees on every wait; one elected lane issues the copies.
      if (!grid_aborted) {
        const bool issuer = elect_one();
        const uint32_t sq = sbase + kOffQ;
        const uint32_t skv = sbase + kOffKV;
        if (issuer) {
          const uint32_t q_full = kPair ? mapa_shared(bar(kBarQFull), 0) : bar(kBarQFull);
          if (leader) mbar_expect_tx(bar(kBarQFull), (kPair ? 4 : 2) * kTileBytes);
          for (int t = 0; t < 2; ++t)
            for (int hh = 0; hh < 2; ++hh) {
              if constexpr (kPair)
                tma_load_3d_pair(sq + t * kTileBytes + hh * kHalfBytes, &tmap_q, q_full, hh * 64, m0 + t * kBlockM,
                                 head);
              else
                tma_load_3d(sq + t * kTileBytes + hh * kHalfBytes, &tmap_q, q_full, hh * 64, m0 + t * kBlockM, head);
            }
        }
        __syncwarp();
        int it = 0;
        for (int j = 0; j < n_kv; ++j) {
          bool ok = true;
          for (int kv = 0; kv < 2; ++kv, ++it) {
            const int st = it % kRing;
            if (it >= kRing) {
              // the stage's previous item (it - kRing) is free once release e has completed:
              // K_r (item 2r) after S_1(r), V_r (item 2r + 1) after S_1(r + 1)
              const int e = (it - kRing + 1) / 2;
              if (!__all_sync(0xffffffffu,
                              mbar_wait(bar(kBarRel + e % kRel), uint32_t(e / kRel) & 1u, ctx, kStatusTimeoutKV))) {
                ok = false;
                break;
              }
            }
            const uint32_t dst = skv + st * kStage;
            if (issuer) {
              if constexpr (kPair) {
                const uint32_t full = mapa_shared(bar(kBarKVFull + st), 0);
                if (leader) mbar_expect_tx(bar(kBarKVFull + st), kTileBytes);
                if (kv == 0) {  // K: this CTA's 64 keys, both 64-column blocks (64-row boxes)
                  for (int hh = 0; hh < 2; ++hh)
                    tma_load_3d_pair(dst + hh * (kStage / 2), &tmap_k, full, hh * 64, j * kBlockN + 64 * int(rank),
                                     head);
                } else {  // V: all 128 keys, this CTA's 64 head-dimension columns
                  tma_load_3d_pair(dst, &tmap_v, full, 64 * int(rank), j * kBlockN, head);
                }
              } else {
                const CUtensorMap* m = kv ? &tmap_v : &tmap_k;
                mbar_expect_tx(bar(kBarKVFull + st), kTileBytes);
                tma_load_3d(dst, m, bar(kBarKVFull + st), 0, j * kBlockN, head);
                tma_load_3d(dst + kHalfBytes, m, bar(kBarKVFull + st), 64, j * kBlockN, head);
              }
            }
            __syncwarp();
          }
          if (!ok) break;
        }
        // Every issued copy must land before the CTA may exit (the pair's copies all count on the
        // even CTA's barriers; the odd CTA cannot leave before the final cluster barrier).
        if (leader && issuer) {
          auto drain = [&](uint32_t b, uint32_t par) {
            if constexpr (kPair)
              pair::drain_wait_pair(b, par, p.status);
            else
              drain_wait(b, par, p.status);
          };
          drain(bar(kBarQFull), 0);
          for (int st = 0; st < kRing; ++st) {
            const int cnt = it / kRing + (st < it % kRing ? 1 : 0);
            if (cnt > 0) drain(bar(kBarKVFull + st), uint32_t(cnt - 1) & 1u);
          }
        }
        __syncwarp();
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issuer (even CTA)
      // The whole warp runs the loop and agrees on every wait; one elected lane issues the MMAs
      // and commits.
      if (leader && !grid_aborted) {
        const bool issuer = elect_one();
        const uint32_t sq = sbase + kOffQ;
        const uint32_t skv = sbase + kOffKV;
        const bool rec = blockIdx.x == 0 && blockIdx.y == 0 && issuer;
        // waits on barriers that the other CTA's threads or copies complete take cluster scope
        auto wait_x = [&](uint32_t b, uint32_t par, int code) -> bool {
          bool got;
          if constexpr (kPair)
            got = mbar_wait_cluster(b, par, ctx, code);
          else
            got = mbar_wait(b, par, ctx, code);
          return __all_sync(0xffffffffu, got);
        };
        auto wait_full = [&](int st_it) -> bool {
          return wait_x(bar(kBarKVFull + st_it % kRing), uint32_t(st_it / kRing) & 1u, kStatusTimeoutKV);
        };
        auto commit = [&](int b) {
          if (issuer) {
            if constexpr (kPair)
              mma_commit_pair(bar(b), 0x3);
            else
              mma_commit(bar(b));
          }
          __syncwarp();
        };
        auto qk = [&](int t, uint32_t k_base) {
          if (issuer) {
            if constexpr (kPair)
              pair::issue_qk_pair(tmem + col_s(t), sq + t * kTileBytes, k_base);
            else
              issue_qk(tmem + col_s(t), sq + t * kTileBytes, k_base);
          }
          __syncwarp();
        };
        auto pv_head = [&](int t, uint32_t v_base, bool acc) {
          if (issuer) {
            if constexpr (kPair)
              pair::issue_pv_pair_steps<0, 2 * kSplit>(tmem + col_o(t), tmem + col_p(t), v_base, acc);
            else
              issue_pv_steps<0, 2 * kSplit>(tmem + col_o(t), tmem + col_p(t), v_base, acc);
          }
          __syncwarp();
        };
        auto pv_tail = [&](int t, uint32_t v_base) {
          if (issuer) {
            if constexpr (kPair)
              pair::issue_pv_pair_steps<2 * kSplit, 8 - 2 * kSplit>(tmem + col_o(t), tmem + col_p(t), v_base, true);
            else
              issue_pv_steps<2 * kSplit, 8 - 2 * kSplit>(tmem + col_o(t), tmem + col_p(t), v_base, true);
          }
          __syncwarp();
        };
        bool ok = wait_x(bar(kBarQFull), 0, kStatusTimeoutQ) && wait_full(0);
        if (ok) {
          tc_fence_after();
          qk(0, skv);
          commit(kBarSFull + 0);
          qk(1, skv);
          commit(kBarSFull + 1);
        }
        for (int j = 0; ok && j < n_kv; ++j) {
          prof_mark<kProf>(p, rec, 2, j, 0);
          const int it_v = 2 * j + 1, it_k = 2 * j + 2;
          const bool next = j + 1 < n_kv;
          // smem operands arrive by TMA, ordered by the mbarrier wait alone; a tcgen05 fence is
          // needed only after the waits on P, which other threads wrote with tcgen05.st.
          if (!(ok = wait_full(it_v))) break;
          const uint32_t sv = skv + (it_v % kRing) * kStage;
          const uint32_t sk = skv + (it_k % kRing) * kStage;
          const uint32_t ph = uint32_t(j) & 1u;
          prof_mark<kProf>(p, rec, 2, j, 1);
          for (int t = 0; t < 2; ++t) {
            if (!(ok = wait_x(bar(kBarPSplit + t), ph, kStatusTimeoutP))) break;
            prof_mark<kProf>(p, rec, 2, j, 2 + 3 * t);
            tc_fence_after();
            pv_head(t, sv, j > 0);
            if (!(ok = wait_x(bar(kBarPLast + t), ph, kStatusTimeoutP))) break;
            prof_mark<kProf>(p, rec, 2, j, 3 + 3 * t);
            tc_fence_after();
            pv_tail(t, sv);
            // every tcgen05.commit drains the tensor pipe (~100 clk), so a tile commits once per
            // iteration (S ready, which also certifies its P V) and O only after the last P V
            if (!next) commit(kBarODone + t);
            if (next) {
              if (t == 0 && !(ok = wait_full(it_k))) break;  // overlaps the queued P*V work
              qk(t, sk);
              commit(kBarSFull + t);
            }
            prof_mark<kProf>(p, rec, 2, j, 4 + 3 * t);
          }
        }
        // Every issued MMA must retire before TMEM is released.
        if (issuer) {
          if constexpr (kPair) {
            mma_commit_pair(bar(kBarDrain), 0x1);
            pair::drain_wait_pair(bar(kBarDrain), 0, p.status);
          } else {
            mma_commit(bar(kBarDrain));
            drain_wait(bar(kBarDrain), 0, p.status);
          }
        }
        __syncwarp();
      }
    }
  } else {
    regs_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;  // Q tile
    const int quad = warp & 3;      // TMEM lane quadrant this warp may access
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + col_s(t);
    const uint32_t tP = tmem + lane_off + col_p(t);
    const uint32_t tO = tmem + lane_off + col_o(t);
    const float c = p.scale_log2;
    const uint64_t c2 = f2_pack(c, c);
    const int tail_valid = p.s_kv - (n_kv - 1) * kBlockN;
    float m_run = -INFINITY;
    uint64_t l_a = f2_pack(0.f, 0.f), l_b = f2_pack(0.f, 0.f);  // packed partial row sums
    bool ok = !grid_aborted;
    const bool rec = blockIdx.x == 0 && blockIdx.y == 0 && quad == 0 && lane == 0;
    // P hand-off: every thread's stores are complete and fenced; then one arrival per thread on
    // this CTA's barrier, or (pair form) one per warp on the even CTA's barrier
    auto hand_over = [&](int b) {
      tmem_st_wait();
      tc_fence_before();
      if constexpr (kPair) {
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(bar(b), 0));
      } else {
        mbar_arrive(bar(b));
      }
    };

    for (int j = 0; ok && j < n_kv; ++j) {
      prof_mark<kProf>(p, rec, t, j, 0);
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarSFull + t), uint32_t(j) & 1u, ctx, kStatusTimeoutS));
      if (!ok) break;
      // S_1(j) ready: every MMA reading K_j and V_(j-1) has retired; hand their stages back
      if (t == 1 && quad == 0 && lane == 0) mbar_arrive(bar(kBarRel + j % kRel));
      prof_mark<kProf>(p, rec, t, j, 1);
      tc_fence_after();
      // S in two 64-column halves: the second half's load is in flight while the first half's
      // maximum is taken
      uint32_t sa[64], sb[64];
      tmem_ld64_wait(tS, sa);
      tmem_ld64_nowait(tS + 64, sb);
      float s[128];
#pragma unroll
      for (int i = 0; i < 64; ++i) s[i] = __uint_as_float(sa[i]);
      const bool tail = j == n_kv - 1 && tail_valid < kBlockN;
      if (tail) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= tail_valid) s[i] = -INFINITY;
      }
      // row max over the tile's 128 keys: four chains of three-input maxima
      float mx0 = fmax3(s[0], s[1], s[2]), mx1 = fmax3(s[3], s[4], s[5]);
      float mx2 = fmax3(s[6], s[7], s[8]), mx3 = fmax3(s[9], s[10], s[11]);
#pragma unroll
      for (int i = 12; i < 60; i += 8) {
        mx0 = fmax3(mx0, s[i], s[i + 1]);
        mx1 = fmax3(mx1, s[i + 2], s[i + 3]);
        mx2 = fmax3(mx2, s[i + 4], s[i + 5]);
        mx3 = fmax3(mx3, s[i + 6], s[i + 7]);
      }
      mx0 = fmax3(mx0, s[60], s[61]);
      mx1 = fmax3(mx1, s[62], s[63]);
      tmem_ld64_wait_on(sb);
#pragma unroll
      for (int i = 0; i < 64; ++i) s[64 + i] = __uint_as_float(sb[i]);
      if (tail) {
#pragma unroll
        for (int i = 64; i < 128; ++i)
          if (i >= tail_valid) s[i] = -INFINITY;
      }
      prof_mark<kProf>(p, rec, t, j, 2);
#pragma unroll
      for (int i = 64; i < 120; i += 8) {
        mx0 = fmax3(mx0, s[i], s[i + 1]);
        mx1 = fmax3(mx1, s[i + 2], s[i + 3]);
        mx2 = fmax3(mx2, s[i + 4], s[i + 5]);
        mx3 = fmax3(mx3, s[i + 6], s[i + 7]);
      }
      mx0 = fmax3(mx0, s[120], s[121]);
      mx1 = fmax3(mx1, s[122], s[123]);
      mx2 = fmax3(mx2, s[124], s[125]);
      mx3 = fmax3(mx3, s[126], s[127]);
      const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c);
      if (j == 0) {
        m_run = m_new;
      } else {
        // Rescale O (and l) of the rows whose running max grew by more than 2^8. O_t is
        // quiescent here (S_t(j) ready implies every earlier P_t V has retired).
        const bool need = m_new > m_run + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float f = need ? ex2_approx(m_run - m_new) : 1.0f;
          if (need) {
            l_a = f2_fma(l_a, f2_pack(f, f), f2_pack(0.f, 0.f));
            l_b = f2_fma(l_b, f2_pack(f, f), f2_pack(0.f, 0.f));
            m_run = m_new;
          }
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
      prof_mark<kProf>(p, rec, t, j, 3);
      if (kPingPong && (t == 1 || j > 0)) {
        const uint32_t par = t == 0 ? uint32_t(j - 1) & 1u : uint32_t(j) & 1u;
        ok = __all_sync(0xffffffffu, mbar_wait(bar(kBarTok + t), par, ctx, kStatusTimeoutS));
        if (!ok) break;
      }
      // exponentials in four 32-key chunks, each stored as bf16 P as soon as it is done; the
      // fp32 values stay in s[] for the row sum, which is taken after P has been handed over
      const uint64_t nm2 = f2_pack(-m_run, -m_run);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int e = 32 * k + 2 * i;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(s[e], s[e + 1]), c2, nm2), x0, x1);
          ex2_pair<kEmuMask, kEmuChunks>(x0, x1, k, i, s[e], s[e + 1]);
          pk[i] = pack_bf16x2(s[e], s[e + 1]);
        }
        tmem_st16(tP + 16 * k, pk);
        if (k == kSplit - 1) {
          hand_over(kBarPSplit + t);
          prof_mark<kProf>(p, rec, t, j, 4);
        }
      }
      if (kPingPong) mbar_arrive(bar(kBarTok + (t ^ 1)));  // hand the exp phase over
      hand_over(kBarPLast + t);
      prof_mark<kProf>(p, rec, t, j, 5);
#pragma unroll
      for (int i = 0; i < 128; i += 4) {
        l_a = f2_add(l_a, f2_pack(s[i], s[i + 1]));
        l_b = f2_add(l_b, f2_pack(s[i + 2], s[i + 3]));
      }
    }
    float la0, la1, lb0, lb1;
    f2_unpack(l_a, la0, la1);
    f2_unpack(l_b, lb0, lb1);
    const float l_run = (la0 + la1) + (lb0 + lb1);
    if (ok) {
      ok = __all_sync(0xffffffffu,
                      mbar_wait(bar(kBarODone + t), 0, ctx, kStatusTimeoutO));
    }
    // Peer outputs (o_peer) are staged in this tile's Q buffer (its last Q*K^T has retired) and
    // stored as whole 256-byte rows, 16 threads per row, so every warp store writes two contiguous
    // rows across NVLink instead of 32 scattered 16-byte pieces. Chunk c of row r sits at
    // c ^ (r & 15) in the staged row.
    const bool peer = p.o_peer != nullptr;
    const int r_in = quad * 32 + lane;
    const uint32_t stage = sbase + kOffQ + uint32_t(t) * kTileBytes;
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / l_run;
      const int row = m0 + t * kBlockM + r_in;
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
        if (peer) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            st_shared_u4(stage + uint32_t(r_in) * 256u + ((uint32_t(4 * c4 + i) ^ uint32_t(r_in & 15)) << 4),
                         make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]));
        } else if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c4 * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
    if (peer) {
      // every warp of the tile reaches this barrier (each wait above is bounded). The copy-out reads
      // rows that other warps staged, so the tile sends nothing unless all four warps finished:
      // after an abort no peer receives stale staging rows, and the status word marks the call failed
      const bool tile_ok = named_bar_and(1 + t, 128, ok);
      if (tile_ok) {
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const int kk = i * 128 + r_in;  // chunk kk & 15 of staged row kk >> 4
          const int sr = kk >> 4, ch = kk & 15;
          const long long grow = (long long)m0 + t * kBlockM + sr;
          if (grow < p.s_q) {
            const uint4 v = ld_shared_u4(stage + uint32_t(sr) * 256u + ((uint32_t(ch) ^ uint32_t(sr & 15)) << 4));
            __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.o_peer[grow / p.o_rank_rows]) +
                               (long long)head * p.o_head_stride + (grow % p.o_rank_rows) * p.o_row_stride + 8 * ch;
            *reinterpret_cast<uint4*>(d) = v;
          }
        }
      }
      __threadfence_system();  // peer stores visible before the host-side barrier
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // the pair MMAs into this CTA's TMEM have retired
  if (warp == 2) {
    tc_fence_after();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem, 512);
    else
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
      issue_pv_steps<0, 8>(tmem + 128, tmem + 64, sbase, false);
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

// Bounded-wait known-answer kernel: the path every kernel here takes when a wait runs out,
// exercised on purpose. Thread 0 starts a TMA load of one 128x128 tile (a copy in flight), then
// waits with the caller's limit on an mbarrier that nothing ever arrives on; warps 1-3 wait for
// thread 0's hand-off, which never comes. When the limit passes, the waiters record
// kStatusTimeoutKat and raise the CTA's abort flag (which also releases the other waiters),
// thread 0 drains its copy, and the CTA frees its TMEM and returns: the GPU stays usable and
// the host reads the code from the status word.
__global__ void __launch_bounds__(128, 1)
    kat_wait_kernel(const __grid_constant__ CUtensorMap tmap, int* status, unsigned long long limit_ns) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTileBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5;
  const uint32_t b_full = smem_u32(&bars[0]), b_never = smem_u32(&bars[1]), b_handoff = smem_u32(&bars[2]);
  if (threadIdx.x == 0) {
    mbar_init(b_full, 1);
    mbar_init(b_never, 1);
    mbar_init(b_handoff, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  WaitCtx ctx{abort_flag, status};
  ctx.limit_ns = limit_ns;
  if (threadIdx.x == 0) {
    mbar_expect_tx(b_full, kTileBytes);
    for (int hh = 0; hh < 2; ++hh) tma_load_3d(sbase + hh * kHalfBytes, &tmap, b_full, hh * 64, 0, 0);
    if (mbar_wait(b_never, 0, ctx, kStatusTimeoutKat)) mbar_arrive(b_handoff);
    drain_wait(b_full, 0, status);
  } else if (warp != 0) {
    mbar_wait(b_handoff, 0, ctx, kStatusTimeoutKat);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
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

// [n_heads][rows][128] bf16 with element strides (row_stride, head_stride); box 64 x box_rows x 1, SW128.
static int make_head_map(CUtensorMap* map, const void* base, long long rows, long long n_heads,
                         long long row_stride, long long head_stride, unsigned box_rows = 128) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return H3_ERR_DRIVER;
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)n_heads};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride * 2, (cuuint64_t)head_stride * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
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

// Tensor maps of one call: Q and V in 64-column x 128-row boxes; K in 128-row boxes (1-SM form)
// or 64-row boxes (pair form: each SM stages half of a K tile).
struct Maps {
  CUtensorMap q, k, k_half, v;
};

template <bool kPair, uint32_t kEmuMask, uint32_t kEmuChunks, int kSplit, bool kPingPong, bool kProf>
static int launch_variant(cudaStream_t st, const Maps& m, const Params& p) {
  auto* kern = attn_fwd_kernel<kPair, kEmuMask, kEmuChunks, kSplit, kPingPong, kProf>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
    return H3_ERR_LAUNCH;
  // one CTA per 256 query rows; the pair form launches whole two-CTA clusters (512 rows each)
  const unsigned ctas = kPair ? 2u * unsigned((p.s_q + 2 * kRowsPerCta - 1) / (2 * kRowsPerCta))
                              : unsigned((p.s_q + kRowsPerCta - 1) / kRowsPerCta);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, (unsigned)p.n_heads);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kPair ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, m.q, kPair ? m.k_half : m.k, m.v, p) != cudaSuccess) return H3_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

// Schedule variants: (SM-pair MMAs, FMA-pipe exp2 pair positions in a 32-key chunk, chunks that
// use them, P hand-off after kSplit of the 4 chunks, softmax ping-pong). Variants with the same
// exp2 placement compute bit-identical results.
template <bool kProf>
static int launch_schedule(int variant, cudaStream_t st, const Maps& m, const Params& p) {
  switch (variant) {
    case 0: return launch_variant<false, 0x0000u, 0x0u, 3, false, kProf>(st, m, p);
    case 1: return launch_variant<true, 0x0000u, 0x0u, 3, false, kProf>(st, m, p);
    case 2: return launch_variant<false, 0x0000u, 0x0u, 2, false, kProf>(st, m, p);
    case 3: return launch_variant<false, 0x0000u, 0x0u, 3, true, kProf>(st, m, p);
    case 4: return launch_variant<false, 0x5555u, 0x6u, 3, false, kProf>(st, m, p);
    case 5: return launch_variant<false, 0x1111u, 0x7u, 3, false, kProf>(st, m, p);
    case 6: return launch_variant<false, 0x4444u, 0x6u, 3, false, kProf>(st, m, p);
    case 7: return launch_variant<false, 0x0000u, 0x0u, 4, false, kProf>(st, m, p);
    case 8: return launch_variant<true, 0x5555u, 0x6u, 3, false, kProf>(st, m, p);
    default: return H3_ERR_UNSUPPORTED;
  }
}

constexpr int kDefaultVariant = 0;

static int attn_fwd_impl(const void* q, const void* k, const void* v, void* o, int64_t n_heads, int64_t s_q,
                         int64_t s_kv, int64_t q_head_stride, int64_t q_row_stride, int64_t kv_head_stride,
                         int64_t kv_row_stride, int64_t o_rank_rows, int64_t o_rank_stride, int64_t o_head_stride,
                         int64_t o_row_stride, float softmax_scale, int32_t* status, int32_t variant,
                         long long* prof, int prof_iters, void* stream,
                         const unsigned long long* o_peer = nullptr) {
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

  const long long qhs = n_heads > 1 ? q_head_stride : s_q * q_row_stride;
  const long long kvhs = n_heads > 1 ? kv_head_stride : s_kv * kv_row_stride;
  // K maps: whole 128-key tiles (1-SM form) and 64-key halves (each SM of the pair form)
  Maps m;
  int rc;
  if ((rc = make_head_map(&m.q, q, s_q, n_heads, q_row_stride, qhs)) != H3_OK) return rc;
  if ((rc = make_head_map(&m.k, k, s_kv, n_heads, kv_row_stride, kvhs)) != H3_OK) return rc;
  if ((rc = make_head_map(&m.k_half, k, s_kv, n_heads, kv_row_stride, kvhs, 64)) != H3_OK) return rc;
  if ((rc = make_head_map(&m.v, v, s_kv, n_heads, kv_row_stride, kvhs)) != H3_OK) return rc;

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
  p.prof = prof;
  p.prof_iters = prof_iters;
  p.o_peer = o_peer;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (prof != nullptr) return launch_schedule<true>(variant, st, m, p);
  return launch_schedule<false>(variant, st, m, p);
}

extern "C" int h3_attn_fwd_variant(const void* q, const void* k, const void* v, void* o, int64_t n_heads,
                                   int64_t s_q, int64_t s_kv, int64_t q_head_stride, int64_t q_row_stride,
                                   int64_t kv_head_stride, int64_t kv_row_stride, int64_t o_rank_rows,
                                   int64_t o_rank_stride, int64_t o_head_stride, int64_t o_row_stride,
                                   float softmax_scale, int32_t* status, int32_t variant, void* stream) {
  return attn_fwd_impl(q, k, v, o, n_heads, s_q, s_kv, q_head_stride, q_row_stride, kv_head_stride, kv_row_stride,
                       o_rank_rows, o_rank_stride, o_head_stride, o_row_stride, softmax_scale, status, variant,
                       nullptr, 0, stream);
}

extern "C" int h3_attn_fwd_profile(const void* q, const void* k, const void* v, void* o, int64_t n_heads,
                                   int64_t s_q, int64_t s_kv, int64_t q_head_stride, int64_t q_row_stride,
                                   int64_t kv_head_stride, int64_t kv_row_stride, int64_t o_rank_rows,
                                   int64_t o_rank_stride, int64_t o_head_stride, int64_t o_row_stride,
                                   float softmax_scale, int32_t* status, int32_t variant, long long* trace,
                                   int64_t trace_iters, void* stream) {
  if (!trace || trace_iters < 1 || trace_iters > (1 << 20)) return H3_ERR_SHAPE;
  return attn_fwd_impl(q, k, v, o, n_heads, s_q, s_kv, q_head_stride, q_row_stride, kv_head_stride, kv_row_stride,
                       o_rank_rows, o_rank_stride, o_head_stride, o_row_stride, softmax_scale, status, variant, trace,
                       (int)trace_iters, stream);
}

extern "C" int h3_attn_fwd(const void* q, const void* k, const void* v, void* o, int64_t n_heads, int64_t s_q,
                           int64_t s_kv, int64_t q_head_stride, int64_t q_row_stride, int64_t kv_head_stride,
                           int64_t kv_row_stride, int64_t o_rank_rows, int64_t o_rank_stride, int64_t o_head_stride,
                           int64_t o_row_stride, float softmax_scale, int32_t* status, void* stream) {
  return h3_attn_fwd_variant(q, k, v, o, n_heads, s_q, s_kv, q_head_stride, q_row_stride, kv_head_stride,
                             kv_row_stride, o_rank_rows, o_rank_stride, o_head_stride, o_row_stride, softmax_scale,
                             status, kDefaultVariant, stream);
}

extern "C" int h3_attn_fwd_peer(const void* q, const void* k, const void* v, void* o_local, const uint64_t* o_peer,
                                int64_t n_ranks, int64_t n_heads, int64_t s_q, int64_t s_kv, int64_t q_head_stride,
                                int64_t q_row_stride, int64_t kv_head_stride, int64_t kv_row_stride,
                                int64_t o_rank_rows, int64_t o_head_stride, int64_t o_row_stride, float softmax_scale,
                                int32_t* status, void* stream) {
  if (!o_peer) return H3_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(o_peer) & 7u) return H3_ERR_ALIGN;
  // the epilogue indexes o_peer[row / o_rank_rows]: the table must cover every query row
  if (n_ranks < 1 || n_ranks > 65536 || o_rank_rows < 1 || s_q > n_ranks * o_rank_rows) return H3_ERR_SHAPE;
  if (kDefaultVariant != 0) return H3_ERR_UNSUPPORTED;  // the peer epilogue lives in attn_fwd_kernel
  return attn_fwd_impl(q, k, v, o_local, n_heads, s_q, s_kv, q_head_stride, q_row_stride, kv_head_stride,
                       kv_row_stride, o_rank_rows, 0, o_head_stride, o_row_stride, softmax_scale, status,
                       kDefaultVariant, nullptr, 0, stream, reinterpret_cast<const unsigned long long*>(o_peer));
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

extern "C" int h3_wait_kat(const void* tile, int64_t limit_ns, int32_t* status, void* stream) {
  if (!tile || !status) return H3_ERR_NULL;
  if (!aligned16(tile) || (reinterpret_cast<uintptr_t>(status) & 3u)) return H3_ERR_ALIGN;
  if (limit_ns < 1000 || limit_ns > 10ll * 1000 * 1000 * 1000) return H3_ERR_SHAPE;
  CUtensorMap tm;
  int rc;
  if ((rc = make_head_map(&tm, tile, 128, 1, 128, 128 * 128)) != H3_OK) return rc;
  const int smem = 1024 + kTileBytes + 64;
  if (cudaFuncSetAttribute(kat_wait_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return H3_ERR_LAUNCH;
  kat_wait_kernel<<<1, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(tm, status,
                                                                            (unsigned long long)limit_ns);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}
