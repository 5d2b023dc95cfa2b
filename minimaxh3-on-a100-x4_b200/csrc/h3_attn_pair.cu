// CTA-pair (2-SM) building blocks for the attention kernel: tcgen05.mma.cta_group::2 with
// M = 256, where each CTA of the pair holds 128 rows of A and D and half of B (N/2).
//   S = Q K^T: B = K split by keys (CTA r holds keys [64r, 64r+64) of the tile)
//   O += P V : B = V split by head dimension (CTA r holds d in [64r, 64r+64))
// This file holds the pair tile known-answer kernels (cf. attn_sm80/microtest.py:10-26) and the
// SM-pair attention kernels (schedule variants 13-15 and 20 of h3_attn_fwd_variant).
#include "h3_ptx.cuh"
#include "h3attn.h"

namespace h3 {
namespace pair {

constexpr uint32_t kQTileBytes = 128u * 128u * 2u;  // 128 rows x 128 bf16 (two 64-column SW128 blocks)
constexpr uint32_t kHalfK = 64u * 128u * 2u;        // 64 keys x 128 d (two 8 KB SW128 blocks)
constexpr uint32_t kHalfV = 128u * 64u * 2u;        // 128 keys x 64 d (one SW128 block)

// S (+)= Q K^T for the pair: A = this CTA's 128 Q rows (K-major, 64-column blocks 16 KB apart),
// B = this CTA's 64 keys (K-major, 64-column blocks 8 KB apart). Issued by the leader only.
__device__ __forceinline__ void issue_qk_pair(uint32_t d_tmem, uint32_t a_base, uint32_t b_base) {
  constexpr uint32_t idesc = idesc_bf16_f32(256, 128, 0, 0);
  const uint64_t ad = smem_desc_sw128(a_base, 16, 1024), bd = smem_desc_sw128(b_base, 16, 1024);
  const uint32_t alo = uint32_t(ad), ahi = uint32_t(ad >> 32), blo = uint32_t(bd), bhi = uint32_t(bd >> 32);
#define H3_QK2_STEP(OA, OB) \
  "add.u32 la, %1, " #OA ";\n\t add.u32 lb, %3, " #OB ";\n\t" \
  "mov.b64 da, {la, %2};\n\t mov.b64 db, {lb, %4};\n\t" \
  "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, pt;\n\t"
  asm volatile(
      "{\n\t.reg .pred pf, pt;\n\t.reg .b32 la, lb;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 pf, %0, %0;\n\t setp.eq.b32 pt, %0, %0;\n\t"
      "mov.b64 da, {%1, %2};\n\t mov.b64 db, {%3, %4};\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, pf;\n\t"
      H3_QK2_STEP(2, 2) H3_QK2_STEP(4, 4) H3_QK2_STEP(6, 6)
      H3_QK2_STEP(1024, 512) H3_QK2_STEP(1026, 514) H3_QK2_STEP(1028, 516) H3_QK2_STEP(1030, 518)
      "}\n" ::"r"(d_tmem), "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc)
      : "memory");
#undef H3_QK2_STEP
}

// O (+)= P V over 64 keys of the pair (half = 0: keys 0..63, 1: keys 64..127): P from TMEM
// at p_tmem + p_half_cols*half (8 columns per 16-key step), V = this CTA's 64 d-columns of the 128-key
// tile (MN-major, one SW128 block, 8-key groups 1 KB apart, 16-key steps 2 KB apart).
__device__ __forceinline__ void issue_pv_pair(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_base, int half,
                                              bool accumulate, uint32_t p_half_cols = 32) {
  constexpr uint32_t idesc = idesc_bf16_f32(256, 128, 0, 1);
  const uint64_t bd = smem_desc_sw128(v_base + uint32_t(half) * 4u * 2048u, kHalfV, 1024);
  const uint32_t blo = uint32_t(bd), bhi = uint32_t(bd >> 32);
  const uint32_t pa = p_tmem + uint32_t(half) * p_half_cols;
#define H3_PV2_STEP(KK) \
  "add.u32 ta, %1, " #KK "*8;\n\t add.u32 lb, %2, " #KK "*128;\n\t mov.b64 db, {lb, %3};\n\t" \
  "tcgen05.mma.cta_group::2.kind::f16 [%0], [ta], db, %4, pt;\n\t"
  asm volatile(
      "{\n\t.reg .pred pf, pt;\n\t.reg .b32 ta, lb;\n\t.reg .b64 db;\n\t"
      "setp.ne.b32 pf, %5, 0;\n\t setp.eq.b32 pt, %5, %5;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], db, %4, pf;\n\t"
      H3_PV2_STEP(1) H3_PV2_STEP(2) H3_PV2_STEP(3)
      "}\n" ::"r"(d_tmem), "r"(pa), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
#undef H3_PV2_STEP
}

__device__ __forceinline__ void drain_wait_pair(uint32_t bar, uint32_t parity, int* status) {
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_acq_cluster(bar, parity)) {
    if (globaltimer_ns() - t0 > H3_WAIT_LIMIT_NS) {
      atomicCAS(status, 0, kStatusTimeoutDrain);
      return;
    }
  }
}

// ---------------------------------------------------------------- pair KATs
// S[256][128] fp32 = Q[256][128] . K[128][128]^T with CTA r holding Q rows [128r, 128r+128)
// and keys [64r, 64r+64).
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    kat_pair_qk_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                       float* s_out, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQTileBytes + kHalfK);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t b_full = smem_u32(&bars[0]), b_done = smem_u32(&bars[1]);
  if (threadIdx.x == 0) {
    mbar_init(b_full, 1);
    mbar_init(b_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(smem_u32(tmem_slot), 128);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, status};
  if (threadIdx.x == 0) {
    const uint32_t full_leader = mapa_shared(b_full, 0);
    if (rank == 0) mbar_expect_tx(b_full, 2 * (kQTileBytes + kHalfK));
    for (int hh = 0; hh < 2; ++hh) {
      tma_load_3d_pair(sb + hh * (kQTileBytes / 2), &tmap_q, full_leader, hh * 64, 128 * rank, 0);
      tma_load_3d_pair(sb + kQTileBytes + hh * (kHalfK / 2), &tmap_k, full_leader, hh * 64, 64 * rank, 0);
    }
    if (rank == 0) {
      if (mbar_wait_cluster(b_full, 0, ctx, kStatusTimeoutKat)) {
        tc_fence_after();
        issue_qk_pair(tmem, sb, sb + kQTileBytes);
      }
      mma_commit_pair(b_done, 0x3);
    }
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait(b_done, 0, ctx, kStatusTimeoutKat));
  if (ok) {
    tc_fence_after();
    const int row = 128 * rank + warp * 32 + lane;
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t r[32];
      tmem_ld32_wait(tmem + (uint32_t(warp * 32) << 16) + c4 * 32, r);
      for (int i = 0; i < 32; ++i) s_out[row * 128 + c4 * 32 + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 128);
  }
}

// O[256][128] fp32 = P[256][128] . V[128][128]: P rows written into each CTA's TMEM as the
// softmax writes them, CTA r holding V[:, 64r:64r+64].
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    kat_pair_pv_kernel(const __nv_bfloat16* p_in, const __grid_constant__ CUtensorMap tmap_v, float* o_out,
                       int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kHalfV);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t b_full = smem_u32(&bars[0]), b_done = smem_u32(&bars[1]);
  if (threadIdx.x == 0) {
    mbar_init(b_full, 1);
    mbar_init(b_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(smem_u32(tmem_slot), 256);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, status};
  const uint32_t lane_off = uint32_t(warp * 32) << 16;
  {
    const int row = 128 * rank + warp * 32 + lane;
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
  cluster_sync_all();  // both CTAs' P are in TMEM before the leader issues
  if (threadIdx.x == 0) {
    const uint32_t full_leader = mapa_shared(b_full, 0);
    if (rank == 0) mbar_expect_tx(b_full, 2 * kHalfV);
    tma_load_3d_pair(sb, &tmap_v, full_leader, 64 * rank, 0, 0);
    if (rank == 0) {
      if (mbar_wait_cluster(b_full, 0, ctx, kStatusTimeoutKat)) {
        tc_fence_after();
        issue_pv_pair(tmem + 128, tmem + 64, sb, 0, false);
        issue_pv_pair(tmem + 128, tmem + 64, sb, 1, true);
      }
      mma_commit_pair(b_done, 0x3);
    }
  }
  const bool ok = __all_sync(0xffffffffu, mbar_wait(b_done, 0, ctx, kStatusTimeoutKat));
  if (ok) {
    tc_fence_after();
    const int row = 128 * rank + warp * 32 + lane;
    for (int c4 = 0; c4 < 4; ++c4) {
      uint32_t r[32];
      tmem_ld32_wait(tmem + lane_off + 128 + c4 * 32, r);
      for (int i = 0; i < 32; ++i) o_out[row * 128 + c4 * 32 + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 256);
  }
}

constexpr float kPairRescaleThreshold = 8.0f;  // log2 units: P <= 256

// ---------------------------------------------------------------- attention on SM pairs
// Cluster of two CTAs (one per SM), each owning ONE 128-row Q tile of the same head; the pair
// covers 256 query rows. The leader (even) CTA's MMA thread issues cta_group::2 MMAs for both:
// each SM reads only half of every K and V tile (keys / d split), and S is double-buffered in
// TMEM (S_0 columns [0,128), S_1 [128,256), O [256,384)), so S(j+1) = Q K_{j+1}^T is computed
// while the softmax works on S(j): the softmax runs back to back instead of waiting for the
// P*V -> next Q*K^T chain. Each CTA: warp 0 TMA producer + TMEM allocator, warp 1 MMA issuer
// (leader only), then one of three softmax layouts (kSoft):
//   0: warps 4..7, one query row per thread;
//   1: warps 4..11, two warps per TMEM lane quarter, each owning 64 keys of every row: the two
//      exchange their row maxima through shared memory before exponentiating, so both halves
//      use one running max per row;
//   2: warps 4..11, two warps per TMEM lane quarter, each owning 16 rows (16-lane TMEM shapes,
//      four threads per row): no exchange, the two warps of a sub-partition run independently.
// Layouts 1 and 2 put two softmax warps on every SM sub-partition to keep its MUFU unit busy.
constexpr int kPairThreads = 256;
constexpr int kSplitThreads = 384;
constexpr int kPairStages = 10;  // ring of 16 KB stages: K halves (64 keys x 128 d), V halves (128 keys x 64 d)
constexpr uint32_t kStageBytes = 16384;
constexpr uint32_t kPOffQ = 0;
constexpr uint32_t kPOffRing = kQTileBytes;
constexpr uint32_t kPOffBars = kPOffRing + kPairStages * kStageBytes;

enum PairBar : int {
  kPbQFull = 0,                             // leader: Q tiles of both CTAs landed
  kPbKVFull = 1,                            // leader: both halves of a ring stage landed
  kPbKVEmpty = kPbKVFull + kPairStages,     // both: stage free again (multicast commit)
  kPbSFull = kPbKVEmpty + kPairStages,      // both: S buffer b ready (multicast commit)
  // The hand-off barriers come one per S buffer (tile j uses [j & 1], phase j >> 1): with S
  // double-buffered a softmax warp can run one tile ahead of the slowest warp of the pair, and
  // a single barrier would then see arrivals of two tiles in one phase.
  kPbPFullA = kPbSFull + 2,                 // leader: first 64 keys of P in TMEM in both CTAs
  kPbPFullB = kPbPFullA + 2,                // leader: last 64 keys of P in both CTAs
  kPbODoneA = kPbPFullB + 2,                // both: first-half P*V retired
  kPbODone = kPbODoneA + 2,                 // both: P*V retired
  kPbDrain = kPbODone + 2,                  // leader: every issued MMA retired
  kPbCount = kPbDrain + 1
};
constexpr uint32_t kPOffX = kPOffBars + 512;  // float [2 parity][2 key half][128 rows]: row-max exchange
constexpr uint32_t kPairSmemBytes = 1024 + kPOffX + 2 * 2 * 128 * 4;
static_assert(kPbCount * 8 + 16 <= 512, "barrier block overlaps the exchange buffer");

struct PairParams {
  int s_q, s_kv, n_kv_tiles;
  float scale_log2;
  __nv_bfloat16* o;
  long long o_rank_rows, o_rank_stride, o_head_stride, o_row_stride;
  int* status;
  long long* prof;
  int prof_iters;
};

template <bool kProf>
__device__ __forceinline__ void pmark(const PairParams& p, bool rec, int role, int j, int point) {
  if (kProf && rec && j < p.prof_iters) p.prof[((long long)role * p.prof_iters + j) * 8 + point] = clock64();
}

template <bool kProf, int kSoft>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kSoft > 0 ? kSplitThreads : kPairThreads, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                     const __grid_constant__ CUtensorMap tmap_v, const PairParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPOffBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kPbCount);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int head = blockIdx.y;
  const int m0 = (blockIdx.x >> 1) * 256 + 128 * int(rank);
  const int n_kv = p.n_kv_tiles;

  if (threadIdx.x == 0) {
    mbar_init(bar(kPbQFull), 1);
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(bar(kPbKVFull + s), 1);
      mbar_init(bar(kPbKVEmpty + s), 1);
    }
    mbar_init(bar(kPbSFull + 0), 1);
    mbar_init(bar(kPbSFull + 1), 1);
    for (int b = 0; b < 2; ++b) {
      // one arrival per softmax warp of both CTAs that hands over that half of P
      mbar_init(bar(kPbPFullA + b), kSoft == 2 ? 16 : 8);
      mbar_init(bar(kPbPFullB + b), kSoft == 2 ? 16 : 8);
      mbar_init(bar(kPbODoneA + b), 1);
      mbar_init(bar(kPbODone + b), 1);
    }
    mbar_init(bar(kPbDrain), 1);
    *abort_flag = (*reinterpret_cast<volatile int*>(p.status) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_v);
    }
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers and TMEM of both CTAs exist before anything remote touches them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, p.status};
  const bool grid_aborted = *abort_flag != 0;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0 && !grid_aborted) {
      const uint32_t sq = sbase + kPOffQ;
      const uint32_t ring = sbase + kPOffRing;
      if (rank == 0) mbar_expect_tx(bar(kPbQFull), 2 * kQTileBytes);
      const uint32_t q_leader = mapa_shared(bar(kPbQFull), 0);
      for (int hh = 0; hh < 2; ++hh)
        tma_load_3d_pair(sq + hh * (kQTileBytes / 2), &tmap_q, q_leader, hh * 64, m0, head);
      int it = 0;
      bool ok = true;
      auto next_stage = [&](uint32_t& dst, uint32_t& full_leader) -> bool {
        const int st = it % kPairStages;
        if (!mbar_wait(bar(kPbKVEmpty + st), (uint32_t(it / kPairStages) & 1u) ^ 1u, ctx, kStatusTimeoutKV))
          return false;
        if (rank == 0) mbar_expect_tx(bar(kPbKVFull + st), 2 * kStageBytes);
        dst = ring + st * kStageBytes;
        full_leader = mapa_shared(bar(kPbKVFull + st), 0);
        ++it;
        return true;
      };
      auto load_k = [&](int kj) -> bool {
        uint32_t dst, fb;
        if (!next_stage(dst, fb)) return false;
        for (int hh = 0; hh < 2; ++hh)
          tma_load_3d_pair(dst + hh * (kHalfK / 2), &tmap_k, fb, hh * 64, kj * 128 + 64 * int(rank), head);
        return true;
      };
      auto load_v = [&](int vj) -> bool {
        uint32_t dst, fb;
        if (!next_stage(dst, fb)) return false;
        tma_load_3d_pair(dst, &tmap_v, fb, 64 * int(rank), vj * 128, head);
        return true;
      };
      ok = load_k(0) && (n_kv < 2 || load_k(1));
      for (int j = 0; ok && j < n_kv; ++j) {
        ok = load_v(j);
        if (ok && j + 2 < n_kv) ok = load_k(j + 2);
      }
      if (rank == 0) {
        // every copy of both CTAs counts on the leader's barriers: drain them before exit
        drain_wait_pair(bar(kPbQFull), 0, p.status);
        for (int st = 0; st < kPairStages; ++st) {
          const int cnt = it / kPairStages + (st < it % kPairStages ? 1 : 0);
          if (cnt > 0) drain_wait_pair(bar(kPbKVFull + st), uint32_t(cnt - 1) & 1u, p.status);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (rank == 0 && lane == 0 && !grid_aborted) {
      constexpr uint32_t kPHalfCols = kSoft == 2 ? 64u : 32u;
      const uint32_t sq = sbase + kPOffQ;
      const uint32_t ring = sbase + kPOffRing;
      const bool rec = blockIdx.x == 0 && blockIdx.y == 0;
      int it = 0;
      auto take = [&](uint32_t& base, int& st) -> bool {
        st = it % kPairStages;
        const bool got =
            mbar_wait_cluster(bar(kPbKVFull + st), uint32_t(it / kPairStages) & 1u, ctx, kStatusTimeoutKV);
        base = ring + st * kStageBytes;
        ++it;
        return got;
      };
      bool ok = mbar_wait_cluster(bar(kPbQFull), 0, ctx, kStatusTimeoutQ);
      for (int b = 0; ok && b < 2 && b < n_kv; ++b) {
        uint32_t kb;
        int st;
        if (!(ok = take(kb, st))) break;
        issue_qk_pair(tmem + 128u * b, sq, kb);
        mma_commit_pair(bar(kPbSFull + b), 0x3);
        mma_commit_pair(bar(kPbKVEmpty + st), 0x3);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        pmark<kProf>(p, rec, 2, j, 0);
        const int b = j & 1;
        const uint32_t ph = uint32_t(j >> 1) & 1u;
        // P halves: columns [64, 128) of the S buffer, or [32, 64) and [96, 128) for layout 2
        // (each half written over the S columns it was computed from)
        const uint32_t pcol = 128u * b + (kSoft == 2 ? 32u : 64u);
        uint32_t vb;
        int stv;
        if (!(ok = take(vb, stv))) break;
        pmark<kProf>(p, rec, 2, j, 1);
        if (!(ok = mbar_wait_cluster(bar(kPbPFullA + b), ph, ctx, kStatusTimeoutP))) break;
        pmark<kProf>(p, rec, 2, j, 2);
        tc_fence_after();
        issue_pv_pair(tmem + 256, tmem + pcol, vb, 0, j > 0, kPHalfCols);
        mma_commit_pair(bar(kPbODoneA + b), 0x3);
        if (!(ok = mbar_wait_cluster(bar(kPbPFullB + b), ph, ctx, kStatusTimeoutP))) break;
        pmark<kProf>(p, rec, 2, j, 3);
        tc_fence_after();
        issue_pv_pair(tmem + 256, tmem + pcol, vb, 1, true, kPHalfCols);
        mma_commit_pair(bar(kPbODone + b), 0x3);
        mma_commit_pair(bar(kPbKVEmpty + stv), 0x3);
        pmark<kProf>(p, rec, 2, j, 4);
        if (j + 2 < n_kv) {
          uint32_t kb;
          int stk;
          if (!(ok = take(kb, stk))) break;
          pmark<kProf>(p, rec, 2, j, 5);
          issue_qk_pair(tmem + 128u * b, sq, kb);  // S(j+2) reuses S(j)'s buffer after P(j)*V
          mma_commit_pair(bar(kPbSFull + b), 0x3);
          mma_commit_pair(bar(kPbKVEmpty + stk), 0x3);
        }
        pmark<kProf>(p, rec, 2, j, 6);
      }
      mma_commit_pair(bar(kPbDrain), 0x1);
      drain_wait_pair(bar(kPbDrain), 0, p.status);
    }
  } else if (kSoft == 1 && warp >= 4) {
    // ------------------------------------------------------------ key-split softmax + epilogue
    const int quad = warp & 3;
    const int hc = (warp - 4) >> 2;  // this warp's keys: [64 hc, 64 hc + 64) of every tile
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    const float c = p.scale_log2;
    const int tail_valid = p.s_kv - (n_kv - 1) * 128;
    float* xchg = reinterpret_cast<float*>(smem + kPOffX);
    const int r_in = quad * 32 + lane;
    const int bar_id = 1 + quad;  // named barrier of the two warps sharing this lane quarter
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = !grid_aborted;
    const bool rec = blockIdx.x == 0 && blockIdx.y == 0 && warp == 4 && lane == 0;
    for (int j = 0; j < n_kv; ++j) {
      const int b = j & 1;
      const uint32_t tS = tmem + lane_off + 128u * b;
      pmark<kProf>(p, rec, 0, j, 0);
      const bool okw =
          ok && __all_sync(0xffffffffu, mbar_wait(bar(kPbSFull + b), uint32_t(j >> 1) & 1u, ctx, kStatusTimeoutS));
      pmark<kProf>(p, rec, 0, j, 1);
      uint32_t sv[64];
      float mx = -INFINITY;
      if (okw) {
        tc_fence_after();
        tmem_ld64_wait(tS + 64u * hc, sv);
        if (j == n_kv - 1) {
          const int lim = tail_valid - 64 * hc;
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= lim) sv[i] = __float_as_uint(-INFINITY);
        }
        float x0 = __uint_as_float(sv[0]), x1 = __uint_as_float(sv[1]);
        float x2 = __uint_as_float(sv[2]), x3 = __uint_as_float(sv[3]);
#pragma unroll
        for (int i = 4; i < 64; i += 4) {
          x0 = fmaxf(x0, __uint_as_float(sv[i]));
          x1 = fmaxf(x1, __uint_as_float(sv[i + 1]));
          x2 = fmaxf(x2, __uint_as_float(sv[i + 2]));
          x3 = fmaxf(x3, __uint_as_float(sv[i + 3]));
        }
        mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
      }
      // Exchange the half maxima (slot parity b: the partner read slot b of tile j-2 before the
      // barrier of tile j-1). The barrier also orders the partner's S load before this warp's P
      // store into the same TMEM columns, and ANDs the two warps' progress flags so that both
      // leave together.
      xchg[(b * 2 + hc) * 128 + r_in] = mx;
      tc_fence_before();
      ok = named_bar_and(bar_id, 64, okw);
      if (!ok) break;
      tc_fence_after();
      const float m_tile = fmaxf(mx, xchg[(b * 2 + (hc ^ 1)) * 128 + r_in]) * c;
      pmark<kProf>(p, rec, 0, j, 2);
      if (j == 0) {
        m_run = m_tile;  // O is not written before P(0)*V (accumulate off)
      } else {
        // both warps of the quarter take the same decision per row; the key-half-0 warp
        // rescales all of O once P(j-1)*V has retired, before it hands over P(j)
        const bool need = m_tile > m_run + kPairRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float f = need ? ex2_approx(m_run - m_tile) : 1.0f;
          if (need) {
            l_run *= f;
            m_run = m_tile;
          }
          if (hc == 0) {
            const int ot = j - 1;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(bar(kPbODone + (ot & 1)), uint32_t(ot >> 1) & 1u, ctx, kStatusTimeoutO))) {
              ok = false;  // the partner learns it at the next exchange
            } else {
              tc_fence_after();
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
        }
      }
      if (ok) {
        const float neg_m = -m_run;
        uint32_t pk[32];
        float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int e = 2 * i;
          const float e0 = ex2_approx(fmaf(__uint_as_float(sv[e]), c, neg_m));
          const float e1 = ex2_approx(fmaf(__uint_as_float(sv[e + 1]), c, neg_m));
          const float e2 = ex2_approx(fmaf(__uint_as_float(sv[e + 2]), c, neg_m));
          const float e3 = ex2_approx(fmaf(__uint_as_float(sv[e + 3]), c, neg_m));
          l0 += e0;
          l1 += e1;
          l2 += e2;
          l3 += e3;
          pk[i] = pack_bf16x2(e0, e1);
          pk[i + 1] = pack_bf16x2(e2, e3);
        }
        l_run += (l0 + l1) + (l2 + l3);
        tmem_st32(tS + 64 + 32 * hc, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(bar((hc == 0 ? kPbPFullA : kPbPFullB) + b), 0));
      }
      pmark<kProf>(p, rec, 0, j, 3);
    }
    if (ok) {
      // P(n-1)*V retires after every earlier MMA of the issuing thread
      const int lt = n_kv - 1;
      const bool okw =
          __all_sync(0xffffffffu, mbar_wait(bar(kPbODone + (lt & 1)), uint32_t(lt >> 1) & 1u, ctx, kStatusTimeoutO));
      // the row sum is the two halves' sums added in one fixed order (slot parity of tile n,
      // last read at tile n-2)
      const int sb = n_kv & 1;
      xchg[(sb * 2 + hc) * 128 + r_in] = l_run;
      ok = named_bar_and(bar_id, 64, okw);
      if (ok) {
        tc_fence_after();
        const float other = xchg[(sb * 2 + (hc ^ 1)) * 128 + r_in];
        const float inv = 1.0f / (hc == 0 ? l_run + other : other + l_run);
        const int row = m0 + r_in;
        const bool valid = row < p.s_q;
        const long long rr = valid ? row : 0;
        __nv_bfloat16* dst = p.o + (rr / p.o_rank_rows) * p.o_rank_stride + (long long)head * p.o_head_stride +
                             (rr % p.o_rank_rows) * p.o_row_stride + 64 * hc;
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t o[32];
          tmem_ld32_wait(tO + 64 * hc + c2 * 32, o);
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
          if (valid) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c2 * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
        }
      }
    }
  } else if (kSoft == 2 && warp >= 4) {
    // ------------------------------------------------------------ row-split softmax + epilogue
    const int hq = (warp - 4) >> 2;  // which 16 lanes of the quarter
    const int quad = warp & 3;       // TMEM lane quarter this warp may access
    const int t0 = lane & 3, t1 = lane >> 2;  // thread holds rows t1, t1 + 8; columns 8k + 2 t0 (+1)
    const uint32_t lane_off = uint32_t(32 * quad + 16 * hq) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    const float c = p.scale_log2;
    const int tail_valid = p.s_kv - (n_kv - 1) * 128;
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_part[2] = {0.f, 0.f};  // this thread's share of each row's sum
    bool ok = !grid_aborted;
    const bool rec = blockIdx.x == 0 && blockIdx.y == 0 && (warp == 4 || warp == 8) && lane == 0;

    // Rows whose max grew by more than 2^8 rescale O and l once the P*V behind `o_bar`
    // (phase o_parity) has retired; returns false on abort.
    auto rescale = [&](const float (&m_new)[2], uint32_t o_bar, uint32_t o_parity) -> bool {
      const bool need0 = m_new[0] > m_run[0] + kPairRescaleThreshold;
      const bool need1 = m_new[1] > m_run[1] + kPairRescaleThreshold;
      if (!__any_sync(0xffffffffu, need0 || need1)) return true;
      if (!__all_sync(0xffffffffu, mbar_wait(o_bar, o_parity, ctx, kStatusTimeoutO))) return false;
      tc_fence_after();
      const float f0 = need0 ? ex2_approx(m_run[0] - m_new[0]) : 1.0f;
      const float f1 = need1 ? ex2_approx(m_run[1] - m_new[1]) : 1.0f;
      if (need0) {
        l_part[0] *= f0;
        m_run[0] = m_new[0];
      }
      if (need1) {
        l_part[1] *= f1;
        m_run[1] = m_new[1];
      }
#pragma unroll 1
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[16];
        tmem_ld_16x256b_x4_wait(tO + c4 * 32, o);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * ((i & 2) ? f1 : f0));
        tmem_st_16x256b_x4(tO + c4 * 32, o);
      }
      tmem_st_wait();
      return true;
    };

    for (int j = 0; ok && j < n_kv; ++j) {
      const int b = j & 1;
      const uint32_t tS = tmem + lane_off + 128u * b;
      pmark<kProf>(p, rec, hq, j, 0);
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kPbSFull + b), uint32_t(j >> 1) & 1u, ctx, kStatusTimeoutS));
      if (!ok) break;
      pmark<kProf>(p, rec, hq, j, 1);
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sr[32];
        tmem_ld_16x256b_x8_wait(tS + 64 * h, sr);
        float s[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = __uint_as_float(sr[i]);
        if (j == n_kv - 1 && tail_valid < 128) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = 64 * h + 8 * (i >> 2) + 2 * t0 + (i & 1);
            if (key >= tail_valid) s[i] = -INFINITY;
          }
        }
        float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
#pragma unroll
        for (int k = 1; k < 8; ++k) {
          mx0 = fmaxf(mx0, fmaxf(s[4 * k], s[4 * k + 1]));
          mx1 = fmaxf(mx1, fmaxf(s[4 * k + 2], s[4 * k + 3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float m_new[2] = {fmaxf(m_run[0], mx0 * c), fmaxf(m_run[1], mx1 * c)};
        if (j == 0 && h == 0) {
          m_run[0] = m_new[0];  // O is not written before P(0)*V (accumulate off)
          m_run[1] = m_new[1];
        } else {
          // h = 0: O holds the sum through P(j-1) (o_done of tile j-1); h = 1: through the
          // first half of P(j) (o_done_a of tile j). S(j) was issued after P(j-2)*V, so neither
          // barrier can be more than one phase behind the awaited one.
          const int ot = h == 0 ? j - 1 : j;
          if (!(ok = rescale(m_new, bar((h == 0 ? kPbODone : kPbODoneA) + (ot & 1)), uint32_t(ot >> 1) & 1u)))
            break;
        }
        const float nm0 = -m_run[0], nm1 = -m_run[1];
        float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
        uint32_t pk[16];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float e00 = ex2_approx(fmaf(s[4 * k], c, nm0));
          const float e01 = ex2_approx(fmaf(s[4 * k + 1], c, nm0));
          const float e10 = ex2_approx(fmaf(s[4 * k + 2], c, nm1));
          const float e11 = ex2_approx(fmaf(s[4 * k + 3], c, nm1));
          a0 += e00;
          a1 += e01;
          b0 += e10;
          b1 += e11;
          pk[2 * k] = pack_bf16x2(e00, e01);
          pk[2 * k + 1] = pack_bf16x2(e10, e11);
        }
        l_part[0] += a0 + a1;
        l_part[1] += b0 + b1;
        tmem_st_16x128b_x8(tS + 32 + 64 * h, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(bar((h == 0 ? kPbPFullA : kPbPFullB) + b), 0));
        pmark<kProf>(p, rec, hq, j, 2 + h);
      }
    }
    if (ok) {
      // P(n-1)*V retires after every earlier MMA of the issuing thread
      const int lt = n_kv - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kPbODone + (lt & 1)), uint32_t(lt >> 1) & 1u, ctx, kStatusTimeoutO));
    }
    if (ok) {
      tc_fence_after();
      float l0 = l_part[0], l1 = l_part[1];
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      const float inv[2] = {1.0f / l0, 1.0f / l1};
      __nv_bfloat16* dst[2];
      bool valid[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = m0 + 32 * quad + 16 * hq + t1 + 8 * r;
        valid[r] = row < p.s_q;
        const long long rr = valid[r] ? row : 0;
        dst[r] = p.o + (rr / p.o_rank_rows) * p.o_rank_stride + (long long)head * p.o_head_stride +
                 (rr % p.o_rank_rows) * p.o_row_stride;
      }
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t o[16];
        tmem_ld_16x256b_x4_wait(tO + c4 * 32, o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int col = 32 * c4 + 8 * k + 2 * t0;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const uint32_t w = pack_bf16x2(__uint_as_float(o[4 * k + 2 * r]) * inv[r],
                                           __uint_as_float(o[4 * k + 2 * r + 1]) * inv[r]);
            if (valid[r]) *reinterpret_cast<uint32_t*>(dst[r] + col) = w;
          }
        }
      }
    }
  } else if (kSoft == 0 && warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue (both CTAs)
    const int quad = warp & 3;
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    const float c = p.scale_log2;
    const int tail_valid = p.s_kv - (n_kv - 1) * 128;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = !grid_aborted;
    const bool rec = blockIdx.x == 0 && blockIdx.y == 0 && warp == 4 && lane == 0;

    // exp2 of one 64-key half against m_use; also returns the half's raw max
    auto exps = [&](const float* s, int h, float m_use, uint32_t (&pk)[32], float& lsum, float& mx) {
      const float neg_m = -m_use;
      float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
      float x0 = s[0], x1 = s[1], x2 = s[2], x3 = s[3];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const int e = 2 * i;
        x0 = fmaxf(x0, s[e]);
        x1 = fmaxf(x1, s[e + 1]);
        x2 = fmaxf(x2, s[e + 2]);
        x3 = fmaxf(x3, s[e + 3]);
        const float e0 = ex2_approx(fmaf(s[e], c, neg_m));
        const float e1 = ex2_approx(fmaf(s[e + 1], c, neg_m));
        const float e2 = ex2_approx(fmaf(s[e + 2], c, neg_m));
        const float e3 = ex2_approx(fmaf(s[e + 3], c, neg_m));
        l0 += e0;
        l1 += e1;
        l2 += e2;
        l3 += e3;
        pk[i] = pack_bf16x2(e0, e1);
        pk[i + 1] = pack_bf16x2(e2, e3);
      }
      lsum = (l0 + l1) + (l2 + l3);
      mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
    };
    // Rows whose max grew by more than 2^8 rescale O and l once the P*V behind `o_bar`
    // (phase o_parity) has retired; returns false on abort.
    auto rescale = [&](float m_new, uint32_t o_bar, uint32_t o_parity, bool& any) -> bool {
      const bool need = m_new > m_run + kPairRescaleThreshold;
      any = __any_sync(0xffffffffu, need);
      if (!any) return true;
      if (!__all_sync(0xffffffffu, mbar_wait(o_bar, o_parity, ctx, kStatusTimeoutO))) return false;
      tc_fence_after();
      const float f = need ? ex2_approx(m_run - m_new) : 1.0f;
      if (need) {
        l_run *= f;
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
      return true;
    };

    for (int j = 0; ok && j < n_kv; ++j) {
      const int b = j & 1;
      const uint32_t tS = tmem + lane_off + 128u * b;
      pmark<kProf>(p, rec, 0, j, 0);
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kPbSFull + b), uint32_t(j >> 1) & 1u, ctx, kStatusTimeoutS));
      if (!ok) break;
      pmark<kProf>(p, rec, 0, j, 1);
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
      if (j == n_kv - 1 && tail_valid < 128) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= tail_valid) s[i] = -INFINITY;
      }
      pmark<kProf>(p, rec, 0, j, 2);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (j == 0 && h == 0) {  // no running max yet: take the first half's max first
          float x = s[0];
#pragma unroll
          for (int i = 1; i < 64; ++i) x = fmaxf(x, s[i]);
          m_run = x * c;
        }
        // exponentiate against the running max and check the half's max afterwards; the rare
        // half whose max jumps by more than 2^8 rescales O and is exponentiated again.
        uint32_t pk[32];
        float lsum, mx;
        exps(s + 64 * h, h, m_run, pk, lsum, mx);
        pmark<kProf>(p, rec, 0, j, 3 + 3 * h);
        const float m_new = fmaxf(m_run, mx * c);
        bool redo = false;
        // h = 0: O holds the sum through P(j-1) (o_done of tile j-1); h = 1: through the first
        // half of P(j) (o_done_a of tile j). S(j) was issued after P(j-2)*V, so neither barrier
        // can be more than one phase behind the awaited one.
        const int ot = h == 0 ? j - 1 : j;
        if (!(ok = rescale(m_new, bar((h == 0 ? kPbODone : kPbODoneA) + (ot & 1)), uint32_t(ot >> 1) & 1u, redo)))
          break;
        if (redo) exps(s + 64 * h, h, m_run, pk, lsum, mx);
        l_run += lsum;
        tmem_st32(tS + 64 + 32 * h, pk);
        tmem_st_wait();
        if (h == 0) pmark<kProf>(p, rec, 0, j, 4);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(bar((h == 0 ? kPbPFullA : kPbPFullB) + b), 0));
        pmark<kProf>(p, rec, 0, j, 5 + 2 * h);
      }
    }
    if (ok) {
      // P(n-1)*V retires after every earlier MMA of the issuing thread
      const int lt = n_kv - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kPbODone + (lt & 1)), uint32_t(lt >> 1) & 1u, ctx, kStatusTimeoutO));
    }
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / l_run;
      const int row = m0 + quad * 32 + lane;
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
  cluster_sync_all();  // the leader's MMAs into this CTA's TMEM have retired; nothing remote is pending
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ---------------------------------------------------------------- SM pairs, two Q tiles per CTA
// The schedule of the 1-SM kernel -- two 128-row Q tiles per CTA, one softmax warpgroup per tile
// (one query row per thread), P written over columns [64,128) of S in TMEM, the next Q*K^T of a
// tile issued after its P*V -- with every MMA a cta_group::2 pair MMA on tile t of both CTAs (256
// rows): K split by keys, V split by head dimension, so each SM stages and reads only half of
// every K and V tile (6 KB of shared-memory operands per Q*K^T MMA instead of 8 KB).
constexpr int kP2Threads = 384;  // warp 0 TMA producer, warp 1 MMA (leader), warp 2 TMEM, warps 4..11 softmax
constexpr int kP2Stages = 10;    // 16 KB half tiles: K (64 keys x 128 d) or V (128 keys x 64 d)
constexpr uint32_t kP2OffQ = 0;
constexpr uint32_t kP2OffRing = 2 * kQTileBytes;
constexpr uint32_t kP2OffBars = kP2OffRing + kP2Stages * kStageBytes;
enum P2Bar : int {
  kP2QFull = 0,                       // leader: all four Q tiles of the pair landed
  kP2KVFull = 1,                      // leader: both halves of a ring stage landed
  kP2KVEmpty = kP2KVFull + kP2Stages, // both: stage consumed (multicast commit)
  kP2SFull = kP2KVEmpty + kP2Stages,  // [t] both: S_t ready (multicast commit)
  kP2PFullA = kP2SFull + 2,           // [t] leader: first 64 keys of P_t from the 8 softmax warps of both CTAs
  kP2PFullB = kP2PFullA + 2,          // [t] leader: last 64 keys
  kP2ODoneA = kP2PFullB + 2,          // [t] both: first-half P_t V retired
  kP2ODone = kP2ODoneA + 2,           // [t] both: P_t V retired
  kP2Drain = kP2ODone + 2,            // leader: every issued MMA retired
  kP2NumBars = kP2Drain + 1
};
constexpr uint32_t kP2SmemBytes = 1024 + kP2OffBars + kP2NumBars * 8 + 16;
static_assert(kP2SmemBytes <= 232448, "pair kernel shared memory exceeds the per-CTA limit");
__host__ __device__ constexpr uint32_t p2_col_s(int t) { return uint32_t(t) * 128u; }
__host__ __device__ constexpr uint32_t p2_col_p(int t) { return uint32_t(t) * 128u + 64u; }
__host__ __device__ constexpr uint32_t p2_col_o(int t) { return 256u + uint32_t(t) * 128u; }

template <bool kProf>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kP2Threads, 1)
    attn_pair2_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const PairParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kP2OffBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kP2NumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int head = blockIdx.y;
  const int m0 = (blockIdx.x >> 1) * 512 + 256 * int(rank);  // this CTA's rows: tile t = m0 + 128 t
  const int n_kv = p.n_kv_tiles;

  if (threadIdx.x == 0) {
    mbar_init(bar(kP2QFull), 1);
    for (int s = 0; s < kP2Stages; ++s) {
      mbar_init(bar(kP2KVFull + s), 1);
      mbar_init(bar(kP2KVEmpty + s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(kP2SFull + t), 1);
      mbar_init(bar(kP2PFullA + t), 8);
      mbar_init(bar(kP2PFullB + t), 8);
      mbar_init(bar(kP2ODoneA + t), 1);
      mbar_init(bar(kP2ODone + t), 1);
    }
    mbar_init(bar(kP2Drain), 1);
    *abort_flag = (*reinterpret_cast<volatile int*>(p.status) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 2) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers and TMEM of both CTAs exist before anything remote touches them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, p.status};
  const bool grid_aborted = *abort_flag != 0;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs): Q, K_0, V_0, K_1, ...
    if (lane == 0 && !grid_aborted) {
      const uint32_t sq = sbase + kP2OffQ;
      const uint32_t ring = sbase + kP2OffRing;
      if (rank == 0) mbar_expect_tx(bar(kP2QFull), 4 * kQTileBytes);
      const uint32_t q_leader = mapa_shared(bar(kP2QFull), 0);
      for (int t = 0; t < 2; ++t)
        for (int hh = 0; hh < 2; ++hh)
          tma_load_3d_pair(sq + t * kQTileBytes + hh * (kQTileBytes / 2), &tmap_q, q_leader, hh * 64, m0 + 128 * t,
                           head);
      int it = 0;
      auto next_stage = [&](uint32_t& dst, uint32_t& full_leader) -> bool {
        const int st = it % kP2Stages;
        if (!mbar_wait(bar(kP2KVEmpty + st), (uint32_t(it / kP2Stages) & 1u) ^ 1u, ctx, kStatusTimeoutKV))
          return false;
        if (rank == 0) mbar_expect_tx(bar(kP2KVFull + st), 2 * kStageBytes);
        dst = ring + st * kStageBytes;
        full_leader = mapa_shared(bar(kP2KVFull + st), 0);
        ++it;
        return true;
      };
      auto load_k = [&](int kj) -> bool {
        uint32_t dst, fb;
        if (!next_stage(dst, fb)) return false;
        for (int hh = 0; hh < 2; ++hh)
          tma_load_3d_pair(dst + hh * (kHalfK / 2), &tmap_k, fb, hh * 64, kj * 128 + 64 * int(rank), head);
        return true;
      };
      auto load_v = [&](int vj) -> bool {
        uint32_t dst, fb;
        if (!next_stage(dst, fb)) return false;
        tma_load_3d_pair(dst, &tmap_v, fb, 64 * int(rank), vj * 128, head);
        return true;
      };
      bool ok = load_k(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        ok = load_v(j);
        if (ok && j + 1 < n_kv) ok = load_k(j + 1);
      }
      if (rank == 0) {
        // every copy of both CTAs counts on the leader's barriers: drain them before exit
        drain_wait_pair(bar(kP2QFull), 0, p.status);
        for (int st = 0; st < kP2Stages; ++st) {
          const int cnt = it / kP2Stages + (st < it % kP2Stages ? 1 : 0);
          if (cnt > 0) drain_wait_pair(bar(kP2KVFull + st), uint32_t(cnt - 1) & 1u, p.status);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (rank == 0 && lane == 0 && !grid_aborted) {
      const uint32_t sq = sbase + kP2OffQ;
      const uint32_t ring = sbase + kP2OffRing;
      const bool rec = blockIdx.x == 0 && blockIdx.y == 0;
      int it = 0;
      auto take = [&](uint32_t& base, int& st) -> bool {
        st = it % kP2Stages;
        const bool got =
            mbar_wait_cluster(bar(kP2KVFull + st), uint32_t(it / kP2Stages) & 1u, ctx, kStatusTimeoutKV);
        base = ring + st * kStageBytes;
        ++it;
        return got;
      };
      bool ok = mbar_wait_cluster(bar(kP2QFull), 0, ctx, kStatusTimeoutQ);
      uint32_t kb = 0, vb = 0;
      int stk = 0, stv = 0;
      if (ok && (ok = take(kb, stk))) {
        for (int t = 0; t < 2; ++t) {
          issue_qk_pair(tmem + p2_col_s(t), sq + t * kQTileBytes, kb);
          mma_commit_pair(bar(kP2SFull + t), 0x3);
        }
        mma_commit_pair(bar(kP2KVEmpty + stk), 0x3);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        pmark<kProf>(p, rec, 2, j, 0);
        const uint32_t ph = uint32_t(j) & 1u;
        const bool next = j + 1 < n_kv;
        if (!(ok = take(vb, stv))) break;
        pmark<kProf>(p, rec, 2, j, 1);
        for (int t = 0; t < 2; ++t) {
          if (!(ok = mbar_wait_cluster(bar(kP2PFullA + t), ph, ctx, kStatusTimeoutP))) break;
          pmark<kProf>(p, rec, 2, j, 2 + 3 * t);
          tc_fence_after();
          issue_pv_pair(tmem + p2_col_o(t), tmem + p2_col_p(t), vb, 0, j > 0);
          mma_commit_pair(bar(kP2ODoneA + t), 0x3);
          if (!(ok = mbar_wait_cluster(bar(kP2PFullB + t), ph, ctx, kStatusTimeoutP))) break;
          pmark<kProf>(p, rec, 2, j, 3 + 3 * t);
          tc_fence_after();
          issue_pv_pair(tmem + p2_col_o(t), tmem + p2_col_p(t), vb, 1, true);
          mma_commit_pair(bar(kP2ODone + t), 0x3);
          if (t == 1) mma_commit_pair(bar(kP2KVEmpty + stv), 0x3);
          if (next) {
            if (t == 0 && !(ok = take(kb, stk))) break;  // overlaps the queued P*V work
            issue_qk_pair(tmem + p2_col_s(t), sq + t * kQTileBytes, kb);  // S_t(j+1) after P_t(j) V
            mma_commit_pair(bar(kP2SFull + t), 0x3);
            if (t == 1) mma_commit_pair(bar(kP2KVEmpty + stk), 0x3);
          }
          pmark<kProf>(p, rec, 2, j, 4 + 3 * t);
        }
      }
      mma_commit_pair(bar(kP2Drain), 0x1);
      drain_wait_pair(bar(kP2Drain), 0, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue (both CTAs)
    const int t = (warp - 4) >> 2;  // Q tile
    const int quad = warp & 3;      // TMEM lane quadrant this warp may access
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + p2_col_s(t);
    const uint32_t tP = tmem + lane_off + p2_col_p(t);
    const uint32_t tO = tmem + lane_off + p2_col_o(t);
    const float c = p.scale_log2;
    const int tail_valid = p.s_kv - (n_kv - 1) * 128;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = !grid_aborted;
    const bool rec = blockIdx.x == 0 && blockIdx.y == 0 && quad == 0 && lane == 0;

    // Rescale O (and l) of the rows whose running max grew by more than 2^8; `o_ready` says
    // whether every P*V accumulated so far has retired.
    auto rescale = [&](float m_new, uint32_t o_bar, uint32_t o_parity, bool o_ready) -> bool {
      const bool need = m_new > m_run + kPairRescaleThreshold;
      if (!__any_sync(0xffffffffu, need)) return true;
      if (!o_ready && !__all_sync(0xffffffffu, mbar_wait(o_bar, o_parity, ctx, kStatusTimeoutO))) return false;
      tc_fence_after();
      const float f = need ? ex2_approx(m_run - m_new) : 1.0f;
      if (need) {
        l_run *= f;
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
      return true;
    };

    for (int j = 0; ok && j < n_kv; ++j) {
      pmark<kProf>(p, rec, t, j, 0);
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kP2SFull + t), uint32_t(j) & 1u, ctx, kStatusTimeoutS));
      if (!ok) break;
      pmark<kProf>(p, rec, t, j, 1);
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
      if (j == n_kv - 1 && tail_valid < 128) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= tail_valid) s[i] = -INFINITY;
      }
      pmark<kProf>(p, rec, t, j, 2);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float mx0 = s[64 * h], mx1 = s[64 * h + 1], mx2 = s[64 * h + 2], mx3 = s[64 * h + 3];
#pragma unroll
        for (int i = 4; i < 64; i += 4) {
          mx0 = fmaxf(mx0, s[64 * h + i]);
          mx1 = fmaxf(mx1, s[64 * h + i + 1]);
          mx2 = fmaxf(mx2, s[64 * h + i + 2]);
          mx3 = fmaxf(mx3, s[64 * h + i + 3]);
        }
        const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c);
        if (j == 0 && h == 0) {
          m_run = m_new;
        } else if (h == 0) {
          // S_t(j) ready implies every earlier P_t V has retired (issued before it by the same thread)
          if (!(ok = rescale(m_new, 0, 0, true))) break;
        } else {
          if (!(ok = rescale(m_new, bar(kP2ODoneA + t), uint32_t(j) & 1u, false))) break;
        }
        pmark<kProf>(p, rec, t, j, 3 + 2 * h);
        const float neg_m = -m_run;
        float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int e = 64 * h + 2 * i;
          const float e0 = ex2_approx(fmaf(s[e], c, neg_m));
          const float e1 = ex2_approx(fmaf(s[e + 1], c, neg_m));
          const float e2 = ex2_approx(fmaf(s[e + 2], c, neg_m));
          const float e3 = ex2_approx(fmaf(s[e + 3], c, neg_m));
          l0 += e0;
          l1 += e1;
          l2 += e2;
          l3 += e3;
          pk[i] = pack_bf16x2(e0, e1);
          pk[i + 1] = pack_bf16x2(e2, e3);
        }
        l_run += (l0 + l1) + (l2 + l3);
        tmem_st32(tP + 32 * h, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(bar((h == 0 ? kP2PFullA : kP2PFullB) + t), 0));
        pmark<kProf>(p, rec, t, j, 4 + 2 * h);
      }
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kP2ODone + t), uint32_t(n_kv - 1) & 1u, ctx, kStatusTimeoutO));
    }
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / l_run;
      const int row = m0 + 128 * t + quad * 32 + lane;
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
  cluster_sync_all();  // the leader's MMAs into this CTA's TMEM have retired; nothing remote is pending
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ---------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [n_heads][rows][128] bf16 with element strides; box 64 x box_rows x 1, SW128.
int make_map(CUtensorMap* map, const void* base, long long rows, long long n_heads, long long row_stride,
             long long head_stride, int box_rows) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) != cudaSuccess ||
      qres != cudaDriverEntryPointSuccess)
    return H3_ERR_DRIVER;
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)n_heads};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride * 2, (cuuint64_t)head_stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = reinterpret_cast<EncodeTiledFn>(fn)(
      map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3_OK : H3_ERR_TENSOR_MAP;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <bool kProf>
static int launch_pair2(dim3 grid, cudaStream_t st, const CUtensorMap& tq, const CUtensorMap& tk,
                        const CUtensorMap& tv, const PairParams& pp) {
  auto* kern = attn_pair2_kernel<kProf>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kP2SmemBytes) != cudaSuccess)
    return H3_ERR_LAUNCH;
  kern<<<grid, kP2Threads, kP2SmemBytes, st>>>(tq, tk, tv, pp);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

template <bool kProf, int kSoft>
static int launch_pair(dim3 grid, cudaStream_t st, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                       const PairParams& pp) {
  auto* kern = attn_pair_kernel<kProf, kSoft>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairSmemBytes) != cudaSuccess)
    return H3_ERR_LAUNCH;
  kern<<<grid, kSoft > 0 ? kSplitThreads : kPairThreads, kPairSmemBytes, st>>>(tq, tk, tv, pp);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

// Arguments already validated by the caller (h3_attn_fwd_variant / _profile).
int launch_attn(const void* q, const void* k, const void* v, void* o, long long n_heads, long long s_q, long long s_kv,
                long long q_head_stride, long long q_row_stride, long long kv_head_stride, long long kv_row_stride,
                long long o_rank_rows, long long o_rank_stride, long long o_head_stride, long long o_row_stride,
                float scale_log2, int* status, int variant, long long* prof, int prof_iters, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_map(&tq, q, s_q, n_heads, q_row_stride, q_head_stride, 128)) != H3_OK) return rc;
  if ((rc = make_map(&tk, k, s_kv, n_heads, kv_row_stride, kv_head_stride, 64)) != H3_OK) return rc;
  if ((rc = make_map(&tv, v, s_kv, n_heads, kv_row_stride, kv_head_stride, 128)) != H3_OK) return rc;
  PairParams pp;
  pp.s_q = (int)s_q;
  pp.s_kv = (int)s_kv;
  pp.n_kv_tiles = (int)((s_kv + 127) / 128);
  pp.scale_log2 = scale_log2;
  pp.o = reinterpret_cast<__nv_bfloat16*>(o);
  pp.o_rank_rows = o_rank_rows;
  pp.o_rank_stride = o_rank_stride;
  pp.o_head_stride = o_head_stride;
  pp.o_row_stride = o_row_stride;
  pp.status = status;
  pp.prof = prof;
  pp.prof_iters = prof_iters;
  if (variant == 20) {
    dim3 grid2((unsigned)(2 * ((s_q + 511) / 512)), (unsigned)n_heads);
    return prof != nullptr ? launch_pair2<true>(grid2, st, tq, tk, tv, pp) : launch_pair2<false>(grid2, st, tq, tk, tv, pp);
  }
  dim3 grid((unsigned)(2 * ((s_q + 255) / 256)), (unsigned)n_heads);
  if (prof != nullptr) {
    if (variant == 13) return launch_pair<true, 0>(grid, st, tq, tk, tv, pp);
    if (variant == 14) return launch_pair<true, 1>(grid, st, tq, tk, tv, pp);
    if (variant == 15) return launch_pair<true, 2>(grid, st, tq, tk, tv, pp);
    return H3_ERR_UNSUPPORTED;
  }
  switch (variant) {
    case 13: return launch_pair<false, 0>(grid, st, tq, tk, tv, pp);
    case 14: return launch_pair<false, 1>(grid, st, tq, tk, tv, pp);
    case 15: return launch_pair<false, 2>(grid, st, tq, tk, tv, pp);

    default: return H3_ERR_UNSUPPORTED;
  }
}

}  // namespace pair
}  // namespace h3

using namespace h3::pair;

extern "C" int h3_tile_kat_pair_qk(const void* q, const void* k, float* s_out, int32_t* status, void* stream) {
  if (!q || !k || !s_out || !status) return H3_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(s_out)) return H3_ERR_ALIGN;
  CUtensorMap tq, tk;
  int rc;
  if ((rc = make_map(&tq, q, 256, 1, 128, 256 * 128, 128)) != H3_OK) return rc;
  if ((rc = make_map(&tk, k, 128, 1, 128, 128 * 128, 64)) != H3_OK) return rc;
  const int smem = 1024 + kQTileBytes + kHalfK + 64;
  if (cudaFuncSetAttribute(kat_pair_qk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return H3_ERR_LAUNCH;
  kat_pair_qk_kernel<<<2, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, s_out, status);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_tile_kat_pair_pv(const void* p_in, const void* v, float* o_out, int32_t* status, void* stream) {
  if (!p_in || !v || !o_out || !status) return H3_ERR_NULL;
  if (!aligned16(p_in) || !aligned16(v) || !aligned16(o_out)) return H3_ERR_ALIGN;
  CUtensorMap tv;
  int rc;
  if ((rc = make_map(&tv, v, 128, 1, 128, 128 * 128, 128)) != H3_OK) return rc;
  const int smem = 1024 + kHalfV + 64;
  if (cudaFuncSetAttribute(kat_pair_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return H3_ERR_LAUNCH;
  kat_pair_pv_kernel<<<2, 128, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(p_in), tv, o_out, status);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}
