// CTA-pair (2-SM) MMA building blocks: tcgen05.mma.cta_group::2 with M = 256, issued by the
// even CTA of a two-CTA cluster for both. Each CTA holds 128 rows of A and of D (in its own
// TMEM) and half of B (N/2):
//   S = Q K^T: B = K split by keys (CTA r holds keys [64r, 64r+64) of a 128-key tile)
//   O += P V : B = V split by head dimension (CTA r holds d in [64r, 64r+64))
// Used by the attention kernel's pair form and by the pair tile known-answer kernels.
#pragma once
#include "h3_ptx.cuh"

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

// O (+)= P V over K steps [kFirst, kFirst + kSteps) of a 128-key tile (16 keys per step) for the
// pair: P from TMEM, 8 columns per step; V = this CTA's 64 d-columns of the tile (MN-major, one
// SW128 block, 8-key groups 1 KB apart, steps 2 KB apart). `accumulate` applies to the first
// step. One asm block per call.
template <int kFirst, int kSteps>
__device__ __forceinline__ void issue_pv_pair_steps(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_base,
                                                    bool accumulate) {
  static_assert(kFirst >= 0 && kSteps >= 0 && kFirst + kSteps <= 8, "8 K steps per tile");
  if constexpr (kSteps > 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(256, 128, 0, 1);
    const uint64_t bd = smem_desc_sw128(v_base + uint32_t(kFirst) * 2048u, kHalfV, 1024);
    const uint32_t blo = uint32_t(bd), bhi = uint32_t(bd >> 32);
    const uint32_t pa = p_tmem + uint32_t(kFirst) * 8u;
#define H3_PV2_STEP(KK) \
  "add.u32 ta, %1, " #KK "*8;\n\t add.u32 lb, %2, " #KK "*128;\n\t mov.b64 db, {lb, %3};\n\t" \
  "tcgen05.mma.cta_group::2.kind::f16 [%0], [ta], db, %4, pt;\n\t"
#define H3_PV2_HEAD \
  "{\n\t.reg .pred pf, pt;\n\t.reg .b32 ta, lb;\n\t.reg .b64 db;\n\t" \
  "setp.ne.b32 pf, %5, 0;\n\t setp.eq.b32 pt, %5, %5;\n\t mov.b64 db, {%2, %3};\n\t" \
  "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], db, %4, pf;\n\t"
#define H3_PV2_ARGS ::"r"(d_tmem), "r"(pa), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate ? 1u : 0u) : "memory"
    if constexpr (kSteps == 1) {
      asm volatile(H3_PV2_HEAD "}\n" H3_PV2_ARGS);
    } else if constexpr (kSteps == 2) {
      asm volatile(H3_PV2_HEAD H3_PV2_STEP(1) "}\n" H3_PV2_ARGS);
    } else if constexpr (kSteps == 4) {
      asm volatile(H3_PV2_HEAD H3_PV2_STEP(1) H3_PV2_STEP(2) H3_PV2_STEP(3) "}\n" H3_PV2_ARGS);
    } else if constexpr (kSteps == 6) {
      asm volatile(H3_PV2_HEAD H3_PV2_STEP(1) H3_PV2_STEP(2) H3_PV2_STEP(3) H3_PV2_STEP(4) H3_PV2_STEP(5)
                   "}\n" H3_PV2_ARGS);
    } else if constexpr (kSteps == 8) {
      asm volatile(H3_PV2_HEAD H3_PV2_STEP(1) H3_PV2_STEP(2) H3_PV2_STEP(3) H3_PV2_STEP(4) H3_PV2_STEP(5)
                       H3_PV2_STEP(6) H3_PV2_STEP(7) "}\n" H3_PV2_ARGS);
    } else {
      static_assert(kSteps == 1 || kSteps == 2 || kSteps == 4 || kSteps == 6 || kSteps == 8, "step count");
    }
#undef H3_PV2_ARGS
#undef H3_PV2_HEAD
#undef H3_PV2_STEP
  }
}

// Bounded wait (cluster-scope acquire) that ignores the abort flag: used while draining copies
// and MMAs of both CTAs before exit.
__device__ __forceinline__ void drain_wait_pair(uint32_t bar, uint32_t parity, int* status) {
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_acq_cluster_sleep(bar, parity)) {
    if (globaltimer_ns() - t0 > H3_WAIT_LIMIT_NS) {
      atomicCAS(status, 0, kStatusTimeoutDrain);
      return;
    }
  }
}

}  // namespace pair
}  // namespace h3
