// CTA-pair (2-SM) tile known-answer kernels (cf. attn_sm80/microtest.py:10-26): one pair
// Q K^T and one pair P V tile through the same TMA / descriptor / tcgen05.mma.cta_group::2 path
// that the attention kernel's pair form and the projection GEMM use (operand split per
// h3_pair.cuh, TMEM layout).
#include "h3_pair.cuh"
#include "h3attn.h"

namespace h3 {
namespace pair {

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
        issue_pv_pair_steps<0, 8>(tmem + 128, tmem + 64, sb, false);
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

// ---------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [n_heads][rows][128] bf16 with element strides; box 64 x box_rows x 1, SW128.
static int make_map(CUtensorMap* map, const void* base, long long rows, long long n_heads, long long row_stride,
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
