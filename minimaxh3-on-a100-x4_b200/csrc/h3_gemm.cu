// Token-sharded projection GEMM for the attention layer and the SwiGLU FFN:
//   C[m][n] = sum_k A[m][k] * W[n][k]      (bf16 in, fp32 accumulate, bf16 out)
// W is an nn.Linear weight ([out][in], K contiguous). It replaces the qkv_proj / out_proj calls
// of the reference's attention forward (harness/sp_runtime.py:93, :126) and the FFN's fc1 and
// swiglu-into-fc2 linears (harness/sp_blockloop.py:169-170).
//
// Every output row is computed by exactly one tile with one fixed K order (64-wide k-blocks in
// ascending order, four K=16 MMAs each, no split-K), so a row's result does not depend on how
// many rows the call has or where the row sits: token-sharded calls on W ranks give the same
// bits as the 1-GPU call, which is what makes the W-way layer bit-exact.
//
// Layout: persistent clusters of two CTAs (one per SM). A pair tile is 256 rows x 256 columns:
// CTA r stages A rows [128r, 128r+128) and W rows for columns [128r, 128r+128), and the leader's
// single thread issues tcgen05.mma.cta_group::2 (M=256, N=256, K=16), leaving each CTA a
// 128 x 256 fp32 accumulator in TMEM. Two accumulators (512 columns) alternate between tiles so
// the epilogue of one tile overlaps the main loop of the next. A is read through a 3-D tensor
// map [chunks][rows][chunk_cols]: plain row-major A is one chunk; the head->seq receive buffer
// [H][rows][128] is read in place as A[rows][H*128] (out_proj without an unpack pass).
// SwiGLU epilogue: W holds [gate; up] (2F rows); CTA 0 stages gate rows, CTA 1 the matching up
// rows, so accumulator column c (gate) and c + 128 (up) of a row sit in the same thread.
#include <algorithm>

#include "h3_ptx.cuh"
#include "h3attn.h"

namespace h3 {
namespace gemm {

constexpr int kThreads = 192;  // warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps 2..5 epilogue
constexpr int kStages = 6;
constexpr uint32_t kTileBytes = 128u * 64u * 2u;  // 128 rows x 64 bf16 (one SW128 block)
constexpr uint32_t kStageBytes = 2 * kTileBytes;  // A tile + W tile
constexpr uint32_t kOffBars = kStages * kStageBytes;
// Every tcgen05.commit drains the tensor pipe (~100 clk), against 512 clk of MMA work per k-block,
// so ring stages are released kRelEvery k-blocks at a time: release e (one commit, reaching both
// CTAs) frees the stages of k-blocks [kRelEvery e, kRelEvery e + kRelEvery). The producer waits
// release (it - kStages) / kRelEvery before reusing a stage; release barriers are used round
// robin, and with kRel > (kStages - 1) / kRelEvery every parity wait stays within one phase.
constexpr int kRelEvery = 2;
constexpr int kRel = 3;
static_assert(kRel * kRelEvery > kStages - 1, "release barriers too few for the ring");
enum : int {
  kFull = 0,                      // leader: both CTAs' A and W tiles of a stage landed
  kRelease = kFull + kStages,     // both: k-block group consumed (multicast commit), round robin
  kAccFull = kRelease + kRel,     // both: accumulator b complete (multicast commit)
  kAccEmpty = kAccFull + 2,       // leader: accumulator b drained by the epilogue warps of both CTAs
  kDrain = kAccEmpty + 2,         // leader: every issued MMA retired
  kNumBars = kDrain + 1
};
constexpr uint32_t kSmemBytes = 1024 + kOffBars + kNumBars * 8 + 16;

struct Params {
  int m, n_out, n_kb, kc_blocks;  // k-block kb reads A chunk kb / kc_blocks at column 64 * (kb % kc_blocks)
  int n_m, n_n, n_tiles;
  int swiglu, f;                  // swiglu: CTA r's W rows start at r * f + 128 * nb
  int group_m;                    // rasterisation: row tiles per group (their A rows stay in L2)
  __nv_bfloat16* c;
  long long ldc;
  int* status;
};

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& mb, int& nb) {
  const int per_group = p.group_m * p.n_n;
  const int group = t / per_group;
  const int first_m = group * p.group_m;
  const int gm = min(p.group_m, p.n_m - first_m);
  const int r = t - group * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// One 64-wide k-block: four M=256 N=256 K=16 pair MMAs (descriptors step 32 B along K).
__device__ __forceinline__ void issue_kblock(uint32_t d_tmem, uint32_t a_base, uint32_t b_base, bool accumulate) {
  constexpr uint32_t idesc = idesc_bf16_f32(256, 256, 0, 0);
  const uint64_t ad = smem_desc_sw128(a_base, 16, 1024), bd = smem_desc_sw128(b_base, 16, 1024);
  const uint32_t alo = uint32_t(ad), ahi = uint32_t(ad >> 32), blo = uint32_t(bd), bhi = uint32_t(bd >> 32);
#define H3_GEMM_STEP(O) \
  "add.u32 la, %1, " #O ";\n\t add.u32 lb, %3, " #O ";\n\t" \
  "mov.b64 da, {la, %2};\n\t mov.b64 db, {lb, %4};\n\t" \
  "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, pt;\n\t"
  asm volatile(
      "{\n\t.reg .pred pf, pt;\n\t.reg .b32 la, lb;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 pf, %6, 0;\n\t setp.eq.b32 pt, %6, %6;\n\t"
      "mov.b64 da, {%1, %2};\n\t mov.b64 db, {%3, %4};\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, pf;\n\t"
      H3_GEMM_STEP(2) H3_GEMM_STEP(4) H3_GEMM_STEP(6)
      "}\n" ::"r"(d_tmem), "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
#undef H3_GEMM_STEP
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void drain_wait_cluster(uint32_t bar, uint32_t parity, int* status) {
  uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_acq_cluster(bar, parity)) {
    if (globaltimer_ns() - t0 > H3_WAIT_LIMIT_NS) {
      atomicCAS(status, 0, kStatusTimeoutDrain);
      return;
    }
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cid = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(bar(kFull + s), 1);
    for (int r = 0; r < kRel; ++r) mbar_init(bar(kRelease + r), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kAccFull + b), 1);
      mbar_init(bar(kAccEmpty + b), 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(bar(kDrain), 1);
    *abort_flag = (*reinterpret_cast<volatile int*>(p.status) != 0) ? 1 : 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
  }
  tc_fence_before();
  cluster_sync_all();  // barriers and TMEM of both CTAs exist before anything remote touches them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const WaitCtx ctx{abort_flag, p.status};
  const bool grid_aborted = *abort_flag != 0;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    // The whole warp runs the loop and agrees on every wait; one elected lane issues the copies.
    if (!grid_aborted) {
      const bool issuer = elect_one();
      int it = 0;
      bool ok = true;
      for (int t = cid; ok && t < p.n_tiles; t += n_clusters) {
        int mb, nb;
        tile_coords(p, t, mb, nb);
        const int a_row = mb * 256 + 128 * int(rank);
        const int w_row = p.swiglu ? int(rank) * p.f + 128 * nb : nb * 256 + 128 * int(rank);
        for (int kb = 0; kb < p.n_kb; ++kb, ++it) {
          const int st = it % kStages;
          if (it >= kStages) {
            const int e = (it - kStages) / kRelEvery;
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(bar(kRelease + e % kRel), uint32_t(e / kRel) & 1u, ctx,
                                                        kStatusTimeoutKV))))
              break;
          }
          if (issuer) {
            if (rank == 0) mbar_expect_tx(bar(kFull + st), 2 * kStageBytes);
            const uint32_t full_leader = mapa_shared(bar(kFull + st), 0);
            const uint32_t dst = sbase + st * kStageBytes;
            tma_load_3d_pair(dst, &tmap_a, full_leader, 64 * (kb % p.kc_blocks), a_row, kb / p.kc_blocks);
            tma_load_3d_pair(dst + kTileBytes, &tmap_w, full_leader, 64 * kb, w_row, 0);
          }
          __syncwarp();
        }
      }
      if (rank == 0 && issuer) {
        // every copy of both CTAs counts on the leader's barriers: drain them before exit
        for (int st = 0; st < kStages; ++st) {
          const int cnt = it / kStages + (st < it % kStages ? 1 : 0);
          if (cnt > 0) drain_wait_cluster(bar(kFull + st), uint32_t(cnt - 1) & 1u, p.status);
        }
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    // The whole warp runs the loop and agrees on every wait; one elected lane issues the MMAs and
    // commits (a lane-0-only issuer falls behind when other warps issue at full rate).
    if (rank == 0 && !grid_aborted) {
      const bool issuer = elect_one();
      int it = 0, i = 0;
      bool ok = true;
      for (int t = cid; ok && t < p.n_tiles; t += n_clusters, ++i) {
        const int b = i & 1;
        // accumulator b is free once the epilogue drained the tile that used it two tiles ago
        if (!(ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar(kAccEmpty + b), (uint32_t(i >> 1) & 1u) ^ 1u, ctx,
                                                             kStatusTimeoutO))))
          break;
        tc_fence_after();
        const uint32_t d = tmem + 256u * b;
        for (int kb = 0; kb < p.n_kb; ++kb, ++it) {
          const int st = it % kStages;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait_cluster(bar(kFull + st), uint32_t(it / kStages) & 1u, ctx,
                                                               kStatusTimeoutKV))))
            break;
          tc_fence_after();
          const uint32_t a_base = sbase + st * kStageBytes;
          if (issuer) {
            issue_kblock(d, a_base, a_base + kTileBytes, kb > 0);
            if (it % kRelEvery == kRelEvery - 1) mma_commit_pair(bar(kRelease + (it / kRelEvery) % kRel), 0x3);
          }
          __syncwarp();
        }
        if (ok && issuer) mma_commit_pair(bar(kAccFull + b), 0x3);
        __syncwarp();
      }
      if (issuer) {
        mma_commit_pair(bar(kDrain), 0x1);
        drain_wait_cluster(bar(kDrain), 0, p.status);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int quad = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    bool ok = !grid_aborted;
    int i = 0;
    for (int t = cid; ok && t < p.n_tiles; t += n_clusters, ++i) {
      const int b = i & 1;
      int mb, nb;
      tile_coords(p, t, mb, nb);
      ok = __all_sync(0xffffffffu, mbar_wait(bar(kAccFull + b), uint32_t(i >> 1) & 1u, ctx, kStatusTimeoutS));
      if (!ok) break;
      tc_fence_after();
      const int row = mb * 256 + 128 * int(rank) + quad * 32 + lane;
      const bool valid = row < p.m;
      const uint32_t acc = tmem + lane_off + 256u * b;
      if (!p.swiglu) {
        const int n0 = nb * 256;
        __nv_bfloat16* dst = p.c + (long long)(valid ? row : 0) * p.ldc + n0;
#pragma unroll 1
        for (int c32 = 0; c32 < 8; ++c32) {
          uint32_t r[32];
          tmem_ld32_wait(acc + 32 * c32, r);
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) w[e] = pack_bf16x2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
          if (valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (n0 + 32 * c32 + 8 * q < p.n_out)
                *reinterpret_cast<uint4*>(dst + 32 * c32 + 8 * q) = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2],
                                                                                w[4 * q + 3]);
          }
        }
      } else {
        // out = bf16(bf16(silu(g)) * u), g and u the bf16-rounded gate / up projections
        const int n0 = nb * 128;
        __nv_bfloat16* dst = p.c + (long long)(valid ? row : 0) * p.ldc + n0;
#pragma unroll 1
        for (int c32 = 0; c32 < 4; ++c32) {
          uint32_t g[32], u[32];
          tmem_ld32_wait(acc + 32 * c32, g);
          tmem_ld32_wait(acc + 128 + 32 * c32, u);
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float v[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float gx = bf16_round(__uint_as_float(g[2 * e + h]));
              const float ux = bf16_round(__uint_as_float(u[2 * e + h]));
              const float sx = bf16_round(gx / (1.0f + __expf(-gx)));
              v[h] = sx * ux;
            }
            w[e] = pack_bf16x2(v[0], v[1]);
          }
          if (valid) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(dst + 32 * c32 + 8 * q) = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2],
                                                                              w[4 * q + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(bar(kAccEmpty + b), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs into this CTA's TMEM have retired; nothing remote is pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ---------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [outer][rows][inner] bf16 with element strides; box 64 x 128 x 1, SW128, zero fill out of range.
static int make_map(CUtensorMap* map, const void* base, long long inner, long long rows, long long outer,
                    long long row_stride, long long outer_stride) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) != cudaSuccess ||
      qres != cudaDriverEntryPointSuccess)
    return H3_ERR_DRIVER;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)outer};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride * 2, (cuuint64_t)outer_stride * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = reinterpret_cast<EncodeTiledFn>(fn)(
      map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3_OK : H3_ERR_TENSOR_MAP;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace gemm
}  // namespace h3

using namespace h3::gemm;

extern "C" int h3_gemm_bf16(const void* a, int64_t m, int64_t a_chunks, int64_t a_chunk_cols, int64_t a_chunk_stride,
                            int64_t a_row_stride, const void* w, int64_t n_out, int64_t w_row_stride, void* c,
                            int64_t c_row_stride, int32_t epilogue, int32_t* status, void* stream) {
  if (!a || !w || !c || !status) return H3_ERR_NULL;
  if (!aligned16(a) || !aligned16(w) || !aligned16(c)) return H3_ERR_ALIGN;
  if (m < 1 || a_chunks < 1 || a_chunk_cols < 8 || n_out < 8 || (epilogue != 0 && epilogue != 1)) return H3_ERR_SHAPE;
  if (m > (1ll << 31) - 256 || a_chunks > 65535 || a_chunk_cols * a_chunks > (1ll << 24)) return H3_ERR_SHAPE;
  if (a_chunk_cols % 8 || (a_chunks > 1 && a_chunk_cols % 64) || n_out % 8) return H3_ERR_SHAPE;
  if (epilogue == 1 && n_out % 128) return H3_ERR_SHAPE;
  if (a_row_stride % 8 || a_row_stride < a_chunk_cols || w_row_stride % 8 || c_row_stride % 8 ||
      w_row_stride < a_chunk_cols * a_chunks || c_row_stride < n_out)
    return H3_ERR_STRIDE;
  if (a_chunks > 1 && (a_chunk_stride % 8 || a_chunk_stride < m * a_row_stride)) return H3_ERR_STRIDE;
  const long long k = a_chunk_cols * a_chunks;
  const long long w_rows = epilogue == 1 ? 2 * n_out : n_out;
  CUtensorMap ta, tw;
  int rc;
  if ((rc = make_map(&ta, a, a_chunk_cols, m, a_chunks, a_row_stride, a_chunks > 1 ? a_chunk_stride : m * a_row_stride)) !=
      H3_OK)
    return rc;
  if ((rc = make_map(&tw, w, k, w_rows, 1, w_row_stride, w_rows * w_row_stride)) != H3_OK) return rc;
  Params p;
  p.m = (int)m;
  p.n_out = (int)n_out;
  p.kc_blocks = (int)((a_chunk_cols + 63) / 64);
  p.n_kb = p.kc_blocks * (int)a_chunks;
  p.n_m = (int)((m + 255) / 256);
  p.n_n = epilogue == 1 ? (int)(n_out / 128) : (int)((n_out + 255) / 256);
  p.n_tiles = p.n_m * p.n_n;
  p.swiglu = epilogue;
  p.f = (int)n_out;
  p.c = reinterpret_cast<__nv_bfloat16*>(c);
  p.ldc = c_row_stride;
  p.status = status;
  // Consecutive tiles walk every column tile of a group of 16 row tiles: the group's A rows are
  // reused from L2 while W streams past, and W is read from DRAM once per group. Under the power
  // cap less DRAM traffic means a higher clock: at M=42000, groups of 16 run the qkv / fc1 / fc2
  // shapes 5-11 % faster than groups of 8 (4 and 24 are slower; column-major groups are equal).
  p.group_m = 16;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return H3_ERR_CUDA;
  const int clusters = std::max(1, std::min(p.n_tiles, sms / 2));
  if (cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
    return H3_ERR_LAUNCH;
  gemm_kernel<<<2 * clusters, kThreads, kSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(ta, tw, p);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}
