// HBM-bound data-movement kernels around the Ulysses all-to-alls:
//   * qknorm_rope_pack: per-head RMSNorm (+ RoPE) of q and k fused with writing q, k, v
//     straight into the seq->head send layout (harness/sp_runtime.py:93-104, :69)
//   * seq_to_head_unpack: receive-side reorder of that exchange (sp_runtime.py:71)
//   * head_to_seq_unpack: head-major -> token-major rows ahead of out_proj (:125)
// All traffic is 16-byte vectors; every warp touches whole 128-byte lines.
#include "h3_ptx.cuh"
#include "h3attn.h"

namespace h3 {
namespace pack {

constexpr int kD = 128;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Per-row arithmetic of the fused pack. Lane g (0..7) of an 8-lane group holds elements
// [8g, 8g+8) and [64+8g, 64+8g+8) of one 128-element head row, so every rotary pair
// (i, i+64) is in one thread. Sum of squares: the lane's 16 squares in element order,
// then an xor-butterfly over the group (distances 4, 2, 1). All products and sums are
// separately rounded fp32 operations (no contraction) so the CPU restatement in oracle/
// reproduces every bit. `m` holds the lane's 8 rotation matrices (m00, m01, m10, m11).
__device__ __forceinline__ void norm_rope_row(const uint4& u0, const uint4& u1, const float (&wf)[16],
                                              const float4 (&m)[8], bool has_rope, float eps, uint4& o0, uint4& o1) {
  float x[16];
  bf16x8_to_f32(u0, x);
  bf16x8_to_f32(u1, x + 8);
  float acc = __fmul_rn(x[0], x[0]);
#pragma unroll
  for (int i = 1; i < 16; ++i) acc = __fadd_rn(acc, __fmul_rn(x[i], x[i]));
  const unsigned full = 0xffffffffu;
  acc = __fadd_rn(acc, __shfl_xor_sync(full, acc, 4));
  acc = __fadd_rn(acc, __shfl_xor_sync(full, acc, 2));
  acc = __fadd_rn(acc, __shfl_xor_sync(full, acc, 1));
  const float mean = __fmul_rn(acc, 0.0078125f);  // / 128, exact
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  float y[16];  // a missing weight is 1.0f: (x * r) * 1 == x * r exactly
#pragma unroll
  for (int i = 0; i < 16; ++i) y[i] = __fmul_rn(__fmul_rn(x[i], r), wf[i]);
  if (has_rope) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = y[i], b = y[8 + i];
      y[i] = __fadd_rn(__fmul_rn(m[i].x, a), __fmul_rn(m[i].y, b));
      y[8 + i] = __fadd_rn(__fmul_rn(m[i].z, a), __fmul_rn(m[i].w, b));
    }
  }
  o0 = f32_to_bf16x8(y);
  o1 = f32_to_bf16x8(y + 8);
}

// One warp per token (grid-stride): the token's rotation table row (1 KB) is loaded into
// registers once and reused for its q and k heads; the warp's four 8-lane groups walk the
// token's 2*n_heads q/k head rows, kRowsInFlight rows per group per step so that many 16-byte
// load pairs per lane are in flight, then copy its n_heads v rows unchanged (no arithmetic).
// Every lane joins every shuffle of the q/k loop (rows past the end are clamped and not stored),
// so any n_heads works.
constexpr int kRowsInFlight = 2;
constexpr int kVRowsInFlight = 4;

__global__ void __launch_bounds__(256, 2) qknorm_rope_pack_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    long long in_row_stride, const float* __restrict__ rope, long long rope_row_stride,
    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw, float eps,
    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out,
    long long s_l, int n_heads, int heads_per_rank, long long out_rank_stride, long long out_head_stride,
    const unsigned long long* __restrict__ rank_base, long long tensor_stride, long long row_offset) {
  const int lane = threadIdx.x & 31;
  const int g = lane & 7;
  const int grp = lane >> 3;
  const long long warp_id = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = ((long long)gridDim.x * blockDim.x) >> 5;
  const int n_qk = 2 * n_heads;
  // destination of head row h of tensor `tensor` (0 q, 1 k, 2 v) for token `tok`: the destination
  // rank's buffer (a peer's memory over NVLink) laid out [tensor][head][row], or one local send
  // buffer addressed by rank / head strides
  auto dst_row = [&](int tensor, int h, long long tok) -> __nv_bfloat16* {
    return rank_base != nullptr
               ? reinterpret_cast<__nv_bfloat16*>(rank_base[h / heads_per_rank]) + tensor * tensor_stride +
                     (long long)(h % heads_per_rank) * out_head_stride + (row_offset + tok) * kD
               : (tensor == 0 ? q_out : (tensor == 1 ? k_out : v_out)) + (long long)(h / heads_per_rank) * out_rank_stride +
                     (long long)(h % heads_per_rank) * out_head_stride + tok * kD;
  };
  for (long long tok = warp_id; tok < s_l; tok += n_warps) {
    float4 m[8] = {};
    if (rope != nullptr) {
      const float4* mr = reinterpret_cast<const float4*>(rope + tok * rope_row_stride) + 8 * g;
#pragma unroll
      for (int i = 0; i < 8; ++i) m[i] = __ldg(mr + i);
    }
    for (int base = 0; base < n_qk; base += 4 * kRowsInFlight) {
      int rr[kRowsInFlight];
      uint4 u[kRowsInFlight][2];
#pragma unroll
      for (int pr = 0; pr < kRowsInFlight; ++pr) {
        const int r = base + 4 * pr + grp;
        rr[pr] = r;
        const int rc = r < n_qk ? r : n_qk - 1;
        const int tensor = rc >= n_heads ? 1 : 0, h = rc - tensor * n_heads;
        const __nv_bfloat16* src = (tensor == 0 ? q : k) + tok * in_row_stride + (long long)h * kD;
        u[pr][0] = __ldg(reinterpret_cast<const uint4*>(src + 8 * g));
        u[pr][1] = __ldg(reinterpret_cast<const uint4*>(src + 64 + 8 * g));
      }
#pragma unroll
      for (int pr = 0; pr < kRowsInFlight; ++pr) {
        const int r = rr[pr];
        const int rc = r < n_qk ? r : n_qk - 1;
        const int tensor = rc >= n_heads ? 1 : 0, h = rc - tensor * n_heads;
        uint4 o0, o1;
        float wsel[16];  // this row's RMSNorm weight (L1-resident), 1.0 when absent
        const __nv_bfloat16* w = tensor == 0 ? qw : kw;
        if (w != nullptr) {
          bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(w + 8 * g)), wsel);
          bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(w + 64 + 8 * g)), wsel + 8);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) wsel[i] = 1.0f;
        }
        norm_rope_row(u[pr][0], u[pr][1], wsel, m, rope != nullptr, eps, o0, o1);
        if (r < n_qk) {
          __nv_bfloat16* dst = dst_row(tensor, h, tok);
          reinterpret_cast<uint4*>(dst + 8 * g)[0] = o0;
          reinterpret_cast<uint4*>(dst + 64 + 8 * g)[0] = o1;
        }
      }
    }
    // v rows: copies, kVRowsInFlight per 8-lane group in flight
    for (int base = 0; base < n_heads; base += 4 * kVRowsInFlight) {
      uint4 u[kVRowsInFlight][2];
#pragma unroll
      for (int pr = 0; pr < kVRowsInFlight; ++pr) {
        const int h = base + 4 * pr + grp;
        if (h < n_heads) {
          const __nv_bfloat16* src = v + tok * in_row_stride + (long long)h * kD;
          u[pr][0] = __ldg(reinterpret_cast<const uint4*>(src + 8 * g));
          u[pr][1] = __ldg(reinterpret_cast<const uint4*>(src + 64 + 8 * g));
        }
      }
#pragma unroll
      for (int pr = 0; pr < kVRowsInFlight; ++pr) {
        const int h = base + 4 * pr + grp;
        if (h < n_heads) {
          __nv_bfloat16* dst = dst_row(2, h, tok);
          reinterpret_cast<uint4*>(dst + 8 * g)[0] = u[pr][0];
          reinterpret_cast<uint4*>(dst + 64 + 8 * g)[0] = u[pr][1];
        }
      }
    }
  }
  if (rank_base != nullptr) __threadfence_system();  // peer stores visible before the host-side barrier
}

// Chunk (r, t, h) of s_l*128 contiguous elements moves to out_t[h][r*s_l ...]: grid.y
// enumerates chunks, grid.x strides 16-byte vectors inside a chunk.
__global__ void __launch_bounds__(256) seq_to_head_unpack_kernel(const uint4* __restrict__ recv,
                                                                  uint4* __restrict__ out, int world,
                                                                  int heads_per_rank, long long s_l, int n_tensors,
                                                                  long long recv_rank_stride,
                                                                  long long recv_tensor_stride,
                                                                  long long out_tensor_stride) {
  const int chunk = blockIdx.y;
  const int h = chunk % heads_per_rank;
  const int t = (chunk / heads_per_rank) % n_tensors;
  const int r = chunk / (heads_per_rank * n_tensors);
  const long long nvec = s_l * (kD / 8);
  // strides are in bf16 elements; 8 elements per uint4
  const uint4* src = recv + (r * recv_rank_stride + t * recv_tensor_stride + (long long)h * s_l * kD) / 8;
  uint4* dst = out + (t * out_tensor_stride + (long long)h * world * s_l * kD + (long long)r * s_l * kD) / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __ldg(src + i);
}

// out[j][h][:] = in[h][j][:] for 256-byte rows: one warp per row pair, 16 B per lane.
__global__ void __launch_bounds__(256) head_to_seq_unpack_kernel(const uint4* __restrict__ in,
                                                                  uint4* __restrict__ out, int n_heads,
                                                                  long long s_l) {
  const long long rows = (long long)n_heads * s_l;
  const long long first = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 4;  // 16 lanes per row
  const int l = threadIdx.x & 15;
  const long long stride = ((long long)gridDim.x * blockDim.x) >> 4;
  for (long long rid = first; rid < rows; rid += stride) {
    const long long j = rid / n_heads;  // output-major walk: consecutive rows write consecutive memory
    const int h = (int)(rid % n_heads);
    out[rid * 16 + l] = __ldg(in + ((long long)h * s_l + j) * 16 + l);
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int grid_for(long long work_items, int per_block, int max_blocks) {
  long long b = (work_items + per_block - 1) / per_block;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return (int)b;
}

}  // namespace pack
}  // namespace h3

using namespace h3::pack;

extern "C" int h3_version(void) { return H3ATTN_VERSION; }

extern "C" int h3_qknorm_rope_pack(const void* q, const void* k, const void* v, int64_t in_row_stride,
                                   const float* rope, int64_t rope_row_stride, const void* q_weight,
                                   const void* k_weight, float eps, void* q_out, void* k_out, void* v_out,
                                   int64_t s_l, int64_t n_heads, int64_t heads_per_rank, int64_t out_rank_stride,
                                   int64_t out_head_stride, void* stream) {
  if (!q || !k || !v || !q_out || !k_out || !v_out) return H3_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(q_out) || !aligned16(k_out) ||
      !aligned16(v_out) || (rope && !aligned16(rope)) || (q_weight && !aligned16(q_weight)) ||
      (k_weight && !aligned16(k_weight)))
    return H3_ERR_ALIGN;
  if (s_l < 1 || n_heads < 1 || heads_per_rank < 1 || n_heads % heads_per_rank) return H3_ERR_SHAPE;
  if (s_l > (1ll << 31) || n_heads > 65535 || s_l * 3 * n_heads > (1ll << 40)) return H3_ERR_SHAPE;
  if (in_row_stride < n_heads * 128 || (in_row_stride % 8) || (out_rank_stride % 8) || (out_head_stride % 8) ||
      (rope && (rope_row_stride < 256 || (rope_row_stride % 4))))
    return H3_ERR_STRIDE;
  if (!(eps >= 0.f)) return H3_ERR_SHAPE;
  // one warp per token, 8 warps per block, grid-stride: up to 8 resident blocks per SM
  const int blocks = grid_for(s_l, 8, 148 * 8);
  qknorm_rope_pack_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      reinterpret_cast<const __nv_bfloat16*>(v), in_row_stride, rope, rope_row_stride,
      reinterpret_cast<const __nv_bfloat16*>(q_weight), reinterpret_cast<const __nv_bfloat16*>(k_weight), eps,
      reinterpret_cast<__nv_bfloat16*>(q_out), reinterpret_cast<__nv_bfloat16*>(k_out),
      reinterpret_cast<__nv_bfloat16*>(v_out), s_l, (int)n_heads, (int)heads_per_rank, out_rank_stride,
      out_head_stride, nullptr, 0, 0);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_qknorm_rope_pack_peer(const void* q, const void* k, const void* v, int64_t in_row_stride,
                                        const float* rope, int64_t rope_row_stride, const void* q_weight,
                                        const void* k_weight, float eps, const uint64_t* rank_base,
                                        int64_t n_ranks, int64_t tensor_stride, int64_t head_stride,
                                        int64_t row_offset, int64_t s_l, int64_t n_heads, int64_t heads_per_rank,
                                        void* stream) {
  if (!q || !k || !v || !rank_base) return H3_ERR_NULL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (rope && !aligned16(rope)) ||
      (q_weight && !aligned16(q_weight)) || (k_weight && !aligned16(k_weight)) ||
      (reinterpret_cast<uintptr_t>(rank_base) & 7u))
    return H3_ERR_ALIGN;
  if (s_l < 1 || n_heads < 1 || heads_per_rank < 1 || n_heads % heads_per_rank || row_offset < 0) return H3_ERR_SHAPE;
  if (s_l > (1ll << 31) || n_heads > 65535 || s_l * 3 * n_heads > (1ll << 40)) return H3_ERR_SHAPE;
  // the kernel indexes rank_base[head / heads_per_rank]: the table must cover every destination
  if (n_ranks < 1 || n_heads / heads_per_rank > n_ranks) return H3_ERR_SHAPE;
  if (in_row_stride < n_heads * 128 || (in_row_stride % 8) || (tensor_stride % 8) || (head_stride % 8) ||
      tensor_stride < 0 || head_stride < 0 || (rope && (rope_row_stride < 256 || (rope_row_stride % 4))))
    return H3_ERR_STRIDE;
  if (!(eps >= 0.f)) return H3_ERR_SHAPE;
  const int blocks = grid_for(s_l, 8, 148 * 8);
  qknorm_rope_pack_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      reinterpret_cast<const __nv_bfloat16*>(v), in_row_stride, rope, rope_row_stride,
      reinterpret_cast<const __nv_bfloat16*>(q_weight), reinterpret_cast<const __nv_bfloat16*>(k_weight), eps,
      nullptr, nullptr, nullptr, s_l, (int)n_heads, (int)heads_per_rank, 0, head_stride,
      reinterpret_cast<const unsigned long long*>(rank_base), tensor_stride, row_offset);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_seq_to_head_unpack(const void* recv, void* out, int64_t world, int64_t heads_per_rank,
                                     int64_t s_l, int64_t n_tensors, int64_t recv_rank_stride,
                                     int64_t recv_tensor_stride, int64_t out_tensor_stride, void* stream) {
  if (!recv || !out) return H3_ERR_NULL;
  if (!aligned16(recv) || !aligned16(out)) return H3_ERR_ALIGN;
  if (world < 1 || heads_per_rank < 1 || s_l < 1 || n_tensors < 1) return H3_ERR_SHAPE;
  if (world * heads_per_rank * n_tensors > 65535) return H3_ERR_SHAPE;
  if ((recv_rank_stride % 8) || (recv_tensor_stride % 8) || (out_tensor_stride % 8)) return H3_ERR_STRIDE;
  const long long nvec = s_l * 16;
  dim3 grid((unsigned)grid_for(nvec, 256, 64), (unsigned)(world * heads_per_rank * n_tensors));
  seq_to_head_unpack_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(recv), reinterpret_cast<uint4*>(out), (int)world, (int)heads_per_rank, s_l,
      (int)n_tensors, recv_rank_stride, recv_tensor_stride, out_tensor_stride);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_head_to_seq_unpack(const void* recv, void* out, int64_t n_heads, int64_t s_l, void* stream) {
  if (!recv || !out) return H3_ERR_NULL;
  if (!aligned16(recv) || !aligned16(out)) return H3_ERR_ALIGN;
  if (n_heads < 1 || s_l < 1 || n_heads > 65535) return H3_ERR_SHAPE;
  const long long rows = n_heads * s_l;
  head_to_seq_unpack_kernel<<<grid_for(rows * 16, 256, 148 * 16), 256, 0,
                              reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(recv), reinterpret_cast<uint4*>(out), (int)n_heads, s_l);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width,
                          int64_t rows, void* stream) {
  if (!dst || !src) return H3_ERR_NULL;
  if (width < 1 || rows < 1 || dst_pitch < width || src_pitch < width) return H3_ERR_SHAPE;
  return cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch, (size_t)width, (size_t)rows,
                           cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
             ? H3_OK
             : H3_ERR_CUDA;
}

extern "C" int h3_status_read(const int32_t* status, void* stream) {
  if (!status) return H3_ERR_NULL;
  int32_t host = 0;
  if (cudaMemcpyAsync(&host, status, sizeof(int32_t), cudaMemcpyDeviceToHost,
                      reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return H3_ERR_CUDA;
  if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return H3_ERR_CUDA;
  return host;
}
