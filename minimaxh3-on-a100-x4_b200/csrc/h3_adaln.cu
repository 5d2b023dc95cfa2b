// AdaLN modulation and gated residuals of the DiT block, one HBM pass each (HBM-bound).
//
// The host model's block (the timed replica at harness/sp_runtime.py:203-218) does, per token row
// in modulation segment `row` (tokens outside every segment -- the SP pad tail -- are copied):
//   h  = LN(x) * (1 + scale[row]) + shift[row]        (_mod_scale_shift after norm1 / norm2)
//   x' = x + gate[row] * y                            (_mod_gate: attention / FFN residual)
// as separate torch ops, each rounding to bf16. These kernels keep that rounding order:
//   bf16(1 + scale), bf16(LN(x) * that), bf16(... + shift);  bf16(gate * y), bf16(x + ...)
// with LN = (x - mean) / sqrt(var + eps) in fp32 (biased variance, no affine), rounded to bf16.
// h3_norm_modulate optionally applies a gated residual first and normalises its result (the
// attention residual fused with norm2), so the block needs three passes over [rows][hidden].
// One CTA per token row: the row (hidden <= 8192) stays in registers (as bf16) between the
// statistics and the output; 16-byte loads and stores; every row is computed independently of the
// others.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "h3attn.h"

namespace h3 {
namespace adaln {

constexpr int kThreads = 256;
constexpr int kMaxVec = 4;  // 16-byte vectors per thread: hidden <= 8 * 256 * 4 = 8192

__device__ __forceinline__ float rb(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&b);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Sum over the CTA; fixed order (warp butterfly, then warp 0 over the warp partials).
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kThreads / 32 ? red[lane] : 0.f;
  if (warp == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[kThreads / 32] = t;
  }
  __syncthreads();
  const float r = red[kThreads / 32];
  __syncthreads();  // red is reused by the next call
  return r;
}

struct NormParams {
  const __nv_bfloat16* x;
  long long x_stride;
  const __nv_bfloat16* y;  // residual branch output or nullptr
  long long y_stride;
  const __nv_bfloat16* gate;
  __nv_bfloat16* x_out;  // residual result (nullptr: not stored)
  long long x_out_stride;
  const __nv_bfloat16* shift;
  const __nv_bfloat16* scale;
  long long mod_stride;  // row stride of gate / shift / scale (modulation rows)
  const int32_t* seg_row;  // per token: modulation row, or -1
  __nv_bfloat16* h;
  long long h_stride;
  int hidden;
  float eps;
};

// kVec vectors of 8 per thread hold the row, kept as bf16 (every value the statistics and the
// output read is bf16-representable: x itself, or the bf16-rounded residual), so 3 vectors
// (hidden <= 6144, H3's 5376) fit 32 registers and eight rows per SM are in flight; 4 cover the
// rest. All of a row's x / y loads are issued before anything is stored: the compiler cannot move
// a load above a store to x_out (which it must assume may alias), and one round trip to DRAM per
// row instead of one per vector is what keeps HBM busy.
template <int kVec, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks) norm_modulate_kernel(const NormParams p) {
  __shared__ float red[kThreads / 32 + 1];
  const long long r = blockIdx.x;
  const int m = p.seg_row[r];
  const int n_vec = p.hidden >> 3;
  const bool res = p.y != nullptr && m >= 0;
  uint4 v[kVec], yv[kVec];
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n_vec) {
      v[i] = *reinterpret_cast<const uint4*>(p.x + r * p.x_stride + 8 * c);
      if (res) yv[i] = *reinterpret_cast<const uint4*>(p.y + r * p.y_stride + 8 * c);
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n_vec) {
      if (res) {
        float a[8], y[8], g[8];
        unpack8(v[i], a);
        unpack8(yv[i], y);
        unpack8(*reinterpret_cast<const uint4*>(p.gate + m * p.mod_stride + 8 * c), g);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = rb(a[e] + rb(g[e] * y[e]));
        v[i] = pack8(a);
      }
      if (p.x_out != nullptr) *reinterpret_cast<uint4*>(p.x_out + r * p.x_out_stride + 8 * c) = v[i];
      float f[8];
      unpack8(v[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += f[e];
    }
  }
  const float mean = block_sum(s, red) / float(p.hidden);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n_vec) {
      float f[8];
      unpack8(v[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = f[e] - mean;
        q += d * d;
      }
    }
  }
  const float rstd = rsqrtf(block_sum(q, red) / float(p.hidden) + p.eps);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < n_vec) {
      float o[8], f[8];
      unpack8(v[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = rb((f[e] - mean) * rstd);
      if (m >= 0) {
        float sh[8], sc[8];
        unpack8(*reinterpret_cast<const uint4*>(p.shift + m * p.mod_stride + 8 * c), sh);
        unpack8(*reinterpret_cast<const uint4*>(p.scale + m * p.mod_stride + 8 * c), sc);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rb(rb(o[e] * rb(1.0f + sc[e])) + sh[e]);
      }
      *reinterpret_cast<uint4*>(p.h + r * p.h_stride + 8 * c) = pack8(o);
    }
  }
}

// out = x + gate[row] * y on segment tokens, x elsewhere; one 16-byte vector per thread.
__global__ void __launch_bounds__(256) gated_residual_kernel(const __nv_bfloat16* x, long long x_stride,
                                                             const __nv_bfloat16* y, long long y_stride,
                                                             const __nv_bfloat16* gate, long long gate_stride,
                                                             const int32_t* seg_row, __nv_bfloat16* out,
                                                             long long out_stride, long long rows, int n_vec) {
  const long long total = rows * n_vec;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / n_vec;
    const int c = int(i - r * n_vec);
    const int m = seg_row[r];
    float a[8];
    unpack8(*reinterpret_cast<const uint4*>(x + r * x_stride + 8 * c), a);
    if (m >= 0) {
      float b[8], g[8];
      unpack8(*reinterpret_cast<const uint4*>(y + r * y_stride + 8 * c), b);
      unpack8(*reinterpret_cast<const uint4*>(gate + m * gate_stride + 8 * c), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] = rb(a[e] + rb(g[e] * b[e]));
    }
    *reinterpret_cast<uint4*>(out + r * out_stride + 8 * c) = pack8(a);
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace adaln
}  // namespace h3

using namespace h3::adaln;

extern "C" int h3_norm_modulate(const void* x, int64_t x_row_stride, const void* y, int64_t y_row_stride,
                                const void* gate, void* x_out, int64_t x_out_row_stride, const void* shift,
                                const void* scale, int64_t mod_row_stride, const int32_t* seg_row, void* h,
                                int64_t h_row_stride, int64_t rows, int64_t hidden, float eps, void* stream) {
  if (!x || !shift || !scale || !seg_row || !h || (y && !gate)) return H3_ERR_NULL;
  if (!aligned16(x) || !aligned16(shift) || !aligned16(scale) || !aligned16(h) || (y && !aligned16(y)) ||
      (gate && !aligned16(gate)) || (x_out && !aligned16(x_out)))
    return H3_ERR_ALIGN;
  if (rows < 1 || rows > (1ll << 31) - 1 || hidden < 8 || hidden % 8 || hidden > 8 * kThreads * kMaxVec ||
      !(eps >= 0.f))
    return H3_ERR_SHAPE;
  if (x_row_stride % 8 || x_row_stride < hidden || h_row_stride % 8 || h_row_stride < hidden || mod_row_stride % 8 ||
      mod_row_stride < hidden || (y && (y_row_stride % 8 || y_row_stride < hidden)) ||
      (x_out && (x_out_row_stride % 8 || x_out_row_stride < hidden)))
    return H3_ERR_STRIDE;
  NormParams p;
  p.x = reinterpret_cast<const __nv_bfloat16*>(x);
  p.x_stride = x_row_stride;
  p.y = reinterpret_cast<const __nv_bfloat16*>(y);
  p.y_stride = y_row_stride;
  p.gate = reinterpret_cast<const __nv_bfloat16*>(gate);
  p.x_out = reinterpret_cast<__nv_bfloat16*>(x_out);
  p.x_out_stride = x_out_row_stride;
  p.shift = reinterpret_cast<const __nv_bfloat16*>(shift);
  p.scale = reinterpret_cast<const __nv_bfloat16*>(scale);
  p.mod_stride = mod_row_stride;
  p.seg_row = seg_row;
  p.h = reinterpret_cast<__nv_bfloat16*>(h);
  p.h_stride = h_row_stride;
  p.hidden = (int)hidden;
  p.eps = eps;
  if (hidden <= 8 * kThreads * 3)
    norm_modulate_kernel<3, 8><<<(unsigned)rows, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  else
    norm_modulate_kernel<kMaxVec, 6><<<(unsigned)rows, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_gated_residual(const void* x, int64_t x_row_stride, const void* y, int64_t y_row_stride,
                                 const void* gate, int64_t gate_row_stride, const int32_t* seg_row, void* out,
                                 int64_t out_row_stride, int64_t rows, int64_t hidden, void* stream) {
  if (!x || !y || !gate || !seg_row || !out) return H3_ERR_NULL;
  if (!aligned16(x) || !aligned16(y) || !aligned16(gate) || !aligned16(out)) return H3_ERR_ALIGN;
  if (rows < 1 || hidden < 8 || hidden % 8 || hidden > (1 << 24)) return H3_ERR_SHAPE;
  if (x_row_stride % 8 || y_row_stride % 8 || gate_row_stride % 8 || out_row_stride % 8 || x_row_stride < hidden ||
      y_row_stride < hidden || gate_row_stride < hidden || out_row_stride < hidden)
    return H3_ERR_STRIDE;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return H3_ERR_CUDA;
  const long long total = rows * (hidden / 8);
  const long long blocks = (total + 255) / 256;
  const unsigned grid = (unsigned)(blocks < 8ll * sms ? blocks : 8ll * sms);
  gated_residual_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), x_row_stride, reinterpret_cast<const __nv_bfloat16*>(y), y_row_stride,
      reinterpret_cast<const __nv_bfloat16*>(gate), gate_row_stride, seg_row, reinterpret_cast<__nv_bfloat16*>(out),
      out_row_stride, rows, (int)(hidden / 8));
  return cudaGetLastError() == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}
