// h3_attn_layer_noalloc: the single-GPU attention layer (fused qk-RMSNorm + RoPE pack,
// then exact attention) for callers that cannot allocate device memory.
//
// Who needs it: a caller that owns no CUDA allocator of its own -- for example plain C,
// ctypes or another language's FFI code embedded in a host application whose device
// memory is all held by that application's caching allocator. Such a caller can hand us
// its input and output buffers, but a cudaMalloc of its own for our intermediate would
// either fail or eat into memory the host application has already reserved.
//
// The intermediate (the packed q, k, v in head-major layout) and the attention kernel's
// status word live in one file-scope static device array instead: kStatusBytes for the
// status word followed by kPackedMaxBytes for q/k/v, 64 MiB + 256 B in total. Every GPU
// that loads this library keeps that array until the process exits. A call needs
// 3 * s * n_heads * 128 * 2 bytes of it (s * n_heads <= 87381, e.g. 56 heads x 1560
// tokens); larger calls are rejected with H3_ERR_SCRATCH_LIMIT before anything runs.
//
// Host code cannot use the array's name as a device address, so the first call on each
// device (with that device current) looks the address up with cudaGetSymbolAddress and
// caches it; make that first call before any stream capture on that device. Every call
// shares the array and it keeps the last call's contents: the status word is cleared at
// the start of each call; the packed area is fully rewritten for the part a call reads.
// Calls whose work overlaps on the GPU (other streams, other host threads) race on the
// array. The call waits for its stream to drain so it can return the kernel's status.
#include <atomic>
#include <cmath>
#include <cstdint>

#include "h3_ptx.cuh"
#include "h3attn.h"

namespace {

constexpr size_t kStatusBytes = 256;
constexpr size_t kPackedMaxBytes = size_t(64) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kStatusBytes + kPackedMaxBytes];

std::atomic<unsigned char*> g_scratch_addr[kMaxDevices];

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_for_current_device(unsigned char** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return H3_ERR_CUDA;
  unsigned char* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || addr == nullptr) return H3_ERR_CUDA;
    p = static_cast<unsigned char*>(addr);
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return H3_OK;
}

}  // namespace

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" int h3_attn_layer_noalloc(const void* qkv, int64_t qkv_row_stride, const float* rope,
                                     int64_t rope_row_stride, const void* q_weight, const void* k_weight, float eps,
                                     void* o, int64_t s, int64_t n_heads, float softmax_scale, void* stream) {
  // Every argument is checked here, before anything is enqueued: a call that one of the two
  // kernels would reject must not leave the other half-done in the shared array.
  if (!qkv || !o) return H3_ERR_NULL;
  if (!aligned16(qkv) || !aligned16(o) || (rope && !aligned16(rope)) || (q_weight && !aligned16(q_weight)) ||
      (k_weight && !aligned16(k_weight)))
    return H3_ERR_ALIGN;
  if (s < 1 || n_heads < 1 || n_heads > 65535 || s > (int64_t(1) << 31) - 512) return H3_ERR_SHAPE;
  // q, k and v are the three column blocks of one row: the row must hold all three
  if (qkv_row_stride < 3 * n_heads * 128 || (qkv_row_stride % 8) ||
      (rope && (rope_row_stride < 256 || (rope_row_stride % 4))))
    return H3_ERR_STRIDE;
  if (!(eps >= 0.f) || !(softmax_scale > 0.f) || !std::isfinite(softmax_scale)) return H3_ERR_SHAPE;
  const int64_t head_elems = s * 128;
  if (n_heads > (int64_t)(kPackedMaxBytes / (3 * 2 * (size_t)head_elems))) return H3_ERR_SCRATCH_LIMIT;
  unsigned char* base = nullptr;
  int rc = scratch_for_current_device(&base);
  if (rc != H3_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t* status = reinterpret_cast<int32_t*>(base);
  __nv_bfloat16* packed = reinterpret_cast<__nv_bfloat16*>(base + kStatusBytes);
  __nv_bfloat16* qh = packed;
  __nv_bfloat16* kh = packed + n_heads * head_elems;
  __nv_bfloat16* vh = packed + 2 * n_heads * head_elems;
  if (cudaMemsetAsync(status, 0, sizeof(int32_t), st) != cudaSuccess) return H3_ERR_CUDA;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(qkv);
  rc = h3_qknorm_rope_pack(x, x + n_heads * 128, x + 2 * n_heads * 128, qkv_row_stride, rope, rope_row_stride,
                           q_weight, k_weight, eps, qh, kh, vh, s, n_heads, n_heads, 0, head_elems, stream);
  if (rc != H3_OK) return rc;
  rc = h3_attn_fwd(qh, kh, vh, o, n_heads, s, s, head_elems, 128, head_elems, 128, s, 0, 128, n_heads * 128,
                   softmax_scale, status, stream);
  if (rc != H3_OK) return rc;
  const int code = h3_status_read(status, stream);
  if (code < 0) return code;
  return code == 0 ? H3_OK : H3_ERR_DEVICE_TIMEOUT;
}
