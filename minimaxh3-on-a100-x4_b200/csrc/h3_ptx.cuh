// Inline-PTX building blocks for the sm_100a kernels of this library:
// mbarriers with bounded waits, TMA tile loads (no cluster multicast anywhere),
// tcgen05 tensor-memory allocation, MMA issue/commit, and TMEM loads/stores.
//
// Every wait here is bounded: after WaitCtx::limit_ns of polling (H3_WAIT_LIMIT_NS unless
// a caller passes its own; measured with %globaltimer) the waiter records an error code in the caller's device status
// word, raises the CTA's abort flag and returns false, so the kernel can wind down
// and return instead of hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#ifndef H3_WAIT_LIMIT_NS
#define H3_WAIT_LIMIT_NS 2000000000ull  // 2 s; a healthy wait here lasts microseconds
#endif

namespace h3 {

// Device status codes (mirrored in include/h3attn.h).
enum : int {
  kStatusOk = 0,
  kStatusTimeoutQ = 1,      // Q tile load never landed
  kStatusTimeoutKV = 2,     // K/V ring wait gave up
  kStatusTimeoutS = 3,      // softmax waited too long for S
  kStatusTimeoutP = 4,      // MMA waited too long for P
  kStatusTimeoutO = 5,      // waited too long for an O accumulation
  kStatusTimeoutDrain = 6,  // teardown drain wait gave up
  kStatusTimeoutKat = 7,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread until the phase completes, for at most kSuspendHintNs:
// a waiting warp then sleeps instead of spinning through issue slots that the working warps of
// its SM sub-partition need. It returns as soon as the phase completes.
constexpr uint32_t kSuspendHintNs = 1000000;  // 1 ms between checks of the abort flag / time limit
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Shared state a CTA uses to give up cleanly: `abort` lives in shared memory,
// `status` is the caller's device status word (also read as a grid-wide abort),
// `limit_ns` how long one wait may poll before it gives up.
struct WaitCtx {
  volatile int* abort;
  int* status;
  unsigned long long limit_ns = H3_WAIT_LIMIT_NS;
};

// After every unsuccessful (suspending) try: leave when the CTA aborted, another CTA failed the
// call, or the wait outlived its limit.
__device__ __forceinline__ bool wait_should_stop(const WaitCtx& ctx, uint64_t t0, int code) {
  if (*ctx.abort) return true;
  if (*reinterpret_cast<volatile int*>(ctx.status) != 0) {
    *ctx.abort = 1;
    return true;
  }
  if (globaltimer_ns() - t0 > ctx.limit_ns) {
    atomicCAS(ctx.status, 0, code);
    *ctx.abort = 1;
    return true;
  }
  return false;
}

// Bounded wait on phase `parity` of `bar`. Returns false when the CTA must abort.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& ctx, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (wait_should_stop(ctx, t0, code)) return false;
  }
}

// One lane of a converged warp (elect.sync). A single-thread instruction stream inside a warp
// that runs the same loop on all lanes: an MMA-issuing loop written this way keeps the tensor
// pipe fed while other warps of the SM sub-partition issue at full rate, where a lane-0-only
// branch falls behind.
__device__ __forceinline__ bool elect_one() {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r));
  return r != 0;
}

// ---------------------------------------------------------------- TMA (plain, per CTA)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 3-D tiled load of one box into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format (1 = bf16),
//   bit 15 A major (0 = K), bit 16 B major (0 = K, 1 = MN), 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn_major) << 15) | (uint32_t(b_mn_major) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version bits.
//   bits 0-13 start>>4, 16-29 LBO>>4, 32-45 SBO>>4, 46-47 version (1), 61-63 layout (2 = SW128).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// TMEM loads: 32 lanes x 32 bit, N consecutive columns per thread. The load and
// its wait sit in one asm block so no use of the registers can be scheduled early.
#define H3_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                 "=r"(r[i + 6]), "=r"(r[i + 7])
__device__ __forceinline__ void tmem_ld32_wait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : H3_R8(0), H3_R8(8), H3_R8(16), H3_R8(24)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16_wait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : H3_R8(0), H3_R8(8)
      : "r"(taddr)
      : "memory");
}
// Two 32-column loads in flight, then one wait.
__device__ __forceinline__ void tmem_ld64_wait(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : H3_R8(0), H3_R8(8), H3_R8(16), H3_R8(24), H3_R8(32), H3_R8(40), H3_R8(48), H3_R8(56)
      : "r"(taddr), "r"(taddr + 32u)
      : "memory");
}
// Two 32-column loads issued without waiting; tmem_ld64_wait_on() completes them. The wait
// names the registers as in/out operands, so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld64_nowait(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n"
      : H3_R8(0), H3_R8(8), H3_R8(16), H3_R8(24), H3_R8(32), H3_R8(40), H3_R8(48), H3_R8(56)
      : "r"(taddr), "r"(taddr + 32u)
      : "memory");
}
#undef H3_R8
#define H3_RW8(i) "+r"(r[i + 0]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), "+r"(r[i + 4]), \
                  "+r"(r[i + 5]), "+r"(r[i + 6]), "+r"(r[i + 7])
__device__ __forceinline__ void tmem_ld64_wait_on(uint32_t (&r)[64]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : H3_RW8(0), H3_RW8(8), H3_RW8(16), H3_RW8(24), H3_RW8(32), H3_RW8(40), H3_RW8(48), H3_RW8(56)
               :
               : "memory");
}
#undef H3_RW8

// Per-warpgroup register budgets (setmaxnreg): a warpgroup gives registers back to the
// CTA's pool or takes more from it. The counts must fit the registers the CTA was launched
// with (threads x registers per thread at launch).
template <int kRegs>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegs));
}
template <int kRegs>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegs));
}

#define H3_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                 "r"(r[i + 6]), "r"(r[i + 7])
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n" ::"r"(taddr),
      H3_W8(0), H3_W8(8)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n" ::"r"(taddr),
      H3_W8(0), H3_W8(8), H3_W8(16), H3_W8(24)
      : "memory");
}
#undef H3_W8
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16-lane TMEM shapes (a warp addresses 16 lanes starting at the lane field of taddr).
// 16x256b: thread (t0 + 4*t1) of the warp gets, per repeat k (8 columns), registers
//   [4k+0], [4k+1] = lane t1,     columns 8k+2*t0, 8k+2*t0+1
//   [4k+2], [4k+3] = lane t1 + 8, the same columns
// 16x128b: per repeat k (4 columns): [2k+0] = lane t1, column 4k+t0; [2k+1] = lane t1 + 8.
#define H3_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                 "=r"(r[i + 6]), "=r"(r[i + 7])
__device__ __forceinline__ void tmem_ld_16x256b_x8_wait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : H3_R8(0), H3_R8(8), H3_R8(16), H3_R8(24)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_16x256b_x4_wait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : H3_R8(0), H3_R8(8)
      : "r"(taddr)
      : "memory");
}
#undef H3_R8
#define H3_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                 "r"(r[i + 6]), "r"(r[i + 7])
__device__ __forceinline__ void tmem_st_16x128b_x8(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x128b.x8.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n" ::"r"(taddr),
      H3_W8(0), H3_W8(8)
      : "memory");
}
__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n" ::"r"(taddr),
      H3_W8(0), H3_W8(8)
      : "memory");
}
#undef H3_W8

// ---------------------------------------------------------------- 2-SM (CTA pair) helpers
// A cluster of two CTAs on two SMs: tcgen05 ops with cta_group::2 are issued by the even CTA
// (the leader) for both; each CTA keeps its own half of the A rows and of B (N/2), and its own
// rows of D in its own TMEM.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA in the cluster. Release at CTA scope: what the arrival
// publishes here is tensor-memory state, ordered by tcgen05.wait::st and
// tcgen05.fence::before_thread_sync ahead of it; a cluster-scope release costs ~1000 cycles
// (it waits out the thread's outstanding global writes) and orders nothing more that matters.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Named barrier over n_threads (whole warps).
__device__ __forceinline__ void named_bar_sync(int id, int n_threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n_threads) : "memory");
}
__device__ __forceinline__ void st_shared_u4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}
// Named barrier over n_threads (whole warps) returning the AND of every thread's `v`.
__device__ __forceinline__ bool named_bar_and(int id, int n_threads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(id), "r"(n_threads)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool mbar_try_wait_acq_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait_acq_cluster_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (for barriers that peer CTAs arrive on).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, const WaitCtx& ctx, int code) {
  if (mbar_try_wait_acq_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_acq_cluster_sleep(bar, parity)) return true;
    if (wait_should_stop(ctx, t0, code)) return false;
  }
}
// 3-D tile load into this CTA's shared memory whose completion is counted on an mbarrier that
// may live in the peer CTA of the pair (cluster address). No multicast.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive once on the mbarrier at offset `bar` in every CTA of `cta_mask` when all tcgen05 ops
// this thread issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               ::"r"(bar), "h"(cta_mask)
               : "memory");
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed fp32 pairs (sm_100 f32x2 ALU forms): each lane is an IEEE round-to-nearest
// operation, identical to its scalar counterpart, at one issue slot per pair.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// max(a, b, c) in one instruction.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair on the FMA pipe (relieves MUFU, which issues 16 exponentials per clock per
// SM): x is clamped at -127, n = floor(x) comes from the 1.5*2^23 shifter added with
// round-toward-minus-infinity, f = x - n lies in [0, 1), 2^f = 1 + c1 f + c2 f^2 + c3 f^3 with
// minimax relative error 8.6e-5 (linear-programming fit, csrc/gen_exp2_poly.py), and n is added
// straight into the exponent field: the shifter's low bits hold n, and shifting them up by 23
// drops the shifter's own exponent bits. p(f) lies in [1, 2), so any n >= -127 leaves a valid
// (at worst subnormal) fp32; x = -inf (a masked key) gives f = 0, p = 1 and exactly +0. Every
// step is one IEEE-rounded operation in a fixed order, so results do not depend on launch shape.
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& y0, float& y1) {
  const uint64_t shifter = 0x4B4000004B400000ull;  // 1.5 * 2^23, twice
  const uint64_t k3 = 0x3D9DD56E3D9DD56Eull;       // 7.706724107e-02f
  const uint64_t k2 = 0x3E691BC43E691BC4ull;       // 2.276449800e-01f
  const uint64_t k1 = 0x3F31F32A3F31F32Aull;       // 6.951166391e-01f
  const uint64_t one = 0x3F8000003F800000ull;      // 1.0f
  uint32_t r0, r1;
  asm("{\n\t.reg .f32 a, b;\n\t.reg .b64 xc, t, n, f, q;\n\t.reg .b32 q0, q1, t0, t1;\n\t"
      "max.f32 a, %2, 0fC2FE0000;\n\t"
      "max.f32 b, %3, 0fC2FE0000;\n\t"
      "mov.b64 xc, {a, b};\n\t"
      "add.rm.f32x2 t, xc, %4;\n\t"
      "sub.rn.f32x2 n, t, %4;\n\t"
      "sub.rn.f32x2 f, xc, n;\n\t"
      "fma.rn.f32x2 q, f, %5, %6;\n\t"
      "fma.rn.f32x2 q, q, f, %7;\n\t"
      "fma.rn.f32x2 q, q, f, %8;\n\t"
      "mov.b64 {q0, q1}, q;\n\t"
      "mov.b64 {t0, t1}, t;\n\t"
      "mad.lo.u32 %0, t0, 8388608, q0;\n\t"
      "mad.lo.u32 %1, t1, 8388608, q1;\n\t}\n"
      : "=r"(r0), "=r"(r1)
      : "f"(x0), "f"(x1), "l"(shifter), "l"(k3), "l"(k2), "l"(k1), "l"(one));
  y0 = __uint_as_float(r0);
  y1 = __uint_as_float(r1);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x (low 16 bits) = lo
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace h3
