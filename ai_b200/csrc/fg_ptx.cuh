// Inline-PTX building blocks for sm_100a: mbarriers with bounded waits,
// TMA tile loads, tcgen05 (TMEM allocation, MMA issue, commit, loads) and
// the shared-memory matrix descriptor for 128-byte-swizzled K-major tiles.
//
// Every wait in this library is bounded: a pipeline wait that does not
// complete within the device's wait limit (DeviceStatus, 2 s by default)
// sets the CTA's abort flag and the device error word, and returns false,
// so a kernel that meets a broken pipeline ends with an error status the
// host reads instead of hanging the GPU. The teardown waits for a CTA's own
// copies and MMAs in flight always use the fixed kWaitTimeoutNs.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace fg {

// Error codes written into the device error word (first writer wins).
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,      // consumer waited too long for a TMA stage
  kDevTimeoutEmpty = 2,     // producer waited too long for a free stage
  kDevTimeoutAccFull = 3,   // epilogue waited too long for an accumulator
  kDevTimeoutAccEmpty = 4,  // MMA waited too long for the epilogue
  kDevTimeoutDrain = 5,     // teardown waited too long for in-flight work
  kDevBadArgs = 6,          // a kernel saw arguments it cannot handle
};

// Default limit of a pipeline wait, and the fixed limit of the teardown
// waits that let a CTA's own copies and MMAs finish before it retires.
constexpr uint64_t kWaitTimeoutNs = 2000ull * 1000ull * 1000ull;  // 2 s

// The per-device status block kernels receive as `int* gerr`: the error
// word first, then the pipeline-wait limit in nanoseconds (set from the
// host, fg_set_wait_limit). 16 bytes, zero error and kWaitTimeoutNs when
// created.
struct DeviceStatus {
  int err;
  int reserved;
  unsigned long long wait_limit_ns;
};
static_assert(sizeof(DeviceStatus) == 16, "status block layout");

__device__ __forceinline__ uint64_t wait_limit_ns(const int* gerr) {
  return reinterpret_cast<const volatile DeviceStatus*>(gerr)->wait_limit_ns;
}

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
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up after
// the device's wait limit (gerr's status block), or as soon as another role of the CTA has aborted
// (*abort != 0); on a timeout it raises the abort flag and records `code`.
// A try_wait on an open phase holds the thread for a while (about 4 µs on
// B200, whatever suspend-time hint it is given), so the limit is checked
// between tries: a wait gives up at the first check past the limit, i.e.
// waits shorter than one try never do. The time is taken before the first
// try, so a limit below one try binds on every wait that outlasts a try.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          int* gerr, int code) {
  const uint64_t t0 = globaltimer_ns();
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t limit = wait_limit_ns(gerr);
  while (true) {
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit) {
      *abort = 1;
      atomicCAS(gerr, 0, code);
      return false;
    }
    if (mbar_try_wait(bar, parity)) return true;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load, no multicast: box at element coordinates (x inner, y outer).
// x must be a multiple of 4 (16 bytes of fp32); callers pass multiples of 32.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled store of a shared-memory box to global memory at element
// coordinates (x inner, y outer), tracked by bulk groups; the parts of the
// box outside the tensor are not written. x must be a multiple of 4, y >= 0.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
// The same for a 3-D tensor, coordinates (x inner, y, z outer).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N committed store groups still read shared memory.
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until every committed store group has completed.
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) · B(smem desc)ᵀ, TF32 inputs, FP32 accumulate.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---------------------------------------------------------------- CTA pairs
// A cluster of two CTAs on two SMs sharing one tcgen05 MMA (cta_group::2):
// each CTA holds half of A's rows and half of B's rows in its own shared
// memory and its half of the accumulator rows in its own TMEM; one thread
// of the even CTA issues the MMA for both.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `addr` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Every thread of both CTAs; orders memory at cluster scope.
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of the other CTA of the pair (address from
// mapa_shared), with the instruction's default semantics. The signals sent
// this way between the pair's CTAs order shared-memory tiles (made visible
// to the tensor core's async proxy first) and TMEM reads against the pair
// MMA; an arrive with .release.cluster costs about 1.5k cycles each, which
// at one per pipeline stage is more than the stage's MMA time.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// mbar_wait for a barrier that threads of the other CTA arrive on.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort,
                                                  int* gerr, int code) {
  const uint64_t t0 = globaltimer_ns();
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t limit = wait_limit_ns(gerr);
  while (true) {
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit) {
      *abort = 1;
      atomicCAS(gerr, 0, code);
      return false;
    }
    if (mbar_try_wait_cluster(bar, parity)) return true;
  }
}
// Same warp index in both CTAs; both receive the same TMEM address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Pair MMA, M = 256 (128 rows per CTA), TF32 inputs, FP32 accumulate; the
// descriptors address the same shared-memory offsets in both CTAs.
__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the mbarrier at offset `bar` of every CTA in `cta_mask`
// when the pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// D(tmem) (+)= A(smem desc) · B(smem desc)ᵀ, BF16 inputs, FP32 accumulate.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) · B(smem desc)ᵀ, BF16 inputs: A is [128 rows (lanes) ×
// K], two bf16 per 32-bit column, lower K index in the low half.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Pair MMA, M = 256 (128 rows per CTA), FP16 inputs, FP32 accumulate.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor: kind::f16 with FP16 A and B, FP32 accumulator, K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4)                                 // D format: F32
         | (0u << 7)                               // A format: F16
         | (0u << 10)                              // B format: F16
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// fp16x2 packing: `lo_elem` in bits 0-15, `hi_elem` in bits 16-31, round to nearest.
__device__ __forceinline__ uint32_t pack_f16x2(float lo_elem, float hi_elem) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_elem), "f"(lo_elem));
  return r;
}
// Named barrier over `nthreads` threads (whole warps) with an AND of `v`:
// every participant gets true only if all passed true. Shared-memory
// accesses before it are ordered before those after it for all of them.
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v ? 1 : 0), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// 2^k as a float for k in [-126, 127] (exact).
__host__ __device__ __forceinline__ float pow2f(int k) {
#ifdef __CUDA_ARCH__
  return __int_as_float((127 + k) << 23);
#else
  uint32_t u = static_cast<uint32_t>(127 + k) << 23;
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}

// Instruction descriptor: kind::f16 with BF16 A and B, FP32 accumulator, K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4)                                 // D format: F32
         | (1u << 7)                               // A format: BF16
         | (1u << 10)                              // B format: BF16
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// Each thread of the warp writes 16 consecutive 32-bit columns of its lane.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// bf16x2 packing: `lo_elem` in bits 0-15, `hi_elem` in bits 16-31, round to nearest.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo_elem, float hi_elem) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_elem), "f"(lo_elem));
  return r;
}
__device__ __forceinline__ float bf16_round_f32(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (and its smem operands may be overwritten).
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzling: rows of 128 bytes (32 fp32), 8-row swizzle atoms
// 1024 bytes apart. The tile base must be 1024-byte aligned; stepping along
// K inside the 128-byte row is done by adding the byte offset to `saddr`.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);     // start address
  d |= static_cast<uint64_t>(1u) << 16;                   // leading byte offset (unused)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;           // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1u) << 46;                   // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                   // SWIZZLE_128B
  return d;
}

// The same descriptor for rows of SW bytes (128 or 64) written by TMA with
// the matching swizzle: 8-row atoms 8·SW bytes apart, layout type
// SWIZZLE_128B (2) or SWIZZLE_64B (4); the tile base must be 8·SW aligned.
template <int SW>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  static_assert(SW == 128 || SW == 64, "swizzle width");
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>((8u * SW) >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(SW == 128 ? 2u : 4u) << 61;
  return d;
}

// Instruction descriptor: kind::tf32, FP32 accumulator, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4)                                 // D format: F32
         | (2u << 7)                               // A format: TF32
         | (2u << 10)                              // B format: TF32
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------- split-TF32
// The high part keeps the 19 bits a TF32 operand carries (sign, exponent,
// 10 mantissa bits); the low part is the exact fp32 remainder. hi + lo == x
// exactly, and lo carries the bits the tensor core would otherwise drop.
__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}
__device__ __forceinline__ float tf32_lo(float x) { return x - tf32_hi(x); }

}  // namespace fg
