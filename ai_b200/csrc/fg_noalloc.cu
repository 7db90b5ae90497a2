// fg_matmul_noalloc: the product of fg_matmul with its scratch space in a
// fixed, library-owned device array instead of memory allocated per call.
//
// Who needs it: callers that must not allocate device memory during a call
// — a host whose own allocator has reserved the GPU's memory up front (a
// cudaMalloc from inside the library would then fail or fragment that
// pool), and latency-critical callers that cannot afford the implicit
// synchronisation cudaMalloc/cudaFree may cause. This entry point calls no
// cudaMalloc, cudaFree or other allocating routine.
//
// The scratch is the file-scope array below (kScratchBytes, 32 MiB), which
// every GPU that loads the library holds until the process exits. The CUDA
// driver reserves it when it loads this file's module on a device: at the
// first call on that device under lazy module loading (the CUDA 12
// default), or when the context is created under CUDA_MODULE_LOADING=EAGER.
// A caller whose allocator reserves the GPU's memory up front should make
// one call (or set eager loading) before that reservation. In host code the
// array's name is only a host-side stand-in, so the device address is
// obtained with cudaGetSymbolAddress, once per device, with that device
// current, on the first call made on it; that first call should therefore
// come before any stream capture. All calls share the one array: calls
// that overlap on the GPU (different streams, or concurrent host threads)
// race on it and must be serialised by the caller. A bounded wait that
// gives up in one of its kernels is recorded in the entry point's own
// status block, which fg_synchronize reads and clears (FG_ETIMEOUT).
#include <mutex>

#include "fg_internal.h"
#include "fg_kernels.cuh"
#include "fg_ptx.cuh"

namespace fg {
namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

// Every element a call reads from here is written earlier in the same call
// (the split / pack kernels fill exactly the rows and columns the GEMM's
// tensor maps cover), so nothing needs clearing between calls.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];
// Status block of the kernels this entry point launches: their
// bounded-wait timeouts are recorded in its first word, and their wait
// limit is read from it (DeviceStatus). It is registered with the runtime
// at set-up, so fg_synchronize reads and clears it like the library's own.
static __device__ __align__(16) DeviceStatus g_noalloc_status = {0, 0, kWaitTimeoutNs};

struct DevicePointers {
  unsigned char* scratch = nullptr;
  int* err = nullptr;
  bool ready = false;
};
std::mutex g_mu;
DevicePointers g_dev[kMaxDevices];

int device_pointers(DevicePointers* out) {
  int dev = 0;
  FG_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(FG_ENODEV, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  DevicePointers& d = g_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(FG_ECUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    }
    void* q = nullptr;
    e = cudaGetSymbolAddress(&q, g_noalloc_status);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(FG_ECUDA, "cudaGetSymbolAddress(status block) failed: %s", cudaGetErrorString(e));
    }
    FG_TRY(register_status_block(dev, static_cast<int*>(q)));
    d.scratch = static_cast<unsigned char*>(p);
    d.err = static_cast<int*>(q);
    d.ready = true;
  }
  *out = d;
  return FG_OK;
}

}  // namespace
}  // namespace fg

using namespace fg;

extern "C" int fg_matmul_noalloc(int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx,
                                 const float* w, int64_t ldw, int w_transposed, float* out,
                                 int64_t ldo, const fg_epilogue* epi, int precision,
                                 void* stream) {
  clear_error();
  if (m < 0 || n < 0 || k <= 0 || m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
    return set_error(FG_EINVAL, "fg_matmul_noalloc: bad shape m=%lld n=%lld k=%lld",
                     (long long)m, (long long)n, (long long)k);
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "fg_matmul_noalloc: unknown precision %d", precision);
  if (m == 0 || n == 0) return FG_OK;
  if (!x || !w || !out) return set_error(FG_EINVAL, "fg_matmul_noalloc: null operand");
  if (ldx < k || ldo < n || (w_transposed ? ldw < k : ldw < n))
    return set_error(FG_EINVAL, "fg_matmul_noalloc: leading dimension smaller than the row");
  if (epi && epi->act != FG_ACT_NONE && epi->act != FG_ACT_RELU && epi->act != FG_ACT_GELU)
    return set_error(FG_EINVAL, "fg_matmul_noalloc: unknown activation %d", epi->act);
  if (epi && ((epi->mul && epi->ldm < n) || (epi->residual && epi->ldr < n)))
    return set_error(FG_EINVAL, "fg_matmul_noalloc: Mul/Residual leading dimension smaller than n");

  const MatmulPlan plan = plan_matmul(m, n, k, x, ldx, w, ldw, w_transposed, precision);
  if (plan.total() > kScratchBytes)
    return set_error(FG_EINVAL,
                     "fg_matmul_noalloc: needs %zu bytes of scratch for m=%lld n=%lld k=%lld, "
                     "more than its fixed %zu-byte array; use fg_matmul",
                     plan.total(), (long long)m, (long long)n, (long long)k, kScratchBytes);
  DevicePointers dp;
  FG_TRY(device_pointers(&dp));
  return matmul_run(plan, m, n, k, x, ldx, w, ldw, w_transposed, out, ldo, epi, dp.scratch, dp.err,
                    static_cast<cudaStream_t>(stream));
}
