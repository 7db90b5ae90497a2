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
// every GPU that loads the library holds until the process exits. In host
// code the array's name is only a host-side stand-in, so the device
// address is obtained with cudaGetSymbolAddress, once per device, with that
// device current, on the first call made on it; that first call should
// therefore come before any stream capture. All calls share the one array:
// calls that overlap on the GPU (different streams, or concurrent host
// threads) race on it and must be serialised by the caller.
#include <mutex>

#include "fg_internal.h"
#include "fg_kernels.cuh"

namespace fg {
namespace {

constexpr size_t kScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

// Every element a call reads from here is written earlier in the same call
// (the split / pack kernels fill exactly the rows and columns the GEMM's
// tensor maps cover), so nothing needs clearing between calls.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];
// Bounded-wait timeouts of kernels launched by this entry point are
// recorded here (the call itself never blocks to read it back).
static __device__ int g_noalloc_err;

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
    e = cudaGetSymbolAddress(&q, g_noalloc_err);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(FG_ECUDA, "cudaGetSymbolAddress(error word) failed: %s", cudaGetErrorString(e));
    }
    d.scratch = static_cast<unsigned char*>(p);
    d.err = static_cast<int*>(q);
    d.ready = true;
  }
  *out = d;
  return FG_OK;
}

size_t round256(size_t v) { return (v + 255) / 256 * 256; }

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
  if (precision != FG_PREC_SPLIT_TF32 && precision != FG_PREC_TF32)
    return set_error(FG_EINVAL, "fg_matmul_noalloc: unknown precision %d", precision);
  if (m == 0 || n == 0) return FG_OK;
  if (!x || !w || !out) return set_error(FG_EINVAL, "fg_matmul_noalloc: null operand");
  if (ldx < k || ldo < n || (w_transposed ? ldw < k : ldw < n))
    return set_error(FG_EINVAL, "fg_matmul_noalloc: leading dimension smaller than the row");
  if (epi && epi->act != FG_ACT_NONE && epi->act != FG_ACT_RELU && epi->act != FG_ACT_GELU)
    return set_error(FG_EINVAL, "fg_matmul_noalloc: unknown activation %d", epi->act);
  if (epi && ((epi->mul && epi->ldm < n) || (epi->residual && epi->ldr < n)))
    return set_error(FG_EINVAL, "fg_matmul_noalloc: Mul/Residual leading dimension smaller than n");

  // Scratch plan: x split (or re-strided) into [m, kp] parts, w transposed
  // to [n, kp] when given as [k, n], and w split into [n, kp] parts.
  const bool split = precision == FG_PREC_SPLIT_TF32;
  const int64_t kp = (k + 3) / 4 * 4;
  const bool a_direct = !split && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 4 == 0;
  const bool b_direct = !split && w_transposed && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                        ldw % 4 == 0;
  const size_t a_bytes = round256(size_t(m) * kp * 4), b_bytes = round256(size_t(n) * kp * 4);
  size_t need = 0;
  if (!a_direct) need += a_bytes * (split ? 2 : 1);
  if (!w_transposed) need += b_bytes;
  if (!b_direct) need += b_bytes * (split ? 2 : 1);
  if (need > kScratchBytes)
    return set_error(FG_EINVAL,
                     "fg_matmul_noalloc: needs %zu bytes of scratch for m=%lld n=%lld k=%lld, "
                     "more than its fixed %zu-byte array; use fg_matmul",
                     need, (long long)m, (long long)n, (long long)k, kScratchBytes);

  DevicePointers dp;
  FG_TRY(device_pointers(&dp));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* cur = dp.scratch;
  auto take = [&](size_t bytes) {
    float* r = reinterpret_cast<float*>(cur);
    cur += bytes;
    return r;
  };

  GemmEpilogue e;
  e.out = out;
  e.ldo = ldo;
  if (epi) {
    e.bias = epi->bias;
    e.rowscale = epi->row_scale;
    e.act = epi->act;
    e.mul = epi->mul;
    e.ldm = epi->ldm;
    e.residual = epi->residual;
    e.ldr = epi->ldr;
  }
  GemmArgs g;
  g.M = int(m);
  g.Nb = int(n);
  g.K = int(k);
  if (a_direct) {
    g.A = x;
    g.lda = ldx;
  } else {
    float* ahi = take(a_bytes);
    float* alo = split ? take(a_bytes) : nullptr;
    FG_TRY(split_copy_2d(x, ldx, m, k, ahi, alo, kp, split ? 1 : 0, s));
    g.A = ahi;
    g.A_lo = alo;
    g.lda = kp;
  }
  const float* bsrc = w;
  int64_t ldb_src = ldw;
  if (!w_transposed) {
    float* bt = take(b_bytes);
    FG_TRY(transpose_f32(w, ldw, k, n, bt, kp, s));
    bsrc = bt;
    ldb_src = kp;
  }
  if (b_direct) {
    g.B = w;
    g.ldb = ldw;
  } else {
    float* bhi = take(b_bytes);
    float* blo = split ? take(b_bytes) : nullptr;
    FG_TRY(split_copy_2d(bsrc, ldb_src, n, k, bhi, blo, kp, split ? 1 : 0, s));
    g.B = bhi;
    g.B_lo = blo;
    g.ldb = kp;
  }
  g.epi = e;
  return gemm_tn(g, dp.err, s);
}
