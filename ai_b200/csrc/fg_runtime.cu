// Library runtime: thread-local error messages, device queries, the
// per-device status block kernels report bounded-wait timeouts into (and
// read their wait limit from), and the device-memory helpers of the C ABI.
#include <mutex>
#include <vector>

#include <atomic>

#include "fg_internal.h"

namespace fg {

namespace {
thread_local std::string t_last_error;
std::mutex g_mu;
std::vector<int*> g_dev_err;    // per device status block, lazily allocated
std::vector<int*> g_extra_err;  // per device: the no-allocation entry point's block
std::vector<unsigned long long> g_wait_limit;  // per device, 0 = default
std::vector<int> g_sms;
std::vector<cudaMemPool_t> g_pools;  // per device: op-level scratch

// Host image of the device status block (fg_ptx.cuh DeviceStatus).
struct DeviceStatusHost {
  int err;
  int reserved;
  unsigned long long wait_limit_ns;
};
constexpr unsigned long long kDefaultWaitLimitNs = 2000ull * 1000ull * 1000ull;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

void clear_error() { t_last_error.clear(); }
const char* last_error() { return t_last_error.c_str(); }

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (int(g_sms.size()) <= dev) g_sms.resize(dev + 1, 0);
  if (g_sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = n > 0 ? n : 148;
  }
  return g_sms[dev];
}

// Status block of the current device: the error word (zeroed at
// allocation) followed by the pipeline-wait limit. Allocated on first use.
int device_error_word(int** out) {
  int dev = 0;
  FG_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_mu);
  if (int(g_dev_err.size()) <= dev) g_dev_err.resize(dev + 1, nullptr);
  if (g_dev_err[dev] == nullptr) {
    DeviceStatusHost init{0, 0, kDefaultWaitLimitNs};
    if (int(g_wait_limit.size()) > dev && g_wait_limit[dev] != 0) init.wait_limit_ns = g_wait_limit[dev];
    int* p = nullptr;
    FG_CUDA_TRY(cudaMalloc(&p, sizeof(DeviceStatusHost)));
    FG_CUDA_TRY(cudaMemcpy(p, &init, sizeof(init), cudaMemcpyHostToDevice));
    g_dev_err[dev] = p;
  }
  *out = g_dev_err[dev];
  return FG_OK;
}

int register_status_block(int dev, int* block) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (int(g_extra_err.size()) <= dev) g_extra_err.resize(dev + 1, nullptr);
  g_extra_err[dev] = block;
  if (int(g_wait_limit.size()) > dev && g_wait_limit[dev] != 0) {
    const unsigned long long v = g_wait_limit[dev];
    FG_CUDA_TRY(cudaMemcpy(reinterpret_cast<char*>(block) + 8, &v, sizeof(v), cudaMemcpyHostToDevice));
  }
  return FG_OK;
}

// Synchronises the current device and converts a recorded kernel timeout
// into FG_ETIMEOUT, resetting the error words. Reads the library's status
// block and the one registered by the no-allocation entry point; allocates
// nothing (a block not yet created holds no record).
int check_device_error_word() {
  FG_CUDA_TRY(cudaDeviceSynchronize());
  int dev = 0;
  FG_CUDA_TRY(cudaGetDevice(&dev));
  int* words[2] = {nullptr, nullptr};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int(g_dev_err.size()) > dev) words[0] = g_dev_err[dev];
    if (int(g_extra_err.size()) > dev) words[1] = g_extra_err[dev];
  }
  int first = 0;
  for (int* w : words) {
    if (!w) continue;
    int v = 0;
    FG_CUDA_TRY(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) {
      const int zero = 0;
      FG_CUDA_TRY(cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice));
      if (!first) first = v;
    }
  }
  if (first) return set_error(FG_ETIMEOUT, "a device wait gave up (kernel status %d)", first);
  return FG_OK;
}

int set_wait_limit(int dev, unsigned long long ns) {
  int* blocks[2] = {nullptr, nullptr};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int(g_wait_limit.size()) <= dev) g_wait_limit.resize(dev + 1, 0);
    g_wait_limit[dev] = ns;
    if (int(g_dev_err.size()) > dev) blocks[0] = g_dev_err[dev];
    if (int(g_extra_err.size()) > dev) blocks[1] = g_extra_err[dev];
  }
  for (int* b : blocks)
    if (b) FG_CUDA_TRY(cudaMemcpy(reinterpret_cast<char*>(b) + 8, &ns, sizeof(ns), cudaMemcpyHostToDevice));
  return FG_OK;
}

// Library-owned stream-ordered pool per device for the op-level calls'
// scratch (operand splits, transposes, attention operands). Its release
// threshold is unlimited, so memory freed at the end of one call stays
// reserved and the next call reuses it without mapping new pages (with the
// device's default pool, whose threshold is 0, every synchronisation
// returned the memory and every call paid for mapping it again).
int scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
  *p = nullptr;
  if (bytes == 0) return FG_OK;
  int dev = 0;
  FG_CUDA_TRY(cudaGetDevice(&dev));
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int(g_pools.size()) <= dev) g_pools.resize(dev + 1, nullptr);
    if (!g_pools[dev]) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      cudaMemPool_t mp = nullptr;
      FG_CUDA_TRY(cudaMemPoolCreate(&mp, &props));
      cuuint64_t keep = ~cuuint64_t(0);
      FG_CUDA_TRY(cudaMemPoolSetAttribute(mp, cudaMemPoolAttrReleaseThreshold, &keep));
      g_pools[dev] = mp;
    }
    pool = g_pools[dev];
  }
  if (cudaMallocFromPoolAsync(p, bytes, pool, s) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return set_error(FG_ENOMEM, "scratch allocation of %zu bytes failed", bytes);
  }
  return FG_OK;
}

void scratch_free(void* p, cudaStream_t s) {
  if (p) cudaFreeAsync(p, s);
}

int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> cached{nullptr};
  if (!cached.load()) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || f == nullptr) {
      cudaGetLastError();
      return set_error(FG_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
    }
    cached.store(reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f));
  }
  *fn = cached.load();
  return FG_OK;
}

}  // namespace fg

extern "C" {

const char* fg_last_error(void) { return fg::last_error(); }

int fg_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int good = 0;
  for (int d = 0; d < n; ++d) {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
    if (major == 10) ++good;
  }
  return good;
}

int fg_malloc(int device, int64_t bytes, void** out) {
  if (!out || bytes < 0) return fg::set_error(FG_EINVAL, "fg_malloc: bad arguments");
  FG_CUDA_TRY(cudaSetDevice(device));
  *out = nullptr;
  if (bytes == 0) return FG_OK;
  if (cudaMalloc(out, size_t(bytes)) != cudaSuccess) {
    cudaGetLastError();
    return fg::set_error(FG_ENOMEM, "fg_malloc: %lld bytes", (long long)bytes);
  }
  return FG_OK;
}

int fg_free(int device, void* ptr) {
  FG_CUDA_TRY(cudaSetDevice(device));
  if (ptr) FG_CUDA_TRY(cudaFree(ptr));
  return FG_OK;
}

int fg_memcpy_h2d(int device, void* dst, const void* src, int64_t bytes) {
  FG_CUDA_TRY(cudaSetDevice(device));
  if (bytes > 0) FG_CUDA_TRY(cudaMemcpy(dst, src, size_t(bytes), cudaMemcpyHostToDevice));
  return FG_OK;
}

int fg_memcpy_d2h(int device, void* dst, const void* src, int64_t bytes) {
  FG_CUDA_TRY(cudaSetDevice(device));
  if (bytes > 0) FG_CUDA_TRY(cudaMemcpy(dst, src, size_t(bytes), cudaMemcpyDeviceToHost));
  return FG_OK;
}

int fg_synchronize(int device) {
  FG_CUDA_TRY(cudaSetDevice(device));
  return fg::check_device_error_word();
}

int fg_set_wait_limit(int device, int64_t nanoseconds) {
  fg::clear_error();
  if (nanoseconds < 0) return fg::set_error(FG_EINVAL, "fg_set_wait_limit: negative limit");
  FG_CUDA_TRY(cudaSetDevice(device));
  FG_CUDA_TRY(cudaDeviceSynchronize());
  const unsigned long long ns =
      nanoseconds == 0 ? fg::kDefaultWaitLimitNs : static_cast<unsigned long long>(nanoseconds);
  return fg::set_wait_limit(device, ns);
}

}  // extern "C"
