// Downstream of the embeddings: fiber/ai's cluster package
// (cluster/cluster.go) on device buffers — Normalize (:19-28),
// Similarities (:185-190), Nearest (:136-148) and KMeans with k-means++
// seeding (:43-133). As in the reference, every similarity matrix is one
// product on the tensor cores (the split-TF32 GEMM of fg_gemm.cu); the rest
// is memory-bound row work:
//   - argmax over a row of similarities keeps the first maximum, as
//     tensor.Argmax (tensor/reduce.go:269-297);
//   - a centre's sum adds its rows in row order in float32 (the
//     reference's loop, cluster.go:101-108): rows are stably sorted by
//     centre, then one thread per (centre, column) walks its rows in order,
//     so the sums do not depend on scheduling;
//   - the k-means++ draws come from a restatement of Go's math/rand/v2 PCG
//     (128-bit LCG, DXSM output; O'Neill's published PCG constants) with
//     Rand.IntN (Lemire's multiply-and-reject) and Rand.Float64 (53 bits),
//     seeded as KMeans seeds it, and the weighted pick walks the weights in
//     float64 on the host exactly as cluster.go:67-79 does.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include <cub/device/device_radix_sort.cuh>

#include "fg_internal.h"
#include "fg_kernels.cuh"

namespace fg {
namespace {

constexpr int kRowWarps = 8;  // rows per 256-thread block in the row kernels

int64_t round_up4(int64_t v) { return (v + 3) / 4 * 4; }

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// out = x / ‖x‖ per row; a zero row stays zero (its norm is taken as 1).
__global__ void __launch_bounds__(256) normalize_rows_kernel(const float* __restrict__ x, int64_t ldx,
                                                             int64_t n, int d, float* __restrict__ out,
                                                             int64_t ldo) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  if (row >= n) return;
  const float* xr = x + row * ldx;
  float ss = 0.f;
  for (int j = lane; j < d; j += 32) ss = __fmaf_rn(xr[j], xr[j], ss);
  ss = warp_sum_f(ss);
  float norm = __fsqrt_rn(ss);
  if (norm == 0.f) norm = 1.f;
  float* orow = out + row * ldo;
  for (int j = lane; j < d; j += 32) orow[j] = __fdiv_rn(xr[j], norm);
}

// best[i] = max(best[i], x_i · c) — one k-means++ round (cluster.go:60-66).
// A NaN similarity never replaces the best, as `sim > best` never holds.
__global__ void __launch_bounds__(256) dot_max_kernel(const float* __restrict__ x, int64_t ldx, int64_t n,
                                                      int d, const float* __restrict__ c,
                                                      float* __restrict__ best) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kRowWarps + (threadIdx.x >> 5);
  if (row >= n) return;
  const float* xr = x + row * ldx;
  float acc = 0.f;
  for (int j = lane; j < d; j += 32) acc = __fmaf_rn(xr[j], __ldg(c + j), acc);
  acc = warp_sum_f(acc);
  if (lane == 0 && acc > best[row]) best[row] = acc;
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    p[i] = v;
}

// Per row of sim [n, k]: the first column holding the maximum (a NaN in
// column 0 keeps column 0, later NaNs are skipped, as tensor.Argmax's
// `v > best` scan does) and its value. LPR lanes share a row (LPR = 32 /
// rows per warp), each scanning columns sub, sub + LPR, …; with `index`
// holding the previous assignment, changed rows are counted before it is
// overwritten; `sizes` counts rows per column.
template <int LPR>
__global__ void __launch_bounds__(256) argmax_rows_kernel(const float* __restrict__ sim, int64_t lds, int64_t n,
                                                          int k, int32_t* __restrict__ index,
                                                          float* __restrict__ value, int32_t* __restrict__ changed,
                                                          int32_t* __restrict__ sizes) {
  constexpr int kRowsPerWarp = 32 / LPR;
  const int lane = threadIdx.x & 31, sub = lane % LPR;
  const int64_t row = (int64_t(blockIdx.x) * kRowWarps + (threadIdx.x >> 5)) * kRowsPerWarp + lane / LPR;
  const bool live = row < n;
  const float* s = sim + (live ? row : 0) * lds;
  float best = -INFINITY;
  int bi = -1;
  if (live) {
    for (int j = sub; j < k; j += LPR) {
      const float v = s[j];
      if (v > best || (bi < 0 && v == best)) {  // v == -inf still claims the slot
        best = v;
        bi = j;
      }
    }
  }
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi >= 0 && (bi < 0 || ob > best || (ob == best && oi < bi))) {
      best = ob;
      bi = oi;
    }
  }
  if (!live || sub != 0) return;
  const float first = s[0];
  if (isnan(first) || bi < 0) {  // column 0 is the answer when nothing beats it
    best = first;
    bi = 0;
  }
  if (changed && index[row] != bi) atomicAdd(changed, 1);
  index[row] = bi;
  value[row] = best;
  if (sizes) atomicAdd(&sizes[bi], 1);
}

int argmax_rows(const float* sim, int64_t lds, int64_t n, int k, int32_t* index, float* value,
                int32_t* changed, int32_t* sizes, cudaStream_t s) {
  auto grid = [&](int rows_per_warp) { return int((n + int64_t(kRowWarps) * rows_per_warp - 1) / (int64_t(kRowWarps) * rows_per_warp)); };
  if (k <= 16)
    argmax_rows_kernel<4><<<grid(8), 256, 0, s>>>(sim, lds, n, k, index, value, changed, sizes);
  else if (k <= 64)
    argmax_rows_kernel<8><<<grid(4), 256, 0, s>>>(sim, lds, n, k, index, value, changed, sizes);
  else if (k <= 256)
    argmax_rows_kernel<16><<<grid(2), 256, 0, s>>>(sim, lds, n, k, index, value, changed, sizes);
  else
    argmax_rows_kernel<32><<<grid(1), 256, 0, s>>>(sim, lds, n, k, index, value, changed, sizes);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

__global__ void iota_kernel(int32_t* p, int64_t n) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    p[i] = int32_t(i);
}

// sums[c][j] = Σ x[i][j] over the rows i of centre c, added in increasing i
// in float32. rows: all row indices stably sorted by centre; sizes: rows
// per centre. Block (c, 128-column chunk), one thread per column.
__global__ void __launch_bounds__(128) centre_sums_kernel(const float* __restrict__ x, int64_t ldx, int d,
                                                          const int32_t* __restrict__ rows,
                                                          const int32_t* __restrict__ sizes,
                                                          float* __restrict__ sums, int64_t lds) {
  __shared__ int64_t s_off;
  __shared__ int32_t s_rows[128];
  const int c = blockIdx.x;
  const int j = blockIdx.y * 128 + threadIdx.x;
  if (threadIdx.x == 0) {
    int64_t off = 0;
    for (int i = 0; i < c; ++i) off += sizes[i];
    s_off = off;
  }
  __syncthreads();
  const int64_t off = s_off;
  const int cnt = sizes[c];
  float acc = 0.f;
  for (int base = 0; base < cnt; base += 128) {
    const int m = min(128, cnt - base);
    __syncthreads();
    if (threadIdx.x < m) s_rows[threadIdx.x] = rows[off + base + threadIdx.x];
    __syncthreads();
    if (j < d) {
      int r = 0;
      for (; r + 4 <= m; r += 4) {
        const float v0 = x[int64_t(s_rows[r]) * ldx + j];
        const float v1 = x[int64_t(s_rows[r + 1]) * ldx + j];
        const float v2 = x[int64_t(s_rows[r + 2]) * ldx + j];
        const float v3 = x[int64_t(s_rows[r + 3]) * ldx + j];
        acc = __fadd_rn(acc, v0);
        acc = __fadd_rn(acc, v1);
        acc = __fadd_rn(acc, v2);
        acc = __fadd_rn(acc, v3);
      }
      for (; r < m; ++r) acc = __fadd_rn(acc, x[int64_t(s_rows[r]) * ldx + j]);
    }
  }
  if (j < d) sums[int64_t(c) * lds + j] = acc;
}

// The first index of the smallest value (a NaN at 0 keeps 0), one block.
__global__ void __launch_bounds__(1024) argmin_kernel(const float* __restrict__ v, int64_t n, int64_t* out) {
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  float best = INFINITY;
  int64_t bi = -1;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = v[i];
    if (x < best || (bi < 0 && x == best)) {
      best = x;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi >= 0 && (bi < 0 || ob < best || (ob == best && oi < bi))) {
      best = ob;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : INFINITY;
    bi = lane < nw ? si[lane] : -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ob < best || (ob == best && oi < bi))) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) *out = (isnan(v[0]) || bi < 0) ? 0 : bi;
  }
}

int row_grid(int64_t n) { return int((n + kRowWarps - 1) / kRowWarps); }

// Go's math/rand/v2 PCG source and the two Rand methods KMeans uses.
struct GoRand {
  uint64_t hi, lo;
  uint64_t uint64() {
    const unsigned __int128 mul = (static_cast<unsigned __int128>(0x2360ed051fc65da4ULL) << 64) | 0x4385df649fccf645ULL;
    const unsigned __int128 inc = (static_cast<unsigned __int128>(0x5851f42d4c957f2dULL) << 64) | 0x14057b7ef767814fULL;
    unsigned __int128 st = (static_cast<unsigned __int128>(hi) << 64) | lo;
    st = st * mul + inc;
    hi = uint64_t(st >> 64);
    lo = uint64_t(st);
    uint64_t h = hi;  // DXSM output of the new state
    h ^= h >> 32;
    h *= 0xda942042e4dd58b5ULL;
    h ^= h >> 48;
    h *= lo | 1;
    return h;
  }
  uint64_t uint64n(uint64_t n) {
    if ((n & (n - 1)) == 0) return uint64() & (n - 1);
    unsigned __int128 p = static_cast<unsigned __int128>(uint64()) * n;
    uint64_t lo64 = uint64_t(p);
    if (lo64 < n) {
      const uint64_t thresh = (0 - n) % n;
      while (lo64 < thresh) {
        p = static_cast<unsigned __int128>(uint64()) * n;
        lo64 = uint64_t(p);
      }
    }
    return uint64_t(p >> 64);
  }
  int64_t intn(int64_t n) { return int64_t(uint64n(uint64_t(n))); }
  double float64() { return double((uint64() << 11) >> 11) / 9007199254740992.0; }
};

// Stream-ordered scratch from the library's per-device pool: released
// after the work queued on the stream before the release, and kept
// reserved by the pool for the next call.
struct DevScratch {
  cudaStream_t s;
  std::vector<void*> ptrs;
  explicit DevScratch(cudaStream_t st) : s(st) {}
  template <class T>
  int alloc(T** p, size_t count) {
    void* v = nullptr;
    FG_TRY(scratch_alloc(&v, std::max<size_t>(count, 1) * sizeof(T), s));
    ptrs.push_back(v);
    *p = static_cast<T*>(v);
    return FG_OK;
  }
  ~DevScratch() {
    for (void* v : ptrs) scratch_free(v, s);
  }
};

// sim[n, k] (leading dimension lds) = x · cᵀ for centres c [k, d] (rows
// unit length by contract). The product runs on the split-TF32 tensor-core
// GEMM with A = x read in place (its low part made in shared memory) when
// x's rows are 16-byte aligned, else through fg_matmul's packing.
// `cbuf` (optional, 2·k·round4(d) floats) holds the centres' split parts;
// without it they go to scratch from `ds`.
int similarities(const float* x, int64_t ldx, int64_t n, int64_t d, const float* c, int64_t ldc, int64_t k,
                 float* sim, int64_t lds, int precision, DevScratch& ds, cudaStream_t s,
                 float* cbuf = nullptr) {
  const bool a_direct = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 4 == 0;
  if (!a_direct || n > INT32_MAX || d > INT32_MAX || k > INT32_MAX)
    return fg_matmul(n, k, d, x, ldx, c, ldc, 1, sim, lds, nullptr, precision, s);
  int* err = nullptr;
  FG_TRY(device_error_word(&err));
  const int64_t dp = round_up4(d);
  const bool lo_pass = precision != FG_PREC_TF32;
  float *bhi = cbuf, *blo = cbuf ? cbuf + k * dp : nullptr;
  if (!bhi) {
    FG_TRY(ds.alloc(&bhi, size_t(k * dp)));
    if (lo_pass) FG_TRY(ds.alloc(&blo, size_t(k * dp)));
  }
  if (!lo_pass) blo = nullptr;
  FG_TRY(split_copy_2d(c, ldc, k, d, bhi, blo, dp, lo_pass ? 1 : 0, s));
  GemmArgs g;
  g.M = int(n);
  g.Nb = int(k);
  g.K = int(d);
  g.A = x;
  g.lda = ldx;
  g.a_lo_smem = lo_pass;
  g.B = bhi;
  g.B_lo = blo;
  g.ldb = dp;
  g.epi.out = sim;
  g.epi.ldo = lds;
  return gemm_tn(g, err, s);
}

}  // namespace
}  // namespace fg

using namespace fg;

extern "C" {

int fg_normalize_rows(int64_t n, int64_t d, const float* x, int64_t ldx, float* out, int64_t ldo,
                      void* stream) {
  clear_error();
  if (n < 0 || d < 0 || d > INT32_MAX) return set_error(FG_EINVAL, "fg_normalize_rows: bad shape");
  if (n == 0 || d == 0) return FG_OK;
  if (!x || !out || ldx < d || ldo < d) return set_error(FG_EINVAL, "fg_normalize_rows: bad operand");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  normalize_rows_kernel<<<row_grid(n), 256, 0, s>>>(x, ldx, n, int(d), out, ldo);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int fg_similarities(int64_t q, int64_t n, int64_t d, const float* queries, int64_t ldq, const float* docs,
                    int64_t ldd, float* out, int64_t ldo, int precision, void* stream) {
  clear_error();
  if (q < 0 || n < 0 || d <= 0) return set_error(FG_EINVAL, "fg_similarities: shapes [%lld x %lld] and [%lld x %lld]", (long long)q, (long long)d, (long long)n, (long long)d);
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "fg_similarities: unknown precision %d", precision);
  if (q == 0 || n == 0) return FG_OK;
  if (!queries || !docs || !out || ldq < d || ldd < d || ldo < n)
    return set_error(FG_EINVAL, "fg_similarities: bad operand");
  DevScratch ds(static_cast<cudaStream_t>(stream));
  return similarities(queries, ldq, q, d, docs, ldd, n, out, ldo, precision, ds, ds.s);
}

int fg_nearest(int64_t n, int64_t k, int64_t d, const float* x, int64_t ldx, const float* centres, int64_t ldc,
               int32_t* index, float* similarity, int precision, void* stream) {
  clear_error();
  if (n < 0 || k <= 0 || d <= 0 || k > INT32_MAX) return set_error(FG_EINVAL, "fg_nearest: bad shape");
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "fg_nearest: unknown precision %d", precision);
  if (n == 0) return FG_OK;
  if (!x || !centres || !index || !similarity || ldx < d || ldc < d)
    return set_error(FG_EINVAL, "fg_nearest: bad operand");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DevScratch ds(s);
  const int64_t lds = round_up4(k);
  float* sim = nullptr;
  FG_TRY(ds.alloc(&sim, size_t(n * lds)));
  FG_TRY(similarities(x, ldx, n, d, centres, ldc, k, sim, lds, precision, ds, s));
  return argmax_rows(sim, lds, n, int(k), index, similarity, nullptr, nullptr, s);
}

int fg_kmeans(int64_t n, int64_t d, const float* x, int64_t ldx, int k, int iters, uint64_t seed,
              float* centres, int32_t* assignment, float* similarity, int32_t* sizes, int* iterations,
              int precision, void* stream) {
  clear_error();
  if (k <= 0 || int64_t(k) > n) return set_error(FG_EINVAL, "cluster: k must be between 1 and the number of rows");
  if (d <= 0 || d > INT32_MAX || iters < 0) return set_error(FG_EINVAL, "fg_kmeans: bad shape");
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "fg_kmeans: unknown precision %d", precision);
  if (!x || !centres || !assignment || !similarity || !sizes || !iterations || ldx < d)
    return set_error(FG_EINVAL, "fg_kmeans: bad operand");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DevScratch ds(s);
  const int64_t lds = round_up4(k);
  float *best = nullptr, *raw = nullptr, *sim = nullptr;
  int32_t *changed = nullptr, *rows_in = nullptr, *rows = nullptr;
  uint32_t* keys_out = nullptr;
  int64_t* worst_d = nullptr;
  FG_TRY(ds.alloc(&best, size_t(n)));
  FG_TRY(ds.alloc(&raw, size_t(k) * size_t(d)));
  FG_TRY(ds.alloc(&sim, size_t(n * lds)));
  FG_TRY(ds.alloc(&changed, 1));
  FG_TRY(ds.alloc(&rows_in, size_t(n)));
  FG_TRY(ds.alloc(&rows, size_t(n)));
  FG_TRY(ds.alloc(&keys_out, size_t(n)));
  FG_TRY(ds.alloc(&worst_d, 1));
  float* cbuf = nullptr;  // the centres' split parts, reused every round
  FG_TRY(ds.alloc(&cbuf, size_t(2 * k) * size_t(round_up4(d))));
  // sort keys: the assignment, non-negative, read as unsigned
  const uint32_t* keys = reinterpret_cast<const uint32_t*>(assignment);
  int end_bit = 1;
  while ((int64_t(1) << end_bit) < k) ++end_bit;
  size_t sort_bytes = 0;
  FG_CUDA_TRY(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, keys, keys_out, rows_in, rows, n, 0, end_bit, s));
  uint8_t* sort_tmp = nullptr;
  FG_TRY(ds.alloc(&sort_tmp, sort_bytes));
  const size_t row_bytes = size_t(d) * sizeof(float);

  // k-means++ (cluster.go:50-83): the first centre uniformly, each further
  // one with probability ∝ (1 − best similarity)², walked in float64.
  GoRand r{seed, seed ^ 0x9e3779b97f4a7c15ULL};
  std::vector<float> hbest(static_cast<size_t>(n));
  const int64_t first = r.intn(n);
  FG_CUDA_TRY(cudaMemcpyAsync(raw, x + first * ldx, row_bytes, cudaMemcpyDeviceToDevice, s));
  fill_kernel<<<256, 256, 0, s>>>(best, n, -1.f);
  FG_CUDA_TRY(cudaGetLastError());
  for (int c = 1; c < k; ++c) {
    dot_max_kernel<<<row_grid(n), 256, 0, s>>>(x, ldx, n, int(d), raw + int64_t(c - 1) * d, best);
    FG_CUDA_TRY(cudaGetLastError());
    FG_CUDA_TRY(cudaMemcpyAsync(hbest.data(), best, size_t(n) * sizeof(float), cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    double total = 0;
    std::vector<double> w(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) {
      const double di = double(1.0f - hbest[size_t(i)]);  // float32 difference, then widened
      w[size_t(i)] = di * di;
      total += w[size_t(i)];
    }
    double pick = r.float64() * total;
    int64_t idx = n - 1;
    for (int64_t i = 0; i < n; ++i) {
      pick -= w[size_t(i)];
      if (pick <= 0) {
        idx = i;
        break;
      }
    }
    FG_CUDA_TRY(cudaMemcpyAsync(raw + int64_t(c) * d, x + idx * ldx, row_bytes, cudaMemcpyDeviceToDevice, s));
  }
  normalize_rows_kernel<<<row_grid(k), 256, 0, s>>>(raw, d, k, int(d), centres, d);
  FG_CUDA_TRY(cudaGetLastError());

  FG_CUDA_TRY(cudaMemsetAsync(assignment, 0, size_t(n) * sizeof(int32_t), s));
  FG_CUDA_TRY(cudaMemsetAsync(similarity, 0, size_t(n) * sizeof(float), s));
  FG_CUDA_TRY(cudaMemsetAsync(sizes, 0, size_t(k) * sizeof(int32_t), s));
  iota_kernel<<<256, 256, 0, s>>>(rows_in, n);
  FG_CUDA_TRY(cudaGetLastError());
  *iterations = 0;
  std::vector<int32_t> hsizes(static_cast<size_t>(k));
  const float one = 1.0f;
  for (int it = 1; it <= iters; ++it) {
    *iterations = it;
    // assignment: one product and a row argmax (cluster.go:88-99)
    FG_TRY(similarities(x, ldx, n, d, centres, d, k, sim, lds, precision, ds, s, cbuf));
    FG_CUDA_TRY(cudaMemsetAsync(changed, 0, sizeof(int32_t), s));
    FG_CUDA_TRY(cudaMemsetAsync(sizes, 0, size_t(k) * sizeof(int32_t), s));
    FG_TRY(argmax_rows(sim, lds, n, k, assignment, similarity, changed, sizes, s));
    // centre update: rows stably sorted by centre, summed in row order
    FG_CUDA_TRY(cub::DeviceRadixSort::SortPairs(sort_tmp, sort_bytes, keys, keys_out, rows_in, rows, n, 0,
                                                end_bit, s));
    centre_sums_kernel<<<dim3(unsigned(k), unsigned((d + 127) / 128)), 128, 0, s>>>(x, ldx, int(d), rows, sizes,
                                                                                   raw, d);
    FG_CUDA_TRY(cudaGetLastError());
    int32_t hchanged = 0;
    FG_CUDA_TRY(cudaMemcpyAsync(&hchanged, changed, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaMemcpyAsync(hsizes.data(), sizes, size_t(k) * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    for (int c = 0; c < k; ++c) {
      if (hsizes[size_t(c)] != 0) continue;
      // an empty centre restarts on the worst-fitting row (cluster.go:110-118)
      int64_t worst = 0;
      argmin_kernel<<<1, 1024, 0, s>>>(similarity, n, worst_d);
      FG_CUDA_TRY(cudaGetLastError());
      FG_CUDA_TRY(cudaMemcpyAsync(&worst, worst_d, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
      FG_CUDA_TRY(cudaStreamSynchronize(s));
      FG_CUDA_TRY(cudaMemcpyAsync(raw + int64_t(c) * d, x + worst * ldx, row_bytes, cudaMemcpyDeviceToDevice, s));
      FG_CUDA_TRY(cudaMemcpyAsync(similarity + worst, &one, sizeof(float), cudaMemcpyHostToDevice, s));
    }
    normalize_rows_kernel<<<row_grid(k), 256, 0, s>>>(raw, d, k, int(d), centres, d);
    FG_CUDA_TRY(cudaGetLastError());
    if (hchanged == 0 && it > 1) break;
  }
  FG_CUDA_TRY(cudaStreamSynchronize(s));
  return check_device_error_word();
}

}  // extern "C"
