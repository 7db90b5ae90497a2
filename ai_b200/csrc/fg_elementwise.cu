// Memory-bound encoder kernels: one warp per row, the row held in registers,
// float4 loads and stores, warp-shuffle reductions. Products and sums that
// the reference writes as separate float32 operations use the _rn
// intrinsics so the compiler does not contract them into FMAs.
#include <algorithm>
#include <cmath>

#include "fg_kernels.cuh"
#include "fg_ptx.cuh"

namespace fg {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// 1/√(ss/n + eps) with the division and sum in float32 and the root in
// float64, cast back to float32: rmsScale (embed.go:432-438) and
// rmsNormFused (attention.go:328).
__device__ __forceinline__ float rms_inv(float ss, int n, float eps) {
  const float m = __fadd_rn(__fdiv_rn(ss, float(n)), eps);
  return float(1.0 / sqrt(double(m)));
}

__device__ __forceinline__ float sq_acc(float acc, float v) { return __fadd_rn(acc, __fmul_rn(v, v)); }

constexpr int kWarpsPerBlock = 8;

// ---------------------------------------------------------------- gather
// Row `id` of the table, chunk c of a lane: 4 consecutive values.
template <typename TT>
__device__ __forceinline__ float4 table_chunk(const TT* table, int64_t id, int n, int i4);
template <>
__device__ __forceinline__ float4 table_chunk<float>(const float* table, int64_t id, int n, int i4) {
  return __ldg(reinterpret_cast<const float4*>(table + id * n) + i4);
}
template <>
__device__ __forceinline__ float4 table_chunk<uint16_t>(const uint16_t* table, int64_t id, int n, int i4) {
  // bf16 → fp32 is exact: the bf16 bits are the fp32's upper half
  const uint2 h = __ldg(reinterpret_cast<const uint2*>(table + id * n) + i4);
  return make_float4(__uint_as_float(h.x << 16), __uint_as_float(h.x & 0xffff0000u),
                     __uint_as_float(h.y << 16), __uint_as_float(h.y & 0xffff0000u));
}

template <int C4, typename TT>
__global__ void __launch_bounds__(256) embed_kernel(const TT* __restrict__ table, int64_t vocab,
                                                    const int32_t* __restrict__ ids,
                                                    const int32_t* __restrict__ lengths, int B, int T,
                                                    int n, float emb_scale, float eps,
                                                    float* __restrict__ x, float* __restrict__ x_lo,
                                                    float* __restrict__ rowscale, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kWarpsPerBlock + warp;
  if (row >= int64_t(B) * T) return;
  const int b = int(row / T), t = int(row % T);
  const int len = lengths[b];
  float4* xr = reinterpret_cast<float4*>(x + row * n);
  float4* lr = x_lo ? reinterpret_cast<float4*>(x_lo + row * n) : nullptr;
  if (t >= max(len, 1)) {
#pragma unroll
    for (int c = 0; c < C4; ++c) {
      xr[lane + 32 * c] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (lr) lr[lane + 32 * c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (lane == 0) rowscale[row] = rms_inv(0.f, n, eps);
    return;
  }
  int64_t id = (len == 0) ? 0 : int64_t(ids[row]);
  if (id < 0 || id >= vocab) {
    if (lane == 0) atomicCAS(err, 0, kDevBadArgs);
    id = 0;
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < C4; ++c) {
    float4 v = table_chunk<TT>(table, id, n, lane + 32 * c);
    v.x = __fmul_rn(v.x, emb_scale);
    v.y = __fmul_rn(v.y, emb_scale);
    v.z = __fmul_rn(v.z, emb_scale);
    v.w = __fmul_rn(v.w, emb_scale);
    ss = sq_acc(ss, v.x);
    ss = sq_acc(ss, v.y);
    ss = sq_acc(ss, v.z);
    ss = sq_acc(ss, v.w);
    xr[lane + 32 * c] = v;
    if (lr) lr[lane + 32 * c] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
  }
  ss = warp_sum(ss);
  if (lane == 0) rowscale[row] = rms_inv(ss, n, eps);
}

// ------------------------------------------------------- QK-norm + RoPE
// One warp per (row, head). Heads [0, Hq) are queries, [Hq, Hq+Hkv) keys,
// [Hq+Hkv, Hq+2Hkv) values: RMS-normalised with vgain when one is given
// (EmbeddingGemma 2's weight-free v_norm, embed.go:300), and split when a
// lo buffer is given; no RoPE on values.
constexpr int kMaxPairs = 8;  // D ≤ 512
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    float* __restrict__ qkv, float* __restrict__ qkv_lo, int64_t rows, int Hq, int Hkv, int D,
    int heads_done, const float* __restrict__ qgain, const float* __restrict__ kgain,
    const float* __restrict__ vgain, float eps, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int T) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t task = int64_t(blockIdx.x) * kWarpsPerBlock + warp;
  if (task >= rows * heads_done) return;
  const int64_t row = task / heads_done;
  const int head = int(task % heads_done);
  const int half = D / 2;
  const int width = (Hq + 2 * Hkv) * D;
  float* v = qkv + row * width + int64_t(head) * D;
  float* vl = qkv_lo ? qkv_lo + row * width + int64_t(head) * D : nullptr;
  const bool value = head >= Hq + Hkv;
  if (value && !vgain) {  // value head: split only
    for (int i = lane; i < D; i += 32) vl[i] = tf32_lo(v[i]);
    return;
  }
  const float* g = value ? vgain : (head < Hq ? qgain : kgain);
  float a[kMaxPairs], b2[kMaxPairs];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) {
    const int i = lane + 32 * p;
    a[p] = 0.f;
    b2[p] = 0.f;
    if (i < half) {
      a[p] = v[i];
      b2[p] = v[i + half];
    }
  }
  // Σx² in element order within each lane's slice of each half.
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) ss = sq_acc(ss, a[p]);
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) ss = sq_acc(ss, b2[p]);
  ss = warp_sum(ss);
  const float inv = rms_inv(ss, D, eps);
  if (value) {
#pragma unroll
    for (int p = 0; p < kMaxPairs; ++p) {
      const int i = lane + 32 * p;
      if (i < half) {
        const float y1 = __fmul_rn(__fmul_rn(a[p], inv), g[i]);
        const float y2 = __fmul_rn(__fmul_rn(b2[p], inv), g[i + half]);
        v[i] = y1;
        v[i + half] = y2;
        if (vl) {
          vl[i] = tf32_lo(y1);
          vl[i + half] = tf32_lo(y2);
        }
      }
    }
    return;
  }
  const int t = int(row % T);
  const float* c = cos_t + int64_t(t) * half;
  const float* s = sin_t + int64_t(t) * half;
#pragma unroll
  for (int p = 0; p < kMaxPairs; ++p) {
    const int i = lane + 32 * p;
    if (i < half) {
      const float x1 = __fmul_rn(__fmul_rn(a[p], inv), g[i]);
      const float x2 = __fmul_rn(__fmul_rn(b2[p], inv), g[i + half]);
      const float ci = c[i], si = s[i];
      const float y1 = __fsub_rn(__fmul_rn(x1, ci), __fmul_rn(x2, si));
      const float y2 = __fadd_rn(__fmul_rn(x1, si), __fmul_rn(x2, ci));
      v[i] = y1;
      v[i + half] = y2;
      if (vl) {
        vl[i] = tf32_lo(y1);
        vl[i + half] = tf32_lo(y2);
      }
    }
  }
}

// ------------------------------------------------- residual + post-norm
template <int C4>
__global__ void __launch_bounds__(256) residual_postnorm_kernel(
    float* __restrict__ x, Split16Out parts, const float* __restrict__ o,
    const float* __restrict__ gain, float eps, float* __restrict__ rowscale,
    const float* __restrict__ fgain, int64_t rows, int n, float scalar) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kWarpsPerBlock + warp;
  if (row >= rows) return;
  const float4* o4 = reinterpret_cast<const float4*>(o + row * n);
  float4* x4 = reinterpret_cast<float4*>(x + row * n);
  const float4* g4 = reinterpret_cast<const float4*>(gain);
  float4 ov[C4], xv[C4];
  float sso = 0.f;
#pragma unroll
  for (int c = 0; c < C4; ++c) {
    ov[c] = o4[lane + 32 * c];
    sso = sq_acc(sso, ov[c].x);
    sso = sq_acc(sso, ov[c].y);
    sso = sq_acc(sso, ov[c].z);
    sso = sq_acc(sso, ov[c].w);
  }
  sso = warp_sum(sso);
  const float inv_o = rms_inv(sso, n, eps);
  float ssx = 0.f;
#pragma unroll
  for (int c = 0; c < C4; ++c) {
    const float4 g = __ldg(g4 + lane + 32 * c);
    float4 xx = x4[lane + 32 * c];
    xx.x = __fadd_rn(xx.x, __fmul_rn(__fmul_rn(ov[c].x, inv_o), g.x));
    xx.y = __fadd_rn(xx.y, __fmul_rn(__fmul_rn(ov[c].y, inv_o), g.y));
    xx.z = __fadd_rn(xx.z, __fmul_rn(__fmul_rn(ov[c].z, inv_o), g.z));
    xx.w = __fadd_rn(xx.w, __fmul_rn(__fmul_rn(ov[c].w, inv_o), g.w));
    // EmbeddingGemma 2's layer scalar (embed.go:370-371); 1 elsewhere (exact)
    xx.x = __fmul_rn(xx.x, scalar);
    xx.y = __fmul_rn(xx.y, scalar);
    xx.z = __fmul_rn(xx.z, scalar);
    xx.w = __fmul_rn(xx.w, scalar);
    xv[c] = xx;
    ssx = sq_acc(ssx, xx.x);
    ssx = sq_acc(ssx, xx.y);
    ssx = sq_acc(ssx, xx.z);
    ssx = sq_acc(ssx, xx.w);
  }
  ssx = warp_sum(ssx);
  const float inv_x = rms_inv(ssx, n, eps);
  if (fgain) {
    const float4* f4 = reinterpret_cast<const float4*>(fgain);
#pragma unroll
    for (int c = 0; c < C4; ++c) {
      const float4 g = __ldg(f4 + lane + 32 * c);
      float4 y;
      y.x = __fmul_rn(__fmul_rn(xv[c].x, inv_x), g.x);
      y.y = __fmul_rn(__fmul_rn(xv[c].y, inv_x), g.y);
      y.z = __fmul_rn(__fmul_rn(xv[c].z, inv_x), g.z);
      y.w = __fmul_rn(__fmul_rn(xv[c].w, inv_x), g.w);
      x4[lane + 32 * c] = y;
    }
    return;
  }
#pragma unroll
  for (int c = 0; c < C4; ++c) x4[lane + 32 * c] = xv[c];
  if (parts.hi) {
    // the next product's fp16 parts of this row, as its converters would cut them
    const int e = max(-60, min(60, 13 - ilogbf(parts.norm_k / inv_x)));
    const float sc = pow2f(e);
    uint2* h2 = reinterpret_cast<uint2*>(parts.hi + row * n);
    uint2* l2 = reinterpret_cast<uint2*>(parts.lo + row * n);
    const float4* pg4 = reinterpret_cast<const float4*>(parts.gain);
#pragma unroll
    for (int c = 0; c < C4; ++c) {
      const float4 v = xv[c];
      float a0, a1, a2, a3;
      if (parts.gain) {
        const float4 g = __ldg(pg4 + lane + 32 * c);
        a0 = v.x * (g.x * sc); a1 = v.y * (g.y * sc); a2 = v.z * (g.z * sc); a3 = v.w * (g.w * sc);
      } else {
        a0 = v.x * sc; a1 = v.y * sc; a2 = v.z * sc; a3 = v.w * sc;
      }
      const float q0 = tf32_hi(a0), q1 = tf32_hi(a1), q2 = tf32_hi(a2), q3 = tf32_hi(a3);
      h2[lane + 32 * c] = make_uint2(pack_f16x2(q0, q1), pack_f16x2(q2, q3));
      l2[lane + 32 * c] = make_uint2(pack_f16x2(a0 - q0, a1 - q1), pack_f16x2(a2 - q2, a3 - q3));
    }
  }
  if (lane == 0) rowscale[row] = inv_x;
}

// ---------------------------------------------------------------- pooling
__global__ void mean_pool_kernel(const float* __restrict__ h, const int32_t* __restrict__ lengths,
                                 int T, int n, float* __restrict__ pooled,
                                 float* __restrict__ pooled_lo) {
  const int b = blockIdx.x;
  const int col = blockIdx.y * blockDim.x + threadIdx.x;
  if (col >= n) return;
  const int cnt = max(lengths[b], 1);
  const float* base = h + int64_t(b) * T * n + col;
  float acc = 0.f;
#pragma unroll 8
  for (int t = 0; t < cnt; ++t) acc = __fadd_rn(acc, base[int64_t(t) * n]);
  const float inv = __fdiv_rn(1.f, float(cnt));
  const float r = __fmul_rn(acc, inv);
  pooled[int64_t(b) * n + col] = r;
  if (pooled_lo) pooled_lo[int64_t(b) * n + col] = tf32_lo(r);
}

__global__ void l2_kernel(const float* __restrict__ x, int64_t ldx, int B, int dim, int l2,
                          float* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * kWarpsPerBlock + warp;
  if (b >= B) return;
  const float* r = x + int64_t(b) * ldx;
  float ss = 0.f;
  if (l2)
    for (int i = lane; i < dim; i += 32) ss = sq_acc(ss, r[i]);
  ss = warp_sum(ss);
  const float nrm = __fsqrt_rn(__fadd_rn(ss, 1e-12f));
  for (int i = lane; i < dim; i += 32) out[int64_t(b) * dim + i] = l2 ? __fdiv_rn(r[i], nrm) : r[i];
}

// ------------------------------------------------------ op-level generic
__global__ void row_sumsq_kernel(const float* __restrict__ x, int64_t rows, int64_t n, int64_t ldx,
                                 float* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kWarpsPerBlock + warp;
  if (row >= rows) return;
  const float* r = x + row * ldx;
  float ss = 0.f;
  for (int64_t i = lane; i < n; i += 32) ss = sq_acc(ss, r[i]);
  ss = warp_sum(ss);
  if (lane == 0) out[row] = ss;
}

// out may equal x (each row is read in full before it is written).
__global__ void rmsnorm_kernel(const float* x, int64_t rows, int64_t n, const float* __restrict__ g,
                               float eps, float* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * kWarpsPerBlock + warp;
  if (row >= rows) return;
  const float* r = x + row * n;
  float ss = 0.f;
  for (int64_t i = lane; i < n; i += 32) ss = sq_acc(ss, r[i]);
  ss = warp_sum(ss);
  const float inv = rms_inv(ss, int(n), eps);
  for (int64_t i = lane; i < n; i += 32) out[row * n + i] = __fmul_rn(__fmul_rn(r[i], inv), g[i]);
}

__global__ void rope_kernel(const float* __restrict__ x, int64_t rows, int T, int D,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            float* __restrict__ out) {
  const int half = D / 2;
  const int64_t total = rows * half;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = e / half;
    const int i = int(e % half);
    const int t = int(row % T);
    const float c = cos_t[int64_t(t) * half + i], s = sin_t[int64_t(t) * half + i];
    const float x1 = x[row * D + i], x2 = x[row * D + i + half];
    out[row * D + i] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    out[row * D + i + half] = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
  }
}

__global__ void split_copy_kernel(const float* __restrict__ src, int64_t lds, int64_t rows,
                                  int64_t cols, float* __restrict__ hi, float* __restrict__ lo,
                                  int64_t ldd, int truncate_hi) {
  const int64_t total = rows * cols;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / cols, c = e % cols;
    const float v = src[r * lds + c];
    if (hi) hi[r * ldd + c] = truncate_hi ? tf32_hi(v) : v;
    if (lo) lo[r * ldd + c] = tf32_lo(v);
  }
}

int grid_for(int64_t tasks, int per_block) {
  return int(std::max<int64_t>(1, (tasks + per_block - 1) / per_block));
}

}  // namespace

int embed_gather(const float* table, const uint16_t* table_bf16, int64_t vocab, const int32_t* ids,
                 const int32_t* lengths, int B, int T, int hidden, float emb_scale, float eps, float* x,
                 float* x_lo, float* rowscale, int* err, cudaStream_t s) {
  const int64_t rows = int64_t(B) * T;
  if (rows == 0) return FG_OK;
  const int grid = grid_for(rows, kWarpsPerBlock);
  switch (hidden / 128) {
#define FG_EMB(C)                                                                                   \
  case C:                                                                                           \
    if (table_bf16)                                                                                 \
      embed_kernel<C, uint16_t><<<grid, 256, 0, s>>>(table_bf16, vocab, ids, lengths, B, T, hidden, \
                                                     emb_scale, eps, x, x_lo, rowscale, err);       \
    else                                                                                            \
      embed_kernel<C, float><<<grid, 256, 0, s>>>(table, vocab, ids, lengths, B, T, hidden,         \
                                                  emb_scale, eps, x, x_lo, rowscale, err);          \
    break;
    FG_EMB(1) FG_EMB(2) FG_EMB(3) FG_EMB(4) FG_EMB(5) FG_EMB(6) FG_EMB(7) FG_EMB(8)
#undef FG_EMB
    default:
      return set_error(FG_EINVAL, "hidden size %d unsupported (multiple of 128 up to 1024)", hidden);
  }
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int qk_norm_rope(float* qkv, float* qkv_lo, int64_t rows, int Hq, int Hkv, int D,
                 const float* qgain, const float* kgain, const float* vgain, float eps,
                 const float* cos_t, const float* sin_t, int T, cudaStream_t s) {
  if (rows == 0) return FG_OK;
  if (D % 2 != 0 || D / 2 > 32 * kMaxPairs)
    return set_error(FG_EINVAL, "head_dim %d unsupported (even, at most 512)", D);
  const int heads = Hq + Hkv + ((qkv_lo || vgain) ? Hkv : 0);
  const int grid = grid_for(rows * heads, kWarpsPerBlock);
  qk_norm_rope_kernel<<<grid, 256, 0, s>>>(qkv, qkv_lo, rows, Hq, Hkv, D, heads, qgain, kgain, vgain,
                                           eps, cos_t, sin_t, T);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int residual_postnorm(float* x, const Split16Out* parts, const float* o, const float* gain, float eps,
                      float* rowscale, const float* final_gain, int64_t rows, int n,
                      cudaStream_t s, float scalar) {
  if (rows == 0) return FG_OK;
  const Split16Out p16 = parts ? *parts : Split16Out{nullptr, nullptr, nullptr, 0.f};
  const int grid = grid_for(rows, kWarpsPerBlock);
  switch (n / 128) {
#define FG_RES(C) \
  case C: residual_postnorm_kernel<C><<<grid, 256, 0, s>>>(x, p16, o, gain, eps, rowscale, final_gain, rows, n, scalar); break;
    FG_RES(1) FG_RES(2) FG_RES(3) FG_RES(4) FG_RES(5) FG_RES(6) FG_RES(7) FG_RES(8)
#undef FG_RES
    default:
      return set_error(FG_EINVAL, "hidden size %d unsupported (multiple of 128 up to 1024)", n);
  }
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int mean_pool(const float* h, const int32_t* lengths, int B, int T, int n, float* pooled,
              float* pooled_lo, cudaStream_t s) {
  if (B == 0) return FG_OK;
  dim3 grid(unsigned(B), unsigned((n + 127) / 128));
  mean_pool_kernel<<<grid, 128, 0, s>>>(h, lengths, T, n, pooled, pooled_lo);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int l2_normalize(const float* x, int64_t ldx, int B, int dim, int l2, float* out, cudaStream_t s) {
  if (B == 0) return FG_OK;
  l2_kernel<<<grid_for(B, kWarpsPerBlock), 256, 0, s>>>(x, ldx, B, dim, l2, out);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int row_sum_squares(const float* x, int64_t rows, int64_t n, int64_t ldx, float* out,
                    cudaStream_t s) {
  if (rows == 0) return FG_OK;
  row_sumsq_kernel<<<grid_for(rows, kWarpsPerBlock), 256, 0, s>>>(x, rows, n, ldx, out);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int rmsnorm(const float* x, int64_t rows, int64_t n, const float* g, float eps, float* out,
            cudaStream_t s) {
  if (rows == 0) return FG_OK;
  rmsnorm_kernel<<<grid_for(rows, kWarpsPerBlock), 256, 0, s>>>(x, rows, n, g, eps, out);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int rope(const float* x, int64_t rows, int T, int D, const float* cos_t, const float* sin_t,
         float* out, cudaStream_t s) {
  if (rows == 0) return FG_OK;
  const int64_t total = rows * (D / 2);
  const int grid = int(std::min<int64_t>(grid_for(total, 256), int64_t(sm_count()) * 32));
  rope_kernel<<<grid, 256, 0, s>>>(x, rows, T, D, cos_t, sin_t, out);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int split_copy_2d(const float* src, int64_t lds, int64_t rows, int64_t cols, float* hi, float* lo,
                  int64_t ldd, int truncate_hi, cudaStream_t s) {
  const int64_t total = rows * cols;
  if (total == 0) return FG_OK;
  const int grid = int(std::min<int64_t>(grid_for(total, 256), int64_t(sm_count()) * 32));
  split_copy_kernel<<<grid, 256, 0, s>>>(src, lds, rows, cols, hi, lo, ldd, truncate_hi);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

}  // namespace fg
