// Flash-style attention on the SIMT FP32 pipe (first implementation).
//
// Replaces attentionFused / AttentionBlock (tensor/attention.go:130-287,
// internal/blas/attention.go:61-136) for the encoder's masks. Instead of
// adding a materialised −1e9 mask to every score, visibility is index
// arithmetic: key j is visible to query i when j < klen[b] and, on sliding
// layers, |i − j| < window; key tiles with no visible key are never loaded,
// so a local layer costs O(T · 2·window) instead of O(T²). Masked keys get
// weight exactly 0, as the reference's flushing exp gives them
// (internal/kernel/generic.go:283-291).
//
// One CTA: 64 query rows of one head, 256 threads. K/V tiles of 32 keys are
// staged in shared memory; scores and the P·V update are register-blocked.
#include <algorithm>
#include <atomic>
#include <cfloat>

#include "fg_kernels.cuh"

namespace fg {

namespace {

constexpr int kBQ = 64;

// Key tile: 32 keys up to head_dim 256; 16 keys at 512 so that the Q tile
// and the K/V tiles fit in shared memory (203 KB).
template <int DP>
struct AttnSmem {
  static constexpr int kKV = DP > 256 ? 16 : 32;
  static constexpr int kLd = DP + 4;
  static constexpr size_t kFloats = size_t(kBQ) * kLd + 2 * size_t(kKV) * kLd +
                                    size_t(kBQ) * (kKV + 1) + 2 * kBQ;
  static constexpr size_t kBytes = kFloats * 4;
};

__device__ __forceinline__ void load_row(float* dst, const float* src, int D, int DP, bool valid,
                                         bool vec) {
  // cooperative within a warp: lane covers float4 chunks
  const int lane = threadIdx.x & 31;
  if (!valid) {
    for (int c = lane * 4; c < DP; c += 128) *reinterpret_cast<float4*>(dst + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  if (vec) {
    for (int c = lane * 4; c < DP; c += 128) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < D) v = __ldg(reinterpret_cast<const float4*>(src + c));
      *reinterpret_cast<float4*>(dst + c) = v;
    }
  } else {
    for (int c = lane; c < DP; c += 32) dst[c] = c < D ? src[c] : 0.f;
  }
}

template <int DP>
__global__ void __launch_bounds__(256, 1) attn_simt_kernel(const AttnArgs a) {
  using SM = AttnSmem<DP>;
  constexpr int LD = SM::kLd;
  constexpr int kBKV = SM::kKV;
  constexpr int KK = kBKV / 8;  // keys per thread in the score phase
  constexpr int NJ = DP / 64;  // float4 column groups per thread in the P·V phase
  extern __shared__ float4 smem4[];
  float* sm = reinterpret_cast<float*>(smem4);
  float* Qs = sm;
  float* Ks = Qs + kBQ * LD;
  float* Vs = Ks + kBKV * LD;
  float* Ps = Vs + kBKV * LD;
  float* corr_s = Ps + kBQ * (kBKV + 1);
  float* l_s = corr_s + kBQ;

  const int qblk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.Hq / a.Hkv);
  const int i0 = qblk * kBQ;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int qlen = a.qlen ? min(a.qlen[b], a.T) : a.T;
  const int klen = a.klen ? min(a.klen[b], a.S) : a.S;
  float* outp = a.out + b * a.osb + h * a.osh;
  float* outl = a.out_lo ? a.out_lo + b * a.osb + h * a.osh : nullptr;
  const bool vec = (a.D % 4 == 0) && ((a.qst | a.kst | a.vst | a.qsb | a.ksb | a.vsb | a.qsh | a.ksh | a.vsh) % 4 == 0) &&
                   ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                     reinterpret_cast<uintptr_t>(a.v)) & 15) == 0;

  // P·V mapping: 4 rows × (NJ float4) columns per thread.
  const int orow = (tid >> 4) * 4;
  const int ocol = (tid & 15) * 4;

  if (i0 >= qlen) {
    for (int r = warp; r < kBQ; r += 8) {
      const int i = i0 + r;
      if (i >= a.T) break;
      for (int c = tid & 31; c < a.D; c += 32) {
        outp[int64_t(i) * a.ost + c] = 0.f;
        if (outl) outl[int64_t(i) * a.ost + c] = 0.f;
      }
    }
    return;
  }

  const float* qb = a.q + b * a.qsb + h * a.qsh;
  const float* kb = a.k + b * a.ksb + hk * a.ksh;
  const float* vb = a.v + b * a.vsb + hk * a.vsh;
  for (int r = warp; r < kBQ; r += 8) {
    const int i = i0 + r;
    load_row(Qs + r * LD, qb + int64_t(i) * a.qst, a.D, DP, i < a.T, vec);
  }

  int kbeg = 0, kend = klen;
  if (a.window > 0) {
    kbeg = max(0, i0 - a.window + 1);
    kend = min(klen, i0 + kBQ - 1 + a.window);
  }

  // score mapping: rows 2·ty, 2·ty+1; keys tx + 8·kk
  const int ty = tid >> 3, tx = tid & 7;
  float m_r[2] = {-FLT_MAX, -FLT_MAX};
  bool any_r[2] = {false, false};
  float l_r[2] = {0.f, 0.f};
  float o[4][NJ][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[r][j][e] = 0.f;

  for (int j0 = (kbeg / kBKV) * kBKV; j0 < kend; j0 += kBKV) {
    __syncthreads();
    for (int r = warp; r < kBKV; r += 8) {
      const int j = j0 + r;
      load_row(Ks + r * LD, kb + int64_t(j) * a.kst, a.D, DP, j < a.S, vec);
      load_row(Vs + r * LD, vb + int64_t(j) * a.vst, a.D, DP, j < a.S, vec);
    }
    __syncthreads();

    float sc[2][KK];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int kk = 0; kk < KK; ++kk) sc[r][kk] = 0.f;
    const float* q0p = Qs + (2 * ty) * LD;
    const float* q1p = q0p + LD;
#pragma unroll 4
    for (int d = 0; d < DP; d += 4) {
      const float4 q0 = *reinterpret_cast<const float4*>(q0p + d);
      const float4 q1 = *reinterpret_cast<const float4*>(q1p + d);
#pragma unroll
      for (int kk = 0; kk < KK; ++kk) {
        const float4 kv = *reinterpret_cast<const float4*>(Ks + (tx + 8 * kk) * LD + d);
        sc[0][kk] = fmaf(q0.x, kv.x, sc[0][kk]);
        sc[0][kk] = fmaf(q0.y, kv.y, sc[0][kk]);
        sc[0][kk] = fmaf(q0.z, kv.z, sc[0][kk]);
        sc[0][kk] = fmaf(q0.w, kv.w, sc[0][kk]);
        sc[1][kk] = fmaf(q1.x, kv.x, sc[1][kk]);
        sc[1][kk] = fmaf(q1.y, kv.y, sc[1][kk]);
        sc[1][kk] = fmaf(q1.z, kv.z, sc[1][kk]);
        sc[1][kk] = fmaf(q1.w, kv.w, sc[1][kk]);
      }
    }

#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = i0 + 2 * ty + r;
      bool vis[KK];
      float tmax = -FLT_MAX;
      bool tany = false;
#pragma unroll
      for (int kk = 0; kk < KK; ++kk) {
        const int j = j0 + tx + 8 * kk;
        vis[kk] = j < klen && (a.window <= 0 || (i - j < a.window && j - i < a.window));
        if (vis[kk]) {
          tmax = fmaxf(tmax, sc[r][kk]);
          tany = true;
        }
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
        tany = tany | (__shfl_xor_sync(0xffffffffu, int(tany), off) != 0);
      }
      float corr = 1.f;
      if (tany) {
        const float m_new = any_r[r] ? fmaxf(m_r[r], tmax) : tmax;
        corr = any_r[r] ? expf(a.scale * (m_r[r] - m_new)) : 0.f;
        m_r[r] = m_new;
        any_r[r] = true;
      }
      float psum = 0.f;
#pragma unroll
      for (int kk = 0; kk < KK; ++kk) {
        const float p = (vis[kk] && any_r[r]) ? expf(a.scale * (sc[r][kk] - m_r[r])) : 0.f;
        Ps[(2 * ty + r) * (kBKV + 1) + tx + 8 * kk] = p;
        psum += p;
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l_r[r] = l_r[r] * corr + psum;
      if (tx == 0) corr_s[2 * ty + r] = corr;
    }
    __syncthreads();

    float cr[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) cr[r] = corr_s[orow + r];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[r][j][e] *= cr[r];
#pragma unroll 4
    for (int kk = 0; kk < kBKV; ++kk) {
      float p[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) p[r] = Ps[(orow + r) * (kBKV + 1) + kk];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const float4 vv = *reinterpret_cast<const float4*>(Vs + kk * LD + ocol + 64 * j);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          o[r][j][0] = fmaf(p[r], vv.x, o[r][j][0]);
          o[r][j][1] = fmaf(p[r], vv.y, o[r][j][1]);
          o[r][j][2] = fmaf(p[r], vv.z, o[r][j][2]);
          o[r][j][3] = fmaf(p[r], vv.w, o[r][j][3]);
        }
      }
    }
  }

  if (tx == 0) {
    l_s[2 * ty] = l_r[0];
    l_s[2 * ty + 1] = l_r[1];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = i0 + orow + r;
    if (i >= a.T) continue;
    const float l = l_s[orow + r];
    const float inv = (i < qlen && l > 0.f) ? 1.f / l : 0.f;
    float* dst = outp + int64_t(i) * a.ost;
    float* dstl = outl ? outl + int64_t(i) * a.ost : nullptr;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int c = ocol + 64 * j + e;
        if (c < a.D) {
          const float val = o[r][j][e] * inv;
          dst[c] = val;
          if (dstl) dstl[c] = val - __uint_as_float(__float_as_uint(val) & 0xFFFFE000u);
        }
      }
    }
  }
}

template <int DP>
int launch_attn(const AttnArgs& a, cudaStream_t s) {
  auto kern = attn_simt_kernel<DP>;
  const size_t smem = AttnSmem<DP>::kBytes;
  static std::atomic<bool> set[64];  // per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    FG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    set[dev & 63] = true;
  }
  dim3 grid(unsigned((a.T + kBQ - 1) / kBQ), unsigned(a.Hq), unsigned(a.B));
  kern<<<grid, 256, smem, s>>>(a);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

// Rows whose every key is masked. In the reference the additive −1e9 masks
// swamp the raw float32 scores, so such a row's scores are equal on the keys
// hidden by the fewest masks and its output is the plain mean of their
// values (padding and window masks each add −1e9). One warp per row; rows
// with a visible key return at once.
__global__ void attn_masked_rows_kernel(const AttnArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t task = int64_t(blockIdx.x) * 8 + warp;
  const int64_t total = int64_t(a.B) * a.Hq * a.T;
  if (task >= total) return;
  const int i = int(task % a.T);
  const int h = int((task / a.T) % a.Hq);
  const int b = int(task / (int64_t(a.T) * a.Hq));
  const int klen = a.klen ? max(0, min(a.klen[b], a.S)) : a.S;
  const int w = a.window;
  int lo = 0, hi = klen;  // visible keys [lo, hi)
  if (w > 0) {
    lo = max(0, i - w + 1);
    hi = min(klen, i + w);
  }
  if (lo < hi || a.S == 0) return;
  // count of masks hiding key j: (j >= klen) + (window && |i-j| >= w)
  auto cnt = [&](int j) { return int(j >= klen) + int(w > 0 && (i - j >= w || j - i >= w)); };
  int minc = 2;
  for (int j = lane; j < a.S; j += 32) minc = min(minc, cnt(j));
  for (int off = 16; off > 0; off >>= 1) minc = min(minc, __shfl_xor_sync(0xffffffffu, minc, off));
  const int hk = h / (a.Hq / a.Hkv);
  const float* vb = a.v + b * a.vsb + hk * a.vsh;
  float* dst = a.out + b * a.osb + h * a.osh + int64_t(i) * a.ost;
  int n = 0;
  for (int j = 0; j < a.S; ++j) n += cnt(j) == minc;
  const float inv = 1.f / float(n);
  for (int d = lane; d < a.D; d += 32) {
    float acc = 0.f;
    for (int j = 0; j < a.S; ++j)
      if (cnt(j) == minc) acc += vb[int64_t(j) * a.vst + d];
    dst[d] = acc * inv;
  }
}

}  // namespace

int attention_masked_rows(const AttnArgs& a, cudaStream_t s) {
  const int64_t total = int64_t(a.B) * a.Hq * a.T;
  if (total == 0) return FG_OK;
  attn_masked_rows_kernel<<<unsigned((total + 7) / 8), 256, 0, s>>>(a);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int attention_simt(const AttnArgs& a, cudaStream_t s) {
  if (a.B == 0 || a.T == 0) return FG_OK;
  if (a.Hkv <= 0 || a.Hq % a.Hkv != 0)
    return set_error(FG_EINVAL, "attention: %d query heads not a multiple of %d key/value heads", a.Hq, a.Hkv);
  if (a.D <= 0 || a.D > 512) return set_error(FG_EINVAL, "attention: head dimension %d unsupported (1..512)", a.D);
  if (a.T > 65535 * kBQ || a.Hq > 65535 || a.B > 65535) return set_error(FG_EINVAL, "attention: grid too large");
  if (a.D <= 64) return launch_attn<64>(a, s);
  if (a.D <= 128) return launch_attn<128>(a, s);
  if (a.D <= 256) return launch_attn<256>(a, s);
  return launch_attn<512>(a, s);
}

}  // namespace fg
