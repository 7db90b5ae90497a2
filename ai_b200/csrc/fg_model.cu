// EmbeddingGemma encoder model: weight intake and load-time folds
// (gemma.Load, models/gemma/model.go:76-232), device-resident weights, and
// the batch forward (embedBatch → encode → pool → applyHead → l2normalize,
// models/gemma/embed.go:118-240, 381-475) as a sequence of sm_100a kernels
// on one stream.
//
// Device layout (all fp32, row-major, [out, in] = K-major for every
// projection, the layout the tensor cores read without packing):
//   embed      [vocab, hidden]
//   per layer  Wqkv [(Hq+2·Hkv)·D, hidden]  rows q | k | v, pre-norm folded
//              Wo   [hidden, Hq·D]
//              Wgu  [2·ffn, hidden]  gate and up rows interleaved in blocks
//                   of 128 (gate 128j.., up 128j..) so one 256-row tile of B
//                   yields 128 finished GeGLU columns; pre-norm folded
//              Wd   [hidden, ffn]
//              each with its TF32 low part when it is non-zero
//   activations, token-major [B·T, ·]: x (residual stream), qkv, att, gu,
//   tmp; rowscale [B·T]. The split products make their A operand's low part
//   (or fp16 parts) in shared memory from the A tile.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include <cuda_fp16.h>

#include "fg_internal.h"
#include "fg_kernels.cuh"
#include "fg_ptx.cuh"

namespace fg {

namespace {

float bf16_to_f32(uint16_t h) {
  uint32_t u = uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = uint32_t(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ffu;
  uint32_t u;
  if (exp == 0) {
    if (mant == 0) {
      u = sign;
    } else {
      uint32_t e = 127 - 15 + 1;
      while ((mant & 0x400u) == 0) {
        mant <<= 1;
        --e;
      }
      mant &= 0x3ffu;
      u = sign | (e << 23) | (mant << 13);
    }
  } else if (exp == 0x1f) {
    u = sign | 0x7f800000u | (mant << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

struct HostTensor {
  std::vector<int64_t> shape;
  std::vector<float> data;
};

struct DevBuf {
  float* p = nullptr;
  size_t n = 0;
};

// A K-major operand resident on the device with its optional low part.
struct DevMat {
  float* hi = nullptr;
  float* lo = nullptr;  // null when every low part is zero
  int rows = 0, cols = 0;
  // fp16 bits of hi·2^h16_exp when that is exact for every value (the
  // split-fp16 GEMM's B operand), else null
  uint16_t* h16 = nullptr;
  int h16_exp = 0;
  // when not null: h16 is the weight before its fold with this column gain
  // (|gain| <= h16_gmax), which the split-fp16 GEMM applies to A instead
  const float* h16_gain = nullptr;
  float h16_gmax = 1.f;
  // a weight with no exact fp16 form (an fp32 checkpoint): h16 holds the
  // high part (top 11 significant bits of w·2^h16_exp) and h16_lo =
  // fp16(w·2^h16_exp − high), for the three-pass split-fp16 product
  uint16_t* h16_lo = nullptr;
};

// A projection resident as bf16 (FG_WEIGHTS_BF16): [rows, cols] bits and
// the pre-norm gain folded into its columns at widening (null: none).
struct Bf16Mat {
  uint16_t* w = nullptr;
  const float* gain = nullptr;
  bool lo = false;  // the folded values have non-zero split-TF32 low parts
  // with split-fp16: w holds the folded values as fp16 bits of v·2^exp
  // (exact), the split-fp16 GEMM's B operand as it is (gain null, no lo)
  bool f16 = false;
  int exp = 0;
  // f16 with a gain: w is the weight before the fold (the GEMM applies the
  // gain to A; widening folds it), |gain| <= gmax
  float gmax = 1.f;
};

struct Layer {
  DevMat wqkv, wo, wgu, wd;
  bool resident_bf16 = false;  // the four below hold the weights; the DevMats are the workspace
  Bf16Mat bqkv, bo, bgu, bd;
  float* g_in = nullptr;  // pre-attention and pre-FFN gains (1 + w)
  float* g_pf = nullptr;
  float* qgain = nullptr;
  float* kgain = nullptr;
  float* post_attn = nullptr;
  float* post_ffn = nullptr;
  int rope = 0;  // index into the model's rope tables
  // EmbeddingGemma 2 (encode2, embed.go:247-377): this layer's head geometry,
  // the PLE block's gate [P, H] and projection [H, P], the weight-free
  // v_norm (ones), the PLE post-norm and the layer scalar
  int D = 0, Hkv = 0;
  DevMat wpg, wpp;
  float* vgain = nullptr;
  float* ple_post = nullptr;
  float scalar = 1.f;
  // split-fp16 exponents of the O and down projections' inputs, from
  // bounds on the attention output and the gated activations (ok: finite)
  int att_exp = 0, gu_exp = 0;
  bool att_ok = false, gu_ok = false;
};

struct Dense {
  DevMat w;
  int in = 0, out = 0;
  bool tanh = false;
};

}  // namespace

}  // namespace fg

struct fg_model {
  int device = 0;
  fg_config cfg{};
  std::vector<int> sliding;
  std::vector<double> rope_base;
  std::map<std::string, fg::HostTensor> host;
  bool finalized = false;

  // device weights
  float* embed = nullptr;             // fp32 table, or
  uint16_t* embed_bf16 = nullptr;     // the bf16 table when every entry is bf16-exact
  std::vector<fg::Layer> layers;
  float* final_gain = nullptr;
  std::vector<fg::Dense> dense;
  std::vector<float*> rope_cos, rope_sin;    // [max_tokens, D/2]
  // the same for 256-wide heads, position-minor with cos and sin side by
  // side: [D/2][max_tokens][2] (null for other head sizes)
  std::vector<float*> rope_csT;
  std::vector<double> rope_bases;  // distinct bases, index = Layer::rope
  std::vector<void*> allocations;

  // workspace
  int64_t cap_tokens = 0;
  int cap_batch = 0;
  float *x = nullptr, *rowscale = nullptr, *qkv = nullptr, *att = nullptr, *gu = nullptr,
        *tmp = nullptr;
  // the split-fp16 parts of x for the gate/up product ([tokens, H] hi, then
  // lo); those of the attention output and of the gated activations take
  // the place of att and gu, whose fp32 forms are then not written
  uint16_t* x16 = nullptr;
  float *pooled = nullptr, *head_a = nullptr, *head_b = nullptr;
  int32_t* eff_len = nullptr;
  int* err = nullptr;
  void* attn_ws = nullptr;  // split-bf16 operands of the tensor-core attention
  size_t attn_ws_bytes = 0;
  // The fp16 forms the split-fp16 encoder GEMMs read are prepared at
  // finalize wherever the weights have one; use16 is the current forward's
  // choice (FG_PREC_SPLIT: yes; FG_PREC_SPLIT_TF32 / FG_PREC_TF32: no).
  bool h16 = true;
  bool use16 = true;
  int weight_mode = FG_WEIGHTS_F32;
  size_t weight_bytes = 0;  // device bytes allocated by finalize before the activation workspace
  size_t alloc_bytes = 0;
  // FG_WEIGHTS_BF16: one layer's widened fp32 projections (hi and low parts)
  fg::DevMat ws_qkv, ws_o, ws_gu, ws_d;
  // EmbeddingGemma 2: per-layer geometry, the per-layer-embedding projection
  // [L·P, H] and its norm, the embedding projection [E, H], and their
  // workspaces (ple [tokens, L·P], the constant 1/√H row scale, the PLE
  // block's gated activations [tokens, P])
  std::vector<int> head_dim_l, kv_l;
  std::vector<int> rope_dims;  // head dim of each rope table (index = Layer::rope)
  fg::DevMat ple_proj, emb_proj;
  float* ple_gain = nullptr;
  float *ple_buf = nullptr, *ple_scale = nullptr, *gbuf = nullptr;
  // host-API staging
  int32_t* d_ids = nullptr;
  int64_t d_ids_cap = 0;
  int32_t* d_len = nullptr;
  float* d_out = nullptr;
  int64_t d_out_cap = 0;
  int d_len_cap = 0;
  cudaStream_t stream = nullptr;

  // measurement: launch counts and algorithmic work per phase (always),
  // CUDA-event pairs around each launch while profiling is enabled
  bool prof = false;
  struct Mark {
    int phase;
    cudaEvent_t a, b;
  };
  std::vector<Mark> marks;
  std::vector<cudaEvent_t> event_pool;
  int64_t launches[FG_NUM_PHASES] = {};
  double work[FG_NUM_PHASES] = {};

  // CUDA graphs of the device-API forward, per (B, T, dim, precision, ids,
  // lengths, out): a key's first call runs eagerly (it makes any
  // allocation and one-time set-up the shape needs), its second is
  // captured on cap_stream and then launched, later ones launch the graph
  // on the caller's stream. A graph also carries the launch counts and
  // algorithmic work its capture recorded, added on every launch. Graphs
  // are dropped when a buffer they use is freed.
  using GraphKey = std::tuple<int, int, int, int, const void*, const void*, const void*>;
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    int64_t launches[FG_NUM_PHASES] = {};
    double work[FG_NUM_PHASES] = {};
  };
  std::map<GraphKey, Graph> graphs;
  std::set<GraphKey> graph_seen;
  cudaStream_t cap_stream = nullptr;
};

namespace fg {
namespace {

int dev_alloc(fg_model* m, void** p, size_t bytes) {
  if (bytes == 0) bytes = 16;
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return set_error(FG_ENOMEM, "device allocation of %zu bytes failed", bytes);
  }
  m->allocations.push_back(*p);
  m->alloc_bytes += bytes;
  return FG_OK;
}

template <class T>
int dev_alloc_t(fg_model* m, T** p, size_t count) {
  void* v = nullptr;
  FG_TRY(dev_alloc(m, &v, count * sizeof(T)));
  *p = static_cast<T*>(v);
  return FG_OK;
}

int upload(fg_model* m, const std::vector<float>& h, float** out) {
  FG_TRY(dev_alloc_t(m, out, h.size()));
  FG_CUDA_TRY(cudaMemcpy(*out, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
  return FG_OK;
}

// The embedding table stays resident in bf16 (half the bytes: 403 MB
// instead of 805 MB for EmbeddingGemma's 262144 × 768) when every entry is
// a widened bf16 — always so for a bf16 checkpoint — and the gather widens
// it exactly; otherwise it is kept in fp32. FG_EMBED_BF16=0 keeps fp32.
int upload_table(fg_model* m, const std::vector<float>& h, float** f32, uint16_t** b16) {
  *f32 = nullptr;
  *b16 = nullptr;
  const char* env = std::getenv("FG_EMBED_BF16");
  bool exact = !(env && env[0] == '0');
  for (size_t i = 0; exact && i < h.size(); ++i) {
    uint32_t u;
    std::memcpy(&u, &h[i], 4);
    exact = (u & 0xffffu) == 0;
  }
  if (!exact) return upload(m, h, f32);
  std::vector<uint16_t> hb(h.size());
  for (size_t i = 0; i < h.size(); ++i) {
    uint32_t u;
    std::memcpy(&u, &h[i], 4);
    hb[i] = uint16_t(u >> 16);
  }
  FG_TRY(dev_alloc_t(m, b16, hb.size()));
  FG_CUDA_TRY(cudaMemcpy(*b16, hb.data(), hb.size() * sizeof(uint16_t), cudaMemcpyHostToDevice));
  return FG_OK;
}

// bf16 bits of h when every value is a widened bf16 (else false).
bool pack_bf16(const float* h, size_t n, std::vector<uint16_t>& out) {
  out.resize(n);
  for (size_t i = 0; i < n; ++i) {
    uint32_t u;
    std::memcpy(&u, &h[i], 4);
    if (u & 0xffffu) return false;
    out[i] = uint16_t(u >> 16);
  }
  return true;
}

// Whether W'[r][c] = W[r][c]·g[c] (the fold, in fp32) has a non-zero
// split-TF32 low part anywhere. tf32 keeps the top 10 mantissa bits.
bool fold_has_lo(const float* w, const std::vector<float>* g, int64_t rows, int64_t cols) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const float v = g ? w[r * cols + c] * (*g)[size_t(c)] : w[r * cols + c];
      uint32_t u;
      std::memcpy(&u, &v, 4);
      if (u & 0x1fffu) return true;
    }
  return false;
}

struct WidenJob {
  const uint16_t* w;
  const float* gain;
  float* hi;
  float* lo;
  int64_t n4;  // groups of 4 values
  int cols;    // a multiple of 4
  int f16;     // w holds fp16 bits of the folded values times 2^f16_exp
  int f16_exp;
};
struct WidenJobs {
  WidenJob j[4];
};

// Widens bf16 projections, folds the pre-norm gain into their columns and
// splits them for split-TF32, the same fp32 operations upload_mat performs
// on the host-folded weights (fold: w·g; split_tf32: hi = tf32(v),
// lo = v − hi), so the GEMM sees identical operands. blockIdx.y = job.
__global__ void __launch_bounds__(256) widen_fold_kernel(WidenJobs jobs) {
  const WidenJob J = jobs.j[blockIdx.y];
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < J.n4;
       i += int64_t(gridDim.x) * blockDim.x) {
    const uint2 h = __ldg(reinterpret_cast<const uint2*>(J.w) + i);
    float v[4] = {__uint_as_float(h.x << 16), __uint_as_float(h.x & 0xffff0000u),
                  __uint_as_float(h.y << 16), __uint_as_float(h.y & 0xffff0000u)};
    if (J.f16) {
      // exact: an fp16 value times a power of two in fp32's normal range
      const float sc = pow2f(-J.f16_exp);
      v[0] = __half2float(__ushort_as_half(uint16_t(h.x & 0xffffu))) * sc;
      v[1] = __half2float(__ushort_as_half(uint16_t(h.x >> 16))) * sc;
      v[2] = __half2float(__ushort_as_half(uint16_t(h.y & 0xffffu))) * sc;
      v[3] = __half2float(__ushort_as_half(uint16_t(h.y >> 16))) * sc;
    }
    if (J.gain) {
      const int c = int((i * 4) % J.cols);
      const float4 g = __ldg(reinterpret_cast<const float4*>(J.gain + c));
      v[0] = __fmul_rn(v[0], g.x);
      v[1] = __fmul_rn(v[1], g.y);
      v[2] = __fmul_rn(v[2], g.z);
      v[3] = __fmul_rn(v[3], g.w);
    }
    float4 hi, lo;
    hi.x = tf32_hi(v[0]); hi.y = tf32_hi(v[1]); hi.z = tf32_hi(v[2]); hi.w = tf32_hi(v[3]);
    reinterpret_cast<float4*>(J.hi)[i] = hi;
    if (J.lo) {
      lo.x = __fsub_rn(v[0], hi.x); lo.y = __fsub_rn(v[1], hi.y);
      lo.z = __fsub_rn(v[2], hi.z); lo.w = __fsub_rn(v[3], hi.w);
      reinterpret_cast<float4*>(J.lo)[i] = lo;
    }
  }
}

// Uploads a K-major [rows, cols] fp32 matrix and its split-TF32 parts.
// The fp16 bits of v when v is exactly an fp16 value (normal or subnormal).
bool f16_exact(float v, uint16_t* out) {
  uint32_t u;
  std::memcpy(&u, &v, 4);
  const uint32_t sign = (u >> 31) << 15, ex = (u >> 23) & 0xffu, mant = u & 0x7fffffu;
  if (ex == 0) {
    *out = uint16_t(sign);
    return mant == 0;  // fp32 subnormals are far below fp16's range
  }
  if (ex == 0xffu) return false;
  const int e = int(ex) - 127;
  if (e > 15) return false;
  if (e >= -14) {
    if (mant & 0x1fffu) return false;
    *out = uint16_t(sign | (uint32_t(e + 15) << 10) | (mant >> 13));
    return true;
  }
  const int sh = -e - 1;  // value = ((1 << 23) | mant) · 2^(e − 23) = m16 · 2^−24
  if (sh > 24) return false;
  const uint32_t sig = (1u << 23) | mant;
  if (sig & ((1u << sh) - 1)) return false;
  *out = uint16_t(sign | (sig >> sh));
  return true;
}

// Exponent e with bound·2^e in [2^13, 2^14) (a split-fp16 operand scale), or
// false when the bound is not a positive finite number.
bool h16_exponent(double bound, int* e) {
  if (!(bound > 0) || !std::isfinite(bound)) return false;
  *e = 13 - std::ilogb(bound);
  return *e > -100 && *e < 100;
}

// Round-to-nearest-even fp16 bits of an fp32 value (subnormals included;
// the split forms' magnitudes stay below 2^15).
uint16_t f16_rn(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  const uint32_t sign = (u >> 16) & 0x8000u, ex = (u >> 23) & 0xffu, mant = u & 0x7fffffu;
  if (ex == 0xffu) return uint16_t(sign | 0x7c00u | (mant ? 0x200u : 0u));
  const int e = int(ex) - 127;
  if (e > 15) return uint16_t(sign | 0x7c00u);
  if (e >= -14) {
    uint32_t h = (uint32_t(e + 15) << 10) | (mant >> 13);
    const uint32_t r = mant & 0x1fffu;
    if (r > 0x1000u || (r == 0x1000u && (h & 1u))) h += 1;  // a carry moves into the exponent
    return uint16_t(sign | h);
  }
  if (e < -25 || ex == 0) return uint16_t(sign);
  // subnormal: the value in units of 2^-24 is (2^23 + mant)·2^(e + 1)
  const uint32_t m = mant | 0x800000u;
  const int shift = -(e + 1);
  uint32_t q = m >> shift;
  const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
  if (rem > half || (rem == half && (q & 1u))) q += 1;
  return uint16_t(sign | q);
}

// Two fp16 parts of h·2^e (e from the largest |value|): the high part is
// the value's top 11 significant bits (its TF32 truncation), the low part
// the rounded remainder — as the GEMM converters cut A.
int upload_h16_split(fg_model* m, const std::vector<float>& h, DevMat* out) {
  if (!m->h16 || out->h16) return FG_OK;
  double mx = 0;
  for (float v : h) mx = std::max(mx, double(std::fabs(v)));
  int e = 0;
  if (!h16_exponent(mx, &e)) return FG_OK;
  std::vector<uint16_t> hi(h.size()), lo(h.size());
  for (size_t i = 0; i < h.size(); ++i) {
    const float v = std::ldexp(h[i], e);
    uint32_t u;
    std::memcpy(&u, &v, 4);
    u &= 0xFFFFE000u;
    float t;
    std::memcpy(&t, &u, 4);
    hi[i] = f16_rn(t);
    lo[i] = f16_rn(v - t);
  }
  FG_TRY(dev_alloc_t(m, &out->h16, hi.size()));
  FG_TRY(dev_alloc_t(m, &out->h16_lo, lo.size()));
  FG_CUDA_TRY(cudaMemcpy(out->h16, hi.data(), hi.size() * 2, cudaMemcpyHostToDevice));
  FG_CUDA_TRY(cudaMemcpy(out->h16_lo, lo.data(), lo.size() * 2, cudaMemcpyHostToDevice));
  out->h16_exp = e;
  return FG_OK;
}

// h·2^e as fp16 bits, e from the largest |value|, when exact for all.
bool f16_form(const std::vector<float>& h, std::vector<uint16_t>& b, int* e) {
  double mx = 0;
  for (float v : h) mx = std::max(mx, double(std::fabs(v)));
  if (!h16_exponent(mx, e)) return false;
  b.resize(h.size());
  for (size_t i = 0; i < h.size(); ++i)
    if (!f16_exact(std::ldexp(h[i], *e), &b[i])) return false;
  return true;
}

int upload_h16(fg_model* m, const std::vector<float>& h, DevMat* out) {
  std::vector<uint16_t> b;
  int e = 0;
  if (!f16_form(h, b, &e)) return FG_OK;
  FG_TRY(dev_alloc_t(m, &out->h16, b.size()));
  FG_CUDA_TRY(cudaMemcpy(out->h16, b.data(), b.size() * 2, cudaMemcpyHostToDevice));
  out->h16_exp = e;
  return FG_OK;
}

int upload_mat(fg_model* m, const std::vector<float>& h, int rows, int cols, DevMat* out) {
  float* raw = nullptr;
  FG_TRY(upload(m, h, &raw));
  float* lo = nullptr;
  FG_TRY(dev_alloc_t(m, &lo, h.size()));
  int* flag = nullptr;
  FG_TRY(dev_alloc_t(m, &flag, 1));
  FG_CUDA_TRY(cudaMemset(flag, 0, sizeof(int)));
  // hi in place: the truncated TF32 value; lo: the exact remainder
  FG_TRY(split_tf32(raw, raw, lo, int64_t(h.size()), flag, nullptr));
  int any = 0;
  FG_CUDA_TRY(cudaMemcpy(&any, flag, sizeof(int), cudaMemcpyDeviceToHost));
  if (!any) {  // bf16-exact weights: no low pass, release the buffer
    FG_CUDA_TRY(cudaFree(lo));
    m->alloc_bytes -= h.size() * sizeof(float);
    m->allocations.erase(std::find(m->allocations.begin(), m->allocations.end(), static_cast<void*>(lo)));
    lo = nullptr;
  }
  out->hi = raw;
  out->lo = lo;
  out->rows = rows;
  out->cols = cols;
  // a weight with a low part is not fp16-exact (it has more than 11 bits)
  if (m->h16 && !lo) FG_TRY(upload_h16(m, h, out));
  return FG_OK;
}

// The split-fp16 form of a folded projection whose folded values have no
// exact fp16 form: the unfolded weight (bf16 values are), with the fold's
// column gain left for the GEMM to apply to A.
int upload_h16_unfolded(fg_model* m, const std::vector<float>& raw, const float* gain_dev,
                        const std::vector<float>& gain, DevMat* out) {
  if (!m->h16 || out->h16) return FG_OK;
  FG_TRY(upload_h16(m, raw, out));
  if (!out->h16) return FG_OK;
  double gm = 0;
  for (float v : gain) gm = std::max(gm, double(std::fabs(v)));
  out->h16_gain = gain_dev;
  out->h16_gmax = float(gm);
  return FG_OK;
}

// sqrt(Σ_c (w[r][c]·g[c])²) of row r of a [rows, cols] matrix folded with
// the column gain g (fp32 products, as the fold stores them).
double folded_row_norm(const float* w, const std::vector<float>& g, int64_t r, int64_t cols) {
  double s = 0;
  for (int64_t c = 0; c < cols; ++c) {
    const double v = double(w[r * cols + c] * g[size_t(c)]);
    s += v * v;
  }
  return std::sqrt(s);
}

const HostTensor* find(fg_model* m, const std::string& name) {
  auto it = m->host.find(name);
  return it == m->host.end() ? nullptr : &it->second;
}

int need(fg_model* m, const std::string& name, std::vector<int64_t> shape, const HostTensor** out) {
  const HostTensor* t = find(m, name);
  if (!t) return set_error(FG_EINVAL, "gemma: weight %s not found", name.c_str());
  if (t->shape != shape) {
    std::string want, got;
    for (auto s : shape) want += std::to_string(s) + ",";
    for (auto s : t->shape) got += std::to_string(s) + ",";
    return set_error(FG_EINVAL, "gemma: weight %s has shape [%s], want [%s]", name.c_str(), got.c_str(), want.c_str());
  }
  *out = t;
  return FG_OK;
}

// Gemma's (1 + w) norm gain (model.go:131-140).
std::vector<float> plus_one(const HostTensor& t) {
  std::vector<float> g(t.data.size());
  for (size_t i = 0; i < g.size(); ++i) g[i] = t.data[i] + 1.0f;
  return g;
}

// Folds a pre-norm gain into [rows, cols] projection rows: W'[n][k] =
// W[n][k]·g[k] (the reference's diag(g)·Wᵀ on the transposed weight,
// model.go:206-222).
std::vector<float> fold(const std::vector<float>& w, const std::vector<float>& g, int64_t cols) {
  std::vector<float> out(w.size());
  const int64_t rows = int64_t(w.size()) / cols;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = w[r * cols + c] * g[c];
  return out;
}

// [half][P][2]: (cos, sin) of frequency i at position t at (i·P + t)·2,
// from the position-major tables [P][half].
std::vector<float> rope_pairs_position_minor(const std::vector<float>& cs, const std::vector<float>& sn, int64_t P,
                                             int64_t half) {
  std::vector<float> out(size_t(2 * P * half));
  for (int64_t t = 0; t < P; ++t)
    for (int64_t i = 0; i < half; ++i) {
      out[size_t(2 * (i * P + t))] = cs[size_t(t * half + i)];
      out[size_t(2 * (i * P + t) + 1)] = sn[size_t(t * half + i)];
    }
  return out;
}

void rope_table(double base, int T, int D, std::vector<float>& c, std::vector<float>& s) {
  const int half = D / 2;
  std::vector<double> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = std::pow(base, -double(2 * i) / double(D));
  c.resize(size_t(T) * half);
  s.resize(size_t(T) * half);
  for (int t = 0; t < T; ++t)
    for (int i = 0; i < half; ++i) {
      const double a = double(t) * inv[i];
      c[size_t(t) * half + i] = float(std::cos(a));
      s[size_t(t) * half + i] = float(std::sin(a));
    }
}

__global__ void eff_len_kernel(const int32_t* len, int B, int T, int32_t* eff) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) eff[b] = max(min(len[b], T), 1);
}

int ensure_workspace(fg_model* m, int64_t tokens, int batch) {
  const fg_config& c = m->cfg;
  if (tokens > m->cap_tokens) {
    if (m->x) return set_error(FG_EINVAL, "batch of %lld tokens exceeds the workspace (%lld)", (long long)tokens, (long long)m->cap_tokens);
    const int64_t H = c.hidden_size;
    int64_t qkvw = 0, attw = 0;  // widest layer (EmbeddingGemma 2's differ)
    for (int l = 0; l < c.num_layers; ++l) {
      qkvw = std::max<int64_t>(qkvw, int64_t(c.num_heads + 2 * m->kv_l[size_t(l)]) * m->head_dim_l[size_t(l)]);
      attw = std::max<int64_t>(attw, int64_t(c.num_heads) * m->head_dim_l[size_t(l)]);
    }
    const int64_t F = c.intermediate_size;
    FG_TRY(dev_alloc_t(m, &m->x, tokens * H));
    FG_TRY(dev_alloc_t(m, &m->rowscale, tokens));
    FG_TRY(dev_alloc_t(m, &m->qkv, tokens * qkvw));
    FG_TRY(dev_alloc_t(m, &m->att, tokens * attw));
    FG_TRY(dev_alloc_t(m, &m->gu, tokens * F));
    FG_TRY(dev_alloc_t(m, &m->tmp, tokens * std::max(H, attw)));
    if (c.variant != 2) FG_TRY(dev_alloc_t(m, &m->x16, 2 * tokens * H));
    if (c.variant == 2) {
      const int64_t P = c.ple_dim, L = c.num_layers;
      FG_TRY(dev_alloc_t(m, &m->ple_buf, tokens * L * P));
      FG_TRY(dev_alloc_t(m, &m->gbuf, tokens * P));
      FG_TRY(dev_alloc_t(m, &m->ple_scale, tokens));
      // pl·(1/√hidden) as a row scale of the product (embed.go:270)
      const float inv = float(1.0 / std::sqrt(double(H)));
      std::vector<float> hs(static_cast<size_t>(tokens), inv);
      FG_CUDA_TRY(cudaMemcpy(m->ple_scale, hs.data(), hs.size() * sizeof(float), cudaMemcpyHostToDevice));
    }
    m->cap_tokens = tokens;
  }
  if (batch > m->cap_batch) {
    int widest = std::max(c.hidden_size, c.variant == 2 ? c.embedding_dim : 0);
    for (auto& d : m->dense) widest = std::max(widest, std::max(d.in, d.out));
    const int64_t nb = std::max(batch, 1);
    FG_TRY(dev_alloc_t(m, &m->pooled, nb * c.hidden_size));
    FG_TRY(dev_alloc_t(m, &m->head_a, nb * widest));
    FG_TRY(dev_alloc_t(m, &m->head_b, nb * widest));
    FG_TRY(dev_alloc_t(m, &m->eff_len, nb));
    m->cap_batch = int(nb);
  }
  return FG_OK;
}

// The weights EmbeddingGemma 2's Load reads (model.go:142-205 with the
// variant-2 additions), folded as there: norms multiply by the stored
// weight, the input norm folds into Wq/Wk/Wv and the pre-FFN norm into
// Wgate/Wup (model.go:206-222).
int finalize_v2(fg_model* m, int64_t max_tokens) {
  const fg_config& c = m->cfg;
  const int64_t H = c.hidden_size, Hq = c.num_heads, F = c.intermediate_size;
  const int64_t L = c.num_layers, P = c.ple_dim, E = c.embedding_dim;
  if (F % 128 != 0) return set_error(FG_EINVAL, "intermediate_size %lld must be a multiple of 128", (long long)F);
  if (H % 128 != 0 || H > 1024) return set_error(FG_EINVAL, "hidden_size %lld must be a multiple of 128 up to 1024", (long long)H);
  FG_CUDA_TRY(cudaSetDevice(m->device));
  FG_TRY(device_error_word(&m->err));
  const HostTensor* t = nullptr;
  FG_TRY(need(m, "embed_tokens.weight", {c.vocab_size, H}, &t));
  FG_TRY(upload_table(m, t->data, &m->embed, &m->embed_bf16));

  // rope tables per distinct (base, head dim)
  auto rope_index = [&](double base, int D, int* out) -> int {
    for (size_t i = 0; i < m->rope_bases.size(); ++i)
      if (m->rope_bases[i] == base && m->rope_dims[i] == D) {
        *out = int(i);
        return FG_OK;
      }
    std::vector<float> cs, sn;
    rope_table(base, c.max_tokens, D, cs, sn);
    float *dc = nullptr, *ds = nullptr;
    FG_TRY(upload(m, cs, &dc));
    FG_TRY(upload(m, sn, &ds));
    m->rope_cos.push_back(dc);
    m->rope_sin.push_back(ds);
    // position-minor copy for the fused QKV epilogue (256-wide heads)
    float* dT = nullptr;
    if (D == 256) FG_TRY(upload(m, rope_pairs_position_minor(cs, sn, c.max_tokens, D / 2), &dT));
    m->rope_csT.push_back(dT);
    m->rope_bases.push_back(base);
    m->rope_dims.push_back(D);
    *out = int(m->rope_bases.size()) - 1;
    return FG_OK;
  };
  auto gain = [&](const std::string& name, int64_t n, float** out) -> int {
    const HostTensor* g = nullptr;
    FG_TRY(need(m, name, {n}, &g));
    return upload(m, g->data, out);
  };

  m->layers.resize(size_t(L));
  for (int l = 0; l < L; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    Layer& Ly = m->layers[size_t(l)];
    const int64_t D = m->head_dim_l[size_t(l)], Hkv = m->kv_l[size_t(l)];
    Ly.D = int(D);
    Ly.Hkv = int(Hkv);
    FG_TRY(rope_index(m->rope_base[l], int(D), &Ly.rope));
    const HostTensor *in_norm, *pf_norm, *wq, *wk, *wv, *wo, *wg, *wu, *wd, *pg, *pp;
    FG_TRY(need(m, p + "input_layernorm.weight", {H}, &in_norm));
    FG_TRY(need(m, p + "pre_feedforward_layernorm.weight", {H}, &pf_norm));
    FG_TRY(need(m, p + "self_attn.q_proj.weight", {Hq * D, H}, &wq));
    FG_TRY(need(m, p + "self_attn.k_proj.weight", {Hkv * D, H}, &wk));
    FG_TRY(need(m, p + "self_attn.v_proj.weight", {Hkv * D, H}, &wv));
    FG_TRY(need(m, p + "self_attn.o_proj.weight", {H, Hq * D}, &wo));
    FG_TRY(need(m, p + "mlp.gate_proj.weight", {F, H}, &wg));
    FG_TRY(need(m, p + "mlp.up_proj.weight", {F, H}, &wu));
    FG_TRY(need(m, p + "mlp.down_proj.weight", {H, F}, &wd));
    FG_TRY(need(m, p + "ple_block.per_layer_input_gate.weight", {P, H}, &pg));
    FG_TRY(need(m, p + "ple_block.per_layer_projection.weight", {H, P}, &pp));
    const HostTensor* sc = find(m, p + "layer_scalar");
    if (!sc || sc->data.size() != 1) return set_error(FG_EINVAL, "gemma: weight %slayer_scalar not found (one value)", p.c_str());
    Ly.scalar = sc->data[0];

    const std::vector<float>& g_in = in_norm->data;  // no 1 + w in EmbeddingGemma 2
    const std::vector<float>& g_pf = pf_norm->data;
    std::vector<float> rqkv(size_t((Hq + 2 * Hkv) * D * H)), rgu(size_t(2 * F * H));
    std::memcpy(rqkv.data(), wq->data.data(), size_t(Hq * D * H) * 4);
    std::memcpy(rqkv.data() + Hq * D * H, wk->data.data(), size_t(Hkv * D * H) * 4);
    std::memcpy(rqkv.data() + (Hq + Hkv) * D * H, wv->data.data(), size_t(Hkv * D * H) * 4);
    for (int64_t j = 0; j < F / 128; ++j) {
      std::memcpy(rgu.data() + (2 * j) * 128 * H, wg->data.data() + j * 128 * H, size_t(128 * H) * 4);
      std::memcpy(rgu.data() + (2 * j + 1) * 128 * H, wu->data.data() + j * 128 * H, size_t(128 * H) * 4);
    }
    FG_TRY(upload_mat(m, fold(rqkv, g_in, H), int((Hq + 2 * Hkv) * D), int(H), &Ly.wqkv));
    FG_TRY(upload_mat(m, wo->data, int(H), int(Hq * D), &Ly.wo));
    FG_TRY(upload_mat(m, fold(rgu, g_pf, H), int(2 * F), int(H), &Ly.wgu));
    if (m->h16) {
      FG_TRY(upload(m, g_in, &Ly.g_in));
      FG_TRY(upload(m, g_pf, &Ly.g_pf));
      FG_TRY(upload_h16_unfolded(m, rqkv, Ly.g_in, g_in, &Ly.wqkv));
      FG_TRY(upload_h16_unfolded(m, rgu, Ly.g_pf, g_pf, &Ly.wgu));
    }
    FG_TRY(upload_mat(m, wd->data, int(H), int(F), &Ly.wd));
    FG_TRY(upload_mat(m, pg->data, int(P), int(H), &Ly.wpg));
    FG_TRY(upload_mat(m, pp->data, int(H), int(P), &Ly.wpp));
    if (m->h16) {
      // split-fp16 bounds of the O and down inputs: v is RMS-normalised
      // without a weight, so |v| < sqrt(D) and so is the attention output;
      // the gated activations as in EmbeddingGemma (‖rs·x‖ < sqrt(H))
      const double sh = std::sqrt(double(H));
      double bgu = 0;
      for (int64_t k = 0; k < F; ++k) {
        const double bg = sh * folded_row_norm(wg->data.data(), g_pf, k, H);
        const double bu = sh * folded_row_norm(wu->data.data(), g_pf, k, H);
        bgu = std::max(bgu, std::max(bg, 0.2) * bu);
      }
      Ly.att_ok = h16_exponent(std::sqrt(double(D)) * 1.01, &Ly.att_exp);
      Ly.gu_ok = h16_exponent(bgu * 1.01, &Ly.gu_exp);
    }
    FG_TRY(gain(p + "self_attn.q_norm.weight", D, &Ly.qgain));
    FG_TRY(gain(p + "self_attn.k_norm.weight", D, &Ly.kgain));
    FG_TRY(upload(m, std::vector<float>(size_t(D), 1.0f), &Ly.vgain));  // v_norm has no weight
    FG_TRY(gain(p + "post_attention_layernorm.weight", H, &Ly.post_attn));
    FG_TRY(gain(p + "post_feedforward_layernorm.weight", H, &Ly.post_ffn));
    FG_TRY(gain(p + "ple_block.post_per_layer_input_norm.weight", H, &Ly.ple_post));
  }
  FG_TRY(gain("norm.weight", H, &m->final_gain));
  const HostTensor *pm, *ep;
  FG_TRY(need(m, "ple.per_layer_model_projection.weight", {L * P, H}, &pm));
  FG_TRY(upload_mat(m, pm->data, int(L * P), int(H), &m->ple_proj));
  FG_TRY(gain("ple.per_layer_projection_norm.weight", P, &m->ple_gain));
  FG_TRY(need(m, "embedding_projection.weight", {E, H}, &ep));
  FG_TRY(upload_mat(m, ep->data, int(E), int(H), &m->emb_proj));

  int prev = int(E);
  for (int j = 0; j < c.num_dense; ++j) {
    const HostTensor* w = nullptr;
    FG_TRY(need(m, "dense." + std::to_string(j) + ".linear.weight", {c.dense_out[j], c.dense_in[j]}, &w));
    if (c.dense_in[j] != prev) return set_error(FG_EINVAL, "dense layer %d takes %d features, previous gives %d", j, c.dense_in[j], prev);
    if (c.dense_in[j] % 4 != 0) return set_error(FG_EINVAL, "dense layer %d input width must be a multiple of 4", j);
    Dense d;
    d.in = c.dense_in[j];
    d.out = c.dense_out[j];
    d.tanh = c.dense_tanh[j] != 0;
    FG_TRY(upload_mat(m, w->data, d.out, d.in, &d.w));
    m->dense.push_back(d);
    prev = d.out;
  }
  m->host.clear();
  m->weight_bytes = m->alloc_bytes;
  FG_TRY(ensure_workspace(m, std::max<int64_t>(max_tokens, 1), 1));
  FG_CUDA_TRY(cudaDeviceSynchronize());
  m->finalized = true;
  return FG_OK;
}

int finalize(fg_model* m, int64_t max_tokens) {
  if (m->cfg.variant == 2) return finalize_v2(m, max_tokens);
  const fg_config& c = m->cfg;
  const int64_t H = c.hidden_size, D = c.head_dim, Hq = c.num_heads, Hkv = c.num_kv_heads;
  const int64_t F = c.intermediate_size;
  if (F % 128 != 0) return set_error(FG_EINVAL, "intermediate_size %lld must be a multiple of 128", (long long)F);
  if (H % 128 != 0 || H > 1024) return set_error(FG_EINVAL, "hidden_size %lld must be a multiple of 128 up to 1024", (long long)H);
  if (D % 4 != 0 || D > 256) return set_error(FG_EINVAL, "head_dim %lld unsupported (multiple of 4, at most 256)", (long long)D);
  FG_CUDA_TRY(cudaSetDevice(m->device));
  FG_TRY(device_error_word(&m->err));

  const HostTensor* t = nullptr;
  FG_TRY(need(m, "embed_tokens.weight", {c.vocab_size, H}, &t));
  FG_TRY(upload_table(m, t->data, &m->embed, &m->embed_bf16));

  // distinct rope bases
  for (int l = 0; l < c.num_layers; ++l) {
    int idx = -1;
    for (size_t i = 0; i < m->rope_bases.size(); ++i)
      if (m->rope_bases[i] == m->rope_base[l]) idx = int(i);
    if (idx < 0) {
      idx = int(m->rope_bases.size());
      m->rope_bases.push_back(m->rope_base[l]);
      std::vector<float> cs, sn;
      rope_table(m->rope_base[l], c.max_tokens, int(D), cs, sn);
      float *dc = nullptr, *ds = nullptr;
      FG_TRY(upload(m, cs, &dc));
      FG_TRY(upload(m, sn, &ds));
      m->rope_cos.push_back(dc);
      m->rope_sin.push_back(ds);
      float* dT = nullptr;
      FG_TRY(upload(m, rope_pairs_position_minor(cs, sn, c.max_tokens, int(D) / 2), &dT));
      m->rope_csT.push_back(dT);
    }
  }

  m->layers.resize(c.num_layers);
  for (int l = 0; l < c.num_layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    Layer& L = m->layers[l];
    L.rope = 0;
    for (size_t i = 0; i < m->rope_bases.size(); ++i)
      if (m->rope_bases[i] == m->rope_base[l]) L.rope = int(i);
    const HostTensor *in_norm, *pa_norm, *pf_norm, *pff_norm, *qn, *kn, *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    FG_TRY(need(m, p + "input_layernorm.weight", {H}, &in_norm));
    FG_TRY(need(m, p + "post_attention_layernorm.weight", {H}, &pa_norm));
    FG_TRY(need(m, p + "pre_feedforward_layernorm.weight", {H}, &pf_norm));
    FG_TRY(need(m, p + "post_feedforward_layernorm.weight", {H}, &pff_norm));
    FG_TRY(need(m, p + "self_attn.q_norm.weight", {D}, &qn));
    FG_TRY(need(m, p + "self_attn.k_norm.weight", {D}, &kn));
    FG_TRY(need(m, p + "self_attn.q_proj.weight", {Hq * D, H}, &wq));
    FG_TRY(need(m, p + "self_attn.k_proj.weight", {Hkv * D, H}, &wk));
    FG_TRY(need(m, p + "self_attn.v_proj.weight", {Hkv * D, H}, &wv));
    FG_TRY(need(m, p + "self_attn.o_proj.weight", {H, Hq * D}, &wo));
    FG_TRY(need(m, p + "mlp.gate_proj.weight", {F, H}, &wg));
    FG_TRY(need(m, p + "mlp.up_proj.weight", {F, H}, &wu));
    FG_TRY(need(m, p + "mlp.down_proj.weight", {H, F}, &wd));

    const std::vector<float> g_in = plus_one(*in_norm), g_pf = plus_one(*pf_norm);
    const int64_t qkv_rows = (Hq + 2 * Hkv) * D;
    // q|k|v rows and gate/up rows interleaved in blocks of 128 (the GeGLU
    // epilogue's pairing), before any fold
    std::vector<float> rqkv(size_t(qkv_rows * H)), rgu(size_t(2 * F * H));
    std::memcpy(rqkv.data(), wq->data.data(), size_t(Hq * D * H) * 4);
    std::memcpy(rqkv.data() + Hq * D * H, wk->data.data(), size_t(Hkv * D * H) * 4);
    std::memcpy(rqkv.data() + (Hq + Hkv) * D * H, wv->data.data(), size_t(Hkv * D * H) * 4);
    for (int64_t j = 0; j < F / 128; ++j) {
      std::memcpy(rgu.data() + (2 * j) * 128 * H, wg->data.data() + j * 128 * H, size_t(128 * H) * 4);
      std::memcpy(rgu.data() + (2 * j + 1) * 128 * H, wu->data.data() + j * 128 * H, size_t(128 * H) * 4);
    }
    std::vector<uint16_t> bqkv, bo, bgu, bd;
    L.resident_bf16 = m->weight_mode == FG_WEIGHTS_BF16 && pack_bf16(rqkv.data(), rqkv.size(), bqkv) &&
                      pack_bf16(wo->data.data(), wo->data.size(), bo) &&
                      pack_bf16(rgu.data(), rgu.size(), bgu) && pack_bf16(wd->data.data(), wd->data.size(), bd);
    FG_TRY(upload(m, g_in, &L.g_in));
    FG_TRY(upload(m, g_pf, &L.g_pf));
    if (L.resident_bf16) {
      auto put = [&](const std::vector<uint16_t>& b, const float* gain, bool lo, Bf16Mat* out) -> int {
        FG_TRY(dev_alloc_t(m, &out->w, b.size()));
        FG_CUDA_TRY(cudaMemcpy(out->w, b.data(), b.size() * 2, cudaMemcpyHostToDevice));
        out->gain = gain;
        out->lo = lo;
        return FG_OK;
      };
      // with split-fp16, a projection whose folded values have an exact
      // fp16 form stays resident in that form instead (same bytes): the
      // GEMM reads it directly, and plain TF32 widens it
      auto put16 = [&](const std::vector<float>& folded, Bf16Mat* out, bool* done) -> int {
        std::vector<uint16_t> b;
        int e = 0;
        *done = m->h16 && f16_form(folded, b, &e);
        if (!*done) return FG_OK;
        FG_TRY(put(b, nullptr, false, out));
        out->f16 = true;
        out->exp = e;
        return FG_OK;
      };
      bool done = false;
      // else the unfolded weight's fp16 form with the gain (the GEMM puts
      // it on A; widening folds it as the host fold does)
      auto put16g = [&](const std::vector<float>& raw, const float* gain_dev, const std::vector<float>& gain,
                        bool lo, Bf16Mat* out, bool* done) -> int {
        std::vector<uint16_t> b;
        int e = 0;
        *done = m->h16 && f16_form(raw, b, &e);
        if (!*done) return FG_OK;
        FG_TRY(put(b, gain_dev, lo, out));
        out->f16 = true;
        out->exp = e;
        double gm = 0;
        for (float v : gain) gm = std::max(gm, double(std::fabs(v)));
        out->gmax = float(gm);
        return FG_OK;
      };
      FG_TRY(put16(fold(rqkv, g_in, H), &L.bqkv, &done));
      const bool lo_qkv = fold_has_lo(rqkv.data(), &g_in, qkv_rows, H);
      if (!done) FG_TRY(put16g(rqkv, L.g_in, g_in, lo_qkv, &L.bqkv, &done));
      if (!done) FG_TRY(put(bqkv, L.g_in, lo_qkv, &L.bqkv));
      FG_TRY(put16(wo->data, &L.bo, &done));
      if (!done) FG_TRY(put(bo, nullptr, false, &L.bo));
      FG_TRY(put16(fold(rgu, g_pf, H), &L.bgu, &done));
      const bool lo_gu = fold_has_lo(rgu.data(), &g_pf, 2 * F, H);
      if (!done) FG_TRY(put16g(rgu, L.g_pf, g_pf, lo_gu, &L.bgu, &done));
      if (!done) FG_TRY(put(bgu, L.g_pf, lo_gu, &L.bgu));
      FG_TRY(put16(wd->data, &L.bd, &done));
      if (!done) FG_TRY(put(bd, nullptr, false, &L.bd));
      L.wqkv = DevMat{nullptr, nullptr, int(qkv_rows), int(H)};
      L.wo = DevMat{nullptr, nullptr, int(H), int(Hq * D)};
      L.wgu = DevMat{nullptr, nullptr, int(2 * F), int(H)};
      L.wd = DevMat{nullptr, nullptr, int(H), int(F)};
    } else {
      const std::vector<float> fqkv = fold(rqkv, g_in, H), fgu = fold(rgu, g_pf, H);
      FG_TRY(upload_mat(m, fqkv, int(qkv_rows), int(H), &L.wqkv));
      FG_TRY(upload_mat(m, wo->data, int(H), int(Hq * D), &L.wo));
      FG_TRY(upload_mat(m, fgu, int(2 * F), int(H), &L.wgu));
      FG_TRY(upload_mat(m, wd->data, int(H), int(F), &L.wd));
      FG_TRY(upload_h16_unfolded(m, rqkv, L.g_in, g_in, &L.wqkv));
      FG_TRY(upload_h16_unfolded(m, rgu, L.g_pf, g_pf, &L.wgu));
      // weights with no exact fp16 form at all (an fp32 checkpoint): two parts
      FG_TRY(upload_h16_split(m, fqkv, &L.wqkv));
      FG_TRY(upload_h16_split(m, wo->data, &L.wo));
      FG_TRY(upload_h16_split(m, fgu, &L.wgu));
      FG_TRY(upload_h16_split(m, wd->data, &L.wd));
    }
    if (m->h16) {
      // Bounds for the split-fp16 scales of the O and down inputs. With
      // rs = 1/sqrt(mean(x²) + eps), ‖rs·x‖ < sqrt(H), so each projection
      // output is below sqrt(H)·‖W'_row‖ (Cauchy-Schwarz): v, hence the
      // attention output (convex combinations of v rows); gate and up,
      // hence GELU(g)·u (|GELU(g)| <= max(|g|, 0.17)).
      const double sh = std::sqrt(double(H));
      double bv = 0, bgu = 0;
      for (int64_t r = (Hq + Hkv) * D; r < qkv_rows; ++r)
        bv = std::max(bv, sh * folded_row_norm(rqkv.data(), g_in, r, H));
      for (int64_t k = 0; k < F; ++k) {
        const double bg = sh * folded_row_norm(wg->data.data(), g_pf, k, H);
        const double bu = sh * folded_row_norm(wu->data.data(), g_pf, k, H);
        bgu = std::max(bgu, std::max(bg, 0.2) * bu);
      }
      L.att_ok = h16_exponent(bv * 1.01, &L.att_exp);
      L.gu_ok = h16_exponent(bgu * 1.01, &L.gu_exp);
    }

    FG_TRY(upload(m, plus_one(*qn), &L.qgain));
    FG_TRY(upload(m, plus_one(*kn), &L.kgain));
    FG_TRY(upload(m, plus_one(*pa_norm), &L.post_attn));
    FG_TRY(upload(m, plus_one(*pff_norm), &L.post_ffn));
  }
  const HostTensor* fn = nullptr;
  FG_TRY(need(m, "norm.weight", {H}, &fn));
  FG_TRY(upload(m, plus_one(*fn), &m->final_gain));

  int prev = int(H);
  for (int j = 0; j < c.num_dense; ++j) {
    const HostTensor* w = nullptr;
    FG_TRY(need(m, "dense." + std::to_string(j) + ".linear.weight", {c.dense_out[j], c.dense_in[j]}, &w));
    if (c.dense_in[j] != prev) return set_error(FG_EINVAL, "dense layer %d takes %d features, previous gives %d", j, c.dense_in[j], prev);
    if (c.dense_in[j] % 4 != 0) return set_error(FG_EINVAL, "dense layer %d input width must be a multiple of 4", j);
    Dense d;
    d.in = c.dense_in[j];
    d.out = c.dense_out[j];
    d.tanh = c.dense_tanh[j] != 0;
    FG_TRY(upload_mat(m, w->data, d.out, d.in, &d.w));
    m->dense.push_back(d);
    prev = d.out;
  }
  m->host.clear();
  bool any_bf16 = false, lo_qkv = false, lo_gu = false;
  for (const Layer& L : m->layers) {
    any_bf16 |= L.resident_bf16;
    lo_qkv |= L.resident_bf16 && L.bqkv.lo;
    lo_gu |= L.resident_bf16 && L.bgu.lo;
  }
  if (any_bf16) {
    const Layer& L0 = m->layers[0];
    auto ws = [&](const DevMat& shape, bool lo, DevMat* out) -> int {
      *out = DevMat{nullptr, nullptr, shape.rows, shape.cols};
      const size_t n = size_t(shape.rows) * shape.cols;
      FG_TRY(dev_alloc_t(m, &out->hi, n));
      if (lo) FG_TRY(dev_alloc_t(m, &out->lo, n));
      return FG_OK;
    };
    FG_TRY(ws(L0.wqkv, lo_qkv, &m->ws_qkv));
    FG_TRY(ws(L0.wo, false, &m->ws_o));
    FG_TRY(ws(L0.wgu, lo_gu, &m->ws_gu));
    FG_TRY(ws(L0.wd, false, &m->ws_d));
  }
  m->weight_bytes = m->alloc_bytes;
  FG_TRY(ensure_workspace(m, std::max<int64_t>(max_tokens, 1), 1));
  FG_CUDA_TRY(cudaDeviceSynchronize());
  m->finalized = true;
  return FG_OK;
}

cudaEvent_t take_event(fg_model* m) {
  if (!m->event_pool.empty()) {
    cudaEvent_t e = m->event_pool.back();
    m->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

// Brackets the launches of one phase: counts them, adds their algorithmic
// work, and, while profiling, records an event pair on the stream.
struct PhaseScope {
  fg_model* m;
  int phase;
  cudaStream_t s;
  cudaEvent_t a = nullptr;
  PhaseScope(fg_model* m_, int p, cudaStream_t s_, double work, int nlaunch = 1)
      : m(m_), phase(p), s(s_) {
    m->launches[p] += nlaunch;
    m->work[p] += work;
    if (m->prof) {
      a = take_event(m);
      if (a) cudaEventRecord(a, s);
    }
  }
  ~PhaseScope() {
    if (!a) return;
    cudaEvent_t b = take_event(m);
    if (!b) {
      m->event_pool.push_back(a);
      return;
    }
    cudaEventRecord(b, s);
    m->marks.push_back({phase, a, b});
  }
};

double gemm_flops(const GemmArgs& g) {
  const double nout = g.epi.geglu ? g.Nb : g.Nb;
  return 2.0 * double(g.M) * nout * double(g.K);
}

GemmArgs make_gemm(int M, const float* A, const float* A_lo, int64_t lda, const DevMat& B,
                   bool split) {
  GemmArgs g;
  g.M = M;
  g.Nb = B.rows;
  g.K = B.cols;
  g.A = A;
  g.A_lo = split ? A_lo : nullptr;
  g.a_lo_smem = split && A_lo == nullptr;  // low part made in shared memory
  g.lda = lda;
  g.B = B.hi;
  g.B_lo = split ? B.lo : nullptr;
  g.ldb = B.cols;
  return g;
}

// Split-fp16 operands for a split product whose A parts are made in shared
// memory: B's exact fp16 form, and A's exponent from its row scales a_rs
// (1/sqrt(mean(a²) + eps)) or, without them, the static aexp (ok: the bound
// behind it is finite).
void use_h16(const fg_model* m, GemmArgs& g, const DevMat& W, const float* a_rs, bool ok, int aexp) {
  if (!m->h16 || !m->use16 || !g.a_lo_smem || !W.h16 || !ok) return;
  g.B16 = W.h16;
  g.b_exp = W.h16_exp;
  g.a_rs = a_rs;
  g.a_exp_rs = a_rs ? 1 : 0;
  g.a_exp = aexp;
  g.a_gain = W.h16_gain;
  g.a_gain_max = W.h16_gmax;
  g.B16_lo = W.h16_lo;
}

struct Batch {
  int start, count, T;  // positions [start, start+count) of the order; padded length T ≥ 1
};

// The batching of (*Model).Embed (embed.go:46-74): indices stably sorted by
// length (sortIndex, model.go:412), then greedy batches in that order, a
// batch closing when admitting the next sequence would make its padded
// size max_len·count exceed the budget.
void plan_batches(const int* len, int nseq, int64_t budget, std::vector<int>& order, std::vector<Batch>& batches) {
  order.resize(static_cast<size_t>(nseq));
  for (int i = 0; i < nseq; ++i) order[size_t(i)] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return len[a] < len[b]; });
  batches.clear();
  int start = 0, count = 0, max_len = 0;
  for (int k = 0; k < nseq; ++k) {
    const int l = len[order[size_t(k)]];
    int nm = std::max(max_len, l);
    if (count > 0 && int64_t(nm) * (count + 1) > budget) {
      batches.push_back({start, count, std::max(max_len, 1)});
      start = k;
      count = 0;
      max_len = 0;
      nm = l;
    }
    ++count;
    max_len = nm;
  }
  if (count > 0) batches.push_back({start, count, std::max(max_len, 1)});
}

// Destroys the cached forward graphs (before a buffer they use is freed),
// after every launch of them has finished.
void drop_graphs(fg_model* m) {
  if (!m->graphs.empty()) cudaDeviceSynchronize();
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second.exec);
  m->graphs.clear();
  m->graph_seen.clear();
}

// The tensor-core attention's operand workspace, grown (never shrunk) to
// `need` bytes; growing waits for the work already queued on `s`.
int grow_attn_ws(fg_model* m, size_t need, cudaStream_t s) {
  if (need <= m->attn_ws_bytes) return FG_OK;
  drop_graphs(m);
  if (m->attn_ws) {
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    FG_CUDA_TRY(cudaFree(m->attn_ws));
    m->attn_ws = nullptr;
    m->attn_ws_bytes = 0;
  }
  FG_CUDA_TRY(cudaMalloc(&m->attn_ws, need));
  m->attn_ws_bytes = need;
  return FG_OK;
}

// EmbeddingGemma 2's text tower (encode2From, embed.go:247-377), then pool,
// embedding projection, Dense head and L2 (embed.go:381-475). Per layer:
// Q/K/V (row-scaled product) → q/k RMSNorm + RoPE and the weight-free
// v_norm → attention with unscaled scores (tensor cores at head_dim 256,
// the SIMT kernel at the global layers' 512) → O → x += RMSNorm(o) → GeGLU
// FFN → x += RMSNorm(mlp) → PLE block g = GELU(x·Wgate)⊙ple_l, y = g·Wproj
// → x = (x + RMSNorm(y))·scalar; the final norm is fused into the last
// residual kernel.
int forward_v2(fg_model* m, const int32_t* ids, const int32_t* lengths, int B, int T, int dim,
               int precision, float* out, cudaStream_t s) {
  const fg_config& c = m->cfg;
  const bool split = precision != FG_PREC_TF32;
  m->use16 = precision == FG_PREC_SPLIT;
  const int H = c.hidden_size, Hq = c.num_heads, F = c.intermediate_size;
  const int L = c.num_layers, P = c.ple_dim, E = c.embedding_dim;
  const int64_t M = int64_t(B) * T;
  if (M > INT32_MAX) return set_error(FG_EINVAL, "batch too large");
  FG_TRY(ensure_workspace(m, M, B));
  const double act_bytes = double(M) * H * 4.0;
  {
    const double row_read = double(M) * H * (m->embed_bf16 ? 2.0 : 4.0);
    PhaseScope ps(m, FG_PHASE_EMBED, s, row_read + act_bytes + double(M) * 8, 2);
    eff_len_kernel<<<(B + 127) / 128, 128, 0, s>>>(lengths, B, T, m->eff_len);
    FG_CUDA_TRY(cudaGetLastError());
    const float emb_scale = float(std::sqrt(double(H)));
    FG_TRY(embed_gather(m->embed, m->embed_bf16, c.vocab_size, ids, lengths, B, T, H, emb_scale, c.rms_norm_eps,
                        m->x, nullptr, m->rowscale, m->err, s));
  }
  // per-layer embeddings once per pass: RMSNorm_P((x·Wple)·(1/√H)) (embed.go:270-275)
  {
    GemmArgs g = make_gemm(int(M), m->x, nullptr, H, m->ple_proj, split);
    g.epi.out = m->ple_buf;
    g.epi.ldo = int64_t(L) * P;
    g.epi.rowscale = m->ple_scale;
    PhaseScope ps(m, FG_PHASE_GEMM_QKV, s, gemm_flops(g));
    FG_TRY(gemm_tn(g, m->err, s));
    FG_TRY(rmsnorm(m->ple_buf, M * L, P, m->ple_gain, c.rms_norm_eps, m->ple_buf, s));
  }
  for (int l = 0; l < L; ++l) {
    const Layer& Ly = m->layers[size_t(l)];
    const bool last = l == L - 1;
    const int D = Ly.D, Hkv = Ly.Hkv;
    const int qkvw = (Hq + 2 * Hkv) * D, attw = Hq * D;
    AttnArgs a{};
    a.q = m->qkv;
    a.k = m->qkv + int64_t(Hq) * D;
    a.v = m->qkv + int64_t(Hq + Hkv) * D;
    a.out = m->att;
    a.out_lo = nullptr;
    a.qsb = int64_t(T) * qkvw; a.qsh = D; a.qst = qkvw;
    a.ksb = a.qsb; a.ksh = D; a.kst = qkvw;
    a.vsb = a.qsb; a.vsh = D; a.vst = qkvw;
    a.osb = int64_t(T) * attw; a.osh = D; a.ost = attw;
    a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.T = T; a.S = T; a.D = D;
    a.klen = m->eff_len;
    a.qlen = m->eff_len;
    a.window = (c.window > 0 && m->sliding[size_t(l)]) ? c.window : 0;
    a.scale = c.attn_scale;
    // q|k|v = rowscale ⊙ (x · Wqkv'ᵀ)   (embed.go:285-288); on the
    // 256-wide layers the epilogue also applies the q/k norms, RoPE and the
    // v_norm and writes the tensor-core attention's operands
    const bool tc = attn_tc_supported(a);
    const bool fused = tc && D == 256 && m->rope_csT[size_t(Ly.rope)] != nullptr;
    AttnOperands ops{};
    if (tc) FG_TRY(grow_attn_ws(m, attn_tc_workspace_bytes(B, T, T, Hq, Hkv, D), s));
    GemmArgs g = make_gemm(int(M), m->x, nullptr, H, Ly.wqkv, split);
    g.epi.rowscale = m->rowscale;
    use_h16(m, g, Ly.wqkv, m->rowscale, true, 0);
    if (fused) {
      FG_TRY(attn_tc_carve(m->attn_ws, B, T, T, Hq, Hkv, &ops));
      g.epi.qkv_attn = 1;
      g.epi.vnorm = 1;
      g.epi.Hq = Hq;
      g.epi.Hkv = Hkv;
      g.epi.T = T;
      g.epi.qgain = Ly.qgain;
      g.epi.kgain = Ly.kgain;
      g.epi.eps = c.rms_norm_eps;
      g.epi.rope_cs = reinterpret_cast<const float2*>(m->rope_csT[size_t(Ly.rope)]);
      g.epi.rope_ld = c.max_tokens;
      g.epi.q_hi = ops.q_hi;
      g.epi.q_lo = ops.q_lo;
      g.epi.k_hi = ops.k_hi;
      g.epi.k_lo = ops.k_lo;
      g.epi.vt_hi = ops.vt_hi;
      g.epi.vt_lo = ops.vt_lo;
      g.epi.ldt = ops.ldt;
    } else {
      g.epi.out = m->qkv;
      g.epi.ldo = qkvw;
    }
    {
      PhaseScope ps(m, FG_PHASE_GEMM_QKV, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    if (!fused) {
      // q/k RMSNorm + RoPE, v RMSNorm (embed.go:289-317)
      PhaseScope ps(m, FG_PHASE_QK_NORM_ROPE, s, double(M) * (Hq + 2 * Hkv) * D * 8.0);
      FG_TRY(qk_norm_rope(m->qkv, nullptr, M, Hq, Hkv, D, Ly.qgain, Ly.kgain, Ly.vgain, c.rms_norm_eps,
                          m->rope_cos[size_t(Ly.rope)], m->rope_sin[size_t(Ly.rope)], T, s));
    }
    {
      PhaseScope ps(m, FG_PHASE_ATTENTION, s, 0.0);
      if (fused) {
        FG_TRY(attention_tc_operands(a, ops, m->err, s));
      } else if (tc) {
        FG_TRY(attention_tc(a, m->attn_ws, m->attn_ws_bytes, m->err, s));
      } else {
        FG_TRY(attention_simt(a, s));
      }
    }
    // o0 = att · Wo; x += RMSNorm(o0)   (embed.go:336-343)
    g = make_gemm(int(M), m->att, nullptr, attw, Ly.wo, split);
    g.epi.out = m->tmp;
    g.epi.ldo = H;
    use_h16(m, g, Ly.wo, nullptr, Ly.att_ok, Ly.att_exp);
    {
      PhaseScope ps(m, FG_PHASE_GEMM_O, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    {
      PhaseScope ps(m, FG_PHASE_RESIDUAL, s, act_bytes * 3 + double(M) * 4);
      FG_TRY(residual_postnorm(m->x, nullptr, m->tmp, Ly.post_attn, c.rms_norm_eps, m->rowscale, nullptr, M, H, s));
    }
    // FFN as in encode (embed.go:345-357)
    g = make_gemm(int(M), m->x, nullptr, H, Ly.wgu, split);
    g.epi.out = m->gu;
    g.epi.ldo = F;
    g.epi.rowscale = m->rowscale;
    g.epi.geglu = 1;
    use_h16(m, g, Ly.wgu, m->rowscale, true, 0);
    {
      PhaseScope ps(m, FG_PHASE_GEMM_GATE_UP, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    g = make_gemm(int(M), m->gu, nullptr, F, Ly.wd, split);
    g.epi.out = m->tmp;
    g.epi.ldo = H;
    use_h16(m, g, Ly.wd, nullptr, Ly.gu_ok, Ly.gu_exp);
    {
      PhaseScope ps(m, FG_PHASE_GEMM_DOWN, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    {
      PhaseScope ps(m, FG_PHASE_RESIDUAL, s, act_bytes * 3 + double(M) * 4);
      FG_TRY(residual_postnorm(m->x, nullptr, m->tmp, Ly.post_ffn, c.rms_norm_eps, m->rowscale, nullptr, M, H, s));
    }
    // PLE block: g = GELU(x·Wgate) ⊙ ple_l; y0 = g·Wproj;
    // x = (x + RMSNorm(y0))·scalar   (embed.go:359-371)
    g = make_gemm(int(M), m->x, nullptr, H, Ly.wpg, split);
    g.epi.out = m->gbuf;
    g.epi.ldo = P;
    g.epi.act = FG_ACT_GELU;
    g.epi.mul = m->ple_buf + int64_t(l) * P;
    g.epi.ldm = int64_t(L) * P;
    use_h16(m, g, Ly.wpg, m->rowscale, true, 0);  // rowscale: this x's RMS scale
    {
      PhaseScope ps(m, FG_PHASE_GEMM_GATE_UP, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    g = make_gemm(int(M), m->gbuf, nullptr, P, Ly.wpp, split);
    g.epi.out = m->tmp;
    g.epi.ldo = H;
    {
      PhaseScope ps(m, FG_PHASE_GEMM_DOWN, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    {
      PhaseScope ps(m, FG_PHASE_RESIDUAL, s, act_bytes * 3 + double(M) * 4);
      FG_TRY(residual_postnorm(m->x, nullptr, m->tmp, Ly.ple_post, c.rms_norm_eps, m->rowscale,
                               last ? m->final_gain : nullptr, M, H, s, Ly.scalar));
    }
  }
  // pool, embedding projection, Dense head, L2 (embed.go:381-475)
  PhaseScope ps(m, FG_PHASE_POOL_HEAD, s, act_bytes, 3 + int(m->dense.size()));
  FG_TRY(mean_pool(m->x, m->eff_len, B, T, H, m->pooled, nullptr, s));
  float* bufs[2] = {m->head_a, m->head_b};
  GemmArgs g = make_gemm(B, m->pooled, nullptr, H, m->emb_proj, split);
  g.epi.out = bufs[0];
  g.epi.ldo = E;
  FG_TRY(gemm_tn(g, m->err, s));
  const float* cur = bufs[0];
  int width = E;
  for (size_t j = 0; j < m->dense.size(); ++j) {
    const Dense& d = m->dense[j];
    g = make_gemm(B, cur, nullptr, width, d.w, split);
    g.epi.out = bufs[(j + 1) & 1];
    g.epi.ldo = d.out;
    g.epi.act = d.tanh ? kActTanh : FG_ACT_NONE;
    FG_TRY(gemm_tn(g, m->err, s));
    cur = bufs[(j + 1) & 1];
    width = d.out;
  }
  if (dim > width) return set_error(FG_EINVAL, "gemma: Dim(%d) outside 1..%d", dim, width);
  FG_TRY(l2_normalize(cur, width, B, dim, c.l2_normalize, out, s));
  return FG_OK;
}

int forward(fg_model* m, const int32_t* ids, const int32_t* lengths, int B, int T, int dim,
            int precision, float* out, cudaStream_t s) {
  if (m->cfg.variant == 2) return forward_v2(m, ids, lengths, B, T, dim, precision, out, s);
  const fg_config& c = m->cfg;
  const bool split = precision != FG_PREC_TF32;
  m->use16 = precision == FG_PREC_SPLIT;
  const int H = c.hidden_size, D = c.head_dim, Hq = c.num_heads, Hkv = c.num_kv_heads;
  const int F = c.intermediate_size;
  const int64_t M = int64_t(B) * T;
  if (M > INT32_MAX) return set_error(FG_EINVAL, "batch too large");
  FG_TRY(ensure_workspace(m, M, B));
  const int qkvw = (Hq + 2 * Hkv) * D, attw = Hq * D;
  // The split products' A low parts are made in shared memory by the GEMM
  // from the A tile, so no producer writes one.
  float* const x_lo = nullptr;
  float* const att_lo = nullptr;
  float* const gu_lo = nullptr;

  const double act_bytes = double(M) * H * 4.0;
  {
    // table rows read (2 or 4 B per value) + x (+ x_lo) written + ids and rowscale
    const double row_read = double(M) * H * (m->embed_bf16 ? 2.0 : 4.0);
    PhaseScope ps(m, FG_PHASE_EMBED, s, row_read + act_bytes + double(M) * 8, 2);
    eff_len_kernel<<<(B + 127) / 128, 128, 0, s>>>(lengths, B, T, m->eff_len);
    FG_CUDA_TRY(cudaGetLastError());
    const float emb_scale = float(std::sqrt(double(H)));
    FG_TRY(embed_gather(m->embed, m->embed_bf16, c.vocab_size, ids, lengths, B, T, H, emb_scale, c.rms_norm_eps,
                        m->x, x_lo, m->rowscale, m->err, s));
  }

  for (int l = 0; l < c.num_layers; ++l) {
    const Layer& L = m->layers[l];
    const bool last = l == c.num_layers - 1;
    // The layer's projections: resident fp32, or bf16 widened now into the
    // one-layer workspace (the previous layer's GEMMs, earlier on the same
    // stream, have finished reading it).
    DevMat Wqkv = L.wqkv, Wo = L.wo, Wgu = L.wgu, Wd = L.wd;
    if (L.resident_bf16) {
      // A projection resident in its fp16 form is read as it is by the
      // split-fp16 GEMM; the others are widened into the workspace.
      const bool h16ok = split && m->h16 && m->use16 && gemm_h16_applies(int(M));
      const Bf16Mat* src[4] = {&L.bqkv, &L.bo, &L.bgu, &L.bd};
      DevMat* dst[4] = {&Wqkv, &Wo, &Wgu, &Wd};
      const DevMat* ws[4] = {&m->ws_qkv, &m->ws_o, &m->ws_gu, &m->ws_d};
      const bool a_ok[4] = {true, L.att_ok, true, L.gu_ok};
      WidenJobs jobs{};
      int nj = 0;
      double bytes = 0;
      for (int i = 0; i < 4; ++i) {
        const int rows = dst[i]->rows, cols = dst[i]->cols;
        if (h16ok && src[i]->f16 && a_ok[i]) {
          *dst[i] = DevMat{nullptr, nullptr, rows, cols, src[i]->w, src[i]->exp, src[i]->gain, src[i]->gmax};
          continue;
        }
        *dst[i] = DevMat{ws[i]->hi, src[i]->lo ? ws[i]->lo : nullptr, rows, cols};
        const int64_t n = int64_t(rows) * cols;
        jobs.j[nj++] = WidenJob{src[i]->w, src[i]->gain, dst[i]->hi, dst[i]->lo, n / 4, cols,
                                src[i]->f16 ? 1 : 0, src[i]->exp};
        bytes += double(n) * (2 + 4 + (dst[i]->lo ? 4 : 0)) + (src[i]->gain ? cols * 4.0 : 0.0);
      }
      if (nj > 0) {
        PhaseScope ps(m, FG_PHASE_WIDEN, s, bytes);
        widen_fold_kernel<<<dim3(4 * 148, nj), 256, 0, s>>>(jobs);
        FG_CUDA_TRY(cudaGetLastError());
      }
    }
    // attention arguments (embed.go:209, attention.go:130)
    AttnArgs a{};
    a.q = m->qkv;
    a.k = m->qkv + int64_t(Hq) * D;
    a.v = m->qkv + int64_t(Hq + Hkv) * D;
    a.out = m->att;
    a.out_lo = att_lo;
    a.qsb = int64_t(T) * qkvw; a.qsh = D; a.qst = qkvw;
    a.ksb = a.qsb; a.ksh = D; a.kst = qkvw;
    a.vsb = a.qsb; a.vsh = D; a.vst = qkvw;
    a.osb = int64_t(T) * attw; a.osh = D; a.ost = attw;
    a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.T = T; a.S = T; a.D = D;
    a.klen = m->eff_len;
    a.qlen = m->eff_len;
    a.window = (c.window > 0 && m->sliding[l]) ? c.window : 0;
    a.scale = c.attn_scale;
    // Tensor-core attention: the QKV GEMM's epilogue applies QK-norm and
    // RoPE and writes the split-bf16 operands straight into its workspace.
    const bool tc = attn_tc_supported(a);
    AttnOperands ops{};
    if (tc) {
      FG_TRY(grow_attn_ws(m, attn_tc_workspace_bytes(B, T, T, Hq, Hkv), s));
      FG_TRY(attn_tc_carve(m->attn_ws, B, T, T, Hq, Hkv, &ops));
    }
    // Split-fp16 with producer-made operands: the attention kernel, the
    // gated epilogue and the residual write the next product's two fp16
    // parts — the ones its converter warps would cut from the fp32 tile —
    // so the O, down and gate/up products load them by TMA and convert
    // nothing (the same parts, so the same result).
    const bool pre = split && m->h16 && m->use16 && gemm_h16_applies(int(M));
    const bool att16 = pre && tc && Wo.h16 && L.att_ok;
    const bool gu16 = pre && Wd.h16 && L.gu_ok;
    const bool x16 = pre && Wgu.h16;
    uint16_t* const att16_hi = reinterpret_cast<uint16_t*>(m->att);  // in place of att
    uint16_t* const att16_lo = att16_hi + M * attw;
    uint16_t* const gu16_hi = reinterpret_cast<uint16_t*>(m->gu);    // in place of gu
    uint16_t* const gu16_lo = gu16_hi + M * F;
    if (att16) {
      a.out16 = att16_hi;
      a.out16_lo = att16_lo;
      a.out16_exp = L.att_exp;
    }
    // q|k|v = rowscale ⊙ (x · Wqkv'ᵀ)   (embed.go:193-197)
    GemmArgs g = make_gemm(int(M), m->x, x_lo, H, Wqkv, split);
    g.epi.rowscale = m->rowscale;
    use_h16(m, g, Wqkv, m->rowscale, true, 0);
    if (tc) {
      // + QK-norm and RoPE (embed.go:198-207) in the epilogue
      g.epi.qkv_attn = 1;
      g.epi.Hq = Hq;
      g.epi.Hkv = Hkv;
      g.epi.T = T;
      g.epi.qgain = L.qgain;
      g.epi.kgain = L.kgain;
      g.epi.eps = c.rms_norm_eps;
      g.epi.rope_cs = reinterpret_cast<const float2*>(m->rope_csT[L.rope]);
      g.epi.rope_ld = c.max_tokens;
      g.epi.q_hi = ops.q_hi;
      g.epi.q_lo = ops.q_lo;
      g.epi.k_hi = ops.k_hi;
      g.epi.k_lo = ops.k_lo;
      g.epi.vt_hi = ops.vt_hi;
      g.epi.vt_lo = ops.vt_lo;
      g.epi.ldt = ops.ldt;
    } else {
      g.epi.out = m->qkv;
      g.epi.ldo = qkvw;
    }
    {
      PhaseScope ps(m, FG_PHASE_GEMM_QKV, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    if (!tc) {
      // QK-norm + RoPE (embed.go:198-207)
      PhaseScope ps(m, FG_PHASE_QK_NORM_ROPE, s, double(M) * (Hq + Hkv) * D * 8.0);
      FG_TRY(qk_norm_rope(m->qkv, nullptr, M, Hq, Hkv, D, L.qgain, L.kgain, nullptr, c.rms_norm_eps,
                          m->rope_cos[L.rope], m->rope_sin[L.rope], T, s));
    }
    {
      PhaseScope ps(m, FG_PHASE_ATTENTION, s, 0.0);
      if (tc) {
        FG_TRY(attention_tc_operands(a, ops, m->err, s));
      } else {
        FG_TRY(attention_simt(a, s));
      }
    }
    // o0 = att · Wo   (embed.go:212-214)
    g = make_gemm(int(M), m->att, att_lo, attw, Wo, split);
    g.epi.out = m->tmp;
    g.epi.ldo = H;
    use_h16(m, g, Wo, nullptr, L.att_ok, L.att_exp);
    if (att16) {
      g.A16 = att16_hi;
      g.A16_lo = att16_lo;
    }
    {
      PhaseScope ps(m, FG_PHASE_GEMM_O, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    // x += RMSNorm(o0)   (embed.go:216-220), and the FFN pre-norm factor
    {
      PhaseScope ps(m, FG_PHASE_RESIDUAL, s, act_bytes * 3 + double(M) * 4);
      // + the gate/up product's parts, with its pre-norm gain when unfolded
      // and the row bound sqrt(H)·max|gain| the product's exponent takes
      const float bg = Wgu.h16_gain && Wgu.h16_gmax > 0.f ? Wgu.h16_gmax : 0.f;
      const Split16Out parts{m->x16, m->x16 + M * H, Wgu.h16_gain, sqrtf(float(H)) * (bg > 0.f ? bg : 1.f)};
      FG_TRY(residual_postnorm(m->x, x16 ? &parts : nullptr, m->tmp, L.post_attn, c.rms_norm_eps,
                               m->rowscale, nullptr, M, H, s));
    }
    // gu = GELU(rs·x·Wg') ⊙ (rs·x·Wu')   (embed.go:224-227)
    g = make_gemm(int(M), m->x, x_lo, H, Wgu, split);
    g.epi.out = m->gu;
    g.epi.ldo = F;
    g.epi.out_lo = gu_lo;
    g.epi.ldo_lo = F;
    g.epi.rowscale = m->rowscale;
    g.epi.geglu = 1;
    use_h16(m, g, Wgu, m->rowscale, true, 0);
    if (x16) {
      g.A16 = m->x16;
      g.A16_lo = m->x16 + M * H;
      g.a_bound_gain = g.a_gain && g.a_gain_max > 0.f ? g.a_gain_max : 0.f;
      g.a_gain = nullptr;  // applied by the residual
    }
    if (gu16) {
      g.epi.out = nullptr;
      g.epi.out_lo = nullptr;
      g.epi.out16 = gu16_hi;
      g.epi.out16_lo = gu16_lo;
      g.epi.out16_exp = L.gu_exp;
    }
    {
      PhaseScope ps(m, FG_PHASE_GEMM_GATE_UP, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    // mlp0 = gu · Wd   (embed.go:229)
    g = make_gemm(int(M), m->gu, gu_lo, F, Wd, split);
    g.epi.out = m->tmp;
    g.epi.ldo = H;
    use_h16(m, g, Wd, nullptr, L.gu_ok, L.gu_exp);
    if (gu16) {
      g.A16 = gu16_hi;
      g.A16_lo = gu16_lo;
    }
    {
      PhaseScope ps(m, FG_PHASE_GEMM_DOWN, s, gemm_flops(g));
      FG_TRY(gemm_tn(g, m->err, s));
    }
    // x += RMSNorm(mlp0)   (embed.go:231-235); final norm on the last layer (embed.go:237)
    {
      PhaseScope ps(m, FG_PHASE_RESIDUAL, s, act_bytes * 3 + double(M) * 4);
      FG_TRY(residual_postnorm(m->x, nullptr, m->tmp, L.post_ffn, c.rms_norm_eps, m->rowscale,
                               last ? m->final_gain : nullptr, M, H, s));
    }
  }
  if (c.num_layers == 0) return set_error(FG_EINVAL, "model has no layers");

  // pool (embed.go:381-404), head (embed.go:408-429), L2 (embed.go:472-475)
  PhaseScope ps(m, FG_PHASE_POOL_HEAD, s, act_bytes, 2 + int(m->dense.size()));
  FG_TRY(mean_pool(m->x, m->eff_len, B, T, H, m->pooled, nullptr, s));
  const float* cur = m->pooled;
  int width = H;
  float* bufs[2] = {m->head_a, m->head_b};
  for (size_t j = 0; j < m->dense.size(); ++j) {
    const Dense& d = m->dense[j];
    GemmArgs g = make_gemm(B, cur, nullptr, width, d.w, split);
    g.epi.out = bufs[j & 1];
    g.epi.ldo = d.out;
    g.epi.act = d.tanh ? kActTanh : FG_ACT_NONE;
    FG_TRY(gemm_tn(g, m->err, s));
    cur = bufs[j & 1];
    width = d.out;
  }
  if (dim > width) return set_error(FG_EINVAL, "gemma: Dim(%d) outside 1..%d", dim, width);
  FG_TRY(l2_normalize(cur, width, B, dim, c.l2_normalize, out, s));
  return FG_OK;
}

// The forward through the model's graph cache (see fg_model::graphs); the
// eager path while profiling (its event pairs are per launch).
int forward_graphed(fg_model* m, const int32_t* ids, const int32_t* lengths, int B, int T, int dim,
                    int precision, float* out, cudaStream_t s) {
  if (m->prof) return forward(m, ids, lengths, B, T, dim, precision, out, s);
  const fg_model::GraphKey key{B, T, dim, precision, ids, lengths, out};
  auto it = m->graphs.find(key);
  if (it != m->graphs.end()) {
    m->use16 = precision == FG_PREC_SPLIT;
    FG_CUDA_TRY(cudaGraphLaunch(it->second.exec, s));
    for (int i = 0; i < FG_NUM_PHASES; ++i) {
      m->launches[i] += it->second.launches[i];
      m->work[i] += it->second.work[i];
    }
    return FG_OK;
  }
  if (!m->graph_seen.count(key)) {
    if (m->graph_seen.size() >= 64) m->graph_seen.clear();
    m->graph_seen.insert(key);
    return forward(m, ids, lengths, B, T, dim, precision, out, s);
  }
  if (!m->cap_stream) FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking));
  int64_t l0[FG_NUM_PHASES];
  double w0[FG_NUM_PHASES];
  std::copy(m->launches, m->launches + FG_NUM_PHASES, l0);
  std::copy(m->work, m->work + FG_NUM_PHASES, w0);
  FG_CUDA_TRY(cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeThreadLocal));
  const int rc = forward(m, ids, lengths, B, T, dim, precision, out, m->cap_stream);
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(m->cap_stream, &g);
  fg_model::Graph gr;
  for (int i = 0; i < FG_NUM_PHASES; ++i) {
    gr.launches[i] = m->launches[i] - l0[i];
    gr.work[i] = m->work[i] - w0[i];
  }
  // the captured launches did not run: their counts come with the graph
  std::copy(l0, l0 + FG_NUM_PHASES, m->launches);
  std::copy(w0, w0 + FG_NUM_PHASES, m->work);
  cudaError_t ie = cudaErrorUnknown;
  if (rc == FG_OK && ce == cudaSuccess && g) ie = cudaGraphInstantiate(&gr.exec, g, 0);
  if (g) cudaGraphDestroy(g);
  if (ie != cudaSuccess) {
    // not capturable after all: this key stays eager
    cudaGetLastError();
    clear_error();
    m->graph_seen.erase(key);
    return forward(m, ids, lengths, B, T, dim, precision, out, s);
  }
  if (m->graphs.size() >= 16) drop_graphs(m);
  m->graphs[key] = gr;
  m->graph_seen.insert(key);
  FG_CUDA_TRY(cudaGraphLaunch(gr.exec, s));
  for (int i = 0; i < FG_NUM_PHASES; ++i) {
    m->launches[i] += gr.launches[i];
    m->work[i] += gr.work[i];
  }
  return FG_OK;
}

// (*Model).Dim (model.go:336-344): the embedding projection's width for
// EmbeddingGemma 2, else the last Dense layer's, else hidden.
int model_dim(const fg_model* m) {
  if (m->cfg.variant == 2) return m->cfg.embedding_dim;
  return m->cfg.num_dense > 0 ? m->cfg.dense_out[m->cfg.num_dense - 1] : m->cfg.hidden_size;
}

}  // namespace

int model_max_tokens(const fg_model* m) { return m->cfg.max_tokens; }

}  // namespace fg

using namespace fg;

extern "C" {

int fg_model_create(const fg_config* cfg, int device, fg_model** out) {
  clear_error();
  if (!cfg || !out) return set_error(FG_EINVAL, "fg_model_create: null argument");
  *out = nullptr;
  const fg_config& c = *cfg;
  if (c.hidden_size <= 0 || c.num_layers <= 0 || c.num_heads <= 0 || c.num_kv_heads <= 0 ||
      c.head_dim <= 0 || c.vocab_size <= 0 || c.intermediate_size <= 0 || c.max_tokens <= 0)
    return set_error(FG_EINVAL, "gemma: config is missing sizes");
  if (c.head_dim % 2 != 0) return set_error(FG_EINVAL, "gemma: head_dim %d must be even for RoPE", c.head_dim);
  if (c.num_heads % c.num_kv_heads != 0)
    return set_error(FG_EINVAL, "gemma: %d query heads not a multiple of %d key/value heads", c.num_heads, c.num_kv_heads);
  if (c.num_dense < 0 || c.num_dense > FG_MAX_DENSE) return set_error(FG_EINVAL, "gemma: %d dense layers", c.num_dense);
  if (!c.sliding || !c.rope_base) return set_error(FG_EINVAL, "gemma: per-layer sliding / rope_base arrays missing");
  if (c.variant != 0 && c.variant != 2) return set_error(FG_EINVAL, "gemma: unknown variant %d", c.variant);
  if (c.variant == 2) {
    if (c.ple_dim <= 0 || c.ple_dim % 4 != 0 || c.embedding_dim <= 0 || c.embedding_dim % 4 != 0)
      return set_error(FG_EINVAL, "gemma: embedding_gemma2 needs hidden_size_per_layer_input and embedding_dim (multiples of 4)");
    for (int l = 0; l < c.num_layers; ++l) {
      const int D = c.layer_head_dim ? c.layer_head_dim[l] : c.head_dim;
      const int kv = c.layer_kv_heads ? c.layer_kv_heads[l] : c.num_kv_heads;
      if (D <= 0 || D % 4 != 0 || D > 512)
        return set_error(FG_EINVAL, "gemma: layer %d head_dim %d unsupported (multiple of 4, at most 512)", l, D);
      if (kv <= 0 || c.num_heads % kv != 0)
        return set_error(FG_EINVAL, "gemma: layer %d: %d query heads not a multiple of %d key/value heads", l, c.num_heads, kv);
    }
  } else if (c.layer_head_dim || c.layer_kv_heads) {
    return set_error(FG_EINVAL, "gemma: per-layer head geometry is an embedding_gemma2 setting");
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
    cudaGetLastError();
    return set_error(FG_ENODEV, "no CUDA device %d", device);
  }
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (major != 10) return set_error(FG_ENODEV, "device %d is not an sm_100 part (cc %d.x)", device, major);
  auto* m = new fg_model();
  m->device = device;
  m->cfg = c;
  m->sliding.assign(c.sliding, c.sliding + c.num_layers);
  m->rope_base.assign(c.rope_base, c.rope_base + c.num_layers);
  m->cfg.sliding = m->sliding.data();
  m->cfg.rope_base = m->rope_base.data();
  for (int l = 0; l < c.num_layers; ++l) {
    m->head_dim_l.push_back(c.layer_head_dim ? c.layer_head_dim[l] : c.head_dim);
    m->kv_l.push_back(c.layer_kv_heads ? c.layer_kv_heads[l] : c.num_kv_heads);
  }
  m->cfg.layer_head_dim = m->head_dim_l.data();
  m->cfg.layer_kv_heads = m->kv_l.data();
  const char* wm = std::getenv("FG_WEIGHTS");
  if (wm && std::string(wm) == "bf16") m->weight_mode = FG_WEIGHTS_BF16;
  *out = m;
  return FG_OK;
}

int fg_model_set_weight_residency(fg_model* m, int mode) {
  clear_error();
  if (!m) return set_error(FG_EINVAL, "fg_model_set_weight_residency: null model");
  if (m->finalized) return set_error(FG_ESTATE, "fg_model_set_weight_residency after finalize");
  if (mode != FG_WEIGHTS_F32 && mode != FG_WEIGHTS_BF16)
    return set_error(FG_EINVAL, "fg_model_set_weight_residency: unknown mode %d", mode);
  m->weight_mode = mode;
  return FG_OK;
}

int64_t fg_model_weight_bytes(fg_model* m) {
  clear_error();
  if (!m) return set_error(FG_EINVAL, "fg_model_weight_bytes: null model");
  if (!m->finalized) return set_error(FG_ESTATE, "fg_model_weight_bytes before finalize");
  return int64_t(m->weight_bytes);
}

int fg_model_set_weight(fg_model* m, const char* name, int dtype, const int64_t* shape, int ndim,
                        const void* data) {
  clear_error();
  if (!m || !name || (!shape && ndim > 0) || ndim < 0 || ndim > 4)
    return set_error(FG_EINVAL, "fg_model_set_weight: bad arguments");
  if (m->finalized) return set_error(FG_ESTATE, "fg_model_set_weight after finalize");
  int64_t n = 1;
  HostTensor t;
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 0) return set_error(FG_EINVAL, "negative dimension");
    n *= shape[i];
    t.shape.push_back(shape[i]);
  }
  if (n > 0 && !data) return set_error(FG_EINVAL, "fg_model_set_weight: null data for %s", name);
  t.data.resize(size_t(n));
  switch (dtype) {
    case FG_DT_F32:
      std::memcpy(t.data.data(), data, size_t(n) * 4);
      break;
    case FG_DT_BF16: {
      const uint16_t* s = static_cast<const uint16_t*>(data);
      for (int64_t i = 0; i < n; ++i) t.data[i] = bf16_to_f32(s[i]);
      break;
    }
    case FG_DT_F16: {
      const uint16_t* s = static_cast<const uint16_t*>(data);
      for (int64_t i = 0; i < n; ++i) t.data[i] = f16_to_f32(s[i]);
      break;
    }
    default:
      return set_error(FG_EINVAL, "fg_model_set_weight: unknown dtype %d", dtype);
  }
  m->host[name] = std::move(t);
  return FG_OK;
}

int fg_model_finalize(fg_model* m, int64_t max_batch_tokens) {
  clear_error();
  if (!m) return set_error(FG_EINVAL, "null model");
  if (m->finalized) return set_error(FG_ESTATE, "model already finalized");
  if (max_batch_tokens < 0) return set_error(FG_EINVAL, "negative token capacity");
  return finalize(m, max_batch_tokens);
}

int fg_embed_ids_device(fg_model* m, const int32_t* d_ids, const int32_t* d_lengths, int B, int T,
                        int dim, int precision, float* d_out, void* stream) {
  clear_error();
  if (!m) return set_error(FG_EINVAL, "null model");
  if (!m->finalized) return set_error(FG_ESTATE, "embed before fg_model_finalize");
  if (B < 0 || T < 0) return set_error(FG_EINVAL, "negative batch shape");
  if (B == 0) return FG_OK;
  if (T == 0) return set_error(FG_EINVAL, "T must be at least 1");
  if (T > m->cfg.max_tokens) return set_error(FG_EINVAL, "T=%d exceeds max_tokens %d", T, m->cfg.max_tokens);
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "unknown precision %d", precision);
  const int full = model_dim(m);
  if (dim < 1 || dim > full) return set_error(FG_EINVAL, "gemma: Dim(%d) outside 1..%d", dim, full);
  FG_CUDA_TRY(cudaSetDevice(m->device));
  return forward_graphed(m, d_ids, d_lengths, B, T, dim, precision, d_out, static_cast<cudaStream_t>(stream));
}

int fg_embed_ids(fg_model* m, const int32_t* ids, const int32_t* lengths, int B, int T, int dim,
                 int precision, float* out) {
  clear_error();
  if (!m) return set_error(FG_EINVAL, "null model");
  if (!m->finalized) return set_error(FG_ESTATE, "embed before fg_model_finalize");
  if (B < 0 || T < 0) return set_error(FG_EINVAL, "negative batch shape");
  if (B == 0) return FG_OK;
  if (!ids || !lengths || !out) return set_error(FG_EINVAL, "null buffer");
  for (int b = 0; b < B; ++b) {
    if (lengths[b] < 0 || lengths[b] > T)
      return set_error(FG_EINVAL, "length %d of sequence %d outside 0..%d", lengths[b], b, T);
    for (int t = 0; t < lengths[b]; ++t) {
      const int32_t id = ids[int64_t(b) * T + t];
      if (id < 0 || id >= m->cfg.vocab_size)
        return set_error(FG_EINVAL, "token id %d at [%d, %d] outside the vocabulary", id, b, t);
    }
  }
  FG_CUDA_TRY(cudaSetDevice(m->device));
  if (!m->stream) FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  const int64_t nid = int64_t(B) * T;
  if (nid > m->d_ids_cap || B > m->d_len_cap || int64_t(B) * dim > m->d_out_cap) {
    // graphs may hold the staging buffers about to be replaced
    FG_CUDA_TRY(cudaStreamSynchronize(m->stream));
    drop_graphs(m);
  }
  if (nid > m->d_ids_cap) {
    if (m->d_ids) cudaFree(m->d_ids);
    FG_CUDA_TRY(cudaMalloc(&m->d_ids, size_t(nid) * 4));
    m->d_ids_cap = nid;
  }
  if (B > m->d_len_cap) {
    if (m->d_len) cudaFree(m->d_len);
    FG_CUDA_TRY(cudaMalloc(&m->d_len, size_t(B) * 4));
    m->d_len_cap = B;
  }
  const int64_t nout = int64_t(B) * dim;
  if (nout > m->d_out_cap) {
    if (m->d_out) cudaFree(m->d_out);
    FG_CUDA_TRY(cudaMalloc(&m->d_out, size_t(nout) * 4));
    m->d_out_cap = nout;
  }
  FG_CUDA_TRY(cudaMemcpyAsync(m->d_ids, ids, size_t(nid) * 4, cudaMemcpyHostToDevice, m->stream));
  FG_CUDA_TRY(cudaMemcpyAsync(m->d_len, lengths, size_t(B) * 4, cudaMemcpyHostToDevice, m->stream));
  FG_TRY(fg_embed_ids_device(m, m->d_ids, m->d_len, B, T, dim, precision, m->d_out, m->stream));
  FG_CUDA_TRY(cudaMemcpyAsync(out, m->d_out, size_t(nout) * 4, cudaMemcpyDeviceToHost, m->stream));
  FG_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return fg_model_check(m);
}

int fg_plan_batches(const int32_t* lengths, int nseq, int64_t batch_tokens, int32_t* order, int32_t* batch_end) {
  clear_error();
  if (nseq < 0 || batch_tokens < 1) return set_error(FG_EINVAL, "fg_plan_batches: bad arguments");
  if (nseq == 0) return 0;
  if (!lengths || !order || !batch_end) return set_error(FG_EINVAL, "fg_plan_batches: null buffer");
  std::vector<int> len(lengths, lengths + nseq), ord;
  for (int l : len)
    if (l < 0) return set_error(FG_EINVAL, "fg_plan_batches: negative length");
  std::vector<Batch> batches;
  plan_batches(len.data(), nseq, batch_tokens, ord, batches);
  for (int i = 0; i < nseq; ++i) order[i] = ord[size_t(i)];
  for (size_t b = 0; b < batches.size(); ++b) batch_end[b] = batches[b].start + batches[b].count;
  return int(batches.size());
}

int fg_embed_many(fg_model* m, const int32_t* ids, const int64_t* offsets, int nseq, int max_tokens,
                  int64_t batch_tokens, int dim, int precision, float* out) {
  clear_error();
  if (!m) return set_error(FG_EINVAL, "null model");
  if (!m->finalized) return set_error(FG_ESTATE, "embed before fg_model_finalize");
  if (nseq < 0) return set_error(FG_EINVAL, "negative sequence count");
  if (nseq == 0) return FG_OK;
  if (!offsets || !out) return set_error(FG_EINVAL, "null buffer");
  if (batch_tokens < 1) return set_error(FG_EINVAL, "batch_tokens %lld < 1", (long long)batch_tokens);
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "unknown precision %d", precision);
  const int full = model_dim(m);
  if (dim < 1 || dim > full) return set_error(FG_EINVAL, "gemma: Dim(%d) outside 1..%d", dim, full);
  const int cap_t = m->cfg.max_tokens;
  const int max_t = (max_tokens > 0 && max_tokens < cap_t) ? max_tokens : cap_t;
  // truncate (embed.go:38-40), validate
  std::vector<int> len(static_cast<size_t>(nseq));
  if (offsets[0] < 0) return set_error(FG_EINVAL, "offsets[0] = %lld < 0", (long long)offsets[0]);
  for (int i = 0; i < nseq; ++i) {
    const int64_t n = offsets[i + 1] - offsets[i];
    if (n < 0) return set_error(FG_EINVAL, "offsets decrease at sequence %d", i);
    len[size_t(i)] = int(std::min<int64_t>(n, max_t));
    if (len[size_t(i)] > 0 && !ids) return set_error(FG_EINVAL, "null ids");
    for (int t = 0; t < len[size_t(i)]; ++t) {
      const int32_t id = ids[offsets[i] + t];
      if (id < 0 || id >= m->cfg.vocab_size)
        return set_error(FG_EINVAL, "token id %d at [%d, %d] outside the vocabulary", id, i, t);
    }
  }
  std::vector<int> order;
  std::vector<Batch> batches;
  plan_batches(len.data(), nseq, batch_tokens, order, batches);
  int64_t max_bt = 0;
  int max_b = 0;
  size_t attn_need = 0;
  for (const Batch& b : batches) {
    max_bt = std::max<int64_t>(max_bt, int64_t(b.count) * b.T);
    max_b = std::max(max_b, b.count);
    if (m->cfg.head_dim == 256)
      attn_need = std::max(attn_need, attn_tc_workspace_bytes(b.count, b.T, b.T, m->cfg.num_heads, m->cfg.num_kv_heads));
  }
  FG_CUDA_TRY(cudaSetDevice(m->device));
  if (!m->stream) FG_CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  cudaStream_t s = m->stream;
  FG_TRY(ensure_workspace(m, max_bt, max_b));
  FG_TRY(grow_attn_ws(m, attn_need, s));

  // Two slots of pinned staging and device buffers: batch i+1 is packed and
  // copied in (copy stream) while batch i runs (the model's stream), and
  // batch i−1's embeddings are scattered into `out` meanwhile.
  struct Slot {
    int32_t *h_ids = nullptr, *h_len = nullptr, *d_ids = nullptr, *d_len = nullptr;
    float *h_out = nullptr, *d_out = nullptr;
    cudaEvent_t h2d = nullptr, done = nullptr;
  } slot[2];
  cudaStream_t cs = nullptr;
  int rc = FG_OK;
  auto cuda_ok = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && rc == FG_OK) rc = set_error(FG_ECUDA, "fg_embed_many: %s failed: %s", what, cudaGetErrorString(e));
    return rc == FG_OK;
  };
  bool ok = cuda_ok(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "stream");
  for (int k = 0; k < 2 && ok; ++k) {
    Slot& q = slot[k];
    ok = cuda_ok(cudaHostAlloc(reinterpret_cast<void**>(&q.h_ids), size_t(max_bt) * 4, cudaHostAllocDefault), "pinned ids") &&
         cuda_ok(cudaHostAlloc(reinterpret_cast<void**>(&q.h_len), size_t(max_b) * 4, cudaHostAllocDefault), "pinned lengths") &&
         cuda_ok(cudaHostAlloc(reinterpret_cast<void**>(&q.h_out), size_t(max_b) * dim * 4, cudaHostAllocDefault), "pinned out") &&
         cuda_ok(cudaMalloc(&q.d_ids, size_t(max_bt) * 4), "ids") && cuda_ok(cudaMalloc(&q.d_len, size_t(max_b) * 4), "lengths") &&
         cuda_ok(cudaMalloc(&q.d_out, size_t(max_b) * dim * 4), "out") &&
         cuda_ok(cudaEventCreateWithFlags(&q.h2d, cudaEventDisableTiming), "event") &&
         cuda_ok(cudaEventCreateWithFlags(&q.done, cudaEventDisableTiming), "event");
  }
  auto scatter = [&](int bi) {
    const Batch& b = batches[size_t(bi)];
    const Slot& q = slot[bi & 1];
    for (int r = 0; r < b.count; ++r)
      std::memcpy(out + int64_t(order[size_t(b.start + r)]) * dim, q.h_out + int64_t(r) * dim, size_t(dim) * 4);
  };
  const int nb = int(batches.size());
  for (int bi = 0; bi < nb && ok; ++bi) {
    const Batch& b = batches[size_t(bi)];
    Slot& q = slot[bi & 1];
    for (int r = 0; r < b.count; ++r) {
      const int i = order[size_t(b.start + r)];
      const int l = len[size_t(i)];
      int32_t* row = q.h_ids + int64_t(r) * b.T;
      if (l) std::memcpy(row, ids + offsets[i], size_t(l) * 4);
      std::memset(row + l, 0, size_t(b.T - l) * 4);  // right-padded with id 0 (embed.go:124-130)
      q.h_len[r] = l;
    }
    ok = cuda_ok(cudaStreamWaitEvent(cs, q.done, 0), "wait") &&  // the slot's previous batch is finished
         cuda_ok(cudaMemcpyAsync(q.d_ids, q.h_ids, size_t(b.count) * b.T * 4, cudaMemcpyHostToDevice, cs), "copy in") &&
         cuda_ok(cudaMemcpyAsync(q.d_len, q.h_len, size_t(b.count) * 4, cudaMemcpyHostToDevice, cs), "copy in") &&
         cuda_ok(cudaEventRecord(q.h2d, cs), "record") && cuda_ok(cudaStreamWaitEvent(s, q.h2d, 0), "wait");
    if (!ok) break;
    rc = forward(m, q.d_ids, q.d_len, b.count, b.T, dim, precision, q.d_out, s);
    ok = rc == FG_OK &&
         cuda_ok(cudaMemcpyAsync(q.h_out, q.d_out, size_t(b.count) * dim * 4, cudaMemcpyDeviceToHost, s), "copy out") &&
         cuda_ok(cudaEventRecord(q.done, s), "record");
    if (ok && bi > 0) {
      ok = cuda_ok(cudaEventSynchronize(slot[(bi - 1) & 1].done), "sync");
      if (ok) scatter(bi - 1);
    }
  }
  if (ok) {
    ok = cuda_ok(cudaEventSynchronize(slot[(nb - 1) & 1].done), "sync");
    if (ok) scatter(nb - 1);
  }
  cudaStreamSynchronize(s);
  if (cs) {
    cudaStreamSynchronize(cs);
    cudaStreamDestroy(cs);
  }
  for (Slot& q : slot) {
    if (q.h_ids) cudaFreeHost(q.h_ids);
    if (q.h_len) cudaFreeHost(q.h_len);
    if (q.h_out) cudaFreeHost(q.h_out);
    if (q.d_ids) cudaFree(q.d_ids);
    if (q.d_len) cudaFree(q.d_len);
    if (q.d_out) cudaFree(q.d_out);
    if (q.h2d) cudaEventDestroy(q.h2d);
    if (q.done) cudaEventDestroy(q.done);
  }
  if (rc != FG_OK) return rc;
  return fg_model_check(m);
}

int fg_model_check(fg_model* m) {
  if (!m) return set_error(FG_EINVAL, "null model");
  FG_CUDA_TRY(cudaSetDevice(m->device));
  return check_device_error_word();
}

int fg_model_set_profiling(fg_model* m, int enable) {
  clear_error();
  if (!m) return set_error(FG_EINVAL, "null model");
  m->prof = enable != 0;
  return FG_OK;
}

int fg_model_read_profile(fg_model* m, double* ms, int64_t* launches, double* work, int n) {
  clear_error();
  if (!m || n < 0) return set_error(FG_EINVAL, "fg_model_read_profile: bad arguments");
  FG_CUDA_TRY(cudaSetDevice(m->device));
  double acc[FG_NUM_PHASES] = {};
  for (auto& mk : m->marks) {
    float t = 0.f;
    FG_CUDA_TRY(cudaEventSynchronize(mk.b));
    FG_CUDA_TRY(cudaEventElapsedTime(&t, mk.a, mk.b));
    acc[mk.phase] += t;
    m->event_pool.push_back(mk.a);
    m->event_pool.push_back(mk.b);
  }
  m->marks.clear();
  for (int p = 0; p < n && p < FG_NUM_PHASES; ++p) {
    if (ms) ms[p] = acc[p];
    if (launches) launches[p] = m->launches[p];
    if (work) work[p] = m->work[p];
  }
  for (int p = 0; p < FG_NUM_PHASES; ++p) {
    m->launches[p] = 0;
    m->work[p] = 0;
  }
  return FG_OK;
}

void fg_model_destroy(fg_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  cudaDeviceSynchronize();
  for (auto& mk : m->marks) {
    cudaEventDestroy(mk.a);
    cudaEventDestroy(mk.b);
  }
  for (auto e : m->event_pool) cudaEventDestroy(e);
  drop_graphs(m);
  if (m->cap_stream) cudaStreamDestroy(m->cap_stream);
  if (m->attn_ws) cudaFree(m->attn_ws);
  for (void* p : m->allocations) cudaFree(p);
  if (m->d_ids) cudaFree(m->d_ids);
  if (m->d_len) cudaFree(m->d_len);
  if (m->d_out) cudaFree(m->d_out);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

}  // extern "C"
