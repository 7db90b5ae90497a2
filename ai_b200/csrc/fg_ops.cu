// Op-level C ABI: the tensor operations the encoder calls, on device
// pointers. Scratch space for operand splitting and packing is
// stream-ordered on the caller's stream, from the library's per-device
// pool, which keeps it reserved between calls.
#include <cmath>
#include <cstdlib>
#include <string>
#include <vector>

#include "fg_internal.h"
#include "fg_kernels.cuh"

namespace fg {
namespace {

int64_t round4(int64_t v) { return (v + 3) / 4 * 4; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct StreamScratch {
  cudaStream_t s;
  void* p = nullptr;
  explicit StreamScratch(cudaStream_t st) : s(st) {}
  int alloc(size_t bytes) { return scratch_alloc(&p, bytes, s); }
  ~StreamScratch() { scratch_free(p, s); }
};

// cos/sin tables [T, D/2] in float64, stored as float32 (tensor/rope.go:36-50).
void rope_tables(double base, const int32_t* positions, int T, int D, std::vector<float>& cos_t,
                 std::vector<float>& sin_t) {
  const int half = D / 2;
  std::vector<double> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = std::pow(base, -double(2 * i) / double(D));
  cos_t.resize(size_t(T) * half);
  sin_t.resize(size_t(T) * half);
  for (int t = 0; t < T; ++t) {
    const double p = double(positions ? positions[t] : t);
    for (int i = 0; i < half; ++i) {
      const double a = p * inv[i];
      cos_t[size_t(t) * half + i] = float(std::cos(a));
      sin_t[size_t(t) * half + i] = float(std::sin(a));
    }
  }
}

}  // namespace
}  // namespace fg

using namespace fg;

namespace fg {

// Scratch of a product as fg_matmul runs it, and the run itself on a
// given scratch pointer (shared with fg_matmul_noalloc, so both take the
// same path bit for bit).
//   A: read in place when 16-byte aligned with a row stride of whole 16-byte
//      units (a split product then makes A's low part in shared memory);
//      else re-strided into scratch [m, kp] (with its low part when split).
//   B: w given as the transposed view of an [n, k] matrix (K-major, the
//      layout the tensor core reads) is read in place when aligned; [k, n]
//      is transposed into scratch [n, kp]. A split-TF32 product adds B's
//      low part [n, ldb] (the high part is B itself: the tensor core reads
//      its top 19 bits).
//   Split precision (FG_PREC_SPLIT) on SM pairs (m >= 256, n > 128, x read
//   in place) runs split-fp16 instead: B cut into fp16 hi/lo parts [n,
//   kp16] under one power-of-two scale found on the device, A's rows
//   scaled by powers of two from their norms (row_inv_rms) and cut into
//   fp16 parts by the GEMM's converters: A_hi·B_hi + A_hi·B_lo + A_lo·B_hi
//   in kind::f16, the tensor-pipe time of 1.5 TF32 passes instead of 3.
namespace {
size_t round256(size_t v) { return (v + 255) / 256 * 256; }
}  // namespace

MatmulPlan plan_matmul(int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx, const float* w,
                       int64_t ldw, int w_transposed, int precision) {
  MatmulPlan p{};
  p.split = precision != FG_PREC_TF32;
  p.kp = round4(k);
  p.kp16 = (k + 7) / 8 * 8;
  p.a_direct = aligned16(x) && ldx % 4 == 0;
  p.b_direct = w_transposed && aligned16(w) && ldw % 4 == 0;
  p.h16 = precision == FG_PREC_SPLIT && p.a_direct && n > 128 && gemm_h16_applies(int(m));
  p.ldb = p.b_direct ? ldw : p.kp;
  p.a_bytes = p.a_direct ? 0 : round256(size_t(m) * p.kp * 4) * (p.split ? 2 : 1);
  p.bt_bytes = p.b_direct ? 0 : round256(size_t(n) * p.kp * 4);
  p.blo_bytes = (p.split && !p.h16) ? round256(size_t(n) * p.ldb * 4) : 0;
  p.b16_bytes = p.h16 ? 2 * round256(size_t(n) * p.kp16 * 2) : 0;
  p.rs_bytes = p.h16 ? round256(size_t(m) * 4) : 0;
  p.misc_bytes = p.h16 ? 256 : 0;
  return p;
}

int matmul_run(const MatmulPlan& p, int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx,
               const float* w, int64_t ldw, int w_transposed, float* out, int64_t ldo, const fg_epilogue* epi,
               void* scratch, int* err, cudaStream_t s) {
  unsigned char* cur = static_cast<unsigned char*>(scratch);
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
  if (p.a_direct) {
    g.A = x;
    g.lda = ldx;
    g.a_lo_smem = p.split;
  } else {
    const size_t part = p.a_bytes / (p.split ? 2 : 1);
    float* ahi = take(part);
    float* alo = p.split ? take(part) : nullptr;
    FG_TRY(split_copy_2d(x, ldx, m, k, ahi, alo, p.kp, p.split ? 1 : 0, s));
    g.A = ahi;
    g.A_lo = alo;
    g.lda = p.kp;
  }
  if (p.b_direct) {
    g.B = w;
  } else {
    float* bt = take(p.bt_bytes);
    if (w_transposed) {
      FG_TRY(split_copy_2d(w, ldw, n, k, bt, nullptr, p.kp, 0, s));  // re-strided, aligned copy
    } else {
      FG_TRY(transpose_f32(w, ldw, k, n, bt, p.kp, s));
    }
    g.B = bt;
  }
  g.ldb = p.ldb;
  if (p.h16) {
    uint16_t* bhi = reinterpret_cast<uint16_t*>(take(p.b16_bytes / 2));
    uint16_t* blo = reinterpret_cast<uint16_t*>(take(p.b16_bytes / 2));
    float* rs = take(p.rs_bytes);
    unsigned* misc = reinterpret_cast<unsigned*>(take(p.misc_bytes));
    int* bexp = reinterpret_cast<int*>(misc + 1);
    FG_TRY(split_f16_parts(g.B, p.ldb, n, k, bhi, blo, p.kp16, misc, bexp, s));
    FG_TRY(row_inv_rms(x, ldx, m, k, rs, s));
    g.B = nullptr;
    g.B16 = bhi;
    g.B16_lo = blo;
    g.ldb = p.kp16;
    g.b_exp_dev = bexp;
    g.a_lo_smem = true;
    g.a_rs = rs;
    g.a_exp_rs = 1;
  } else if (p.split) {
    float* blo = take(p.blo_bytes);
    FG_TRY(split_copy_2d(g.B, p.ldb, n, k, nullptr, blo, p.ldb, 0, s));
    g.B_lo = blo;
  }
  g.epi = e;
  return gemm_tn(g, err, s);
}

}  // namespace fg

extern "C" {

int fg_matmul(int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx, const float* w,
              int64_t ldw, int w_transposed, float* out, int64_t ldo, const fg_epilogue* epi,
              int precision, void* stream) {
  clear_error();
  if (m < 0 || n < 0 || k < 0 || m > INT32_MAX || n > INT32_MAX || k > INT32_MAX)
    return set_error(FG_EINVAL, "fg_matmul: bad shape m=%lld n=%lld k=%lld", (long long)m, (long long)n, (long long)k);
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "fg_matmul: unknown precision %d", precision);
  if (m == 0 || n == 0) return FG_OK;
  if (!x || !w || !out) return set_error(FG_EINVAL, "fg_matmul: null operand");
  if (ldx < k || ldo < n || (w_transposed ? ldw < k : ldw < n))
    return set_error(FG_EINVAL, "fg_matmul: leading dimension smaller than the row");
  if (epi && epi->act != FG_ACT_NONE && epi->act != FG_ACT_RELU && epi->act != FG_ACT_GELU)
    return set_error(FG_EINVAL, "fg_matmul: unknown activation %d", epi->act);
  if (epi && ((epi->mul && epi->ldm < n) || (epi->residual && epi->ldr < n)))
    return set_error(FG_EINVAL, "fg_matmul: Mul/Residual leading dimension smaller than n");
  if (k == 0) return set_error(FG_EINVAL, "fg_matmul: k = 0 is not supported");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = nullptr;
  FG_TRY(device_error_word(&err));
  const MatmulPlan p = plan_matmul(m, n, k, x, ldx, w, ldw, w_transposed, precision);
  StreamScratch scratch(s);
  FG_TRY(scratch.alloc(p.total()));
  return matmul_run(p, m, n, k, x, ldx, w, ldw, w_transposed, out, ldo, epi, scratch.p, err, s);
}

int fg_row_sum_squares(const float* x, int64_t rows, int64_t n, int64_t ldx, float* out,
                       void* stream) {
  clear_error();
  if (rows < 0 || n < 0 || ldx < n) return set_error(FG_EINVAL, "fg_row_sum_squares: bad shape");
  return row_sum_squares(x, rows, n, ldx, out, static_cast<cudaStream_t>(stream));
}

int fg_rmsnorm(const float* x, int64_t rows, int64_t n, const float* g, float eps, float* out,
               void* stream) {
  clear_error();
  if (rows < 0 || n <= 0) return set_error(FG_EINVAL, "fg_rmsnorm: bad shape");
  return rmsnorm(x, rows, n, g, eps, out, static_cast<cudaStream_t>(stream));
}

int fg_rope(const float* x, int64_t rows, int T, int D, double base, const int32_t* positions,
            float* out, void* stream) {
  clear_error();
  if (D % 2 != 0) return set_error(FG_EINVAL, "fg_rope: head dimension %d must be even", D);
  if (T <= 0 || rows < 0 || rows % T != 0) return set_error(FG_EINVAL, "fg_rope: rows %lld not a multiple of T=%d", (long long)rows, T);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::vector<float> ct, st;
  rope_tables(base, positions, T, D, ct, st);
  const size_t tb = ct.size() * sizeof(float);
  StreamScratch scratch(s);
  FG_TRY(scratch.alloc(2 * tb));
  float* dc = static_cast<float*>(scratch.p);
  float* ds = dc + ct.size();
  if (tb) {
    FG_CUDA_TRY(cudaMemcpyAsync(dc, ct.data(), tb, cudaMemcpyHostToDevice, s));
    FG_CUDA_TRY(cudaMemcpyAsync(ds, st.data(), tb, cudaMemcpyHostToDevice, s));
  }
  FG_TRY(rope(x, rows, T, D, dc, ds, out, s));
  // the host tables must outlive the copies
  FG_CUDA_TRY(cudaStreamSynchronize(s));
  return FG_OK;
}

int fg_attention(const float* q, const float* k, const float* v, int B, int Hq, int Hkv, int T,
                 int S, int D, const int32_t* key_lengths, int window, float scale, float* out,
                 int precision, void* stream) {
  clear_error();
  if (B < 0 || Hq <= 0 || Hkv <= 0 || T < 0 || S < 0 || D <= 0)
    return set_error(FG_EINVAL, "fg_attention: bad shape");
  if (precision != FG_PREC_SPLIT && precision != FG_PREC_TF32 && precision != FG_PREC_SPLIT_TF32)
    return set_error(FG_EINVAL, "fg_attention: unknown precision %d", precision);
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.out_lo = nullptr;
  a.qsb = int64_t(Hq) * T * D; a.qsh = int64_t(T) * D; a.qst = D;
  a.ksb = int64_t(Hkv) * S * D; a.ksh = int64_t(S) * D; a.kst = D;
  a.vsb = a.ksb; a.vsh = a.ksh; a.vst = D;
  a.osb = a.qsb; a.osh = a.qsh; a.ost = D;
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.T = T; a.S = S; a.D = D;
  a.klen = key_lengths;
  a.qlen = nullptr;
  a.window = window;
  a.scale = scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (attn_tc_supported(a)) {
    int* err = nullptr;
    FG_TRY(device_error_word(&err));
    const size_t need = attn_tc_workspace_bytes(B, T, S, Hq, Hkv, D);
    StreamScratch scratch(s);
    FG_TRY(scratch.alloc(need));
    FG_TRY(attention_tc(a, scratch.p, need, err, s));
  } else {
    FG_TRY(attention_simt(a, s));
  }
  return attention_masked_rows(a, s);
}

}  // extern "C"
