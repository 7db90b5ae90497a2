/*
 * fg_oracle.c — CPU restatement of the fiber/ai EmbeddingGemma encoder
 * path. TEST INFRASTRUCTURE ONLY: the checker the parity tests compare the
 * CUDA library against, and the timed CPU baseline of bench.py. The
 * product (ai_b200/, libfgemma.so) never links or calls it.
 *
 * Parity pins: the op-level functions reproduce the reference's own
 * known-answer tests (tests/test_oracle_*.py); the whole model is checked
 * against an independent implementation of the same architecture
 * (Hugging Face transformers Gemma3TextModel, bidirectional), see
 * tests/golden/make_golden.py.
 */
#include "fg_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* The reference's float32 exp (internal/kernel/generic.go:241-307): a
 * Cephes-style exp — round x·log2(e) to an integer n with the 1.5·2^23
 * trick, reduce r = x − n·ln2 in two parts, a degree-5 polynomial in r,
 * then scale by 2^n through the exponent bits; below −87 the result is 0,
 * above 88.376 it is clamped. Restated from the published method. */
static float ref_expf(float v) {
  const float log2e = 1.44269504088896341f, magic = 12582912.0f;
  const float ln2hi = 0.693359375f, ln2lo = -2.12194440e-4f;
  if (v < -87.0f) return 0.0f;
  if (v > 88.3762626647949f) v = 88.3762626647949f;
  const float t = v * log2e + magic;
  const float nf = t - magic;
  float r = v - nf * ln2hi;
  r -= nf * ln2lo;
  float p = 1.9875691500e-4f;
  p = p * r + 1.3981999507e-3f;
  p = p * r + 8.3334519073e-3f;
  p = p * r + 4.1665795894e-2f;
  p = p * r + 1.6666665459e-1f;
  p = p * r + 5.0000001201e-1f;
  p = p * r * r + r + 1.0f;
  uint32_t tb, pb;
  memcpy(&tb, &t, 4);
  memcpy(&pb, &p, 4);
  const int32_t e = (int32_t)tb - 0x4B400000;
  pb += (uint32_t)(e << 23);
  float z;
  memcpy(&z, &pb, 4);
  return z;
}

/* Eigen's float tanh (the reference's genericTanh, generic.go:309-360):
 * x itself below 4e-4, ±1 from |x| ≥ 9, else an odd degree-13 over even
 * degree-6 rational after clamping to ±7.99881. */
static float ref_tanhf(float v) {
  if (v > -0.0004f && v < 0.0004f) return v;
  if (v >= 9.0f) return 1.0f;
  if (v <= -9.0f) return -1.0f;
  const float clamp = 7.99881172180175781f;
  v = v < -clamp ? -clamp : (v > clamp ? clamp : v);
  const float v2 = v * v;
  float p = -2.76076847742355e-16f;
  p = p * v2 + 2.00018790482477e-13f;
  p = p * v2 + -8.60467152213735e-11f;
  p = p * v2 + 5.12229709037114e-08f;
  p = p * v2 + 1.48572235717979e-05f;
  p = p * v2 + 6.37261928875436e-04f;
  p = p * v2 + 4.89352455891786e-03f;
  p *= v;
  float q = 1.19825839466702e-06f;
  q = q * v2 + 1.18534705686654e-04f;
  q = q * v2 + 2.26843463243900e-03f;
  q = q * v2 + 4.89352518554385e-03f;
  return p / q;
}

/* GELU composed from the vector kernels (internal/kernel/math.go:122-143). */
static float ref_gelu(float x) {
  float z = x * x;
  z = z * x;
  z = z * 0.044715f;
  z = x + z;
  z = z * 0.7978845608028654f;
  z = ref_tanhf(z);
  z = z + 1.0f;
  z = z * x;
  return z * 0.5f;
}

/* ------------------------------------------------------------------ */
/* Weights as the reference's Load leaves them: projections transposed to
 * [in, out] (model.go:121-127), norms as 1 + w (model.go:131-140), q/k/v
 * and gate/up scaled row-wise by their pre-norm gain (model.go:206-222),
 * all in float32; RoPE tables per layer in float64 stored as float32
 * (rope.go:36-50). */
typedef struct {
  float *wq, *wk, *wv, *wo, *wgate, *wup, *wdown;
  float *qgain, *kgain, *post_attn, *post_ffn;
  float *cos_t, *sin_t;
} folded_layer;

typedef struct {
  const float* embed;
  int hidden;
  folded_layer* layer;
  int layers;
  float* final_gain;
  float* dense[ORC_MAX_DENSE];
} folded;

static const float* c_row(const float* m, int r, int n) { return m + (size_t)r * n; }

static float* transpose_fold(const float* w, int out, int in, const float* norm) {
  float* t = (float*)malloc((size_t)out * in * sizeof(float));
  for (int o = 0; o < out; ++o)
    for (int i = 0; i < in; ++i) {
      float v = w[(size_t)o * in + i];
      if (norm) v = v * (norm[i] + 1.0f);
      t[(size_t)i * out + o] = v;
    }
  return t;
}

static float* plus_one(const float* w, int n) {
  float* g = (float*)malloc((size_t)n * sizeof(float));
  for (int i = 0; i < n; ++i) g[i] = w[i] + 1.0f;
  return g;
}

static void rope_tables(double base, int T, int D, const int32_t* positions, float** cs, float** sn) {
  const int half = D / 2;
  *cs = (float*)malloc((size_t)T * half * sizeof(float));
  *sn = (float*)malloc((size_t)T * half * sizeof(float));
  double* inv = (double*)malloc((size_t)half * sizeof(double));
  for (int i = 0; i < half; ++i) inv[i] = pow(base, -(double)(2 * i) / (double)D);
  for (int t = 0; t < T; ++t) {
    const double p = (double)(positions ? positions[t] : t);
    for (int i = 0; i < half; ++i) {
      const double a = p * inv[i];
      (*cs)[(size_t)t * half + i] = (float)cos(a);
      (*sn)[(size_t)t * half + i] = (float)sin(a);
    }
  }
  free(inv);
}

static void fold(const orc_config* c, const orc_weights* w, int T, folded* f) {
  const int H = c->hidden, D = c->head_dim;
  f->embed = w->embed;
  f->hidden = H;
  f->layers = c->layers;
  f->layer = (folded_layer*)calloc((size_t)c->layers, sizeof(folded_layer));
  for (int l = 0; l < c->layers; ++l) {
    folded_layer* L = &f->layer[l];
    L->wq = transpose_fold(w->wq[l], c->heads * D, H, w->in_norm[l]);
    L->wk = transpose_fold(w->wk[l], c->kv_heads * D, H, w->in_norm[l]);
    L->wv = transpose_fold(w->wv[l], c->kv_heads * D, H, w->in_norm[l]);
    L->wo = transpose_fold(w->wo[l], H, c->heads * D, NULL);
    L->wgate = transpose_fold(w->wgate[l], c->ffn, H, w->pre_ffn_norm[l]);
    L->wup = transpose_fold(w->wup[l], c->ffn, H, w->pre_ffn_norm[l]);
    L->wdown = transpose_fold(w->wdown[l], H, c->ffn, NULL);
    L->qgain = plus_one(w->q_norm[l], D);
    L->kgain = plus_one(w->k_norm[l], D);
    L->post_attn = plus_one(w->post_attn_norm[l], H);
    L->post_ffn = plus_one(w->post_ffn_norm[l], H);
    rope_tables(c->rope_base[l], T, D, NULL, &L->cos_t, &L->sin_t);
  }
  f->final_gain = plus_one(w->final_norm, H);
  for (int j = 0; j < c->num_dense; ++j)
    f->dense[j] = transpose_fold(w->dense[j], c->dense_out[j], c->dense_in[j], NULL);
}

static void unfold(folded* f, int ndense) {
  for (int l = 0; l < f->layers; ++l) {
    folded_layer* L = &f->layer[l];
    free(L->wq); free(L->wk); free(L->wv); free(L->wo); free(L->wgate); free(L->wup);
    free(L->wdown); free(L->qgain); free(L->kgain); free(L->post_attn); free(L->post_ffn);
    free(L->cos_t); free(L->sin_t);
  }
  free(f->layer);
  free(f->final_gain);
  for (int j = 0; j < ndense; ++j) free(f->dense[j]);
}

/* ------------------------------------------------------------------ */
/* ------------------------------------------------------------------ */
/* Packed AVX-512 kernels of the float32 mode, shaped like the reference's
 * SGEMM (internal/blas/gemm.go:562-702 driving the 14×32 micro-kernel of
 * internal/kernel/kernel_avx512_amd64.s): W packed once per call into
 * 32-column panels [k][32], A packed per 14-row block as [k][14], and a
 * 14×32 register tile of 28 accumulators. Every C element is still one
 * sequential chain of fused multiply-adds over k starting from 0, so the
 * results are bit for bit those of the simple loops (orc_set_fast_kernels(0)
 * selects those; tests compare the two). The attention scores go 16 keys
 * at a time over a transposed K, each lane one key's sequential chain over
 * the head dimension. */
#include <immintrin.h>

static int g_fast = 1;
void orc_set_fast_kernels(int on) { g_fast = on != 0; }

#define ORC_MR 14
#define ORC_NR 32

static void gemm_f32_packed(const float* A, const float* W, int m, int k, int n, float* C) {
  const int np = (n + ORC_NR - 1) / ORC_NR, mb = (m + ORC_MR - 1) / ORC_MR;
  float* Wp = (float*)aligned_alloc(64, (size_t)np * k * ORC_NR * sizeof(float) + 64);
  float* Ap = (float*)aligned_alloc(64, (size_t)mb * k * ORC_MR * sizeof(float) + 64);
  if (!Wp || !Ap) {
    free(Wp);
    free(Ap);
    return;
  }
#pragma omp parallel for schedule(static)
  for (int p = 0; p < np; ++p) {
    const int n0 = p * ORC_NR, cols = (n - n0) < ORC_NR ? (n - n0) : ORC_NR;
    float* dst = Wp + (size_t)p * k * ORC_NR;
    for (int kk = 0; kk < k; ++kk) {
      const float* src = W + (size_t)kk * n + n0;
      for (int j = 0; j < ORC_NR; ++j) dst[(size_t)kk * ORC_NR + j] = j < cols ? src[j] : 0.0f;
    }
  }
#pragma omp parallel for schedule(static)
  for (int b = 0; b < mb; ++b) {
    const int i0 = b * ORC_MR, rows = (m - i0) < ORC_MR ? (m - i0) : ORC_MR;
    float* dst = Ap + (size_t)b * k * ORC_MR;
    for (int kk = 0; kk < k; ++kk)
      for (int r = 0; r < ORC_MR; ++r) dst[(size_t)kk * ORC_MR + r] = r < rows ? A[(size_t)(i0 + r) * k + kk] : 0.0f;
  }
  /* tasks of 8 row blocks × 4 panels: both operands' packed slices stay in L2 */
  const int rb = 8, pb = 4;
  const int tr = (mb + rb - 1) / rb, tp = (np + pb - 1) / pb;
#pragma omp parallel for schedule(dynamic, 1)
  for (int task = 0; task < tr * tp; ++task) {
    const int b0 = (task / tp) * rb, p0 = (task % tp) * pb;
    for (int p = p0; p < p0 + pb && p < np; ++p) {
      const float* wp = Wp + (size_t)p * k * ORC_NR;
      const int n0 = p * ORC_NR, cols = (n - n0) < ORC_NR ? (n - n0) : ORC_NR;
      for (int b = b0; b < b0 + rb && b < mb; ++b) {
        const float* ap = Ap + (size_t)b * k * ORC_MR;
        __m512 c0[ORC_MR], c1[ORC_MR];
        for (int r = 0; r < ORC_MR; ++r) {
          c0[r] = _mm512_setzero_ps();
          c1[r] = _mm512_setzero_ps();
        }
        for (int kk = 0; kk < k; ++kk) {
          const __m512 w0 = _mm512_load_ps(wp + (size_t)kk * ORC_NR);
          const __m512 w1 = _mm512_load_ps(wp + (size_t)kk * ORC_NR + 16);
          const float* a = ap + (size_t)kk * ORC_MR;
#pragma GCC unroll 14
          for (int r = 0; r < ORC_MR; ++r) {
            const __m512 av = _mm512_set1_ps(a[r]);
            c0[r] = _mm512_fmadd_ps(av, w0, c0[r]);
            c1[r] = _mm512_fmadd_ps(av, w1, c1[r]);
          }
        }
        const int i0 = b * ORC_MR, rows = (m - i0) < ORC_MR ? (m - i0) : ORC_MR;
        for (int r = 0; r < rows; ++r) {
          float* crow = C + (size_t)(i0 + r) * n + n0;
          if (cols == ORC_NR) {
            _mm512_storeu_ps(crow, c0[r]);
            _mm512_storeu_ps(crow + 16, c1[r]);
          } else {
            float t[ORC_NR];
            _mm512_storeu_ps(t, c0[r]);
            _mm512_storeu_ps(t + 16, c1[r]);
            for (int j = 0; j < cols; ++j) crow[j] = t[j];
          }
        }
      }
    }
  }
  free(Wp);
  free(Ap);
}

/* s[j] = Σ_d q[d]·K[j][d], j < S, from KT [D][ldt] (K transposed), each
 * score a sequential chain of fused multiply-adds over d from 0. */
static void scores_f32_packed(const float* q, const float* KT, int S, int D, int ldt, float* s) {
  int j0 = 0;
  for (; j0 + 16 <= S; j0 += 16) {
    __m512 acc = _mm512_setzero_ps();
    for (int d = 0; d < D; ++d) acc = _mm512_fmadd_ps(_mm512_set1_ps(q[d]), _mm512_loadu_ps(KT + (size_t)d * ldt + j0), acc);
    _mm512_storeu_ps(s + j0, acc);
  }
  if (j0 < S) {
    const __mmask16 mk = (__mmask16)((1u << (S - j0)) - 1u);
    __m512 acc = _mm512_setzero_ps();
    for (int d = 0; d < D; ++d)
      acc = _mm512_fmadd_ps(_mm512_set1_ps(q[d]), _mm512_maskz_loadu_ps(mk, KT + (size_t)d * ldt + j0), acc);
    _mm512_mask_storeu_ps(s + j0, mk, acc);
  }
}

#define R double
#define SFX(name) name##_f64
#define MADD(a, b, c) fma((a), (b), (c))
#include "fg_oracle_impl.h"
#undef R
#undef SFX
#undef MADD

#define R float
#define SFX(name) name##_f32
#define MADD(a, b, c) fmaf((a), (b), (c))
#include "fg_oracle_impl.h"
#undef R
#undef SFX
#undef MADD

int orc_embed(const orc_config* cfg, const orc_weights* w, const int32_t* ids,
              const int32_t* lengths, int B, int T, int dim, int mode, int threads, float* out) {
  if (!cfg || !w || !ids || !lengths || !out || B < 0 || T <= 0 || dim <= 0) return -1;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  folded f;
  memset(&f, 0, sizeof(f));
  fold(cfg, w, T, &f);
  int rc = mode == ORC_F32 ? embed_f32(cfg, &f, ids, lengths, B, T, dim, out)
                           : embed_f64(cfg, &f, ids, lengths, B, T, dim, out);
  unfold(&f, cfg->num_dense);
  return rc;
}

/* ---- op-level restatements ---------------------------------------- */
void orc_matmul_fused(const float* x, const float* w, int m, int k, int n, const float* bias,
                      const float* row_scale, int act, const float* mul, const float* residual,
                      int mode, float* out) {
  if (mode == ORC_F32) {
    float* a = (float*)malloc((size_t)m * k * sizeof(float));
    float* c = (float*)malloc((size_t)m * n * sizeof(float));
    memcpy(a, x, (size_t)m * k * sizeof(float));
    gemm_f32(a, w, m, k, n, c);
    for (int i = 0; i < m; ++i)
      for (int j = 0; j < n; ++j) {
        float v = c[(size_t)i * n + j];
        if (bias) v += bias[j];
        if (row_scale) v *= row_scale[i];
        if (act == 1) v = v > 0 ? v : 0;
        if (act == 2) v = ref_gelu(v);
        if (mul) v *= mul[(size_t)i * n + j];
        if (residual) v += residual[(size_t)i * n + j];
        out[(size_t)i * n + j] = v;
      }
    free(a);
    free(c);
    return;
  }
  double* a = (double*)malloc((size_t)m * k * sizeof(double));
  double* c = (double*)malloc((size_t)m * n * sizeof(double));
  for (size_t e = 0; e < (size_t)m * k; ++e) a[e] = x[e];
  gemm_f64(a, w, m, k, n, c);
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) {
      double v = c[(size_t)i * n + j];
      if (bias) v += bias[j];
      if (row_scale) v *= row_scale[i];
      if (act == 1) v = v > 0 ? v : 0;
      if (act == 2) v = gelu_mode_f64(v);
      if (mul) v *= mul[(size_t)i * n + j];
      if (residual) v += residual[(size_t)i * n + j];
      out[(size_t)i * n + j] = (float)v;
    }
  free(a);
  free(c);
}

void orc_attention_head(const float* q, const float* k, const float* v, const float* mask, int T,
                        int S, int D, float scale, int mode, float* out) {
  if (mode == ORC_F32) {
    float* s = (float*)malloc((size_t)(S > 0 ? S : 1) * sizeof(float));
    for (int i = 0; i < T; ++i)
      attn_row_f32(q + (size_t)i * D, k, v, S, D, D, NULL, mask ? mask + (size_t)i * S : NULL,
                   scale, s, out + (size_t)i * D, NULL, 0);
    free(s);
    return;
  }
  double* qd = (double*)malloc((size_t)T * D * sizeof(double));
  double* kd = (double*)malloc((size_t)S * D * sizeof(double));
  double* vd = (double*)malloc((size_t)S * D * sizeof(double));
  double* s = (double*)malloc((size_t)(S > 0 ? S : 1) * sizeof(double));
  double* o = (double*)malloc((size_t)D * sizeof(double));
  for (size_t e = 0; e < (size_t)T * D; ++e) qd[e] = q[e];
  for (size_t e = 0; e < (size_t)S * D; ++e) kd[e] = k[e], vd[e] = v[e];
  for (int i = 0; i < T; ++i) {
    attn_row_f64(qd + (size_t)i * D, kd, vd, S, D, D, NULL, mask ? mask + (size_t)i * S : NULL,
                 scale, s, o, NULL, 0);
    for (int d = 0; d < D; ++d) out[(size_t)i * D + d] = (float)o[d];
  }
  free(qd); free(kd); free(vd); free(s); free(o);
}

void orc_rmsnorm(const float* x, int rows, int n, const float* g, float eps, int mode, float* out) {
  if (mode == ORC_F32) {
    float* t = (float*)malloc((size_t)rows * n * sizeof(float));
    memcpy(t, x, (size_t)rows * n * sizeof(float));
    rmsnorm_rows_f32(t, (size_t)rows, n, g, eps, t);
    memcpy(out, t, (size_t)rows * n * sizeof(float));
    free(t);
    return;
  }
  double* t = (double*)malloc((size_t)rows * n * sizeof(double));
  for (size_t e = 0; e < (size_t)rows * n; ++e) t[e] = x[e];
  rmsnorm_rows_f64(t, (size_t)rows, n, g, eps, t);
  for (size_t e = 0; e < (size_t)rows * n; ++e) out[e] = (float)t[e];
  free(t);
}

void orc_rope(const float* x, int rows, int T, int D, double base, const int32_t* positions,
              float* out) {
  float *cs, *sn;
  rope_tables(base, T, D, positions, &cs, &sn);
  const int half = D / 2;
  for (int r = 0; r < rows; ++r) {
    const int t = r % T;
    for (int i = 0; i < half; ++i) {
      const float x1 = x[(size_t)r * D + i], x2 = x[(size_t)r * D + i + half];
      const float c = cs[(size_t)t * half + i], s = sn[(size_t)t * half + i];
      out[(size_t)r * D + i] = x1 * c - x2 * s;
      out[(size_t)r * D + i + half] = x1 * s + x2 * c;
    }
  }
  free(cs);
  free(sn);
}

void orc_window_mask(int n, int w, float* out) {
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) out[(size_t)i * n + j] = (j - i >= w || i - j >= w) ? -1e9f : 0.0f;
}

void orc_padding_mask(const int32_t* lengths, int b, int n, float* out) {
  for (int i = 0; i < b; ++i)
    for (int j = 0; j < n; ++j) out[(size_t)i * n + j] = j >= (lengths[i] > 0 ? lengths[i] : 0) ? -1e9f : 0.0f;
}

void orc_exp_ref(const float* x, int n, float* out) {
  for (int i = 0; i < n; ++i) out[i] = ref_expf(x[i]);
}
void orc_tanh_ref(const float* x, int n, float* out) {
  for (int i = 0; i < n; ++i) out[i] = ref_tanhf(x[i]);
}
void orc_gelu_ref(const float* x, int n, float* out) {
  for (int i = 0; i < n; ++i) out[i] = ref_gelu(x[i]);
}
