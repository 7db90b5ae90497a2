/*
 * fg_oracle.h — CPU restatement of the fiber/ai EmbeddingGemma encoder
 * path, used ONLY as test infrastructure: the checker in tests/, the
 * oracle leg of __graft_entry__.smoke(), and the cpu_baseline leg of
 * bench.py. Nothing in the product (ai_b200/) links or calls it.
 *
 * It restates, in plain C, the reference's algorithm (paths in the fiber/ai
 * repository):
 *   models/gemma/model.go:121-140, 206-222  transpose, (1+w) norms, pre-norm folds
 *   models/gemma/embed.go:160-240           encode (op order, folds, epilogues)
 *   models/gemma/embed.go:381-438, 472-475  pool, applyHead, rmsScale, l2normalize
 *   tensor/attention.go:33-42, 97-107       padding / window masks (−1e9, additive)
 *   internal/blas/attention.go:97-135       mask/scale into raw scores, max, exp, 1/Σ after P·V
 *   tensor/rope.go:36-87                    float64 tables stored as float32, rotate-half
 *   tensor/attention.go:312-337             rmsNormFused
 *   internal/kernel/math.go:117-143         tanh-GELU composition
 *   internal/kernel/generic.go:241-360      exp (Cephes-style, flush below −87) and tanh (Eigen rational)
 *
 * Two arithmetic modes:
 *   ORC_F64: every activation in float64 (weights are the float32 values the
 *            reference's Load produces, folds included). The parity target.
 *   ORC_F32: the reference's own float32 arithmetic: sequential float32
 *            accumulation, the reference's exp and tanh polynomials. Its
 *            distance from ORC_F64 is the reference's own rounding noise.
 */
#ifndef FG_ORACLE_H
#define FG_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_F64 0
#define ORC_F32 1
#define ORC_MAX_DENSE 4

typedef struct {
  int hidden, ffn, layers, heads, kv_heads, head_dim, vocab;
  int window;           /* Config.window() bound; 0 = none */
  float eps;            /* rms_norm_eps */
  float attn_scale;     /* 1/sqrt(query_pre_attn_scalar) */
  const int* sliding;   /* [layers] */
  const double* rope_base; /* [layers] */
  int num_dense;
  int dense_in[ORC_MAX_DENSE], dense_out[ORC_MAX_DENSE], dense_tanh[ORC_MAX_DENSE];
  int l2;
} orc_config;

/* Raw weights as stored (projections [out, in]; norm weights w, not 1+w). */
typedef struct {
  const float* embed; /* [vocab, hidden] */
  const float* const* in_norm;
  const float* const* post_attn_norm;
  const float* const* pre_ffn_norm;
  const float* const* post_ffn_norm;
  const float* const* q_norm;
  const float* const* k_norm;
  const float* const* wq;
  const float* const* wk;
  const float* const* wv;
  const float* const* wo;
  const float* const* wgate;
  const float* const* wup;
  const float* const* wdown;
  const float* final_norm;
  const float* dense[ORC_MAX_DENSE]; /* [out, in] */
} orc_weights;

/* embedBatch (embed.go:118-157) on an already padded batch: ids [B*T]
 * (positions ≥ lengths[b] are replaced by the pad id 0, as embedBatch
 * pads), out [B, dim]. threads ≤ 0: all OpenMP threads. Returns 0 or -1. */
int orc_embed(const orc_config* cfg, const orc_weights* w, const int32_t* ids,
              const int32_t* lengths, int B, int T, int dim, int mode, int threads, float* out);

/* ---- op-level restatements (for known-answer tests) ---- */
/* out[m,n] = epilogue(x[m,k] · w[k,n]) in the given mode; epilogue order
 * bias → row_scale → act (0 none, 1 relu, 2 gelu) → mul → residual. */
void orc_matmul_fused(const float* x, const float* w, int m, int k, int n, const float* bias,
                      const float* row_scale, int act, const float* mul, const float* residual,
                      int mode, float* out);
/* AttentionScaled with an explicit additive mask [T, S] (or NULL) for one
 * head: q [T,D], k/v [S,D]; the reference's AttentionBlock arithmetic. */
void orc_attention_head(const float* q, const float* k, const float* v, const float* mask, int T,
                        int S, int D, float scale, int mode, float* out);
void orc_rmsnorm(const float* x, int rows, int n, const float* g, float eps, int mode, float* out);
void orc_rope(const float* x, int rows, int T, int D, double base, const int32_t* positions,
              float* out);
void orc_window_mask(int n, int w, float* out);   /* [n, n] */
void orc_padding_mask(const int32_t* lengths, int b, int n, float* out); /* [b, n] */
void orc_exp_ref(const float* x, int n, float* out);   /* reference float32 exp */
void orc_tanh_ref(const float* x, int n, float* out);  /* reference float32 tanh */
void orc_gelu_ref(const float* x, int n, float* out);  /* reference float32 GELU */

/* Float32-mode kernels: 1 (default) = the packed AVX-512 GEMM and the
 * 16-keys-at-a-time attention scores; 0 = the simple loops. Both give the
 * same results bit for bit (same fused multiply-add chains in the same
 * order); the switch exists for the test that checks it. */
void orc_set_fast_kernels(int on);

#ifdef __cplusplus
}
#endif

#endif
