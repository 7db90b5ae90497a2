// Launch wrappers of the memory-bound encoder kernels and the attention
// kernel (definitions in fg_elementwise.cu and fg_attention.cu).
#pragma once

#include "fg_internal.h"

namespace fg {

// Embedding gather with √hidden scaling (embed.go:175-176) and the first
// layer's folded pre-norm factor rowscale = 1/√(Σx²/n + eps)
// (matmul_fused.go:125-143, embed.go:432-438). ids/lengths are [B·T]/[B];
// positions at or past max(len, 1) are written as zeros; a length-0
// sequence embeds the pad id 0 at position 0. The table is fp32, or bf16
// (`table_bf16`, used when non-null) widened exactly as it is read
// (safetensors/convert.go:31-38 widens the same bits once at load).
int embed_gather(const float* table, const uint16_t* table_bf16, int64_t vocab, const int32_t* ids,
                 const int32_t* lengths, int B, int T, int hidden, float emb_scale, float eps, float* x,
                 float* x_lo, float* rowscale, int* dev_err, cudaStream_t s);

// Per-head RMSNorm of q and k with their gains (attention.go:292-337), then
// rotate-half RoPE with the layer's cos/sin tables [T, D/2] (rope.go:66-87),
// in place on the token-major qkv buffer [B·T, (Hq+2·Hkv)·D]; v untouched.
// Optional lo buffer (same layout) receives split-TF32 low parts of q, k, v.
int qk_norm_rope(float* qkv, float* qkv_lo, int64_t rows, int Hq, int Hkv, int D,
                 const float* qgain, const float* kgain, const float* vgain, float eps,
                 const float* cos_t, const float* sin_t, int T, cudaStream_t s);

// The next product's split-fp16 A operand written by its producer: row r
// of A·2^e_r (times the column gain when given), e_r = 13 −
// ilogb(norm_k / rs_r) clamped to ±60 from the row's RMS scale rs_r,
// cut into its top 11 significant bits (hi) and the rounded remainder
// (lo), fp16 [rows, n] each — the parts the GEMM's converters would make.
struct Split16Out {
  uint16_t* hi;
  uint16_t* lo;
  const float* gain;  // [n] or null
  float norm_k;       // sqrt(n) · max|gain| (sqrt(n) without a gain)
};

// x ← x + RMSNorm(o, gain) (embed.go:216-220, 231-235), then the next
// pre-norm factor rowscale = 1/√(Σx²/n + eps). parts (optional) receives
// the new x's split-fp16 operand for the next product. x_new is (x +
// RMSNorm(o, gain))·scalar (EmbeddingGemma 2's layer scalar,
// embed.go:370-371; 1 = plain residual). When final_gain is given, x is
// replaced by RMSNorm(x_new, final_gain) instead (embed.go:237) and
// rowscale/parts are not written.
int residual_postnorm(float* x, const Split16Out* parts, const float* o, const float* gain, float eps,
                      float* rowscale, const float* final_gain, int64_t rows, int n,
                      cudaStream_t s, float scalar = 1.0f);

// pooled[b] = mean over t < max(len_b, 1) of h[b, t] (embed.go:381-404);
// pooled_lo (optional) gets its split-TF32 low part.
int mean_pool(const float* h, const int32_t* lengths, int B, int T, int n, float* pooled,
              float* pooled_lo, cudaStream_t s);

// out[b, :dim] = x[b, :dim] / √(Σ x² + 1e-12) (embed.go:472-475), or a copy
// of the first dim columns when l2 == 0.
int l2_normalize(const float* x, int64_t ldx, int B, int dim, int l2, float* out,
                 cudaStream_t s);

// Row sums of squares and RMSNorm for the op-level API.
int row_sum_squares(const float* x, int64_t rows, int64_t n, int64_t ldx, float* out,
                    cudaStream_t s);
int rmsnorm(const float* x, int64_t rows, int64_t n, const float* g, float eps, float* out,
            cudaStream_t s);
int rope(const float* x, int64_t rows, int T, int D, const float* cos_t, const float* sin_t,
         float* out, cudaStream_t s);

// Split a strided [rows, cols] matrix into TF32 high (truncated) and exact
// low parts with leading dimension ldd; hi may be a plain copy when
// truncate_hi == 0; lo may be null.
int split_copy_2d(const float* src, int64_t lds, int64_t rows, int64_t cols, float* hi,
                  float* lo, int64_t ldd, int truncate_hi, cudaStream_t s);

// Attention over strided q/k/v/out (element offsets b·sb + h·sh + t·st, d
// contiguous): softmax(scale·q·kᵀ, masked)·v where key j is visible to query
// i of batch b when j < klen[b] (klen null: S) and, if window > 0,
// |i − j| < window. Query rows i ≥ qlen[b] (qlen null: T) are written as 0.
struct AttnArgs {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  float* out_lo;  // optional split-TF32 low part of out (same strides)
  int64_t qsb, qsh, qst;
  int64_t ksb, ksh, kst;
  int64_t vsb, vsh, vst;
  int64_t osb, osh, ost;
  int B, Hq, Hkv, T, S, D;
  const int32_t* klen;
  const int32_t* qlen;
  int window;
  float scale;
  // tensor-core kernel only: instead of `out`, the next product's split-fp16
  // A operand — out·2^out16_exp cut into fp16 hi (top 11 significant bits)
  // and lo (the rounded remainder), laid out like `out` (row stride ost)
  uint16_t* out16 = nullptr;
  uint16_t* out16_lo = nullptr;
  int out16_exp = 0;
};
int attention_simt(const AttnArgs& a, cudaStream_t s);

// The same attention on the tcgen05 tensor cores (head_dim 256 or 512,
// split-bf16 operands); ws must hold attn_tc_workspace_bytes() for the
// shapes and head dimension D.
size_t attn_tc_workspace_bytes(int B, int T, int S, int Hq, int Hkv, int D = 256);
bool attn_tc_supported(const AttnArgs& a);
int attention_tc(const AttnArgs& a, void* ws, size_t ws_bytes, int* err, cudaStream_t s);
// The split-bf16 operands as the tensor-core kernel reads them: q, k
// token-major [B·T, H·D], Vᵀ per sequence [B·Hkv·D, ldt keys].
struct AttnOperands {
  void* q_hi;
  void* q_lo;
  void* k_hi;
  void* k_lo;
  void* vt_hi;
  void* vt_lo;
  int64_t ldt;
};
// Carves ws (attn_tc_workspace_bytes) into the operand buffers.
int attn_tc_carve(void* ws, int B, int T, int S, int Hq, int Hkv, AttnOperands* o, int D = 256);
// Attention on operands already split (e.g. by the QKV GEMM's epilogue);
// a's q/k/v pointers are not read.
int attention_tc_operands(const AttnArgs& a, const AttnOperands& o, int* err, cudaStream_t s);
// Rewrites the rows that have no visible key with the reference's result for
// them: the mean of the values of the keys hidden by the fewest −1e9 masks.
int attention_masked_rows(const AttnArgs& a, cudaStream_t s);

}  // namespace fg
