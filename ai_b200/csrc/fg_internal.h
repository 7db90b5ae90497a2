// Host-side internals shared by the library's translation units: status
// codes, the thread-local last-error message, CUDA error checks, and the
// launch entry points of each kernel family.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/fgemma.h"

namespace fg {

// Records a formatted message as this thread's last error and returns code.
int set_error(int code, const char* fmt, ...);
void clear_error();
const char* last_error();

#define FG_CUDA_TRY(expr)                                                              \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return ::fg::set_error(FG_ECUDA, "%s failed: %s (%s:%d)", #expr,                 \
                             cudaGetErrorString(e_), __FILE__, __LINE__);              \
  } while (0)

#define FG_TRY(expr)          \
  do {                        \
    int rc_ = (expr);         \
    if (rc_ != FG_OK) return rc_; \
  } while (0)

// Number of SMs of the current device (cached per device).
int sm_count();

// Status block of the current device (error word, then the pipeline-wait
// limit; fg_ptx.cuh DeviceStatus); kernels record bounded-wait timeouts
// there. check_device_error_word() synchronises the device and turns a
// recorded timeout into FG_ETIMEOUT, resetting the word.
int device_error_word(int** out);
int check_device_error_word();
// Registers another status block of device `dev` (the no-allocation entry
// point's static one) for check_device_error_word and the wait limit.
int register_status_block(int dev, int* block);
// Sets device `dev`'s pipeline-wait limit in every status block it has.
int set_wait_limit(int dev, unsigned long long ns);

// The model's sequence cap (fg_config.max_tokens), for callers that split a
// batch before handing it to fg_embed_many.
int model_max_tokens(const fg_model* m);

// Stream-ordered scratch from the library's per-device pool (kept
// reserved between calls); freed back to the pool on the same stream.
int scratch_alloc(void** p, size_t bytes, cudaStream_t s);
void scratch_free(void* p, cudaStream_t s);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// libcuda link dependency); resolved once.
int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn);

// Internal activation code beyond the public FG_ACT_*: tanh (Dense head
// layers with a Tanh activation, models/gemma/model.go:297-303).
constexpr int kActTanh = 3;

// ------------------------------------------------------------------ GEMM
// C[M, Nout] = epilogue(A · Bᵀ) with A [M, K] and B [Nb, K], both row-major
// (K contiguous), on the tcgen05 tensor cores in TF32 with FP32 accumulation.
// Split-TF32: when A_lo / B_lo are given, the passes A·B, A·B_lo and A_lo·B
// are accumulated into the same TMEM tile (the A_lo·B_lo term, ~2^-22 of the
// product, is dropped). A plain-TF32 product passes neither.
struct GemmEpilogue {
  float* out = nullptr;          // [M, Nout]
  int64_t ldo = 0;
  float* out_lo = nullptr;       // optional split-TF32 low part of out
  int64_t ldo_lo = 0;
  const float* rowscale = nullptr;  // [M]
  const float* bias = nullptr;      // [Nout]
  const float* mul = nullptr;       // [M, Nout]
  int64_t ldm = 0;
  const float* residual = nullptr;  // [M, Nout]
  int64_t ldr = 0;
  int act = 0;                      // FG_ACT_*
  int geglu = 0;  // B rows interleaved per 128: gate rows then up rows; out = GELU(rs·g)·(rs·u)
  // gated product only: instead of `out`, the next product's split-fp16 A
  // operand — out·2^out16_exp cut into fp16 hi (top 11 significant bits)
  // and lo (the rounded remainder), [M, Nout] each, 16-byte aligned rows
  uint16_t* out16 = nullptr;
  uint16_t* out16_lo = nullptr;
  int out16_exp = 0;

  // QKV projection → attention operands (BN = 256 = head_dim, so N-tile tn
  // is head tn of q | k | v). For q and k heads: rs·acc, per-head RMSNorm
  // with gains (1+w), rotate-half RoPE at position row % T, written as bf16
  // hi/lo; for v heads: rs·acc written transposed as bf16 hi/lo
  // vt[(b·Hkv + hk)·256 + d][t]. `out` is unused in this mode.
  int qkv_attn = 0;
  int vnorm = 0;  // v heads RMS-normalised (weight-free, EmbeddingGemma 2) before their split
  int Hq = 0, Hkv = 0, T = 0;
  const float* qgain = nullptr;
  const float* kgain = nullptr;
  float eps = 0.f;
  // RoPE factors, position-minor with cos and sin side by side: entry
  // (frequency i, position t) at i·rope_ld + t holds (cos, sin)
  const float2* rope_cs = nullptr;
  int64_t rope_ld = 0;  // >= T
  void* q_hi = nullptr;  // bf16 [M, Hq·256]
  void* q_lo = nullptr;
  void* k_hi = nullptr;  // bf16 [M, Hkv·256]
  void* k_lo = nullptr;
  void* vt_hi = nullptr;  // bf16 [B·Hkv·256, ldt]
  void* vt_lo = nullptr;
  int64_t ldt = 0;
};

struct GemmArgs {
  int M = 0, Nb = 0, K = 0;      // Nb = rows of B (= 2·Nout for geglu)
  const float* A = nullptr;
  const float* A_lo = nullptr;
  int64_t lda = 0;
  const float* B = nullptr;
  const float* B_lo = nullptr;
  int64_t ldb = 0;
  // Split-TF32 without a stored A_lo: the kernel computes A's low part in
  // shared memory from the A tile (A is read from memory once).
  bool a_lo_smem = false;
  // Split-fp16 (with a_lo_smem, M >= 256): B16 = the fp16 bits of B·2^b_exp,
  // exact; A's rows are scaled by 2^e_r (a_exp, or from the epilogue's
  // row scales a_rs / epi.rowscale, 1/sqrt(mean(a²) + eps), when a_exp_rs)
  // so that |A|·2^e_r < 2^14. The products are
  // A_hi·B + A_lo·B in kind::f16; the epilogue undoes the scales exactly.
  const uint16_t* B16 = nullptr;
  // B without an exact fp16 form: B16 its high part, B16_lo = fp16(B·2^b_exp
  // − B16) its low part (the product adds the A_hi·B_lo pass)
  const uint16_t* B16_lo = nullptr;
  int b_exp = 0;
  const int* b_exp_dev = nullptr;  // b_exp in device memory (computed there), overriding b_exp
  int a_exp = 0;
  int a_exp_rs = 0;
  const float* a_rs = nullptr;  // row scales behind a_exp_rs (null: epi.rowscale)
  // Split-fp16 with the pre-norm gain on A: B16 holds the unfolded weight and
  // the converters multiply A's column k by a_gain[k] (|a_gain| <= a_gain_max;
  // K a multiple of 32), the product of a fold W·diag(g) moved to A's side.
  const float* a_gain = nullptr;
  float a_gain_max = 1.f;
  // Split-fp16 with A's two fp16 parts already in memory ([M, lda] each),
  // written by A's producer as the converters would make them: A·2^e_r
  // (times a column gain, whose maximum a_bound_gain enters the row bound
  // sqrt(K)·a_bound_gain/rs) cut into its top 11 significant bits and the
  // rounded remainder (a_exp / a_exp_rs give e_r as above).
  const uint16_t* A16 = nullptr;
  const uint16_t* A16_lo = nullptr;
  float a_bound_gain = 0.f;
  GemmEpilogue epi;
};

int gemm_tn(const GemmArgs& g, int* dev_err, cudaStream_t stream);
// Whether an M-row product can take the split-fp16 pair kernel (CTA pairs
// enabled, M >= 256), the only kernel that reads B16 without B.
bool gemm_h16_applies(int M);

// The op-level product (fg_matmul, fg_matmul_noalloc): its scratch plan
// and its run on a given scratch pointer of plan.total() bytes (fg_ops.cu).
struct MatmulPlan {
  bool a_direct, b_direct, split;
  bool h16;  // split-fp16: B as fp16 hi/lo parts, A's parts made by the converters
  int64_t kp, ldb, kp16;
  size_t a_bytes, bt_bytes, blo_bytes, b16_bytes, rs_bytes, misc_bytes;
  size_t total() const { return a_bytes + bt_bytes + blo_bytes + b16_bytes + rs_bytes + misc_bytes; }
};
MatmulPlan plan_matmul(int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx, const float* w,
                       int64_t ldw, int w_transposed, int precision);
int matmul_run(const MatmulPlan& p, int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx,
               const float* w, int64_t ldw, int w_transposed, float* out, int64_t ldo,
               const fg_epilogue* epi, void* scratch, int* err, cudaStream_t s);

// fp16 parts of a row-major [rows, cols] fp32 matrix (leading dimension
// ld) under one power-of-two scale 2^t chosen on the device from its
// largest magnitude (max·2^t < 2^14): hi = the top 11 significant bits of
// x·2^t, lo = fp16(x·2^t − hi), both [rows, ldo]; t goes to *exp_out.
// scratch_max: one device word this call clears and uses.
int split_f16_parts(const float* x, int64_t ld, int64_t rows, int64_t cols, uint16_t* hi, uint16_t* lo,
                    int64_t ldo, unsigned* scratch_max, int* exp_out, cudaStream_t stream);
// Row scales rs[r] = 1/sqrt(Σ_c x[r, c]² / cols), finite for zero rows: the
// split-fp16 converters' exponent bound (max|x_r| ≤ sqrt(cols)/rs[r]).
int row_inv_rms(const float* x, int64_t ld, int64_t rows, int64_t cols, float* rs, cudaStream_t stream);

// Elementwise split of n floats into TF32 high and exact low parts.
// *any_lo_nonzero (device int, optional) is set to 1 when some low part is non-zero.
int split_tf32(const float* x, float* hi, float* lo, int64_t n, int* any_lo_nonzero,
               cudaStream_t stream);
// dst[c, r] = src[r, c] for a rows×cols row-major src with leading dimension lds.
int transpose_f32(const float* src, int64_t lds, int64_t rows, int64_t cols, float* dst,
                  int64_t ldd, cudaStream_t stream);

}  // namespace fg
