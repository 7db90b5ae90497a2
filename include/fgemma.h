/*
 * fgemma.h — C ABI of the B200 (sm_100a) EmbeddingGemma encoder library.
 *
 * This is the drop-in boundary for the fiber/ai `models/gemma` encoder hot
 * path and the `tensor` operations it calls. Every entry point is plain C:
 * pointers, sizes and status codes, no C++ or torch types. Each function
 * returns FG_OK (0) or a negative FG_E* code and never aborts the process;
 * fg_last_error() returns the calling thread's last message.
 *
 * Reference interfaces replaced (paths inside the fiber/ai repository):
 *   models/gemma/model.go:76-232   gemma.Load (weights → fg_model_* below)
 *   models/gemma/embed.go:118-157  (*Model).embedBatch → fg_embed_ids
 *   models/gemma/embed.go:160-240  (*Model).encode     (inside fg_embed_ids)
 *   models/gemma/embed.go:381-475  pool / applyHead / l2normalize (inside fg_embed_ids)
 *   tensor/matmul.go:19            tensor.MatMul         → fg_matmul
 *   tensor/matmul_fused.go:40      tensor.MatMulFused    → fg_matmul with fg_epilogue
 *   tensor/matmul_fused.go:125     (*Tensor).RowSumSquares → fg_row_sum_squares
 *   tensor/attention.go:67         tensor.AttentionScaled (padding / window masks) → fg_attention
 *   tensor/attention.go:292        tensor.RMSNorm        → fg_rmsnorm
 *   tensor/rope.go:20              tensor.RoPE           → fg_rope
 *
 * Threading: a model is driven by one host thread at a time. Op-level calls
 * take device pointers and a CUDA stream (NULL = legacy default stream) and
 * are asynchronous on that stream unless stated otherwise.
 */
#ifndef FGEMMA_H
#define FGEMMA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FG_OK 0
#define FG_EINVAL (-1)   /* bad argument: shape, stride, alignment, name */
#define FG_ENOMEM (-2)   /* device or host allocation failed */
#define FG_ECUDA (-3)    /* a CUDA runtime/driver call failed */
#define FG_ETIMEOUT (-4) /* a bounded device wait gave up (kernel reported it) */
#define FG_ESTATE (-5)   /* call out of order (e.g. embed before finalize) */
#define FG_ENODEV (-6)   /* no usable sm_100 device */

/* ---- arithmetic modes -------------------------------------------------- */
/* FG_PREC_SPLIT (default): fp32-level products, the arithmetic chosen per
 * product. Products on SM pairs run split-fp16: A as two fp16 parts under
 * a power-of-two row scale; B as exact fp16 under a power-of-two scale
 * where it has such a form (bf16 checkpoint weights: 2 fp16 passes), else
 * as two fp16 parts (3 fp16 passes: A_hi·B_hi + A_hi·B_lo + A_lo·B_hi).
 * Smaller products run split TF32.
 * FG_PREC_SPLIT_TF32: every product as split TF32 (A·B + A·B_lo + A_lo·B,
 * up to 3 TF32 passes), the fp32-level mode without fp16 parts.
 * FG_PREC_TF32: one TF32 pass per product (about 1e-4 relative). */
#define FG_PREC_SPLIT 0
#define FG_PREC_TF32 1
#define FG_PREC_SPLIT_TF32 2

/* ---- activations: blas.Activation, internal/blas/gemm.go:270-274 -------- */
#define FG_ACT_NONE 0
#define FG_ACT_RELU 1
#define FG_ACT_GELU 2 /* tanh approximation, internal/kernel/math.go:117-143 */

/* ---- host weight dtypes: safetensors/convert.go:16-21 -------------------- */
#define FG_DT_F32 0
#define FG_DT_BF16 1
#define FG_DT_F16 2

/* tensor.Fused (tensor/matmul_fused.go:17-23): applied in the order
 * bias → row_scale → act → mul → residual (internal/blas/gemm.go:276-288).
 * NULL pointers are skipped. mul / residual are [m, n] with row strides. */
typedef struct fg_epilogue {
  const float* bias;      /* [n] */
  const float* row_scale; /* [m] */
  int act;                /* FG_ACT_* */
  const float* mul;       /* [m, n] */
  int64_t ldm;
  const float* residual;  /* [m, n] */
  int64_t ldr;
} fg_epilogue;

/* The Config fields encode() reads (models/gemma/config.go:19-37), with the
 * per-layer derivations already resolved by the caller:
 *   window       = Config.window()      (config.go:331-339); 0 = no sliding layers
 *   sliding[l]   = Config.isSliding(l)  (config.go:342)
 *   rope_base[l] = Config.ropeBase(l)   (config.go:346-362)
 *   attn_scale   = 1/sqrt(query_pre_attn_scalar)  (model.go:100)
 * Dense head layers follow modules.json (model.go:277-304). */
#define FG_MAX_DENSE 4
typedef struct fg_config {
  int hidden_size;
  int intermediate_size;
  int num_layers;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int vocab_size;
  int window;
  float rms_norm_eps;
  float attn_scale;
  int max_tokens;          /* sequence cap (model.go:98-109): ≤ 2048, ≤ 8192 for variant 2 */
  const int* sliding;      /* [num_layers] */
  const double* rope_base; /* [num_layers] */
  int num_dense;
  int dense_in[FG_MAX_DENSE];
  int dense_out[FG_MAX_DENSE];
  int dense_tanh[FG_MAX_DENSE];
  int l2_normalize;        /* Normalize module present (model.go:262-263, 305-306) */
  /* EmbeddingGemma 2's text tower (encode2, embed.go:247-377; config.go
   * 286-362): variant = 2, else 0. Its norms multiply by the stored weight
   * (no 1 + w, model.go:128-139); attn_scale is 1 (model.go:105-109);
   * window = sliding_window + 1 (config.go:331-339). */
  int variant;
  const int* layer_head_dim;  /* [num_layers] Config.headDim(l); NULL = head_dim everywhere */
  const int* layer_kv_heads;  /* [num_layers] Config.kvHeads(l); NULL = num_kv_heads */
  int ple_dim;                /* hidden_size_per_layer_input (variant 2) */
  int embedding_dim;          /* embedding_projection output width (variant 2) */
} fg_config;

typedef struct fg_model fg_model;

/* ---- library ----------------------------------------------------------- */
/* Number of CUDA devices of compute capability 10.x. */
int fg_device_count(void);
/* Last error message of the calling thread ("" when none). */
const char* fg_last_error(void);

/* Device memory helpers, so a caller without the CUDA runtime (a cgo
 * binding) can stage tensors. Synchronous. */
int fg_malloc(int device, int64_t bytes, void** out);
int fg_free(int device, void* ptr);
int fg_memcpy_h2d(int device, void* dst, const void* src, int64_t bytes);
int fg_memcpy_d2h(int device, void* dst, const void* src, int64_t bytes);
/* Waits for all work on `device`; returns FG_ETIMEOUT (and clears the
 * record) when a kernel's bounded wait gave up since the last check. */
int fg_synchronize(int device);
/* Limit, in nanoseconds, of every pipeline wait (mbarrier) inside the
 * library's kernels on `device`; 0 restores the default of 2 s. A wait that
 * runs out makes its kernel drain its own copies and MMAs, free its tensor
 * memory and return, and the next fg_synchronize / fg_model_check reports
 * FG_ETIMEOUT. Synchronises the device. No counterpart in the reference
 * (its CPU kernels never wait on hardware). */
int fg_set_wait_limit(int device, int64_t nanoseconds);

/* ---- model: gemma.Load + (*Model).embedBatch ---------------------------- */
/* Creates an empty model on `device` for the given configuration.
 * Replaces the allocation half of gemma.Load (models/gemma/model.go:76-104). */
int fg_model_create(const fg_config* cfg, int device, fg_model** out);

/* Hands one weight to the model, by its safetensors name without the
 * "model." / "language_model." prefixes (model.go:112-119), e.g.
 * "embed_tokens.weight", "layers.3.self_attn.q_proj.weight", "norm.weight";
 * the Dense head layers are "dense.<i>.linear.weight" ([out, in]).
 * data is host memory of the given dtype and shape ([out, in] for
 * projections, as stored); it is copied, the caller keeps ownership.
 * Replaces model.go:142-205 (get / transpose / norm). */
int fg_model_set_weight(fg_model* m, const char* name, int dtype, const int64_t* shape, int ndim,
                        const void* data);

/* Checks every weight is present, applies the (1+w) norm offset and folds
 * the pre-norms into the projections (model.go:131-140, 206-222), splits
 * the projections into TF32 high/low parts and uploads them.
 * max_batch_tokens sizes the device workspace (B·T of the largest call). */
int fg_model_finalize(fg_model* m, int64_t max_batch_tokens);

/* Device residency of the encoder's projection weights, chosen before
 * fg_model_finalize (no counterpart in the reference, whose TODO.md lists
 * "bf16 weight storage expanded during GEMM packing (halves the 1.2 GB)";
 * its bf16 widening is safetensors/convert.go:31-38).
 * FG_WEIGHTS_F32 (default): the gain-folded fp32 projections, their
 * split-TF32 low parts and their fp16 forms for split-fp16 stay resident.
 * FG_WEIGHTS_BF16: every bf16-exact projection stays resident in 2 bytes per
 * value — its fp16 form, read by the split-fp16 GEMM as it is, or bf16 —
 * beside its fp32 pre-norm gain; what a product needs in fp32 is widened,
 * folded and split into one layer's fp32 workspace on the stream just
 * before that layer's GEMMs — the same operands bit for bit, so the
 * embeddings are identical. A layer with a projection that is not
 * bf16-exact stays fp32. Returns FG_ESTATE after finalize. */
#define FG_WEIGHTS_F32 0
#define FG_WEIGHTS_BF16 1
int fg_model_set_weight_residency(fg_model* m, int mode);

/* Device bytes the model's weights occupy (embedding table, projections and
 * their low parts, gains, RoPE tables, the widening workspace). */
int64_t fg_model_weight_bytes(fg_model* m);

/* Embeds B sequences of ids, right-padded to T, and writes [B, dim] float
 * embeddings (mean-pooled, Dense head, Matryoshka-narrowed, L2-normalised)
 * in input order. Host buffers; synchronous. Same semantics as
 * (*Model).embedBatch (models/gemma/embed.go:118-157) after the ids are
 * padded: ids[b*T + t] for t < lengths[b] are read, padding is ignored.
 * lengths[b] may be 0 (pooled as one row, embed.go:386-389). */
int fg_embed_ids(fg_model* m, const int32_t* ids, const int32_t* lengths, int B, int T, int dim,
                 int precision, float* out);

/* (*Model).Embed (models/gemma/embed.go:15-80) after tokenisation, with the
 * host work overlapped with the GPU's. Sequence i is ids[offsets[i] ..
 * offsets[i+1]) (offsets has nseq + 1 entries), truncated to max_tokens
 * (embed.go:38-40; 0 or more than the model's limit = the model's limit).
 * The sequences are stably sorted by length (sortIndex, model.go:412) and
 * cut into greedy batches whose padded size max_len·count stays within
 * batch_tokens (embed.go:58-74; a longer single sequence runs alone), each
 * right-padded with id 0. While one batch runs on the GPU the next is
 * packed into pinned memory and copied in on a second stream, and the
 * previous batch's embeddings are copied out and placed. out is
 * [nseq, dim] in the caller's order. Synchronous. */
int fg_embed_many(fg_model* m, const int32_t* ids, const int64_t* offsets, int nseq, int max_tokens,
                  int64_t batch_tokens, int dim, int precision, float* out);

/* (*Model).Embed (models/gemma/embed.go:15-80) over several GPUs of one
 * process: models[r] (r < nmodels) are models holding the same weights,
 * normally one per GPU (fg_model_create on device r, the same
 * fg_model_set_weight calls, fg_model_finalize). The sequences (as for
 * fg_embed_many, truncated to max_tokens) are stably sorted by length and
 * cut into nmodels contiguous slices of about equal estimated GPU time
 * (fg_plan_split); slice r is embedded by fg_embed_many on models[r] on its
 * own host thread (the calling thread takes slice 0), and every embedding
 * lands in out [nseq, dim] in the caller's order. No collective is needed:
 * sequences never interact. Each slice's result is bitwise what
 * fg_embed_many gives for that slice alone. Synchronous; the first error of
 * any slice is returned, with the slice's model named in the message. */
int fg_embed_many_multi(fg_model* const* models, int nmodels, const int32_t* ids, const int64_t* offsets,
                        int nseq, int max_tokens, int64_t batch_tokens, int dim, int precision, float* out);

/* fg_embed_many_multi's split alone, on the host: lengths [nseq] → order
 * [nseq] (indices stably sorted by increasing length, as sortIndex,
 * models/gemma/model.go:412) and bounds [nparts + 1] (slice r is
 * order[bounds[r] .. bounds[r+1])), cut where the running cost reaches
 * r/nparts of the total. No counterpart in the reference (it embeds on one
 * process). */
int fg_plan_split(const int32_t* lengths, int nseq, int nparts, int32_t* order, int32_t* bounds);

/* The split's estimated GPU time of one sequence of `length` tokens, in
 * units of one token of a 512-token sequence (length 0 counts as 1). */
double fg_sequence_cost(int length);

/* fg_embed_many's batching alone, on the host (no device work): lengths
 * [nseq] → order [nseq] (indices stably sorted by length) and batch_end
 * [number of batches ≤ nseq] (each batch's end position in order). Returns
 * the number of batches, or a negative status. */
int fg_plan_batches(const int32_t* lengths, int nseq, int64_t batch_tokens, int32_t* order, int32_t* batch_end);

/* As fg_embed_ids with device buffers on the model's device, asynchronous
 * on `stream` (a cudaStream_t, NULL = default stream). Repeated calls with
 * the same B, T, dim, precision and buffers run the forward as a CUDA graph
 * (the first call runs it eagerly, the second captures it on a stream of
 * the model's and launches it on `stream`); the result is the same bit
 * for bit, and the graph reads the buffers' contents when it runs, so new
 * ids in the same buffer are what it embeds. While profiling is enabled
 * (fg_model_set_profiling) every call runs eagerly. */
int fg_embed_ids_device(fg_model* m, const int32_t* d_ids, const int32_t* d_lengths, int B, int T,
                        int dim, int precision, float* d_out, void* stream);

/* Reads back the device error word of the last device call and resets it
 * (FG_ETIMEOUT when a bounded wait gave up). Synchronises the model's device. */
int fg_model_check(fg_model* m);

void fg_model_destroy(fg_model* m);

/* Per-phase device timing of forwards, for measurement (no reference
 * counterpart; the reference's bench prints wall times, cmd/bench).
 * While enabled, every kernel launch of fg_embed_ids(_device) is bracketed
 * by CUDA events on its stream. fg_model_read_profile synchronises, writes
 * for each phase p < n the summed milliseconds, launches and algorithmic
 * work (FLOPs for GEMM/attention phases, bytes for memory-bound phases),
 * then clears the record. Launch counts are kept even when disabled. */
#define FG_PHASE_EMBED 0
#define FG_PHASE_GEMM_QKV 1
#define FG_PHASE_QK_NORM_ROPE 2
#define FG_PHASE_ATTENTION 3
#define FG_PHASE_GEMM_O 4
#define FG_PHASE_RESIDUAL 5
#define FG_PHASE_GEMM_GATE_UP 6
#define FG_PHASE_GEMM_DOWN 7
#define FG_PHASE_POOL_HEAD 8
#define FG_PHASE_WIDEN 9 /* bf16-resident projections widened per layer */
#define FG_NUM_PHASES 10
int fg_model_set_profiling(fg_model* m, int enable);
int fg_model_read_profile(fg_model* m, double* ms, int64_t* launches, double* work, int n);

/* ---- tensor operations (device pointers) ------------------------------- */
/* out[m, n] = epilogue(x[m, k] · w) — tensor.MatMul (tensor/matmul.go:19)
 * and tensor.MatMulFused (tensor/matmul_fused.go:40). w is [k, n] row-major
 * with leading dimension ldw, or, when w_transposed != 0, the transposed
 * view of an [n, k] row-major matrix (x · Wᵀ, the `w.T()` case). epi may be
 * NULL. x, and w as a transposed view, are read in place when 16-byte
 * aligned with row strides of whole 16-byte units; other layouts are copied
 * into stream-ordered scratch from a pool the library keeps per device
 * (memory it keeps reserved between calls). FG_PREC_SPLIT with m >= 256,
 * n > 128 and x read in place runs the three-pass split-fp16 product (B's
 * fp16 parts and A's row scales made per call on the device); other split
 * products, and FG_PREC_SPLIT_TF32, run A·B + A·B_lo + A_lo·B in TF32 with
 * B_lo computed per call and A's low part made in shared memory. */
int fg_matmul(int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx, const float* w,
              int64_t ldw, int w_transposed, float* out, int64_t ldo, const fg_epilogue* epi,
              int precision, void* stream);

/* fg_matmul for callers that cannot allocate device memory during a call:
 * a host whose own allocator has reserved the GPU's memory up front (a
 * cudaMalloc from inside the library would fail or fragment that pool), or
 * a latency-critical path that cannot take the implicit synchronisation of
 * cudaMalloc/cudaFree. No counterpart in the reference (its Go code
 * allocates host memory freely). Same arguments and results as fg_matmul;
 * the splitting/packing scratch lives in a fixed 32 MiB device array owned
 * by the library (held by every GPU that loads it, until exit), so calls
 * whose scratch would exceed 32 MiB are refused with FG_EINVAL. The scratch
 * is 4·(2·m + 2·n)·k' bytes at most (k' = k rounded up to 4): none for x
 * when x is 16-byte aligned with a row stride of whole 16-byte units (else
 * 4·2·m·k' in split precision, 4·m·k' in TF32); none for w in TF32 when it
 * is such an aligned transposed view (else 4·n·k' for its K-major copy);
 * plus 4·n·k' for w's low part in split precision. The call itself
 * allocates nothing (no cudaMalloc, cudaFree or allocating library routine),
 * but the CUDA driver reserves the array when it loads the module holding
 * it: at the first call on a device under lazy module loading (the CUDA 12
 * default), or at context creation with CUDA_MODULE_LOADING=EAGER. A caller
 * whose allocator reserves the GPU's memory up front should make one call
 * (or set eager loading) before reserving. The first call on a device also
 * looks up the array's device address (cudaGetSymbolAddress) and should
 * come before any stream capture. All calls share the array: calls that
 * overlap on the GPU race on it and must be serialised by the caller. A
 * bounded wait that gave up inside its kernels is reported by the next
 * fg_synchronize on that device (FG_ETIMEOUT), as for fg_matmul. */
int fg_matmul_noalloc(int64_t m, int64_t n, int64_t k, const float* x, int64_t ldx,
                      const float* w, int64_t ldw, int w_transposed, float* out, int64_t ldo,
                      const fg_epilogue* epi, int precision, void* stream);

/* out[r] = Σ_c x[r, c]² — (*Tensor).RowSumSquares (tensor/matmul_fused.go:125-143). */
int fg_row_sum_squares(const float* x, int64_t rows, int64_t n, int64_t ldx, float* out,
                       void* stream);

/* out = x / sqrt(mean(x²) + eps) · g over the last dimension n —
 * tensor.RMSNorm (tensor/attention.go:292-337). g holds the final gains
 * (the caller adds Gemma's 1 as the reference's Load does). */
int fg_rmsnorm(const float* x, int64_t rows, int64_t n, const float* g, float eps, float* out,
               void* stream);

/* Rotate-half RoPE over contiguous [rows, D] vectors whose slot is
 * (row % T), at positions[slot] — tensor.RoPE (tensor/rope.go:20-87). */
int fg_rope(const float* x, int64_t rows, int T, int D, double base, const int32_t* positions,
            float* out, void* stream);

/* softmax(scale·q·kᵀ + mask)·v for q [B, Hq, T, D], k and v [B, Hkv, S, D]
 * (contiguous), with Hq a multiple of Hkv (grouped-query heads share a KV
 * head, the Expand view of tensor/attention.go:62-66). The mask is the
 * additive −1e9 mask the encoder builds: key j of batch b is hidden when
 * j >= key_lengths[b] (PaddingMask, attention.go:33-42; NULL = none) or,
 * when window > 0, when |i − j| >= window (WindowMask, attention.go:97-107).
 * — tensor.AttentionScaled (tensor/attention.go:67). */
int fg_attention(const float* q, const float* k, const float* v, int B, int Hq, int Hkv, int T,
                 int S, int D, const int32_t* key_lengths, int window, float scale, float* out,
                 int precision, void* stream);

/* ---- cluster: the consumer of the embeddings (cluster/cluster.go) ------ */
/* Device pointers, row-major with leading dimensions; `precision` as for
 * fg_matmul (the similarity products run on the split-TF32 GEMM). */

/* out = every row of x [n, d] scaled to unit length; rows of length zero
 * stay zero — cluster.Normalize (cluster.go:19-28). out may equal x. */
int fg_normalize_rows(int64_t n, int64_t d, const float* x, int64_t ldx, float* out, int64_t ldo,
                      void* stream);

/* out [q, n] = queries [q, d] · docs [n, d]ᵀ, the cosine similarities of
 * unit-length rows — cluster.Similarities (cluster.go:185-190). */
int fg_similarities(int64_t q, int64_t n, int64_t d, const float* queries, int64_t ldq, const float* docs,
                    int64_t ldd, float* out, int64_t ldo, int precision, void* stream);

/* For every row of x [n, d], the index of the most similar of the k
 * centres [k, d] (the first on ties, as tensor.Argmax) and that similarity
 * — cluster.Nearest (cluster.go:136-148). Asynchronous on the stream. */
int fg_nearest(int64_t n, int64_t k, int64_t d, const float* x, int64_t ldx, const float* centres, int64_t ldc,
               int32_t* index, float* similarity, int precision, void* stream);

/* k-means of the unit-length rows of x [n, d] by cosine similarity —
 * cluster.KMeans (cluster.go:43-133): k-means++ seeding driven by Go's
 * math/rand/v2 PCG seeded (seed, seed ^ 0x9e3779b97f4a7c15), then up to
 * `iters` rounds of assignment (one product + row argmax) and centre update
 * (row sums in row order, empty centres restarted on the worst-fitting row,
 * renormalised), stopping after a round in which no row changed centre
 * (from the second round on). Writes centres [k, d] (unit length, leading
 * dimension d), assignment [n], similarity [n] (each row's similarity to
 * its centre), sizes [k] and *iterations. k outside 1..n is FG_EINVAL (the
 * reference panics). Synchronous. */
int fg_kmeans(int64_t n, int64_t d, const float* x, int64_t ldx, int k, int iters, uint64_t seed,
              float* centres, int32_t* assignment, float* similarity, int32_t* sizes, int* iterations,
              int precision, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FGEMMA_H */
