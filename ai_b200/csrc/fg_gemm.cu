// tcgen05 TF32 / split-TF32 GEMM for sm_100a with fused epilogues.
//
// C[M, Nout] = epilogue(A · Bᵀ), A [M, K] and B [Nb, K] row-major (both
// K-major operands, the layout the encoder keeps its [out, in] weights in).
// This replaces the reference's blocked SGEMM (internal/blas/gemm.go:562-702)
// and its epilogue (gemm.go:316-347) on the encoder's hot path.
//
// Structure: a persistent kernel, one CTA per SM, 6 warps.
//   warp 0      TMA producer: 128-byte-swizzled [rows × 32 fp32] tiles of A
//               (and A_lo), B (and B_lo) into a multi-stage smem ring.
//   warp 1      TMEM allocator and MMA issuer: one thread issues
//               tcgen05.mma.kind::tf32 (M=128, N=BN, K=8) per pass, into one
//               of two TMEM accumulators (double buffered, 2·BN columns).
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (one row per
//               thread), fused row scale / bias / activation / gate / mul /
//               residual, optional split of the result into TF32 hi/lo, and
//               the global store; overlaps the next tile's main loop.
// Split-TF32 accumulates A·B + A·B_lo + A_lo·B into the same accumulator;
// an operand whose low part is identically zero (bf16-exact weights) has
// no low pass, which changes nothing in the result.
// Split-fp16 (pair kernel only): when B has an exact fp16 form under a
// power-of-two scale (bf16 weights: 8 significant bits), A is cut into two
// fp16 parts under a per-row power-of-two scale and the product is
// A_hi·B + A_lo·B in kind::f16 — the same 22 bits of A as split-TF32, exact
// products, at the fp16 rate (twice TF32's).
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cudaTypedefs.h>

#include <cuda_fp16.h>

#include "fg_internal.h"
#include "fg_ptx.cuh"

namespace fg {

namespace {

constexpr int kBM = 128;
constexpr int kUmmaK = 8;
constexpr int kThreads = 192;
constexpr int kSmemLimit = 232448;  // 227 KB opt-in dynamic shared memory

struct KParams {
  int M, Nout, K;
  int ntm, ntn, nk;
  GemmEpilogue e;
  int* err;
  int tma_out, tma_out_lo;  // out / out_lo are written by TMA stores (maps m[0] / m[1])
  int tma_out16;            // out16 / out16_lo (fp16 parts) are written by TMA stores (maps m[0] / m[1])
  int tma_qk;               // q / k attention operands are written by TMA stores (maps m[0..3])
  // Split-fp16 pair kernel: A·2^e_r and B·2^b_exp in fp16 (see a_row_exp);
  // the epilogue multiplies each row by 2^-(e_r + b_exp), which is exact.
  int h16;
  int a_exp, a_exp_rs, b_exp;
  const int* b_exp_dev;  // when set, B's exponent as the device computed it (overrides b_exp)
  float a_norm_k;      // sqrt(K): max|a_r| <= sqrt(K) / a_rs[r]
  const float* a_rs;   // A's row scales 1/sqrt(mean(a²) + eps) (a_exp_rs)
  const float* a_gain;  // per-column gain on A (split-fp16 with an unfolded B), or null
};

// Exponent e_r of A row r in the split-fp16 product: |a_r|·2^e_r < 2^14, so
// both fp16 parts are finite and every element down to 2^-17 of the bound
// keeps 22 significant bits. Static (p.a_exp, from a bound on the whole
// operand) or, with p.a_exp_rs, from the row's RMS scale rs = 1/sqrt(ms +
// eps): max|a_r| <= sqrt(K·ms) < sqrt(K)/rs.
__device__ __forceinline__ int a_row_exp(const KParams& p, int row) {
  if (!p.a_exp_rs) return p.a_exp;
  const float rs = row < p.M ? p.a_rs[row] : 1.f;
  const int e = 13 - ilogbf(p.a_norm_k / rs);
  return max(-60, min(60, e));
}

// TMA-store maps of the epilogue outputs: fp32 out / out_lo in m[0] / m[1];
// for the attention-operand epilogue the bf16 q_hi, q_lo, k_hi, k_lo.
struct OutMaps {
  CUtensorMap m[4];
};

// Shared memory of each epilogue warp: two 4 KB boxes of [32 rows × 32
// fp32], 128-byte swizzled and 1024-byte aligned, for TMA stores (one is
// filled while the store of the other still reads it); the QKV epilogue
// uses the first 4.2 KB as a padded [32 × 33] transpose block. The stage
// ring comes first, then these 4 × 8 KB, then the mbarriers.
constexpr uint32_t kEpiWarpBytes = 8192;
constexpr uint32_t kEpiStageBytesAll = 4 * kEpiWarpBytes;

// BK fp32 of K per pipeline stage: 32 (128-byte swizzled rows) or 16
// (64-byte rows: half the bytes per stage, so more stages in flight).
// SA: A's low part is loaded by TMA; CV: it is computed in shared memory
// from the A tile by converter warps (A is then read from memory once).
template <int BN, bool SA, bool SB, int BK, bool CV = false>
struct Cfg {
  static constexpr int kSwizzle = BK * 4;
  static constexpr bool kAlo = SA || CV;
  static constexpr int kThreads = CV ? 320 : 192;
  static constexpr uint32_t kABytes = kBM * BK * 4;
  static constexpr uint32_t kBBytes = BN * BK * 4;
  static constexpr uint32_t kStageBytes = kABytes * (kAlo ? 2 : 1) + kBBytes * (SB ? 2 : 1);
  static constexpr uint32_t kTmaBytes = kStageBytes - (CV ? kABytes : 0);
  static constexpr uint32_t kEpiStageBytes = kEpiStageBytesAll;
  static constexpr int kStagesRaw = (kSmemLimit - 2048 - int(kEpiStageBytes)) / kStageBytes;
  static constexpr int kMaxStages = BK == 16 ? 8 : 6;
  static constexpr int kStages = kStagesRaw > kMaxStages ? kMaxStages : kStagesRaw;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr size_t kSmemBytes = 1024 + size_t(kStages) * kStageBytes + kEpiStageBytes + 256;
  static_assert(kStages >= 2, "tile too large for shared memory");
  static_assert(BK == 16 || BK == 32, "stage depth");
};

// Eigen's rational tanh for float (the method the reference's kernels use,
// internal/kernel/generic.go:309-360): odd degree-13 over even degree-6
// polynomial after clamping to the point where it reaches ±1.
// Written without branches (the rational is always evaluated and the small
// and saturated cases selected afterwards) so that the epilogue can keep
// many independent elements in flight; the results are those of the
// early-return form.
__device__ __forceinline__ float tanh_rational(float x_in) {
  const float c = 7.99881172180175781f;
  const float x = fminf(fmaxf(x_in, -c), c);
  const float x2 = x * x;
  float p = -2.76076847742355e-16f;
  p = p * x2 + 2.00018790482477e-13f;
  p = p * x2 + -8.60467152213735e-11f;
  p = p * x2 + 5.12229709037114e-08f;
  p = p * x2 + 1.48572235717979e-05f;
  p = p * x2 + 6.37261928875436e-04f;
  p = p * x2 + 4.89352455891786e-03f;
  p = p * x;
  float q = 1.19825839466702e-06f;
  q = q * x2 + 1.18534705686654e-04f;
  q = q * x2 + 2.26843463243900e-03f;
  q = q * x2 + 4.89352518554385e-03f;
  float r = p / q;
  r = (x_in > -0.0004f && x_in < 0.0004f) ? x_in : r;
  r = x_in >= 9.f ? 1.f : r;
  r = x_in <= -9.f ? -1.f : r;
  return r;
}

// tanh-GELU in the reference's operation order (internal/kernel/math.go:122-143):
// u = c·(x + 0.044715·x³); 0.5·x·(1 + tanh(u)).
__device__ __forceinline__ float gelu_tanh(float x) {
  float z = x * x;
  z = z * x;
  z = z * 0.044715f;
  z = x + z;
  z = z * 0.7978845608028654f;
  float t = tanh_rational(z);
  t = t + 1.f;
  t = t * x;
  return t * 0.5f;
}

// The same tanh-GELU for the gated FFN epilogue, in the form
// 0.5·x·(1 + tanh(u)) = x·σ(2u) = x / (1 + 2^(−2u·log2 e)) with the hardware
// exp2 and reciprocal: ~10 instructions instead of ~40 (the rational tanh and
// an IEEE division), about 1e-7 relative from the form above. +∞ and −∞
// arguments of the exponential give x and −0.
__device__ __forceinline__ float gelu_sigmoid(float x) {
  const float u = x * fmaf(0.7978845608028654f * 0.044715f, x * x, 0.7978845608028654f);
  return x * rcp_approx(1.f + ex2_approx(u * -2.8853900817779268f));
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == FG_ACT_RELU) return fmaxf(v, 0.f);
  if (act == FG_ACT_GELU) return gelu_tanh(v);
  if (act == kActTanh) return tanh_rational(v);
  return v;
}

__device__ __forceinline__ void store_row32(float* dst, const float (&v)[32], int ncols,
                                            bool vec_ok) {
  if (vec_ok && ncols == 32) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncols) dst[j] = v[j];
  }
}

// A warp's [32 rows × 32 columns] fp32 block, one row per lane in v, is
// written to dst (row of lane 0, first column) through the padded staging
// tile `st` ([32][33], conflict-free both ways): each store instruction
// then writes 32 consecutive floats of one row — one 128-byte segment —
// instead of 32 rows' 16-byte pieces. rows/cols bound the valid block.
__device__ __forceinline__ void warp_store_block(float* st, const float (&v)[32], float* dst,
                                                 int64_t ld, int rows, int cols) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 32; ++j) st[lane * 33 + j] = v[j];
  __syncwarp();
  if (lane < cols) {
#pragma unroll 4
    for (int rr = 0; rr < 32; ++rr)
      if (rr < rows) dst[int64_t(rr) * ld + lane] = st[rr * 33 + lane];
  }
  __syncwarp();
}

// The same block written as bf16 hi/lo parts (64-byte segments per store).
__device__ __forceinline__ void warp_store_block_bf16(float* st, const float (&v)[32],
                                                      __nv_bfloat16* hi, __nv_bfloat16* lo,
                                                      int64_t ld, int rows) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 32; ++j) st[lane * 33 + j] = v[j];
  __syncwarp();
#pragma unroll 4
  for (int rr = 0; rr < 32; ++rr) {
    if (rr < rows) {
      const float y = st[rr * 33 + lane];
      const __nv_bfloat16 h = __float2bfloat16_rn(y);
      hi[int64_t(rr) * ld + lane] = h;
      lo[int64_t(rr) * ld + lane] = __float2bfloat16_rn(y - __bfloat162float(h));
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void store_bf16_split(__nv_bfloat16* hi, __nv_bfloat16* lo, int64_t off,
                                                 float y) {
  const __nv_bfloat16 h = __float2bfloat16_rn(y);
  hi[off] = h;
  lo[off] = __float2bfloat16_rn(y - __bfloat162float(h));
}

// Four 32-column accumulator chunks (TMEM column offsets c0..c3 from taddr)
// under a single wait.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, int c0, int c1, int c2, int c3,
                                         uint32_t (&r)[4][32]) {
  tmem_ld_32x32b_x32(taddr + uint32_t(c0), r[0]);
  tmem_ld_32x32b_x32(taddr + uint32_t(c1), r[1]);
  tmem_ld_32x32b_x32(taddr + uint32_t(c2), r[2]);
  tmem_ld_32x32b_x32(taddr + uint32_t(c3), r[3]);
  tmem_ld_wait();
}

// An epilogue warp's staging area (kEpiWarpBytes) and the number of TMA
// store boxes it has issued (selects which of the two boxes is filled next).
struct EpiStage {
  uint8_t* base;
  int n;
};

// bf16 parts of two fp32 values y0, y1, packed into a word each (y0 in the
// low half): hi = RN(y), lo = RN(y - hi).
__device__ __forceinline__ void split_pack_pair(float y0, float y1, uint32_t& hw, uint32_t& lw) {
  hw = pack_bf16x2(y0, y1);  // one paired round-to-nearest conversion
  const float h0 = __uint_as_float(hw << 16), h1 = __uint_as_float(hw & 0xffff0000u);
  lw = pack_bf16x2(y0 - h0, y1 - h1);
}

// Half `hf` (16 bf16 = 32 bytes) of row `lane` of a [32 rows × 32 bf16] TMA
// box with 64-byte swizzling: 16-byte chunk c of row r sits at chunk
// c ^ ((r / 2) % 4), which spreads eight consecutive rows over all banks.
__device__ __forceinline__ void put_half_row_bf16_sw64(uint8_t* box, int hf, const uint32_t (&w)[8]) {
  const int lane = threadIdx.x & 31;
  uint4* rowp = reinterpret_cast<uint4*>(box + lane * 64);
  const int sw = (lane >> 1) & 3;
  rowp[(2 * hf) ^ sw] = make_uint4(w[0], w[1], w[2], w[3]);
  rowp[(2 * hf + 1) ^ sw] = make_uint4(w[4], w[5], w[6], w[7]);
}

// Epilogue of the QKV projection when it feeds the tensor-core attention:
// the accumulator tile is one head (256 columns). q/k heads: y = rs·acc,
// per-head RMSNorm with gain (attention.go:312-337: v·inv·g, inv from the
// float32 mean and a float64 root), rotate-half RoPE at slot t = row % T
// (rope.go:66-87), then bf16 hi/lo parts, token-major. v heads: rs·acc as
// bf16 hi/lo written transposed per sequence (vt[(b·Hkv+hk)·256 + d][t]).
// tcgen05.ld is warp-collective, so every lane loads even for rows ≥ M.
__device__ __forceinline__ void qkv_attn_epilogue(const GemmEpilogue& e, const OutMaps& om, bool tma_qk,
                                                  uint32_t taddr, int tn, int row, bool row_ok, float rs,
                                                  EpiStage& es, int rows) {
  float* const st = reinterpret_cast<float*>(es.base);
  constexpr int D = 256, H2 = 128;
  // Fields in registers: read through the reference they would be re-read
  // after every global store (the stores might alias them).
  const int Hq = e.Hq, Hkv = e.Hkv, T = e.T;
  if (tn < Hq + Hkv) {
    const bool is_q = tn < Hq;
    const float* const g = is_q ? e.qgain : e.kgain;
    const float eps = e.eps;
    // position-minor table with cos and sin side by side: the warp's 32
    // consecutive rows read one 256-byte segment per column, one load each
    const int t = row % T;
    const int64_t rld = e.rope_ld;
    const float2* const csn = e.rope_cs + t;
    __nv_bfloat16* const hi = static_cast<__nv_bfloat16*>(is_q ? e.q_hi : e.k_hi);
    __nv_bfloat16* const lo = static_cast<__nv_bfloat16*>(is_q ? e.q_lo : e.k_lo);
    const int width = (is_q ? Hq : Hkv) * D;
    const int head = is_q ? tn : tn - Hq;
    // pass 1: Σ y² over the head in four interleaved partial sums (columns
    // ≡ q mod 4 ... in order), so the dependent chain is 64 adds, not 256
    float ss4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int h0 = 0; h0 < D; h0 += 128) {
      uint32_t r[4][32];
      tmem_ld4(taddr, h0, h0 + 32, h0 + 64, h0 + 96, r);
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float y = __fmul_rn(__uint_as_float(r[q][j]), rs);
          ss4[j & 3] = __fmaf_rn(y, y, ss4[j & 3]);
        }
    }
    const float ss = (ss4[0] + ss4[1]) + (ss4[2] + ss4[3]);
    const float m = __fadd_rn(__fdiv_rn(ss, float(D)), eps);
    const float inv = float(1.0 / sqrt(double(m)));
    const int lane = threadIdx.x & 31;
    // the warp's first row, first column of this head
    const int64_t base0 = int64_t(row - lane) * width + int64_t(head) * D;
    // the head's gains spread over the lanes (g[32k + lane] in gq[k]) and
    // taken by shuffle: the same for every row, so no per-element loads
    float gq[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) gq[k] = g[32 * k + lane];
    // pass 2: normalise, rotate the pairs (i, i + 128), split, store
#pragma unroll 1
    for (int c0 = 0; c0 < H2; c0 += 32) {
      uint32_t ra[32], rb[32];
      tmem_ld_32x32b_x32(taddr + uint32_t(c0), ra);
      tmem_ld_32x32b_x32(taddr + uint32_t(H2 + c0), rb);
      tmem_ld_wait();
      const int qq = c0 >> 5;
      const float ga = qq == 0 ? gq[0] : qq == 1 ? gq[1] : qq == 2 ? gq[2] : gq[3];
      const float gb = qq == 0 ? gq[4] : qq == 1 ? gq[5] : qq == 2 ? gq[6] : gq[7];
      // y1 = x1·c - x2·s, y2 = x1·s + x2·c for column j of the chunk
      auto rot = [&](int j, float& y1, float& y2) {
        const int i = c0 + j;
        const float g1 = __shfl_sync(0xffffffffu, ga, j), g2 = __shfl_sync(0xffffffffu, gb, j);
        const float x1 = __fmul_rn(__fmul_rn(__fmul_rn(__uint_as_float(ra[j]), rs), inv), g1);
        const float x2 = __fmul_rn(__fmul_rn(__fmul_rn(__uint_as_float(rb[j]), rs), inv), g2);
        const float2 f = row_ok ? csn[i * rld] : make_float2(0.f, 0.f);
        const float c = f.x, s = f.y;
        y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        y2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
      };
      if (tma_qk) {
        // four [32 × 32] bf16 boxes: y1 hi, y1 lo, y2 hi, y2 lo, filled 16 columns at a time
        if (lane == 0) tma_store_wait_read<0>();  // the previous chunk's stores have read the boxes
        __syncwarp();
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t w[4][8];  // y1 hi, y1 lo, y2 hi, y2 lo: 16 bf16 each
#pragma unroll
          for (int jj = 0; jj < 16; jj += 2) {
            float a1, a2, b1, b2;
            rot(hf * 16 + jj, a1, a2);
            rot(hf * 16 + jj + 1, b1, b2);
            split_pack_pair(a1, b1, w[0][jj / 2], w[1][jj / 2]);
            split_pack_pair(a2, b2, w[2][jj / 2], w[3][jj / 2]);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) put_half_row_bf16_sw64(es.base + q * 2048, hf, w[q]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && rows > 0) {
          const CUtensorMap* mh = &om.m[is_q ? 0 : 2];
          const CUtensorMap* ml = &om.m[is_q ? 1 : 3];
          const uint32_t b = smem_u32(es.base);
          const int col = head * D + c0, r0 = row - lane;
          tma_store_2d(mh, b, col, r0);
          tma_store_2d(ml, b + 2048, col, r0);
          tma_store_2d(mh, b + 4096, col + H2, r0);
          tma_store_2d(ml, b + 6144, col + H2, r0);
          tma_store_commit();
        }
      } else {
        float y1[32], y2[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) rot(j, y1[j], y2[j]);
        warp_store_block_bf16(st, y1, hi + base0 + c0, lo + base0 + c0, width, rows);
        warp_store_block_bf16(st, y2, hi + base0 + H2 + c0, lo + base0 + H2 + c0, width, rows);
      }
    }
  } else {
    const int hk = tn - Hq - Hkv;
    const int b = row / T, t = row % T;
    __nv_bfloat16* const hi = static_cast<__nv_bfloat16*>(e.vt_hi);
    __nv_bfloat16* const lo = static_cast<__nv_bfloat16*>(e.vt_lo);
    const int64_t ldt = e.ldt;
    const int64_t base = (int64_t(b) * Hkv + hk) * D * ldt + t;
    // EmbeddingGemma 2's weight-free v_norm (embed.go:300): y·inv, inv from
    // Σ y² over the head as for q and k; 1 (exact) without it
    float vinv = 1.f;
    if (e.vnorm) {
      float ss = 0.f;
#pragma unroll 1
      for (int h0 = 0; h0 < D; h0 += 128) {
        uint32_t r4[4][32];
        tmem_ld4(taddr, h0, h0 + 32, h0 + 64, h0 + 96, r4);
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float y = __fmul_rn(__uint_as_float(r4[q][j]), rs);
            ss = __fadd_rn(ss, __fmul_rn(y, y));
          }
      }
      vinv = float(1.0 / sqrt(double(__fadd_rn(__fdiv_rn(ss, float(D)), e.eps))));
    }
#pragma unroll 1
    for (int c0 = 0; c0 < D; c0 += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + uint32_t(c0), r);
      tmem_ld_wait();
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          store_bf16_split(hi, lo, base + int64_t(c0 + j) * ldt,
                           __fmul_rn(__fmul_rn(__uint_as_float(r[j]), rs), vinv));
      }
    }
  }
}

// The warp's [32 rows × 32 columns] fp32 block (row `lane` in v) written to
// global memory at (row0, col0) by one TMA store: every lane puts its row
// into the next 128-byte-swizzled staging box (16-byte chunk c of row r at
// chunk c ^ (r % 8), conflict-free), then lane 0 issues the store, which
// writes whole rows of 128 bytes and drops what lies outside the tensor.
__device__ __forceinline__ void store_box_tma(const CUtensorMap* map, EpiStage& es, const float (&v)[32],
                                              int col0, int row0, bool inside) {
  const int lane = threadIdx.x & 31;
  uint8_t* buf = es.base + (es.n & 1) * 4096;
  if (lane == 0) tma_store_wait_read<1>();  // the store that last read this box is done with it
  __syncwarp();
  float4* rowp = reinterpret_cast<float4*>(buf + lane * 128);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    rowp[c ^ (lane & 7)] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  fence_proxy_async_smem();  // generic-proxy writes → visible to the TMA engine
  __syncwarp();
  if (lane == 0 && inside) {
    tma_store_2d(map, smem_u32(buf), col0, row0);
    tma_store_commit();
  }
  ++es.n;
}

// The warp's [32 rows × 32 columns] block (row `lane` in v) written as the
// next product's fp16 parts: a = v·sc cut into hi (a's top 11 significant
// bits) and lo = fp16(a − hi), exactly as the GEMM converters cut A; two
// [32 × 32] fp16 boxes (64-byte rows, 64-byte swizzle: 16-byte chunk j of
// row r at chunk j ^ ((r / 2) % 4)) in the next staging slot, stored by TMA.
__device__ __forceinline__ void store_box16_tma(const CUtensorMap* mhi, const CUtensorMap* mlo, EpiStage& es,
                                                const float (&v)[32], float sc, int col0, int row0, bool inside) {
  const int lane = threadIdx.x & 31;
  uint8_t* buf = es.base + (es.n & 1) * 4096;  // hi box at +0, lo box at +2048
  if (lane == 0) tma_store_wait_read<1>();   // the store that last read this slot is done with it
  __syncwarp();
  uint32_t hw[16], lw[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const float a0 = v[2 * q] * sc, a1 = v[2 * q + 1] * sc;
    const float h0 = tf32_hi(a0), h1 = tf32_hi(a1);
    hw[q] = pack_f16x2(h0, h1);
    lw[q] = pack_f16x2(a0 - h0, a1 - h1);
  }
  const int sw = (lane >> 1) & 3;
  uint4* rh = reinterpret_cast<uint4*>(buf + lane * 64);
  uint4* rl = reinterpret_cast<uint4*>(buf + 2048 + lane * 64);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    rh[j ^ sw] = make_uint4(hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]);
    rl[j ^ sw] = make_uint4(lw[4 * j], lw[4 * j + 1], lw[4 * j + 2], lw[4 * j + 3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && inside) {
    tma_store_2d(mhi, smem_u32(buf), col0, row0);
    tma_store_2d(mlo, smem_u32(buf + 2048), col0, row0);
    tma_store_commit();
  }
  ++es.n;
}

// One accumulator tile through the epilogue, by one of the four epilogue
// warps: its 32 TMEM lanes at `taddr` (BN columns) hold output rows
// row0 .. row0+31 of N-tile tn. Results go out by TMA stores when the
// launch prepared maps for them (p.tma_out / p.tma_out_lo), else by direct
// row stores.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const KParams& p, const OutMaps& om, uint32_t taddr,
                                              int row0, int tn, EpiStage& es) {
  const GemmEpilogue& e = p.e;
  // Fields in registers: read through the reference they would be re-read
  // after every global store (the stores might alias them).
  float* const out = e.out;
  const int64_t ldo = e.ldo;
  float* const out_lo = e.out_lo;
  const int64_t ldo_lo = e.ldo_lo;
  const float* const rowscale = e.rowscale;
  const float* const bias = e.bias;
  const float* const mul = e.mul;
  const int64_t ldm = e.ldm;
  const float* const resid = e.residual;
  const int64_t ldr = e.ldr;
  const int act = e.act;
  const bool geglu = e.geglu != 0;
  const bool qkv = BN == 256 && e.qkv_attn != 0;
  const bool plain = !bias && !mul && !resid && act == FG_ACT_NONE;
  const bool tma = p.tma_out != 0, tma_lo = p.tma_out_lo != 0;
  const int Nout = p.Nout, M = p.M;
  const bool vec_out = (ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
  const bool vec_lo = out_lo && (ldo_lo % 4 == 0) && ((reinterpret_cast<uintptr_t>(out_lo) & 15) == 0);
  const int row = row0 + int(threadIdx.x & 31);
  const bool row_ok = row < M;
  const int rows = max(0, min(32, M - row0));
  float rs = (rowscale && row_ok) ? rowscale[row] : 1.f;
  // split-fp16: undo the operands' power-of-two scales (exact); applied to
  // the accumulator first where a bias is added before the row scale
  const int bexp = p.b_exp_dev ? *p.b_exp_dev : p.b_exp;
  const float fac = p.h16 ? pow2f(-(a_row_exp(p, row) + bexp)) : 1.f;
  if (!bias) rs *= fac;
  if (qkv) {
    qkv_attn_epilogue(e, om, p.tma_qk != 0, taddr, tn, row, row_ok, rs, es, rows);
  } else if (geglu) {
    // Tile columns [0, BN/2) are gate, [BN/2, BN) the matching up columns.
#pragma unroll 1
    for (int c0 = 0; c0 < BN / 2; c0 += 32) {
      uint32_t rg[32], ru[32];
      tmem_ld_32x32b_x32(taddr + uint32_t(c0), rg);
      tmem_ld_32x32b_x32(taddr + uint32_t(BN / 2 + c0), ru);
      tmem_ld_wait();
      const int col0 = tn * (BN / 2) + c0;
      const int ncols = min(32, Nout - col0);
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float g = __uint_as_float(rg[j]) * rs;
        const float u = __uint_as_float(ru[j]) * rs;
        v[j] = gelu_sigmoid(g) * u;
      }
      if (p.tma_out16) {
        store_box16_tma(&om.m[0], &om.m[1], es, v, pow2f(e.out16_exp), col0, row0, ncols > 0 && rows > 0);
        continue;
      }
      if (tma) store_box_tma(&om.m[0], es, v, col0, row0, ncols > 0 && rows > 0);
      else if (row_ok && ncols > 0) store_row32(out + int64_t(row) * ldo + col0, v, ncols, vec_out);
      if (out_lo) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = tf32_lo(v[j]);
        if (tma_lo) store_box_tma(&om.m[1], es, v, col0, row0, ncols > 0 && rows > 0);
        else if (row_ok && ncols > 0) store_row32(out_lo + int64_t(row) * ldo_lo + col0, v, ncols, vec_lo);
      }
    }
  } else {
#pragma unroll 1
    for (int h0 = 0; h0 < BN; h0 += 64) {
      uint32_t r[2][32];
      tmem_ld_32x32b_x32(taddr + uint32_t(h0), r[0]);
      tmem_ld_32x32b_x32(taddr + uint32_t(h0 + 32), r[1]);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int col0 = tn * BN + h0 + 32 * q;
        const int ncols = min(32, Nout - col0);
        if (ncols <= 0) break;  // warp-uniform
        float v[32];
        if (plain) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[q][j]) * rs;
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(r[q][j]);
            if (bias) x *= fac;
            const int col = col0 + j;
            const bool in = row_ok && j < ncols;
            if (bias && j < ncols) x = x + bias[col];
            x = x * rs;
            x = apply_act(x, act);
            if (mul && in) x = x * mul[int64_t(row) * ldm + col];
            if (resid && in) x = x + resid[int64_t(row) * ldr + col];
            v[j] = x;
          }
        }
        if (tma) store_box_tma(&om.m[0], es, v, col0, row0, rows > 0);
        else if (row_ok) store_row32(out + int64_t(row) * ldo + col0, v, ncols, vec_out);
        if (out_lo) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = tf32_lo(v[j]);
          if (tma_lo) store_box_tma(&om.m[1], es, v, col0, row0, rows > 0);
          else if (row_ok) store_row32(out_lo + int64_t(row) * ldo_lo + col0, v, ncols, vec_lo);
        }
      }
    }
  }
}

template <int BN, bool SA, bool SB, int BK, bool CV>
__global__ void __launch_bounds__(Cfg<BN, SA, SB, BK, CV>::kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mAlo,
                     const __grid_constant__ CUtensorMap mB, const __grid_constant__ CUtensorMap mBlo,
                     const __grid_constant__ OutMaps om,
                     const __grid_constant__ KParams p) {
  using C = Cfg<BN, SA, SB, BK, CV>;
  constexpr int S = C::kStages;
  constexpr int kSw = C::kSwizzle;
  constexpr uint32_t kIdesc = idesc_tf32(kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + size_t(S) * C::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + C::kEpiStageBytes);
  // bars[0..S) full, [S..2S) empty, [2S..2S+2) acc_full, [2S+2..2S+4) acc_empty,
  // [2S+4] drain, [2S+5..3S+5) A low part converted
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntiles = p.ntm * p.ntn;

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S + s]); };
  auto accf_bar = [&](int a) { return smem_u32(&bars[2 * S + a]); };
  auto acce_bar = [&](int a) { return smem_u32(&bars[2 * S + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[2 * S + 4]);
  auto conv_bar = [&](int s) { return smem_u32(&bars[2 * S + 5 + s]); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
      if (CV) mbar_init(conv_bar(s), 128);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mA);
    tma_prefetch_desc(&mB);
    if (SA) tma_prefetch_desc(&mAlo);
    if (SB) tma_prefetch_desc(&mBlo);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int armed[S];
#pragma unroll
      for (int s = 0; s < S; ++s) armed[s] = 0;
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x) {
        const int tm = tile / p.ntn, tn = tile % p.ntn;
        for (int kb = 0; kb < p.nk; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) break;
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, C::kTmaBytes);
          armed[stage]++;
          uint32_t dst = smem_u32(smem + size_t(stage) * C::kStageBytes);
          tma_load_2d(dst, &mA, fb, kb * BK, tm * kBM);
          dst += C::kABytes;
          if (SA) tma_load_2d(dst, &mAlo, fb, kb * BK, tm * kBM);
          if (C::kAlo) dst += C::kABytes;
          tma_load_2d(dst, &mB, fb, kb * BK, tn * BN);
          dst += C::kBBytes;
          if (SB) tma_load_2d(dst, &mBlo, fb, kb * BK, tn * BN);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      {
        // Let every load this thread issued land before the CTA retires,
        // also when another role gave up and left stages unconsumed (after
        // a normal run every phase has completed and these return at once).
        for (int s = 0; s < S; ++s) {
          if (armed[s] == 0) continue;
          const uint32_t par = uint32_t(armed[s] - 1) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(full_bar(s), par)) {
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
              atomicCAS(p.err, 0, kDevTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool issued = false;
      for (int tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_par = uint32_t(local >> 1) & 1u;
        if (!mbar_wait(acce_bar(acc), acc_par ^ 1, abort_flag, p.err, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < p.nk; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + size_t(stage) * C::kStageBytes);
          const uint32_t alo_addr = a_addr + C::kABytes;
          const uint32_t b_addr = a_addr + C::kABytes * (C::kAlo ? 2 : 1);
          const uint32_t blo_addr = b_addr + C::kBBytes;
#pragma unroll
          for (int k = 0; k < BK / kUmmaK; ++k) {
            const uint32_t koff = uint32_t(k * kUmmaK * 4);
            const uint64_t da = kmajor_desc<kSw>(a_addr + koff);
            const uint64_t db = kmajor_desc<kSw>(b_addr + koff);
            mma_tf32(d_tmem, da, db, kIdesc, (kb | k) != 0 ? 1u : 0u);
            if (SB) mma_tf32(d_tmem, da, kmajor_desc<kSw>(blo_addr + koff), kIdesc, 1u);
          }
          if (SA) {
            // the low pass after the stage's high pass, the order the
            // shared-memory low part (CV) takes, so both give equal sums
#pragma unroll
            for (int k = 0; k < BK / kUmmaK; ++k) {
              const uint32_t koff = uint32_t(k * kUmmaK * 4);
              mma_tf32(d_tmem, kmajor_desc<kSw>(alo_addr + koff), kmajor_desc<kSw>(b_addr + koff), kIdesc, 1u);
            }
          }
          if (CV) {
            // low pass once the converter warps have written A's low part
            if (!mbar_wait(conv_bar(stage), phase, abort_flag, p.err, kDevTimeoutFull)) {
              ok = false;
              issued = true;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < BK / kUmmaK; ++k) {
              const uint32_t koff = uint32_t(k * kUmmaK * 4);
              mma_tf32(d_tmem, kmajor_desc<kSw>(alo_addr + koff), kmajor_desc<kSw>(b_addr + koff),
                       kIdesc, 1u);
            }
          }
          issued = true;
          mma_commit(empty_bar(stage));
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(accf_bar(acc));
      }
      if (issued) {
        // Every MMA issued above must finish before TMEM is released.
        mma_commit(drain_bar);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain_bar, 0)) {
          if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            atomicCAS(p.err, 0, kDevTimeoutDrain);
            break;
          }
        }
      }
    }
  } else if (CV && warp >= 6) {
    // -------------------------------------------------- converters (warps 6..9)
    // A tile [128 rows × BK fp32] as TMA swizzled it; the low part lands at
    // the same byte offsets of the stage's A_lo slot, so it has the same
    // swizzled layout the MMA descriptor expects.
    const int ct = threadIdx.x - 192;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < ntiles && !*abort_flag; tile += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < p.nk; ++kb) {
        if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err, kDevTimeoutFull)) {
          ok = false;
          break;
        }
        const float4* src = reinterpret_cast<const float4*>(smem + size_t(stage) * C::kStageBytes);
        float4* dst = reinterpret_cast<float4*>(smem + size_t(stage) * C::kStageBytes + C::kABytes);
#pragma unroll
        for (int q = 0; q < int(C::kABytes / 16 / 128); ++q) {
          const float4 v = src[q * 128 + ct];
          dst[q * 128 + ct] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
        }
        fence_proxy_async_smem();  // generic-proxy writes → visible to the tensor core
        mbar_arrive(conv_bar(stage));
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
  } else {
    // -------------------------------------------------- epilogue (warps 2..5)
    const int quad = warp & 3;
    EpiStage es{epi_smem + size_t(warp - 2) * kEpiWarpBytes, 0};
    int local = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_par = uint32_t(local >> 1) & 1u;
      const bool got = mbar_wait(accf_bar(acc), acc_par, abort_flag, p.err, kDevTimeoutAccFull);
      if (!__all_sync(0xffffffffu, got)) break;  // warp-uniform before the collective tcgen05.ld
      tc_fence_after();
      const int tm = tile / p.ntn, tn = tile % p.ntn;
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN);
      epilogue_tile<BN>(p, om, taddr, tm * kBM + quad * 32, tn, es);
      tc_fence_before();
      mbar_arrive(acce_bar(acc));
    }
    if (lane == 0) tma_store_wait_read<0>();  // staging read before the CTA's shared memory goes away
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ------------------------------------------------------- CTA-pair kernel
// The same GEMM on pairs of SMs (a cluster of two CTAs) with the pair MMA
// (tcgen05.mma.cta_group::2, M = 256, N = 256): each CTA loads its 128 rows
// of the A tile and its 128 rows of the 256-row B tile, so every B byte is
// read from shared memory once for 256 output rows instead of 128. That
// halves the B operand traffic through shared memory, which is what limits
// the single-CTA kernel (A, A_lo and B reads by the tensor core plus the
// TMA and converter traffic exceed the shared-memory bandwidth).
//   warp 0      both CTAs: TMA producer into the CTA's own stage ring
//   warp 1      both CTAs: TMEM allocation (pair); even CTA: MMA issuer
//   warps 2..5  both CTAs: epilogue of the CTA's 128 accumulator rows
//   warps 6..9  both CTAs: A_lo converter (CV) and stage-ready signal to
//               the even CTA, whose MMA thread waits for both halves
// Only TMA loads without multicast are used; the MMA completion is
// signalled to both CTAs by a multicast tcgen05.commit.
// CV: A's low part computed in shared memory by the converter warps; SA:
// loaded by TMA from a stored low part; neither: plain TF32. SB: B's low
// part (weights that are not TF32-exact, e.g. folded with non-zero norm
// gains) loaded by TMA, adding the A·B_lo pass. Stage: A | A_lo | B | B_lo.
//
// H16 (split-fp16, with CV): the converters write A·2^e_r as two fp16 parts
// (hi = a's top 11 significant bits, lo = fp16(a − hi): 22 significant
// bits, as split-TF32 keeps) as two 64-byte-swizzled [128 × 32] tiles over
// the fp32 A tile they came from (same 16 KB), B arrives as fp16 (B·2^b
// exactly: bf16 weights; unfolded, with the fold's column gain applied to
// A by the converters, when the folded values have no fp16 form), and each
// stage is 2 × 2 pair MMAs of
// kind::f16 (K = 16) instead of 2 × 4 of kind::tf32 (K = 8) — half the
// tensor-pipe time for the same products. Stage: A (then A_hi | A_lo) | B,
// 24 KB, so 8 stages are in flight.
//
// H16 with SB: B has no exact fp16 form (an fp32 checkpoint, or the
// op-level product's arbitrary operand), so it comes as two fp16 parts under
// one power-of-two scale, B_hi (its top 11 significant bits) and B_lo =
// fp16(B − B_hi), and each stage adds the A_hi·B_lo pass: A_hi·B_hi +
// A_hi·B_lo + A_lo·B_hi (A_lo·B_lo, 2^-22 of the product, is dropped, as in
// split-TF32) — three fp16 passes, the tensor-pipe time of 1.5 TF32 passes.
// Stage: A (then its parts) | B_hi | B_lo = 32 KB, 6 stages.
//
// H16 with SA (not CV): A's two fp16 parts were written by the kernel that
// produced A (the same parts, under the same power-of-two row scale, that
// the converters would make) and are loaded by TMA like B, so the stage
// needs no conversion: A_hi | A_lo | B (| B_lo).
template <bool CV, bool SA = false, bool SB = false, bool H16 = false>
struct PairCfg {
  static_assert(!H16 || (CV != SA), "split-fp16 takes A's parts from the converters or from memory");
  static constexpr int BN = 256, BK = 32;
  static constexpr int kThreads = 320;
  static constexpr bool kLo = CV || SA;
  static constexpr uint32_t kABytes = 128 * BK * 4;  // this CTA's A rows
  static constexpr uint32_t kBBytes = 128 * BK * (H16 ? 2 : 4);  // this CTA's half of the B rows
  static constexpr uint32_t kPartBytes = 128 * BK * 2;  // one fp16 part of A (H16), in A's place
  static constexpr uint32_t kStageBytes =
      H16 ? kABytes + kBBytes * (SB ? 2 : 1) : kABytes * (kLo ? 2 : 1) + kBBytes * (SB ? 2 : 1);
  static constexpr uint32_t kBOffset = H16 ? kABytes : kABytes * (kLo ? 2 : 1);
  // TMA bytes per stage: with H16 the A region (the fp32 tile, or its two
  // fp16 parts loaded as they are) is kABytes either way
  static constexpr uint32_t kTmaBytes = H16 ? kABytes + kBBytes * (SB ? 2 : 1)
                                            : kABytes * (SA ? 2 : 1) + kBBytes * (SB ? 2 : 1);
  static constexpr uint32_t kALoOffset = H16 ? kPartBytes : kABytes;  // where A's low part sits
  // stage-ready arrivals per stage: 2 converter warps per CTA take a stage
  // with split-fp16 conversion, all 4 otherwise (both CTAs)
  static constexpr uint32_t kReadyCount = (H16 && CV) ? 4 : 8;
  static constexpr uint32_t kEpiStageBytes = kEpiStageBytesAll;
  static constexpr int kStagesRaw = (kSmemLimit - 2048 - int(kEpiStageBytes)) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr uint32_t kTmemCols = 512;  // two 256-column accumulators
  static constexpr size_t kSmemBytes = 1024 + size_t(kStages) * kStageBytes + kEpiStageBytes + 256;
  static_assert(kStages >= 3, "stage ring too shallow");
  static_assert(!H16 || kStages % 2 == 0, "the two converter groups take alternate stages");
};

template <bool CV, bool SA = false, bool SB = false, bool H16 = false>
__global__ void __launch_bounds__(320, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mAlo,
                     const __grid_constant__ CUtensorMap mB, const __grid_constant__ CUtensorMap mBlo,
                     const __grid_constant__ OutMaps om, const __grid_constant__ KParams p) {
  using C = PairCfg<CV, SA, SB, H16>;
  constexpr int S = C::kStages;
  constexpr int BN = C::BN, BK = C::BK;
  constexpr uint32_t kIdesc = H16 ? idesc_f16(256, BN) : idesc_tf32(256, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + size_t(S) * C::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + C::kEpiStageBytes);
  // bars[0..S) full (local TMA), [S..2S) empty, [2S..3S) ready (even CTA),
  // [3S..3S+2) acc_full, [3S+2..3S+4) acc_empty (even CTA), [3S+4] drain
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = int(blockIdx.x >> 1), npairs = int(gridDim.x >> 1);
  const int ntiles = p.ntm * p.ntn;

  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S + s]); };
  auto ready_bar = [&](int s) { return smem_u32(&bars[2 * S + s]); };
  auto accf_bar = [&](int a) { return smem_u32(&bars[3 * S + a]); };
  auto acce_bar = [&](int a) { return smem_u32(&bars[3 * S + 2 + a]); };
  const uint32_t drain_bar = smem_u32(&bars[3 * S + 4]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
      mbar_init(ready_bar(s), C::kReadyCount);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), 8);  // 4 epilogue warps in each CTA
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mA);
    tma_prefetch_desc(&mB);
    if (SA) tma_prefetch_desc(&mAlo);
    if (SB) tma_prefetch_desc(&mBlo);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), C::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int armed[S];
#pragma unroll
      for (int s = 0; s < S; ++s) armed[s] = 0;
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < ntiles && !*abort_flag; tile += npairs) {
        const int tm = tile / p.ntn, tn = tile % p.ntn;
        const int arow = tm * 256 + int(rank) * 128, brow = tn * BN + int(rank) * 128;
        for (int kb = 0; kb < p.nk; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) break;
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, C::kTmaBytes);
          armed[stage]++;
          const uint32_t dst = smem_u32(smem + size_t(stage) * C::kStageBytes);
          tma_load_2d(dst, &mA, fb, kb * BK, arow);
          if (SA) tma_load_2d(dst + C::kALoOffset, &mAlo, fb, kb * BK, arow);
          tma_load_2d(dst + C::kBOffset, &mB, fb, kb * BK, brow);
          if (SB) tma_load_2d(dst + C::kBOffset + C::kBBytes, &mBlo, fb, kb * BK, brow);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      {
        // Let every load this thread issued land before the CTA retires,
        // also when another role gave up and left stages unconsumed (after
        // a normal run every phase has completed and these return at once).
        for (int s = 0; s < S; ++s) {
          if (armed[s] == 0) continue;
          const uint32_t par = uint32_t(armed[s] - 1) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(full_bar(s), par)) {
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
              atomicCAS(p.err, 0, kDevTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------ MMA issuer (even CTA)
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool issued = false;
      for (int tile = pair; tile < ntiles && !*abort_flag; tile += npairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_par = uint32_t(local >> 1) & 1u;
        if (!mbar_wait_cluster(acce_bar(acc), acc_par ^ 1, abort_flag, p.err, kDevTimeoutAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < p.nk; ++kb) {
          if (!mbar_wait_cluster(ready_bar(stage), phase, abort_flag, p.err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + size_t(stage) * C::kStageBytes);
          const uint32_t alo_addr = a_addr + C::kABytes;
          const uint32_t b_addr = a_addr + C::kBOffset;
          const uint32_t blo_addr = b_addr + C::kBBytes;
          if constexpr (H16) {
            // hi·B (and hi·B_lo) then lo·B, K = 16 fp16 (32 bytes of the
            // 64-byte rows) per MMA
            const uint32_t hi_addr = a_addr, lo_addr = a_addr + C::kPartBytes;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t da = kmajor_desc<64>(hi_addr + k * 32);
              mma_f16_pair(d_tmem, da, kmajor_desc<64>(b_addr + k * 32), kIdesc, (kb | k) != 0 ? 1u : 0u);
              if (SB) mma_f16_pair(d_tmem, da, kmajor_desc<64>(blo_addr + k * 32), kIdesc, 1u);
            }
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              mma_f16_pair(d_tmem, kmajor_desc<64>(lo_addr + k * 32), kmajor_desc<64>(b_addr + k * 32), kIdesc, 1u);
          } else {
#pragma unroll
          for (int k = 0; k < BK / kUmmaK; ++k) {
            const uint32_t koff = uint32_t(k * kUmmaK * 4);
            const uint64_t da = kmajor_desc<128>(a_addr + koff);
            mma_tf32_pair(d_tmem, da, kmajor_desc<128>(b_addr + koff), kIdesc, (kb | k) != 0 ? 1u : 0u);
            // A·B_lo interleaved as in the single-CTA kernel, so both give equal sums
            if (SB) mma_tf32_pair(d_tmem, da, kmajor_desc<128>(blo_addr + koff), kIdesc, 1u);
          }
          if (C::kLo) {
#pragma unroll
            for (int k = 0; k < BK / kUmmaK; ++k) {
              const uint32_t koff = uint32_t(k * kUmmaK * 4);
              mma_tf32_pair(d_tmem, kmajor_desc<128>(alo_addr + koff), kmajor_desc<128>(b_addr + koff),
                            kIdesc, 1u);
            }
          }
          }
          issued = true;
          mma_commit_pair(empty_bar(stage), 0x3);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(accf_bar(acc), 0x3);
      }
      if (issued) {
        // Every pair MMA issued above must finish before TMEM is released.
        mma_commit_pair(drain_bar, 0x1);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain_bar, 0)) {
          if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            atomicCAS(p.err, 0, kDevTimeoutDrain);
            break;
          }
        }
      }
    }
  } else if (warp >= 6) {
    // -------------------------------------------------- converters (warps 6..9)
    const int ct = threadIdx.x - 192;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    if constexpr (H16 && CV) {
      // Two groups of two warps take alternate stages (even / odd), so two
      // stages are converted at once. In a group, thread gt converts rows
      // gt and gt + 64 of the CTA's 128 A rows: each fp32 row (128-byte
      // swizzled: 16-byte chunk c at c ^ (row & 7)) is read whole, the
      // group's 64 threads meet, then the fp16 hi and lo rows (64-byte
      // swizzled: chunk j at j ^ ((row >> 1) & 3)) go over the tile. Every
      // exit is decided together (the AND of the group's named barrier), so
      // no thread is left waiting at it.
      const int grp = (warp - 6) >> 1;
      const int gt = ct - grp * 64;
      for (int tile = pair; tile < ntiles; tile += npairs) {
        bool ok = true;
        const int row0 = (tile / p.ntn) * 256 + int(rank) * 128;
        const float sc[2] = {pow2f(a_row_exp(p, row0 + gt)), pow2f(a_row_exp(p, row0 + gt + 64))};
        for (int kb = 0; kb < p.nk; ++kb) {
          if ((stage & 1) == grp) {
            const bool got = mbar_wait(full_bar(stage), phase, abort_flag, p.err, kDevTimeoutFull);
            uint8_t* base = smem + size_t(stage) * C::kStageBytes;
            float4 v[2][8];
            if (got) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int r = gt + 64 * h;
                const float4* src = reinterpret_cast<const float4*>(base) + r * 8;
#pragma unroll
                for (int c = 0; c < 8; ++c) v[h][c] = src[c ^ (r & 7)];
              }
            }
            if (!named_bar_and(1 + grp, 64, got)) {
              ok = false;
              break;
            }
            // the columns' gains (a fold moved to A's side), times 2^e_r below:
            // a·(g·2^e) = fl(a·g)·2^e exactly
            const bool gained = p.a_gain != nullptr;
            float4 gq[8];
            if (gained) {
#pragma unroll
              for (int c = 0; c < 8; ++c) gq[c] = __ldg(reinterpret_cast<const float4*>(p.a_gain + kb * BK) + c);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int r = gt + 64 * h;
              uint4* dhi = reinterpret_cast<uint4*>(base) + r * 4;
              uint4* dlo = reinterpret_cast<uint4*>(base + C::kPartBytes) + r * 4;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float4 v0 = v[h][2 * j], v1 = v[h][2 * j + 1];
                const float s = sc[h];
                float a[8];
                if (gained) {
                  const float4 g0 = gq[2 * j], g1 = gq[2 * j + 1];
                  a[0] = v0.x * (g0.x * s); a[1] = v0.y * (g0.y * s); a[2] = v0.z * (g0.z * s); a[3] = v0.w * (g0.w * s);
                  a[4] = v1.x * (g1.x * s); a[5] = v1.y * (g1.y * s); a[6] = v1.z * (g1.z * s); a[7] = v1.w * (g1.w * s);
                } else {
                  a[0] = v0.x * s; a[1] = v0.y * s; a[2] = v0.z * s; a[3] = v0.w * s;
                  a[4] = v1.x * s; a[5] = v1.y * s; a[6] = v1.z * s; a[7] = v1.w * s;
                }
                // hi: a's top 11 significant bits (exact in fp16 above 2^-14,
                // rounded on the subnormal grid below, as lo is: 2^-24 at
                // most for the two, 2^-38 of the row bound); lo = a − hi
                // (exact), rounded to fp16
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float h0 = tf32_hi(a[2 * q]), h1 = tf32_hi(a[2 * q + 1]);
                  hw[q] = pack_f16x2(h0, h1);
                  lw[q] = pack_f16x2(a[2 * q] - h0, a[2 * q + 1] - h1);
                }
                const int pj = j ^ ((r >> 1) & 3);
                dhi[pj] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                dlo[pj] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
              }
            }
            fence_proxy_async_smem();  // generic-proxy writes → visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(mapa_shared(ready_bar(stage), 0));
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
    } else {
    for (int tile = pair; tile < ntiles && !*abort_flag; tile += npairs) {
      bool ok = true;
      for (int kb = 0; kb < p.nk; ++kb) {
        if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err, kDevTimeoutFull)) {
          ok = false;
          break;
        }
        if (CV) {
          const float4* src = reinterpret_cast<const float4*>(smem + size_t(stage) * C::kStageBytes);
          float4* dst = reinterpret_cast<float4*>(smem + size_t(stage) * C::kStageBytes + C::kABytes);
#pragma unroll
          for (int q = 0; q < int(C::kABytes / 16 / 128); ++q) {
            const float4 v = src[q * 128 + ct];
            dst[q * 128 + ct] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
          }
          fence_proxy_async_smem();  // generic-proxy writes → visible to the tensor core
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(ready_bar(stage), 0));
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
    }
  } else {
    // -------------------------------------------------- epilogue (warps 2..5)
    const int quad = warp & 3;
    EpiStage es{epi_smem + size_t(warp - 2) * kEpiWarpBytes, 0};
    int local = 0;
    for (int tile = pair; tile < ntiles; tile += npairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_par = uint32_t(local >> 1) & 1u;
      const bool got = mbar_wait_cluster(accf_bar(acc), acc_par, abort_flag, p.err, kDevTimeoutAccFull);
      if (!__all_sync(0xffffffffu, got)) break;  // warp-uniform before the collective tcgen05.ld
      tc_fence_after();
      const int tm = tile / p.ntn, tn = tile % p.ntn;
      const uint32_t taddr = tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN);
      epilogue_tile<BN>(p, om, taddr, tm * 256 + int(rank) * 128 + quad * 32, tn, es);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(acce_bar(acc), 0));
    }
    if (lane == 0) tma_store_wait_read<0>();  // staging read before the CTA's shared memory goes away
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA releases TMEM or exits while its pair may still use it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encode() { return tensor_map_encoder(&g_encode); }

// Row-major [rows, cols] fp32 matrix, tiles of [box_rows × bk] whose rows of
// bk·4 bytes are swizzled to match the MMA descriptors (128 or 64 bytes).
int make_map(CUtensorMap* m, const float* ptr, int64_t rows, int64_t cols, int64_t ld,
             int box_rows, int bk) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0)
    return set_error(FG_EINVAL, "GEMM operand %p is not 16-byte aligned", (const void*)ptr);
  if (ld % 4 != 0) return set_error(FG_EINVAL, "GEMM row stride %lld is not a multiple of 4 floats", (long long)ld);
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 4};
  cuuint32_t box[2] = {cuuint32_t(bk), cuuint32_t(box_rows)};
  cuuint32_t es[2] = {1u, 1u};
  const CUtensorMapSwizzle sw = bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box,
                        es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FG_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return FG_OK;
}

// Row-major [rows, cols] bf16 matrix, [32 × 32] boxes with 64-byte swizzling.
int make_map_bf16(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld) {
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FG_ECUDA, "cuTensorMapEncodeTiled (bf16) failed (%d)", int(r));
  return FG_OK;
}

// Row-major [rows, cols] fp16 matrix, [box_rows × 32] boxes with 64-byte
// swizzling (the split-fp16 B operand).
int make_map_f16(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || ld % 8 != 0)
    return set_error(FG_EINVAL, "fp16 GEMM operand %p / row stride %lld not 16-byte aligned", ptr, (long long)ld);
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {32u, cuuint32_t(box_rows)};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FG_ECUDA, "cuTensorMapEncodeTiled (fp16) failed (%d)", int(r));
  return FG_OK;
}

// TMA-store maps for the epilogue's outputs ([32 × 32] fp32 boxes, or the
// attention operands' bf16 parts) where the output allows them (16-byte
// aligned, row stride a multiple of 4 floats); other outputs are written by
// direct row stores.
int prepare_out_maps(const GemmArgs& g, KParams& kp, OutMaps* om) {
  auto ok = [](const float* ptr, int64_t ld) {
    return ptr != nullptr && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ld % 4 == 0;
  };
  kp.tma_out = 0;
  kp.tma_out_lo = 0;
  kp.tma_qk = 0;
  kp.tma_out16 = 0;
  if (g.epi.out16) {
    const GemmEpilogue& e = g.epi;
    if (!e.geglu || !e.out16_lo || (reinterpret_cast<uintptr_t>(e.out16) & 15) != 0 ||
        (reinterpret_cast<uintptr_t>(e.out16_lo) & 15) != 0 || kp.Nout % 8 != 0)
      return set_error(FG_EINVAL, "gemm: fp16-parts output needs the gated epilogue and aligned buffers");
    FG_TRY(make_map_f16(&om->m[0], e.out16, g.M, kp.Nout, kp.Nout, 32));
    FG_TRY(make_map_f16(&om->m[1], e.out16_lo, g.M, kp.Nout, kp.Nout, 32));
    kp.tma_out16 = 1;
    return FG_OK;
  }
  if (g.epi.qkv_attn) {
    const GemmEpilogue& e = g.epi;
    const void* ps[4] = {e.q_hi, e.q_lo, e.k_hi, e.k_lo};
    for (const void* q : ps)
      if (!q || (reinterpret_cast<uintptr_t>(q) & 15) != 0) return FG_OK;
    const int64_t wq = int64_t(e.Hq) * 256, wk = int64_t(e.Hkv) * 256;
    FG_TRY(make_map_bf16(&om->m[0], e.q_hi, g.M, wq, wq));
    FG_TRY(make_map_bf16(&om->m[1], e.q_lo, g.M, wq, wq));
    FG_TRY(make_map_bf16(&om->m[2], e.k_hi, g.M, wk, wk));
    FG_TRY(make_map_bf16(&om->m[3], e.k_lo, g.M, wk, wk));
    kp.tma_qk = 1;
    return FG_OK;
  }
  if (ok(g.epi.out, g.epi.ldo)) {
    FG_TRY(make_map(&om->m[0], g.epi.out, g.M, kp.Nout, g.epi.ldo, 32, 32));
    kp.tma_out = 1;
  }
  if (ok(g.epi.out_lo, g.epi.ldo_lo)) {
    FG_TRY(make_map(&om->m[1], g.epi.out_lo, g.M, kp.Nout, g.epi.ldo_lo, 32, 32));
    kp.tma_out_lo = 1;
  }
  return FG_OK;
}

template <int BN, bool SA, bool SB, int BK, bool CV = false>
int launch_variant(const GemmArgs& g, KParams kp, int* dev_err, cudaStream_t stream) {
  using C = Cfg<BN, SA, SB, BK, CV>;
  CUtensorMap mA, mAlo, mB, mBlo;
  FG_TRY(make_map(&mA, g.A, g.M, g.K, g.lda, kBM, BK));
  FG_TRY(make_map(&mB, g.B, g.Nb, g.K, g.ldb, BN, BK));
  if (SA) FG_TRY(make_map(&mAlo, g.A_lo, g.M, g.K, g.lda, kBM, BK)); else mAlo = mA;
  if (SB) FG_TRY(make_map(&mBlo, g.B_lo, g.Nb, g.K, g.ldb, BN, BK)); else mBlo = mB;
  OutMaps om;
  for (CUtensorMap& m : om.m) m = mA;
  FG_TRY(prepare_out_maps(g, kp, &om));
  auto kern = gemm_tf32_kernel<BN, SA, SB, BK, CV>;
  static std::atomic<bool> attr_set[64];  // per device; concurrent host threads may launch
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    FG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(C::kSmemBytes)));
    attr_set[dev & 63] = true;
  }
  const int ntiles = kp.ntm * kp.ntn;
  const int grid = std::max(1, std::min(ntiles, sm_count()));
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(mA, mAlo, mB, mBlo, om, kp);
  FG_CUDA_TRY(cudaGetLastError());
  (void)dev_err;
  return FG_OK;
}

// CTA-pair kernel: 256-row M tiles, 256-column N tiles.
template <bool CV, bool SA = false, bool SB = false, bool H16 = false>
int launch_pair(const GemmArgs& g, KParams kp, int* dev_err, cudaStream_t stream) {
  using C = PairCfg<CV, SA, SB, H16>;
  CUtensorMap mA, mAlo, mB, mBlo;
  if (H16 && SA) {
    FG_TRY(make_map_f16(&mA, g.A16, g.M, g.K, g.lda, 128));
    FG_TRY(make_map_f16(&mAlo, g.A16_lo, g.M, g.K, g.lda, 128));
  } else {
    FG_TRY(make_map(&mA, g.A, g.M, g.K, g.lda, 128, 32));
    if (SA) FG_TRY(make_map(&mAlo, g.A_lo, g.M, g.K, g.lda, 128, 32)); else mAlo = mA;
  }
  if (H16) FG_TRY(make_map_f16(&mB, g.B16, g.Nb, g.K, g.ldb, 128));
  else FG_TRY(make_map(&mB, g.B, g.Nb, g.K, g.ldb, 128, 32));
  if (SB && H16) FG_TRY(make_map_f16(&mBlo, g.B16_lo, g.Nb, g.K, g.ldb, 128));
  else if (SB) FG_TRY(make_map(&mBlo, g.B_lo, g.Nb, g.K, g.ldb, 128, 32));
  else mBlo = mB;
  OutMaps om;
  for (CUtensorMap& m : om.m) m = mA;
  FG_TRY(prepare_out_maps(g, kp, &om));
  kp.ntm = (g.M + 255) / 256;
  kp.h16 = H16 ? 1 : 0;
  auto kern = gemm_pair_kernel<CV, SA, SB, H16>;
  static std::atomic<bool> attr_set[64];  // per device; max_pairs is stored before attr_set
  static std::atomic<int> max_pairs[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (!attr_set[dev & 63]) {
    FG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(C::kSmemBytes)));
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    int n = 0;
    FG_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    if (n < 1) return set_error(FG_ECUDA, "gemm: no CTA pair of this kernel fits on an SM pair");
    max_pairs[dev & 63] = n;
    attr_set[dev & 63] = true;
  }
  const int ntiles = kp.ntm * kp.ntn;
  cfg.gridDim = dim3(2 * std::max(1, std::min(ntiles, max_pairs[dev & 63].load())));
  FG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, mA, mAlo, mB, mBlo, om, kp));
  (void)dev_err;
  return FG_OK;
}

// Pair kernel for 256-wide N tiles (M of at least one pair tile).
bool use_pair(const GemmArgs& g) { return g.M >= 256; }

// A's low part: none (plain TF32), loaded (SA), or computed in shared memory (CV).
template <int BN, bool SB>
int launch_a_mode(const GemmArgs& g, const KParams& kp, int* dev_err, cudaStream_t stream) {
  constexpr int BK = 32;
  if (g.A_lo) return launch_variant<BN, true, SB, BK, false>(g, kp, dev_err, stream);
  if (g.a_lo_smem) return launch_variant<BN, false, SB, BK, true>(g, kp, dev_err, stream);
  return launch_variant<BN, false, SB, BK, false>(g, kp, dev_err, stream);
}

template <int BN>
int launch_b_mode(const GemmArgs& g, const KParams& kp, int* dev_err, cudaStream_t stream) {
  if (g.B_lo) return launch_a_mode<BN, true>(g, kp, dev_err, stream);
  return launch_a_mode<BN, false>(g, kp, dev_err, stream);
}

int dispatch(const GemmArgs& g, KParams& kp, int* dev_err, cudaStream_t stream) {
  kp.nk = (g.K + 31) / 32;
  // split-fp16 with A's parts made by A's producer (fp16 [M, lda], 16-byte rows)
  if (g.A16) {
    if (!g.A16_lo || !g.B16 || !use_pair(g) || !(g.epi.geglu || g.Nb > 128) || g.lda % 8 != 0 || g.ldb % 8 != 0 ||
        g.a_gain || (g.a_exp_rs && !kp.a_rs))
      return set_error(FG_EINVAL, "gemm: pre-split fp16 A needs the split-fp16 pair kernel");
    if (g.epi.geglu) {
      kp.Nout = g.Nb / 2;
      kp.ntn = g.Nb / 256;
    } else {
      kp.Nout = g.Nb;
      kp.ntn = (g.Nb + 255) / 256;
    }
    if (g.B16_lo) return launch_pair<false, true, true, true>(g, kp, dev_err, stream);
    return launch_pair<false, true, false, true>(g, kp, dev_err, stream);
  }
  // split-fp16 where B has an exact fp16 form and A's parts are made here
  const bool h16 = g.B16 && g.a_lo_smem && !g.A_lo && (g.ldb % 8) == 0 && (!g.a_exp_rs || kp.a_rs) &&
                   (!g.a_gain || (g.K % 32 == 0 && (reinterpret_cast<uintptr_t>(g.a_gain) & 15) == 0)) &&
                   use_pair(g) && (g.epi.geglu || g.Nb > 128);
  if (!h16 && !g.B) return set_error(FG_EINVAL, "gemm: B has only an fp16 form and the split-fp16 kernel does not apply");
  if (g.epi.geglu) {
    kp.Nout = g.Nb / 2;
    kp.ntn = g.Nb / 256;
  } else {
    kp.Nout = g.Nb;
    if (g.Nb <= 128) {
      kp.ntn = 1;
      return launch_b_mode<128>(g, kp, dev_err, stream);
    }
    kp.ntn = (g.Nb + 255) / 256;
  }
  if (use_pair(g)) {
    if (h16) {
      if (g.B16_lo) return launch_pair<true, false, true, true>(g, kp, dev_err, stream);
      return launch_pair<true, false, false, true>(g, kp, dev_err, stream);
    }
    if (g.B_lo) {
      if (g.A_lo) return launch_pair<false, true, true>(g, kp, dev_err, stream);
      if (g.a_lo_smem) return launch_pair<true, false, true>(g, kp, dev_err, stream);
      // B_lo without any A low part: the single-CTA kernel below
    } else {
      if (g.A_lo) return launch_pair<false, true>(g, kp, dev_err, stream);
      return g.a_lo_smem ? launch_pair<true>(g, kp, dev_err, stream) : launch_pair<false>(g, kp, dev_err, stream);
    }
  }
  return launch_b_mode<256>(g, kp, dev_err, stream);
}

}  // namespace

bool gemm_h16_applies(int M) {
  GemmArgs g;
  g.M = M;
  return use_pair(g);
}

int gemm_tn(const GemmArgs& g, int* dev_err, cudaStream_t stream) {
  if (g.M <= 0 || g.Nb <= 0 || g.K <= 0) {
    if (g.M == 0 || g.Nb == 0) return FG_OK;
    return set_error(FG_EINVAL, "gemm: bad shape M=%d Nb=%d K=%d", g.M, g.Nb, g.K);
  }
  if (g.epi.out == nullptr && !g.epi.qkv_attn && !g.epi.out16) return set_error(FG_EINVAL, "gemm: no output");
  if (g.epi.qkv_attn && (g.Nb != (g.epi.Hq + 2 * g.epi.Hkv) * 256 || g.epi.T <= 0))
    return set_error(FG_EINVAL, "gemm: attention-operand epilogue needs 256-wide heads");
  if (g.epi.geglu && (g.Nb % 256) != 0)
    return set_error(FG_EINVAL, "gemm: gated product needs B rows in multiples of 256, got %d", g.Nb);
  FG_TRY(get_encode());
  KParams kp;
  kp.M = g.M;
  kp.K = g.K;
  kp.e = g.epi;
  kp.err = dev_err;
  kp.ntm = (g.M + kBM - 1) / kBM;
  kp.h16 = 0;
  kp.a_exp = g.a_exp;
  kp.a_exp_rs = g.a_exp_rs;
  kp.b_exp = g.b_exp;
  kp.b_exp_dev = g.b_exp_dev;
  // all-zero gains make A zero: any exponent serves, keep the bound positive
  // (a_bound_gain: the gain a producer applied to pre-split A parts)
  kp.a_norm_k = sqrtf(float(g.K)) * (g.a_gain && g.a_gain_max > 0.f ? g.a_gain_max
                                     : g.a_bound_gain > 0.f ? g.a_bound_gain : 1.f);
  kp.a_rs = g.a_rs ? g.a_rs : g.epi.rowscale;
  kp.a_gain = g.a_gain;
  return dispatch(g, kp, dev_err, stream);
}

// ---------------------------------------------------------------- helpers
namespace {
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, int64_t n, int* any) {
  int found = 0;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float v = x[i];
    const float h = tf32_hi(v);
    const float l = v - h;
    if (hi) hi[i] = h;
    if (lo) lo[i] = l;
    found |= (l != 0.f);
  }
  if (any && __any_sync(0xffffffffu, found) && (threadIdx.x & 31) == 0) atomicOr(any, 1);
}

__global__ void transpose_kernel(const float* __restrict__ src, int64_t lds, int64_t rows,
                                 int64_t cols, float* __restrict__ dst, int64_t ldd) {
  __shared__ float tile[32][33];
  const int64_t r0 = int64_t(blockIdx.y) * 32, c0 = int64_t(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * lds + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * ldd + r] = tile[threadIdx.x][i];
  }
}
}  // namespace

namespace {
// |x| maximum as float bits (non-negative floats order like their bits)
__global__ void abs_max_kernel(const float* __restrict__ x, int64_t ld, int64_t rows, int64_t cols,
                               unsigned* __restrict__ out) {
  float m = 0.f;
  const int64_t total = rows * cols;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(x[(e / cols) * ld + e % cols]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

__global__ void split_f16_kernel(const float* __restrict__ x, int64_t ld, int64_t rows, int64_t cols,
                                 const unsigned* __restrict__ maxbits, uint16_t* __restrict__ hi,
                                 uint16_t* __restrict__ lo, int64_t ldo, int* __restrict__ exp_out) {
  const float mx = __uint_as_float(*maxbits);
  // max·2^t < 2^14: both parts finite, every element down to 2^-17 of the
  // maximum keeps 22 significant bits
  const int t = mx > 0.f && isfinite(mx) ? max(-60, min(60, 13 - ilogbf(mx))) : 0;
  if (blockIdx.x == 0 && threadIdx.x == 0) *exp_out = t;
  const float sc = pow2f(t);
  const int64_t total = rows * cols;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / cols, c = e % cols;
    const float v = x[r * ld + c] * sc;
    const float h = tf32_hi(v);
    hi[r * ldo + c] = __half_as_ushort(__float2half_rn(h));
    lo[r * ldo + c] = __half_as_ushort(__float2half_rn(v - h));
  }
}

// one warp per row
__global__ void row_inv_rms_kernel(const float* __restrict__ x, int64_t ld, int64_t rows, int64_t cols,
                                   float* __restrict__ rs) {
  const int64_t r = blockIdx.x * int64_t(blockDim.x / 32) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
  for (int64_t c = lane; c < cols; c += 32) {
    const float v = x[r * ld + c];
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) rs[r] = 1.f / sqrtf(fmaxf(ss / float(cols), 1e-30f));
}
}  // namespace

int split_f16_parts(const float* x, int64_t ld, int64_t rows, int64_t cols, uint16_t* hi, uint16_t* lo,
                    int64_t ldo, unsigned* scratch_max, int* exp_out, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return FG_OK;
  FG_CUDA_TRY(cudaMemsetAsync(scratch_max, 0, sizeof(unsigned), stream));
  const int64_t total = rows * cols;
  const int grid = int(std::min<int64_t>((total + 255) / 256, int64_t(sm_count()) * 8));
  abs_max_kernel<<<grid, 256, 0, stream>>>(x, ld, rows, cols, scratch_max);
  FG_CUDA_TRY(cudaGetLastError());
  split_f16_kernel<<<grid, 256, 0, stream>>>(x, ld, rows, cols, scratch_max, hi, lo, ldo, exp_out);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int row_inv_rms(const float* x, int64_t ld, int64_t rows, int64_t cols, float* rs, cudaStream_t stream) {
  if (rows <= 0) return FG_OK;
  const int64_t blocks = (rows + 7) / 8;
  row_inv_rms_kernel<<<unsigned(blocks), 256, 0, stream>>>(x, ld, rows, cols, rs);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int split_tf32(const float* x, float* hi, float* lo, int64_t n, int* any, cudaStream_t stream) {
  if (n <= 0) return FG_OK;
  const int threads = 256;
  const int64_t want = (n + threads - 1) / threads;
  const int grid = int(std::min<int64_t>(want, int64_t(sm_count()) * 16));
  split_tf32_kernel<<<grid, threads, 0, stream>>>(x, hi, lo, n, any);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int transpose_f32(const float* src, int64_t lds, int64_t rows, int64_t cols, float* dst,
                  int64_t ldd, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return FG_OK;
  dim3 grid(unsigned((cols + 31) / 32), unsigned((rows + 31) / 32));
  transpose_kernel<<<grid, dim3(32, 8), 0, stream>>>(src, lds, rows, cols, dst, ldd);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

}  // namespace fg
