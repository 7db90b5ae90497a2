// Flash attention on the tcgen05 tensor cores for head_dim 256 and 512,
// fp32 inputs carried as split-bf16 operands.
//
// Replaces attentionFused / AttentionBlock (tensor/attention.go:130-287,
// internal/blas/attention.go:61-136) on the encoder path. Every fp32
// operand x is held as hi = bf16(x) and lo = bf16(x − hi) (x − hi − lo is
// below 2^-17·|x|); each product accumulates hi·hi + hi·lo + lo·hi in FP32
// TMEM, three kind::f16 MMAs — the cost of 1.5 TF32 passes, with products
// good to ~2^-16 relative. (An fp32 Q tile of 128 rows × 256 is 128 KB per
// part: a TF32 hi/lo pair does not fit shared memory beside the K/V ring,
// the bf16 pair does.)
//
// One CTA per (query tile of 128 rows, query head, sequence), 10 warps:
//   warp 0      TMA producer: Q (hi/lo, resident), then per key tile the K
//               d-chunks and the Vᵀ (d-half × key-half) chunks through a
//               3-stage ring of 32 KB, in the order the MMA warp uses them.
//   warp 1      TMEM allocation (512 columns) and the MMA issuer:
//               S_j = Q·K_jᵀ into one of two 128-column S buffers while the
//               softmax warps work on S_{j−1}; then O += P_{j−1}·V_{j−1}
//               with P read from TMEM (A operand), O in columns 256..511.
//   warps 2..9  softmax, two warps per TMEM lane quadrant (one query row
//               per thread, 64 of the 128 score columns each): visibility by
//               index arithmetic (padding: j < len; sliding layers:
//               |i−j| < window; masked scores become -inf while the row
//               maximum is taken), running max with lazy rescaling (O is
//               rescaled in TMEM only when the max grows by more than 2^8),
//               P = exp2 written back over S as packed bf16 hi/lo; the final
//               1/Σ and the store.
// Head_dim 512 (EmbeddingGemma 2's global layers): Q (256 KB as split
// bf16) does not fit beside the ring, so its d-chunks are streamed through
// the ring with the K chunks they meet, and each CTA produces one 256-wide
// half of the output (O in TMEM stays 256 columns), the two halves of a
// head being two CTAs (blockIdx.y = 2·head + half) that both compute S.
// Key tiles outside a query tile's window or past the sequence length are
// never loaded. Masked keys get weight exactly 0, as the reference's
// flushing exp gives them (internal/kernel/generic.go:283-291).
#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cudaTypedefs.h>

#include "fg_internal.h"
#include "fg_kernels.cuh"
#include "fg_ptx.cuh"

namespace fg {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode_bf16 = nullptr;

constexpr int kQ = 128;    // query rows per CTA
constexpr int kKT = 128;   // keys per tile
constexpr int kD = 256;    // output columns per CTA (the head dimension, or half of 512)
constexpr int kStages = 3;
constexpr uint32_t kChunk = 128 * 64 * 2;           // [128 rows × 64 bf16] = 16 KB
constexpr uint32_t kQBytes = 2 * 4 * kChunk;        // Q hi/lo × 4 d-chunks = 128 KB
constexpr uint32_t kStageBytes = 2 * kChunk;        // hi + lo chunk = 32 KB
// Q, the K/V ring, 256 bytes of barriers, the half-row maxima [8 warps × 32]
constexpr size_t kSmem = 1024 + kQBytes + kStages * kStageBytes + 256 + 1024;
constexpr int kThreads = 320;  // producer, MMA issuer, 8 softmax warps
constexpr uint32_t kIdesc = idesc_bf16(128, 128);
constexpr float kRescaleLog2 = 8.f;  // rescale O when the max grows by more than 2^8

struct Params {
  int B, T, S, Hq, Hkv;
  int window;
  float scale_log2;  // attention scale · log2(e)
  const int32_t* qlen;  // rows computed per sequence (null: T); later rows are written as 0
  const int32_t* klen;  // visible keys per sequence (null: S)
  float* out;
  float* out_lo;
  int64_t osb, osh, ost;
  int* err;
  int tma_out, tma_out_lo;  // out / out_lo written by TMA stores (maps mO / mOlo)
  int tma_out16;            // the output's fp16 parts written instead (maps mO / mOlo: hi / lo)
  float out16_scale;        // 2^out16_exp
  uint16_t *out16, *out16_lo;  // the same parts (zero rows are written directly)
};

// NC 64-column d-chunks per head (4: head_dim 256, Q resident; 8: head_dim
// 512, Q streamed, QS).

__device__ __forceinline__ bool waitb(uint32_t bar, uint32_t par, volatile int* ab, int* err, int code) {
  return mbar_wait(bar, par, ab, err, code);
}

template <int NC, bool QS>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap mQ0, const __grid_constant__ CUtensorMap mQ1,
                   const __grid_constant__ CUtensorMap mK0, const __grid_constant__ CUtensorMap mK1,
                   const __grid_constant__ CUtensorMap mV0, const __grid_constant__ CUtensorMap mV1,
                   const __grid_constant__ CUtensorMap mO, const __grid_constant__ CUtensorMap mOlo,
                   const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // [part][chunk] 16 KB each
  uint8_t* sRing = smem + kQBytes;          // [stage][part] 16 KB each
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + kStages * kStageBytes);
  // bars: 0 Q d-chunk 0 | 1..3 kv_full | 4..6 kv_empty | 7,8 s_full | 9,10 p_full |
  //       11,12 s_free | 13 o_prog | 14 o_final | 15 drain | 16..18 Q d-chunks 1..3 |
  //       19 row-sum halves exchanged | 20..27 half-row maxima written by
  //       both warps of a quadrant (quad · 2 + S buffer)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 28);
  float* red_max = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);  // [8 warps][32 rows]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  constexpr int Dh = NC * 64;  // head dimension
  const int qt = blockIdx.x, b = blockIdx.z;
  const int h = QS ? int(blockIdx.y >> 1) : int(blockIdx.y);
  const int oh = QS ? int(blockIdx.y & 1) : 0;  // output half of a 512-wide head
  const int hk = h / (p.Hq / p.Hkv);
  const int i0 = qt * kQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qlen = p.qlen ? min(p.qlen[b], p.T) : p.T;
  const int klen = p.klen ? max(0, min(p.klen[b], p.S)) : p.S;
  float* obase = p.out + b * p.osb + h * p.osh + oh * kD;
  float* olbase = p.out_lo ? p.out_lo + b * p.osb + h * p.osh + oh * kD : nullptr;
  int kbeg = 0, kend = klen;
  if (p.window > 0) {
    kbeg = max(0, i0 - p.window + 1);
    kend = min(klen, i0 + kQ - 1 + p.window);
  }

  if (i0 >= qlen || kend <= kbeg) {  // no row to compute or no visible key: zeros
    for (int r = warp; r < kQ; r += kThreads / 32) {
      const int i = i0 + r;
      if (i >= p.T) break;
      if (p.tma_out16) {
        // kD fp16 of hi and of lo per row, 16 bytes a lane
        const int64_t off = b * p.osb + h * p.osh + oh * kD + int64_t(i) * p.ost;
        for (int c = lane * 8; c < kD; c += 256) {
          *reinterpret_cast<uint4*>(p.out16 + off + c) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(p.out16_lo + off + c) = make_uint4(0u, 0u, 0u, 0u);
        }
        continue;
      }
      float* o = obase + i * p.ost;
      float* ol = olbase ? olbase + i * p.ost : nullptr;
      for (int c = lane; c < kD; c += 32) {
        o[c] = 0.f;
        if (ol) ol[c] = 0.f;
      }
    }
    return;
  }
  const int kt0 = kbeg / kKT;
  const int ntiles = (kend + kKT - 1) / kKT - kt0;

  auto bar = [&](int k) { return smem_u32(&bars[k]); };
  // Q arrives per 64-column d-chunk (hi and lo), so the first score MMAs
  // start when their chunk has landed rather than after all 128 KB.
  auto q_bar = [&](int c) { return c == 0 ? bar(0) : bar(15 + c); };
  const uint32_t s_full0 = bar(7), p_full0 = bar(9), s_free0 = bar(11);
  const uint32_t o_prog = bar(13), o_final = bar(14), drain = bar(15);

  if (threadIdx.x == 0) {
    for (int c = 0; c < 4; ++c) mbar_init(q_bar(c), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(1 + s), 1);
      mbar_init(bar(4 + s), 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(bar(7 + k), 1);
      mbar_init(bar(9 + k), 256);
      mbar_init(bar(11 + k), 1);
    }
    mbar_init(o_prog, 1);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    mbar_init(bar(19), 8);  // row-sum halves written, one arrive per softmax warp
    for (int k = 0; k < 8; ++k) mbar_init(bar(20 + k), 2);  // one arrive per warp of the pair
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&mQ0);
      tma_prefetch_desc(&mK0);
      tma_prefetch_desc(&mV0);
      const int qrow = b * p.T + i0;
      if (!QS) {
        for (int c = 0; c < 4; ++c) {
          mbar_arrive_expect_tx(q_bar(c), 2 * kChunk);
          tma_load_2d(smem_u32(sQ + (0 * 4 + c) * kChunk), &mQ0, q_bar(c), h * Dh + c * 64, qrow);
          tma_load_2d(smem_u32(sQ + (1 * 4 + c) * kChunk), &mQ1, q_bar(c), h * Dh + c * 64, qrow);
        }
      }
      int armed[kStages] = {0, 0, 0};
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      auto next = [&](const CUtensorMap* m0, const CUtensorMap* m1, int x, int y) {
        if (!waitb(bar(4 + stage), phase ^ 1, abort_flag, p.err, kDevTimeoutEmpty)) return false;
        const uint32_t fb = bar(1 + stage);
        mbar_arrive_expect_tx(fb, kStageBytes);
        armed[stage]++;
        uint8_t* dst = sRing + stage * kStageBytes;
        tma_load_2d(smem_u32(dst), m0, fb, x, y);
        tma_load_2d(smem_u32(dst + kChunk), m1, fb, x, y);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
        return true;
      };
      auto load_k = [&](int j) {
        const int key0 = (kt0 + j) * kKT;
        for (int c = 0; c < NC && ok; ++c) {
          if (QS) ok = next(&mQ0, &mQ1, h * Dh + c * 64, qrow);  // Q chunk c, then the K chunk it meets
          if (ok) ok = next(&mK0, &mK1, hk * Dh + c * 64, b * p.S + key0);
        }
      };
      auto load_v = [&](int j) {
        const int key0 = (kt0 + j) * kKT;
        const int vrow = (b * p.Hkv + hk) * Dh + oh * kD;
        for (int dh = 0; dh < 2 && ok; ++dh)
          for (int kh = 0; kh < 2 && ok; ++kh) ok = next(&mV0, &mV1, key0 + kh * 64, vrow + dh * 128);
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        load_k(j);
        if (j >= 1) load_v(j - 1);
      }
      if (ok) load_v(ntiles - 1);
      {
        // Every load issued above lands before the CTA retires, also when
        // another role gave up and left it unconsumed (after a normal run
        // these phases have completed and the waits return at once).
        for (int s = 0; s < kStages; ++s) {
          if (!armed[s]) continue;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(bar(1 + s), uint32_t(armed[s] - 1) & 1u))
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) break;
        }
        for (int c = 0; c < (QS ? 0 : 4); ++c) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(q_bar(c), 0))
            if (globaltimer_ns() - t0 > kWaitTimeoutNs) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued = false;
      auto pv = [&](int jj) {
        const int sb = jj & 1;
        if (!waitb(bar(9 + sb), uint32_t(jj >> 1) & 1u, abort_flag, p.err, kDevTimeoutAccFull)) return false;
        tc_fence_after();
        const uint32_t tP = tmem + uint32_t(sb * 128);
        for (int dh = 0; dh < 2; ++dh) {
          for (int kh = 0; kh < 2; ++kh) {
            if (!waitb(bar(1 + stage), phase, abort_flag, p.err, kDevTimeoutFull)) return false;
            tc_fence_after();
            const uint32_t v0 = smem_u32(sRing + stage * kStageBytes);
            const uint32_t v1 = v0 + kChunk;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              // keys [16m, 16m + 16): P chunk m / 2, hi at its first 16
              // columns, lo at the next 16 (see the softmax's pass 2)
              const int mk = kh * 4 + kk;
              const uint32_t hcol = uint32_t(32 * (mk >> 1) + 8 * (mk & 1));
              const uint64_t b0 = sw128_kmajor_desc(v0 + kk * 32);
              const uint64_t b1 = sw128_kmajor_desc(v1 + kk * 32);
              const uint32_t d = tO + uint32_t(dh * 128);
              const uint32_t first = (jj == 0 && kh == 0 && kk == 0) ? 0u : 1u;
              mma_bf16_ts(d, tP + hcol, b0, kIdesc, first);       // p_hi · v_hi
              mma_bf16_ts(d, tP + hcol, b1, kIdesc, 1u);          // p_hi · v_lo
              mma_bf16_ts(d, tP + hcol + 16, b0, kIdesc, 1u);     // p_lo · v_hi
            }
            mma_commit(bar(4 + stage));
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        mma_commit(bar(11 + sb));  // S/P buffer free
        mma_commit(o_prog);
        return true;
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        const int sb = j & 1;
        if (j >= 2) {
          if (!waitb(bar(11 + sb), uint32_t((j - 2) >> 1) & 1u, abort_flag, p.err, kDevTimeoutAccEmpty)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        const uint32_t tS = tmem + uint32_t(sb * 128);
        for (int c = 0; c < NC && ok; ++c) {
          uint32_t q0, q1;
          int qstage = 0;
          if (QS) {
            // the Q chunk occupies the ring stage before its K chunk
            if (!waitb(bar(1 + stage), phase, abort_flag, p.err, kDevTimeoutFull)) {
              ok = false;
              break;
            }
            qstage = stage;
            q0 = smem_u32(sRing + stage * kStageBytes);
            q1 = q0 + kChunk;
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1;
            }
          } else {
            if (j == 0 && !waitb(q_bar(c), 0, abort_flag, p.err, kDevTimeoutFull)) {
              ok = false;
              break;
            }
            q0 = smem_u32(sQ + c * kChunk);
            q1 = smem_u32(sQ + (4 + c) * kChunk);
          }
          if (!waitb(bar(1 + stage), phase, abort_flag, p.err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k0 = smem_u32(sRing + stage * kStageBytes);
          const uint32_t k1 = k0 + kChunk;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t a0 = sw128_kmajor_desc(q0 + kk * 32);
            const uint64_t a1 = sw128_kmajor_desc(q1 + kk * 32);
            const uint64_t b0 = sw128_kmajor_desc(k0 + kk * 32);
            const uint64_t b1 = sw128_kmajor_desc(k1 + kk * 32);
            mma_bf16_ss(tS, a0, b0, kIdesc, (c | kk) != 0 ? 1u : 0u);  // q_hi · k_hi
            mma_bf16_ss(tS, a0, b1, kIdesc, 1u);                       // q_hi · k_lo
            mma_bf16_ss(tS, a1, b0, kIdesc, 1u);                       // q_lo · k_hi
          }
          issued = true;
          if (QS) mma_commit(bar(4 + qstage));
          mma_commit(bar(4 + stage));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(bar(7 + sb));
        if (j >= 1 && !pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && pv(ntiles - 1)) mma_commit(o_final);
      if (issued) {
        mma_commit(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0))
          if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            atomicCAS(p.err, 0, kDevTimeoutDrain);
            break;
          }
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    // Two warps per TMEM lane quadrant (warps w and w + 4 hold the same 32
    // query rows): each reads its 64 columns of S once, the two half-row
    // maxima meet in shared memory (both warps then hold the same row
    // maximum, so the same running max and rescale decisions), and each
    // handles its half of the columns — exponentials for 64 columns of S,
    // rescaling and output for 128 columns of O.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int i = i0 + r;
    const uint32_t lane_off = uint32_t(quad * 32) << 16;
    // visible keys of row i: [vlo, vhi)
    int vlo = 0, vhi = klen;
    if (p.window > 0) {
      vlo = max(0, i - p.window + 1);
      vhi = min(klen, i + p.window);
    }
    const float c = p.scale_log2;
    float m = -FLT_MAX;
    bool have = false;
    float l = 0.f;  // this warp's columns only; the halves are added at the end
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      const int key0 = (kt0 + j) * kKT;
      const bool got = waitb(bar(7 + sb), uint32_t(j >> 1) & 1u, abort_flag, p.err, kDevTimeoutAccFull);
      if (!__all_sync(0xffffffffu, got)) {  // warp-uniform before the collective tcgen05.ld
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tS = tmem + lane_off + uint32_t(sb * 128);
      const int lo_c = vlo - key0, hi_c = vhi - key0;  // visible columns [lo_c, hi_c)
      const bool full_row = lo_c <= 0 && hi_c >= kKT;
      const int span = max(0, hi_c - lo_c);  // col is visible iff unsigned(col - lo_c) < span
      // pass 1: this warp's 64 columns of S, kept in registers for pass 2,
      // and their maximum over the visible columns in eight chains; the row
      // maximum is the larger of the two warps' halves, exchanged through
      // shared memory (each warp reads and overwrites only its own columns)
      uint32_t sr[2][32];
      tmem_ld_32x32b_x32(tS + uint32_t(half * 64), sr[0]);
      tmem_ld_32x32b_x32(tS + uint32_t(half * 64 + 32), sr[1]);
      tmem_ld_wait();
      float mt8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mt8[u] = -INFINITY;
      if (full_row) {
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int e = 0; e < 32; ++e) mt8[e & 7] = fmaxf(mt8[e & 7], __uint_as_float(sr[q][e]));
      } else {
        // masked scores become -inf here, whose exponential in pass 2 is
        // exactly 0, so pass 2 is the same for every row
        const int c0 = half * 64 - lo_c;  // column e of this warp's half is visible iff unsigned(c0 + e) < span
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const bool in = unsigned(c0 + q * 32 + e) < unsigned(span);
            const float v = in ? __uint_as_float(sr[q][e]) : -INFINITY;
            sr[q][e] = __float_as_uint(v);
            mt8[e & 7] = fmaxf(mt8[e & 7], v);
          }
      }
      const float mh = fmaxf(fmaxf(fmaxf(mt8[0], mt8[1]), fmaxf(mt8[2], mt8[3])),
                             fmaxf(fmaxf(mt8[4], mt8[5]), fmaxf(mt8[6], mt8[7])));
      float mt;
      {
        // the slot is reused every tile: the partner has read the previous
        // tile's value before it arrived on that tile's P barrier
        if (j >= 1) {
          const bool prev = waitb(bar(9 + ((j - 1) & 1)), uint32_t((j - 1) >> 1) & 1u, abort_flag, p.err,
                                  kDevTimeoutAccFull);
          if (!__all_sync(0xffffffffu, prev)) {
            ok = false;
            break;
          }
        }
        red_max[(half * 4 + quad) * 32 + lane] = mh;
        const uint32_t mx_bar = bar(20 + quad * 2 + sb);
        __syncwarp();
        if (lane == 0) mbar_arrive(mx_bar);
        const bool both = waitb(mx_bar, uint32_t(j >> 1) & 1u, abort_flag, p.err, kDevTimeoutAccFull);
        if (!__all_sync(0xffffffffu, both)) {
          ok = false;
          break;
        }
        mt = fmaxf(mh, red_max[((1 - half) * 4 + quad) * 32 + lane]);
      }
      const bool any = lo_c < hi_c && lo_c < kKT && hi_c > 0;
      float factor = 1.f;
      if (any) {
        if (!have) {
          m = mt;
          have = true;
        } else if ((mt - m) * c > kRescaleLog2) {
          factor = ex2_approx((m - mt) * c);
          m = mt;
        }
      }
      // O rows rescale (this warp's 128 columns): the whole warp takes part
      // if any lane needs it
      const bool need = factor != 1.f;
      if (__any_sync(0xffffffffu, need) && j > 0) {
        const bool done = waitb(o_prog, uint32_t(j - 1) & 1u, abort_flag, p.err, kDevTimeoutAccFull);
        if (!__all_sync(0xffffffffu, done)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t ov[32];
          const uint32_t ta = tO + lane_off + uint32_t(half * 128 + ch * 32);
          tmem_ld_32x32b_x32(ta, ov);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * factor);
          tmem_st_32x32b_x32(ta, ov);
        }
        tmem_st_wait();
      }
      l *= factor;
      // a row with no visible key so far has only -inf scores: 0 keeps their
      // exponentials 0 (m·c of the initial -FLT_MAX could overflow to -inf)
      const float mc = have ? m * c : 0.f;
      // pass 2: probabilities of this warp's 64 columns, split into packed
      // bf16 hi / lo. The 32-column chunk q of S is overwritten by its own
      // P: hi (16 columns of bf16 pairs) at columns 32q.., lo at 32q+16..
      float ps8[8];  // eight independent partial sums
#pragma unroll
      for (int u = 0; u < 8; ++u) ps8[u] = 0.f;
      // (masked scores are -inf since pass 1 and mc is finite, so masked
      // keys and rows with no visible key so far get exact zeros)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t hw[16], lw[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = ex2_approx(fmaf(__uint_as_float(sr[q][2 * e]), c, -mc));
          const float bb = ex2_approx(fmaf(__uint_as_float(sr[q][2 * e + 1]), c, -mc));
          ps8[e & 7] += a + bb;
          const uint32_t h2 = pack_bf16x2(a, bb);  // RN bf16 of both, a in the low half
          const float ah = __uint_as_float(h2 << 16), bh = __uint_as_float(h2 & 0xffff0000u);
          hw[e] = h2;
          lw[e] = pack_bf16x2(a - ah, bb - bh);
        }
        const uint32_t cq = uint32_t((half * 2 + q) * 32);
        tmem_st_32x32b_x16(tS + cq, hw);
        tmem_st_32x32b_x16(tS + cq + 16, lw);
      }
      l += ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar(9 + sb));
    }
    // ---------------------------------------------------------- epilogue
    const bool fin = ok && waitb(o_final, 0, abort_flag, p.err, kDevTimeoutAccFull);
    if (__all_sync(0xffffffffu, fin)) {
      tc_fence_after();
      // row sum = both halves' sums (l of the other warp of the quadrant,
      // through the K/V ring, free now that every MMA has completed)
      float* red = reinterpret_cast<float*>(sRing);
      red[(half * 4 + quad) * 32 + lane] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(19));  // a bounded wait, unlike a named barrier, cannot hang
      waitb(bar(19), 0, abort_flag, p.err, kDevTimeoutAccFull);
      const float l_lo = red[quad * 32 + lane], l_hi = red[(4 + quad) * 32 + lane];
      const float lsum = l_lo + l_hi;  // same order in both warps
      const bool row_ok = i < p.T;
      const float inv = (i < qlen && lsum > 0.f) ? 1.f / lsum : 0.f;
      const int col_base = half * 128;  // this warp's output columns
      if (p.tma_out16) {
        // The next product's fp16 parts of the warp's 32 rows × 128 columns:
        // a = out·2^e cut as the GEMM converters cut A, four 32-column
        // chunks of [32 × 32] hi and lo boxes (64-byte rows and swizzle) in
        // the warp's 16 KB of the Q region, then TMA stores.
        uint8_t* stg = sQ + size_t(warp - 2) * 16384;
        const int tw = i0 + quad * 32;
        const float sc = p.out16_scale;
        const int sw = (lane >> 1) & 3;
#pragma unroll 1
        for (int ch = 0; ch < 4; ch += 2) {
          uint32_t ov[2][32];
          tmem_ld_32x32b_x32(tO + lane_off + uint32_t(col_base + ch * 32), ov[0]);
          tmem_ld_32x32b_x32(tO + lane_off + uint32_t(col_base + ch * 32 + 32), ov[1]);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            uint32_t hw[16], lw[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const float a0 = (__uint_as_float(ov[u][2 * q]) * inv) * sc;
              const float a1 = (__uint_as_float(ov[u][2 * q + 1]) * inv) * sc;
              const float h0 = tf32_hi(a0), h1 = tf32_hi(a1);
              hw[q] = pack_f16x2(h0, h1);
              lw[q] = pack_f16x2(a0 - h0, a1 - h1);
            }
            uint4* rh = reinterpret_cast<uint4*>(stg + (ch + u) * 4096 + lane * 64);
            uint4* rl = reinterpret_cast<uint4*>(stg + (ch + u) * 4096 + 2048 + lane * 64);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              rh[j ^ sw] = make_uint4(hw[4 * j], hw[4 * j + 1], hw[4 * j + 2], hw[4 * j + 3]);
              rl[j ^ sw] = make_uint4(lw[4 * j], lw[4 * j + 1], lw[4 * j + 2], lw[4 * j + 3]);
            }
          }
          // this pair of chunks goes out while the next is staged
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && tw < p.T) {
            for (int u = 0; u < 2; ++u) {
              const int col = h * Dh + oh * kD + col_base + (ch + u) * 32;
              tma_store_3d(&mO, smem_u32(stg + (ch + u) * 4096), col, tw, b);
              tma_store_3d(&mOlo, smem_u32(stg + (ch + u) * 4096 + 2048), col, tw, b);
            }
            tma_store_commit();
          }
        }
        if (lane == 0) tma_store_wait_read<0>();  // the boxes are read; the writes complete on their own
        __syncwarp();
      } else if (p.tma_out) {
        // The warp's 32 rows × 128 columns as four [32 × 32] boxes in its
        // 16 KB of the Q region (every MMA that read Q has completed), then
        // TMA stores; rows past the sequence end fall outside the map.
        uint8_t* stg = sQ + size_t(warp - 2) * 16384;
        const int tw = i0 + quad * 32;
        const int parts = olbase ? 2 : 1;
#pragma unroll 1
        for (int part = 0; part < parts; ++part) {
          if (part == 1) {
            if (lane == 0) tma_store_wait_read<0>();  // the hi boxes have been read
            __syncwarp();
          }
#pragma unroll 1
          for (int ch = 0; ch < 4; ch += 2) {
            uint32_t ov[2][32];
            tmem_ld_32x32b_x32(tO + lane_off + uint32_t(col_base + ch * 32), ov[0]);
            tmem_ld_32x32b_x32(tO + lane_off + uint32_t(col_base + ch * 32 + 32), ov[1]);
            tmem_ld_wait();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              float4* rowp = reinterpret_cast<float4*>(stg + (ch + u) * 4096 + lane * 128);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                float4 v;
                v.x = __uint_as_float(ov[u][4 * e]) * inv;
                v.y = __uint_as_float(ov[u][4 * e + 1]) * inv;
                v.z = __uint_as_float(ov[u][4 * e + 2]) * inv;
                v.w = __uint_as_float(ov[u][4 * e + 3]) * inv;
                if (part == 1) v = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
                rowp[e ^ (lane & 7)] = v;  // 128-byte swizzle: chunk e of row r at e ^ (r % 8)
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && tw < p.T) {
            for (int ch = 0; ch < 4; ++ch)
              tma_store_3d(part ? &mOlo : &mO, smem_u32(stg + ch * 4096), h * Dh + oh * kD + col_base + ch * 32, tw, b);
            tma_store_commit();
          }
        }
        if (lane == 0) tma_store_wait_read<0>();  // the boxes are read; the writes complete on their own
        __syncwarp();
      } else {
        float* o = obase + int64_t(i) * p.ost + col_base;
        float* ol = olbase ? olbase + int64_t(i) * p.ost + col_base : nullptr;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tO + lane_off + uint32_t(col_base + ch * 32), ov);
          tmem_ld_wait();
          if (row_ok) {
            float4* o4 = reinterpret_cast<float4*>(o + ch * 32);
            float4* l4 = ol ? reinterpret_cast<float4*>(ol + ch * 32) : nullptr;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float4 v;
              v.x = __uint_as_float(ov[4 * e]) * inv;
              v.y = __uint_as_float(ov[4 * e + 1]) * inv;
              v.z = __uint_as_float(ov[4 * e + 2]) * inv;
              v.w = __uint_as_float(ov[4 * e + 3]) * inv;
              o4[e] = v;
              if (l4) l4[e] = make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Split of q or k (strided [B, H, T, D] element offsets b·sb + h·sh + t·st)
// into token-major bf16 hi/lo [B·T, H·D]: one thread per 2 elements.
__global__ void split_bf16_rows_kernel(const float* __restrict__ src, int64_t sb, int64_t sh,
                                       int64_t st, int B, int T, int H, int D,
                                       __nv_bfloat16* __restrict__ hi,
                                       __nv_bfloat16* __restrict__ lo) {
  const int cols = H * D;
  const int64_t rows = int64_t(B) * T;
  const int64_t total = rows * (cols / 2);
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / (cols / 2);
    const int cc = int(e % (cols / 2)) * 2;
    const int b = int(r / T), t = int(r % T), hd = cc / D, d = cc % D;
    const float2 v = *reinterpret_cast<const float2*>(src + b * sb + hd * sh + t * st + d);
    const __nv_bfloat16 h0 = __float2bfloat16_rn(v.x), h1 = __float2bfloat16_rn(v.y);
    __nv_bfloat162 hh;
    hh.x = h0;
    hh.y = h1;
    __nv_bfloat162 ll;
    ll.x = __float2bfloat16_rn(v.x - __bfloat162float(h0));
    ll.y = __float2bfloat16_rn(v.y - __bfloat162float(h1));
    *reinterpret_cast<__nv_bfloat162*>(hi + r * cols + cc) = hh;
    *reinterpret_cast<__nv_bfloat162*>(lo + r * cols + cc) = ll;
  }
}

// V (strided, fp32) → Vᵀ bf16 hi/lo [B·Hkv·D rows, ldt keys], 32 keys ×
// 32 dims per block through shared memory.
__global__ void transpose_v_kernel(const float* __restrict__ v, int64_t sb, int64_t sh, int64_t st,
                                   int B, int T, int Hkv, int D, __nv_bfloat16* __restrict__ hi,
                                   __nv_bfloat16* __restrict__ lo, int64_t ldt) {
  __shared__ float tile[32][33];
  const int t0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int bh = blockIdx.z;  // b * Hkv + hk
  const int b = bh / Hkv, hk = bh % Hkv;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int t = t0 + r;
    tile[r][threadIdx.x] = t < T ? v[b * sb + hk * sh + int64_t(t) * st + d0 + threadIdx.x] : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int d = d0 + r, t = t0 + threadIdx.x;
    if (t < T) {
      const float x = tile[threadIdx.x][r];
      const __nv_bfloat16 h = __float2bfloat16_rn(x);
      const int64_t off = (int64_t(bh) * D + d) * ldt + t;
      hi[off] = h;
      lo[off] = __float2bfloat16_rn(x - __bfloat162float(h));
    }
  }
}

int make_map_bf16(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems,
                  int box_rows) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || (ld_elems * 2) % 16 != 0)
    return set_error(FG_EINVAL, "attention operand alignment");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld_elems) * 2};
  cuuint32_t box[2] = {64u, cuuint32_t(box_rows)};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = g_encode_bf16(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                             box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FG_ECUDA, "cuTensorMapEncodeTiled (bf16) failed (%d)", int(r));
  return FG_OK;
}

// fp32 output viewed as [B][T][cols] (row stride ost, sequence stride osb,
// in elements), [1 × 32 × 32] boxes with 128-byte swizzling.
int make_map_out3d(CUtensorMap* m, const float* ptr, int B, int T, int64_t cols, int64_t ost, int64_t osb) {
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(T), cuuint64_t(B)};
  cuuint64_t strides[2] = {cuuint64_t(ost) * 4, cuuint64_t(osb) * 4};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = g_encode_bf16(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims, strides, box,
                             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FG_ECUDA, "cuTensorMapEncodeTiled (attention output) failed (%d)", int(r));
  return FG_OK;
}

// fp16 output parts viewed as [B][T][cols] (row stride ost, sequence stride
// osb, in elements), [1 × 32 × 32] boxes with 64-byte swizzling.
int make_map_out16_3d(CUtensorMap* m, const uint16_t* ptr, int B, int T, int64_t cols, int64_t ost, int64_t osb) {
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(T), cuuint64_t(B)};
  cuuint64_t strides[2] = {cuuint64_t(ost) * 2, cuuint64_t(osb) * 2};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = g_encode_bf16(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t*>(ptr), dims, strides, box,
                             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FG_ECUDA, "cuTensorMapEncodeTiled (attention fp16 output) failed (%d)", int(r));
  return FG_OK;
}

}  // namespace

size_t attn_tc_workspace_bytes(int B, int T, int S, int Hq, int Hkv, int D) {
  const int64_t ldt = (S + 7) / 8 * 8;
  return size_t(B) * T * Hq * D * 2 * 2 + size_t(B) * S * Hkv * D * 2 * 2 +
         size_t(B) * Hkv * D * ldt * 2 * 2 + 8 * 256;
}

bool attn_tc_supported(const AttnArgs& a) {
  const bool al = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                    reinterpret_cast<uintptr_t>(a.v)) & 7) == 0 &&
                  ((a.qsb | a.qsh | a.qst | a.ksb | a.ksh | a.kst) % 2) == 0;
  const bool out_al = (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                      ((a.osb | a.osh | a.ost) % 4) == 0 &&
                      (!a.out_lo || (reinterpret_cast<uintptr_t>(a.out_lo) & 15) == 0);
  return (a.D == 256 || a.D == 512) && a.Hkv > 0 && a.Hq % a.Hkv == 0 && al && out_al && a.T > 0 && a.S > 0 &&
         int64_t(a.B) * a.T < (int64_t(1) << 31) && int64_t(a.B) * a.S < (int64_t(1) << 31);
}

int attn_tc_carve(void* ws, int B, int T, int S, int Hq, int Hkv, AttnOperands* o, int D) {
  const int kD = D;  // the head dimension for the layout below
  const int64_t ldt = (S + 7) / 8 * 8;
  const int64_t MQ = int64_t(B) * T, MK = int64_t(B) * S;
  auto align = [](uint8_t* q) { return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q) + 255) & ~uintptr_t(255)); };
  uint8_t* w = align(static_cast<uint8_t*>(ws));
  o->q_hi = w;
  w = align(w + size_t(MQ) * Hq * kD * 2);
  o->q_lo = w;
  w = align(w + size_t(MQ) * Hq * kD * 2);
  o->k_hi = w;
  w = align(w + size_t(MK) * Hkv * kD * 2);
  o->k_lo = w;
  w = align(w + size_t(MK) * Hkv * kD * 2);
  o->vt_hi = w;
  w = align(w + size_t(B) * Hkv * kD * ldt * 2);
  o->vt_lo = w;
  o->ldt = ldt;
  return FG_OK;
}

int attention_tc_operands(const AttnArgs& a, const AttnOperands& o, int* err, cudaStream_t s) {
  const int B = a.B, T = a.T, S = a.S, Hq = a.Hq, Hkv = a.Hkv;
  if (B == 0) return FG_OK;
  if ((a.D != 256 && a.D != 512) || Hkv <= 0 || Hq % Hkv != 0 || T <= 0 || S <= 0)
    return set_error(FG_EINVAL, "tensor-core attention: unsupported shape");
  const int Dh = a.D;
  FG_TRY(tensor_map_encoder(&g_encode_bf16));
  const int64_t MQ = int64_t(B) * T, MK = int64_t(B) * S;
  CUtensorMap mq0, mq1, mk0, mk1, mv0, mv1;
  FG_TRY(make_map_bf16(&mq0, o.q_hi, MQ, Hq * Dh, Hq * Dh, 128));
  FG_TRY(make_map_bf16(&mq1, o.q_lo, MQ, Hq * Dh, Hq * Dh, 128));
  FG_TRY(make_map_bf16(&mk0, o.k_hi, MK, Hkv * Dh, Hkv * Dh, 128));
  FG_TRY(make_map_bf16(&mk1, o.k_lo, MK, Hkv * Dh, Hkv * Dh, 128));
  FG_TRY(make_map_bf16(&mv0, o.vt_hi, int64_t(B) * Hkv * Dh, S, o.ldt, 128));
  FG_TRY(make_map_bf16(&mv1, o.vt_lo, int64_t(B) * Hkv * Dh, S, o.ldt, 128));
  Params prm;
  prm.B = B;
  prm.T = T;
  prm.S = S;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.window = a.window;
  prm.scale_log2 = a.scale * 1.4426950408889634f;
  prm.qlen = a.qlen;
  prm.klen = a.klen;
  prm.out = a.out;
  prm.out_lo = a.out_lo;
  prm.osb = a.osb;
  prm.osh = a.osh;
  prm.ost = a.ost;
  prm.err = err;
  // Output as a [B][T][cols] tensor with row stride ost: TMA stores when
  // the heads are contiguous 256-column blocks and the strides allow it.
  CUtensorMap mo = mq0, mol = mq0;
  auto tma_ok = [&](const float* ptr) {
    return ptr && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && a.osh == Dh && a.ost % 4 == 0 &&
           a.osb % 4 == 0 && a.ost >= int64_t(Hq) * Dh && a.osb >= int64_t(T) * a.ost;
  };
  prm.tma_out = 0;
  prm.tma_out_lo = 0;
  prm.tma_out16 = 0;
  prm.out16_scale = 1.f;
  prm.out16 = nullptr;
  prm.out16_lo = nullptr;
  if (a.out16) {
    // the next product's fp16 parts, through TMA only
    auto ok16 = [&](const uint16_t* ptr) {
      return ptr && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && a.osh == Dh && a.ost % 8 == 0 &&
             a.osb % 8 == 0 && a.ost >= int64_t(Hq) * Dh && a.osb >= int64_t(T) * a.ost;
    };
    if (!ok16(a.out16) || !ok16(a.out16_lo) || a.out16_exp < -126 || a.out16_exp > 127)
      return set_error(FG_EINVAL, "attention: fp16-parts output needs aligned contiguous heads");
    FG_TRY(make_map_out16_3d(&mo, a.out16, B, T, Hq * Dh, a.ost, a.osb));
    FG_TRY(make_map_out16_3d(&mol, a.out16_lo, B, T, Hq * Dh, a.ost, a.osb));
    prm.tma_out16 = 1;
    prm.out16_scale = std::ldexp(1.0f, a.out16_exp);
    prm.out16 = a.out16;
    prm.out16_lo = a.out16_lo;
  } else if (tma_ok(a.out) && (a.out_lo == nullptr || tma_ok(a.out_lo))) {
    FG_TRY(make_map_out3d(&mo, a.out, B, T, Hq * Dh, a.ost, a.osb));
    if (a.out_lo) FG_TRY(make_map_out3d(&mol, a.out_lo, B, T, Hq * Dh, a.ost, a.osb));
    prm.tma_out = 1;
    prm.tma_out_lo = a.out_lo ? 1 : 0;
  }
  static std::atomic<bool> attr[64][2];  // per device and head width
  int dev = 0;
  cudaGetDevice(&dev);
  const int wide = Dh == 512 ? 1 : 0;
  if (!attr[dev & 63][wide]) {
    if (wide)
      FG_CUDA_TRY(cudaFuncSetAttribute(attn_tc_kernel<8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem)));
    else
      FG_CUDA_TRY(cudaFuncSetAttribute(attn_tc_kernel<4, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem)));
    attr[dev & 63][wide] = true;
  }
  if ((T + kQ - 1) / kQ > 65535 || B > 65535 || Hq * (wide + 1) > 65535)
    return set_error(FG_EINVAL, "attention grid too large");
  dim3 grid(unsigned((T + kQ - 1) / kQ), unsigned(Hq * (wide + 1)), unsigned(B));
  if (wide)
    attn_tc_kernel<8, true><<<grid, kThreads, kSmem, s>>>(mq0, mq1, mk0, mk1, mv0, mv1, mo, mol, prm);
  else
    attn_tc_kernel<4, false><<<grid, kThreads, kSmem, s>>>(mq0, mq1, mk0, mk1, mv0, mv1, mo, mol, prm);
  FG_CUDA_TRY(cudaGetLastError());
  return FG_OK;
}

int attention_tc(const AttnArgs& a, void* ws, size_t ws_bytes, int* err, cudaStream_t s) {
  if (!attn_tc_supported(a)) return set_error(FG_EINVAL, "tensor-core attention: unsupported shape or alignment");
  const int B = a.B, T = a.T, S = a.S, Hq = a.Hq, Hkv = a.Hkv;
  if (B == 0) return FG_OK;
  const int Dh = a.D;
  if (ws_bytes < attn_tc_workspace_bytes(B, T, S, Hq, Hkv, Dh))
    return set_error(FG_EINVAL, "attention workspace too small");
  AttnOperands o;
  FG_TRY(attn_tc_carve(ws, B, T, S, Hq, Hkv, &o, Dh));
  const int64_t MQ = int64_t(B) * T, MK = int64_t(B) * S;
  auto bf = [](void* p) { return static_cast<__nv_bfloat16*>(p); };
  auto grid_of = [](int64_t n) { return int(std::min<int64_t>((n + 255) / 256, int64_t(sm_count()) * 16)); };
  split_bf16_rows_kernel<<<grid_of(MQ * Hq * Dh / 2), 256, 0, s>>>(a.q, a.qsb, a.qsh, a.qst, B, T, Hq, Dh, bf(o.q_hi), bf(o.q_lo));
  split_bf16_rows_kernel<<<grid_of(MK * Hkv * Dh / 2), 256, 0, s>>>(a.k, a.ksb, a.ksh, a.kst, B, S, Hkv, Dh, bf(o.k_hi), bf(o.k_lo));
  dim3 tg(unsigned((S + 31) / 32), unsigned(Dh / 32), unsigned(B * Hkv));
  transpose_v_kernel<<<tg, dim3(32, 8), 0, s>>>(a.v, a.vsb, a.vsh, a.vst, B, S, Hkv, Dh, bf(o.vt_hi), bf(o.vt_lo), o.ldt);
  FG_CUDA_TRY(cudaGetLastError());
  return attention_tc_operands(a, o, err, s);
}

}  // namespace fg
