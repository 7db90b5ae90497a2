/*
 * Mode-generic body of the oracle, included twice by fg_oracle.c with
 *   R = double, SFX(name) = name##_f64, MADD = fma    (ORC_F64)
 *   R = float,  SFX(name) = name##_f32, MADD = fmaf   (ORC_F32)
 * MADD is the fused multiply-add the reference's SIMD dot and GEMM
 * kernels accumulate with.
 * Test infrastructure only (see fg_oracle.h).
 */

/* C[m,n] = A[m,k] · W[k,n], row-major, W in the reference's [in, out]
 * layout; each C element accumulates sequentially over k (the order of the
 * reference's micro-kernel, internal/kernel/kernel_avx512_amd64.s), in R. */
static void SFX(gemm)(const R* A, const float* W, int m, int k, int n, R* C) {
  if (sizeof(R) == sizeof(float) && g_fast) {
    gemm_f32_packed((const float*)A, W, m, k, n, (float*)C);
    return;
  }
#pragma omp parallel for schedule(dynamic, 1)
  for (int i0 = 0; i0 < m; i0 += 4) {
    const int rows = (m - i0) < 4 ? (m - i0) : 4;
    for (int n0 = 0; n0 < n; n0 += 64) {
      const int cols = (n - n0) < 64 ? (n - n0) : 64;
      R acc[4][64];
      for (int r = 0; r < 4; ++r)
        for (int j = 0; j < 64; ++j) acc[r][j] = 0;
      for (int kk = 0; kk < k; ++kk) {
        const float* w = W + (size_t)kk * n + n0;
        R a[4];
        for (int r = 0; r < 4; ++r) a[r] = r < rows ? A[(size_t)(i0 + r) * k + kk] : 0;
        if (cols == 64) {
          for (int r = 0; r < 4; ++r)
            for (int j = 0; j < 64; ++j) acc[r][j] = MADD(a[r], (R)w[j], acc[r][j]);
        } else {
          for (int r = 0; r < 4; ++r)
            for (int j = 0; j < cols; ++j) acc[r][j] = MADD(a[r], (R)w[j], acc[r][j]);
        }
      }
      for (int r = 0; r < rows; ++r)
        for (int j = 0; j < cols; ++j) C[(size_t)(i0 + r) * n + n0 + j] = acc[r][j];
    }
  }
}

/* rmsScale (embed.go:432-438): float32(1/√(float64(ss/n + eps))) in the
 * reference; all float64 in the f64 mode. */
static R SFX(rms_inv)(R ss, int n, float eps) {
  if (sizeof(R) == sizeof(float)) {
    const float m = (float)ss / (float)n + eps;
    return (R)(float)(1.0 / sqrt((double)m));
  }
  return (R)(1.0 / sqrt((double)ss / (double)n + (double)eps));
}

/* rmsNormFused (attention.go:312-337) on rows of n. */
static void SFX(rmsnorm_rows)(R* x, size_t rows, int n, const float* g, float eps, R* out) {
#pragma omp parallel for schedule(static)
  for (size_t r = 0; r < rows; ++r) {
    const R* v = x + r * n;
    R ss = 0;
    for (int i = 0; i < n; ++i) ss = MADD(v[i], v[i], ss);
    const R inv = SFX(rms_inv)(ss, n, eps);
    for (int i = 0; i < n; ++i) out[r * n + i] = v[i] * inv * (R)g[i];
  }
}

static R SFX(exp_mode)(R v) {
  if (sizeof(R) == sizeof(float)) return (R)ref_expf((float)v);
  return v < -87.0 ? 0.0 : exp((double)v);
}

static R SFX(gelu_mode)(R x) {
  if (sizeof(R) == sizeof(float)) return (R)ref_gelu((float)x);
  return 0.5 * x * (1.0 + tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)));
}

static R SFX(tanh_mode)(R x) {
  if (sizeof(R) == sizeof(float)) return (R)ref_tanhf((float)x);
  return tanh((double)x);
}

/* One attention row against one head (internal/blas/attention.go:97-135):
 * raw scores s = q·k, the additive mask joins as mask/scale, the max is
 * taken over the whole row, weights exp(scale·s − scale·max) (masked ones
 * flush to exactly 0), P·V, then ×1/Σ. maskcnt[j] counts the −1e9 masks
 * hiding key j (padding, window), so the mask value is −1e9·maskcnt[j]. */
static void SFX(attn_row)(const R* q, const R* K, const R* V, int S, int D, int ld,
                          const unsigned char* maskcnt, const float* fmask, float scale, R* s,
                          R* out, const R* KT, int ldt) {
  if (sizeof(R) == sizeof(float) && KT) {
    scores_f32_packed((const float*)q, (const float*)KT, S, D, ldt, (float*)s);
  } else {
    for (int j = 0; j < S; ++j) {
      R acc = 0;
      for (int d = 0; d < D; ++d) acc = MADD(q[d], K[(size_t)j * ld + d], acc);
      s[j] = acc;
    }
  }
  const R inv_scale = (R)(1.0f / scale);
  if (sizeof(R) == sizeof(float)) {
    /* float32: add mask·(1/scale) exactly as Axpy does, max, ExpSum */
    for (int j = 0; j < S; ++j) {
      float mv = fmask ? fmask[j] : (float)(-1e9 * (double)(maskcnt ? maskcnt[j] : 0));
      if (mv != 0.0f) s[j] = (R)((float)s[j] + (float)inv_scale * mv);
    }
    float mx = -INFINITY;
    for (int j = 0; j < S; ++j) mx = (float)s[j] > mx ? (float)s[j] : mx;
    const float a = scale, b = -scale * mx;
    float sum = 0;
    for (int j = 0; j < S; ++j) {
      float z = a * (float)s[j] + b;
      z = ref_expf(z);
      s[j] = z;
      sum += z;
    }
    const float inv = 1.0f / sum;
    for (int d = 0; d < D; ++d) out[d] = 0;
    for (int j = 0; j < S; ++j) {
      const R p = s[j];
      if (p == 0) continue;
      for (int d = 0; d < D; ++d) out[d] = MADD(p, V[(size_t)j * ld + d], out[d]);
    }
    for (int d = 0; d < D; ++d) out[d] = (R)((float)out[d] * inv);
    return;
  }
  /* float64: the same algorithm; the −1e9 mask swamps the raw scores in
   * float32, so a row whose keys are all hidden gets equal weights on the
   * keys hidden the fewest times — kept here by comparing mask counts. */
  int minc = 1 << 30;
  for (int j = 0; j < S; ++j) {
    const int cnt = fmask ? (fmask[j] != 0.0f) : (maskcnt ? maskcnt[j] : 0);
    if (cnt < minc) minc = cnt;
  }
  double mx = -INFINITY;
  if (fmask) {
    for (int j = 0; j < S; ++j) {
      s[j] = s[j] + (double)fmask[j] * (double)inv_scale;
      mx = s[j] > mx ? s[j] : mx;
    }
  } else {
    for (int j = 0; j < S; ++j) {
      const int cnt = maskcnt ? maskcnt[j] : 0;
      if (cnt == minc && (double)s[j] > mx) mx = s[j];
    }
  }
  double sum = 0;
  for (int j = 0; j < S; ++j) {
    double p;
    if (fmask) {
      p = SFX(exp_mode)((R)((double)scale * (double)s[j] - (double)scale * mx));
    } else {
      const int cnt = maskcnt ? maskcnt[j] : 0;
      if (cnt != minc) p = 0;
      else if (minc == 0) p = exp((double)scale * ((double)s[j] - mx));
      else p = 1; /* every key hidden: the float32 scores are all equal */
    }
    s[j] = (R)p;
    sum += p;
  }
  for (int d = 0; d < D; ++d) out[d] = 0;
  for (int j = 0; j < S; ++j) {
    const R p = s[j];
    if (p == 0) continue;
    for (int d = 0; d < D; ++d) out[d] += p * V[(size_t)j * ld + d];
  }
  const double inv = 1.0 / sum;
  for (int d = 0; d < D; ++d) out[d] = (R)((double)out[d] * inv);
}

/* RoPE rotate-half (rope.go:66-87) on a head vector at slot t. */
static void SFX(rope_vec)(R* v, int D, const float* cs, const float* sn, int t) {
  const int half = D / 2;
  for (int i = 0; i < half; ++i) {
    const R x1 = v[i], x2 = v[i + half];
    const R c = (R)cs[(size_t)t * half + i], s = (R)sn[(size_t)t * half + i];
    v[i] = x1 * c - x2 * s;
    v[i + half] = x1 * s + x2 * c;
  }
}

/* encode → pool → applyHead → l2normalize (embed.go:160-240, 381-429, 472-475). */
static int SFX(embed)(const orc_config* c, const folded* fw, const int32_t* ids,
                      const int32_t* lengths, int B, int T, int dim, float* out) {
  const int H = c->hidden, D = c->head_dim, Hq = c->heads, Hkv = c->kv_heads, F = c->ffn;
  const size_t M = (size_t)B * T;
  const int qw = Hq * D, kw = Hkv * D;
  R* x = (R*)malloc(M * H * sizeof(R));
  R* xs = (R*)malloc(M * H * sizeof(R));
  R* scale = (R*)malloc(M * sizeof(R));
  R* q = (R*)malloc(M * qw * sizeof(R));
  R* kk = (R*)malloc(M * kw * sizeof(R));
  R* vv = (R*)malloc(M * kw * sizeof(R));
  R* att = (R*)malloc(M * qw * sizeof(R));
  R* t1 = (R*)malloc(M * (F > H ? F : H) * sizeof(R));
  R* t2 = (R*)malloc(M * (F > H ? F : H) * sizeof(R));
  if (!x || !xs || !scale || !q || !kk || !vv || !att || !t1 || !t2) {
    free(x); free(xs); free(scale); free(q); free(kk); free(vv); free(att); free(t1); free(t2);
    return -1;
  }
  /* x = embed.Rows(flat) · float32(√hidden)  (embed.go:175-176) */
  const float emb_scale = (float)sqrt((double)H);
#pragma omp parallel for schedule(static)
  for (size_t r = 0; r < M; ++r) {
    const int b = (int)(r / T), t = (int)(r % T);
    const int id = t < lengths[b] ? ids[r] : 0; /* embedBatch pads with id 0 */
    const float* e = c_row(fw->embed, id, H);
    for (int i = 0; i < H; ++i) {
      if (sizeof(R) == sizeof(float)) x[r * H + i] = (R)(e[i] * emb_scale);
      else x[r * H + i] = (R)e[i] * (R)emb_scale;
    }
  }
  const int win = c->window;
  for (int l = 0; l < c->layers; ++l) {
    const folded_layer* L = &fw->layer[l];
    const int sliding = c->sliding[l] && win > 0 && T > win;
    /* folded pre-norm: rowscale = rmsScale(RowSumSquares(x)) (embed.go:193-194) */
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < M; ++r) {
      R ss = 0;
      for (int i = 0; i < H; ++i) ss = MADD(x[r * H + i], x[r * H + i], ss);
      scale[r] = SFX(rms_inv)(ss, H, c->eps);
    }
    SFX(gemm)(x, L->wq, (int)M, H, qw, q);
    SFX(gemm)(x, L->wk, (int)M, H, kw, kk);
    SFX(gemm)(x, L->wv, (int)M, H, kw, vv);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < M; ++r) {
      for (int i = 0; i < qw; ++i) q[r * qw + i] *= scale[r];
      for (int i = 0; i < kw; ++i) kk[r * kw + i] *= scale[r];
      for (int i = 0; i < kw; ++i) vv[r * kw + i] *= scale[r];
    }
    /* QK-norm (embed.go:198-199), RoPE (embed.go:206-207) */
    SFX(rmsnorm_rows)(q, M * Hq, D, L->qgain, c->eps, q);
    SFX(rmsnorm_rows)(kk, M * Hkv, D, L->kgain, c->eps, kk);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < M; ++r) {
      const int t = (int)(r % T);
      for (int h = 0; h < Hq; ++h) SFX(rope_vec)(q + r * qw + (size_t)h * D, D, L->cos_t, L->sin_t, t);
      for (int h = 0; h < Hkv; ++h) SFX(rope_vec)(kk + r * kw + (size_t)h * D, D, L->cos_t, L->sin_t, t);
    }
    /* attention with PaddingMask (+ WindowMask on sliding layers) (embed.go:168-186, 209);
     * float32 with the fast kernels: K transposed per (sequence, KV head) to
     * [D][T] so the scores go 16 keys at a time */
    R* kt = NULL;
    if (sizeof(R) == sizeof(float) && g_fast) {
      kt = (R*)malloc(M * kw * sizeof(R));
      if (kt) {
#pragma omp parallel for schedule(static) collapse(2)
        for (int b = 0; b < B; ++b)
          for (int hk = 0; hk < Hkv; ++hk) {
            R* dst = kt + ((size_t)b * Hkv + hk) * D * T;
            for (int t = 0; t < T; ++t)
              for (int d = 0; d < D; ++d) dst[(size_t)d * T + t] = kk[((size_t)b * T + t) * kw + (size_t)hk * D + d];
          }
      }
    }
#pragma omp parallel
    {
      R* s = (R*)malloc((size_t)T * sizeof(R));
      unsigned char* mc = (unsigned char*)malloc((size_t)T);
#pragma omp for schedule(dynamic, 4) collapse(2)
      for (int b = 0; b < B; ++b)
        for (int i = 0; i < T; ++i) {
          for (int j = 0; j < T; ++j) {
            int cnt = j >= lengths[b];
            if (sliding && (j - i >= win || i - j >= win)) cnt++;
            mc[j] = (unsigned char)cnt;
          }
          for (int h = 0; h < Hq; ++h) {
            const int hk = h / (Hq / Hkv);
            const R* qr = q + ((size_t)b * T + i) * qw + (size_t)h * D;
            const R* Kb = kk + (size_t)b * T * kw + (size_t)hk * D;
            const R* Vb = vv + (size_t)b * T * kw + (size_t)hk * D;
            R* o = att + ((size_t)b * T + i) * qw + (size_t)h * D;
            const R* KTb = kt ? kt + ((size_t)b * Hkv + hk) * D * T : NULL;
            SFX(attn_row)(qr, Kb, Vb, T, D, kw, mc, NULL, c->attn_scale, s, o, KTb, T);
          }
        }
      free(s);
      free(mc);
    }
    free(kt);
    /* o = RMSNorm(att·Wo, 1+postAttn); x += o (embed.go:212-220) */
    SFX(gemm)(att, L->wo, (int)M, qw, H, t1);
    SFX(rmsnorm_rows)(t1, M, H, L->post_attn, c->eps, t1);
#pragma omp parallel for schedule(static)
    for (size_t e = 0; e < M * H; ++e) x[e] = x[e] + t1[e];
    /* FFN (embed.go:224-235) */
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < M; ++r) {
      R ss = 0;
      for (int i = 0; i < H; ++i) ss = MADD(x[r * H + i], x[r * H + i], ss);
      scale[r] = SFX(rms_inv)(ss, H, c->eps);
    }
    SFX(gemm)(x, L->wup, (int)M, H, F, t1);
    SFX(gemm)(x, L->wgate, (int)M, H, F, t2);
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < M; ++r)
      for (int i = 0; i < F; ++i) {
        const R up = t1[r * F + i] * scale[r];
        const R g = t2[r * F + i] * scale[r];
        t2[r * F + i] = SFX(gelu_mode)(g) * up;
      }
    SFX(gemm)(t2, L->wdown, (int)M, F, H, t1);
    SFX(rmsnorm_rows)(t1, M, H, L->post_ffn, c->eps, t1);
#pragma omp parallel for schedule(static)
    for (size_t e = 0; e < M * H; ++e) x[e] = x[e] + t1[e];
  }
  /* final norm (embed.go:237) */
  SFX(rmsnorm_rows)(x, M, H, fw->final_gain, c->eps, xs);
  /* pool (embed.go:381-404) */
  int width = H;
  for (int j = 0; j < c->num_dense; ++j)
    if (c->dense_out[j] > width) width = c->dense_out[j];
  R* cur = (R*)calloc((size_t)B * width, sizeof(R));
  R* nxt = (R*)calloc((size_t)B * width, sizeof(R));
  for (int b = 0; b < B; ++b) {
    int n = lengths[b];
    if (n == 0) n = 1;
    R* dst = cur + (size_t)b * H;
    for (int t = 0; t < n; ++t)
      for (int i = 0; i < H; ++i) dst[i] += xs[((size_t)b * T + t) * H + i];
    R inv;
    if (sizeof(R) == sizeof(float)) inv = (R)(1.0f / (float)n);
    else inv = (R)(1.0 / (double)n);
    for (int i = 0; i < H; ++i) dst[i] *= inv;
  }
  /* head (embed.go:408-429) */
  int cw = H;
  for (int j = 0; j < c->num_dense; ++j) {
    SFX(gemm)(cur, fw->dense[j], B, c->dense_in[j], c->dense_out[j], nxt);
    if (c->dense_tanh[j])
      for (size_t e = 0; e < (size_t)B * c->dense_out[j]; ++e) nxt[e] = SFX(tanh_mode)(nxt[e]);
    R* tmp = cur;
    cur = nxt;
    nxt = tmp;
    cw = c->dense_out[j];
  }
  /* narrow + l2normalize (embed.go:421-427, 472-475) */
  for (int b = 0; b < B; ++b) {
    const R* v = cur + (size_t)b * cw;
    R ss = 0;
    for (int i = 0; i < dim; ++i) ss += v[i] * v[i];
    R nrm;
    if (sizeof(R) == sizeof(float)) nrm = (R)sqrtf((float)ss + 1e-12f);
    else nrm = (R)sqrt((double)ss + 1e-12);
    for (int i = 0; i < dim; ++i) out[(size_t)b * dim + i] = c->l2 ? (float)(v[i] / nrm) : (float)v[i];
  }
  free(cur); free(nxt);
  free(x); free(xs); free(scale); free(q); free(kk); free(vv); free(att); free(t1); free(t2);
  return 0;
}
