/* CPU restatement of the sys1rust model forward in C (fp32, OpenMP) -- TEST INFRASTRUCTURE ONLY.
 *
 * Only the tests and bench.py's CPU-baseline leg load this library, as a second checker beside the
 * PyTorch oracle (forward_ref.py) and as a timed CPU baseline; the product library never links or
 * calls it. It computes what `MlxBackend::forward` computes for one row
 * (runtime/crates/laya-mlx/src/lib.rs:1833-1863), in fp32 with fp32 weights:
 *
 *   encode (lib.rs:1525-1693): tok_emb gather, bias-free emb_norm; per layer attn_norm (identity at
 *     layer 0, lib.rs:993-997), Wqkv, rotate-half RoPE at positions 0..L-1 with inverse frequency
 *     exp2(-(i / (hd/2)) * log2(theta)) and the angle p * inv_freq in fp32 (split_rope.metal:46-76),
 *     softmax(q k^T / sqrt(hd)) v over the row's keys, |i - j| <= window on local layers
 *     (lib.rs:1399-1417, config.rs:135-141), Wo + residual, mlp_norm, Wi, GeGLU with the exact
 *     erf GELU (lib.rs:381-510), Wo2 + residual; final_norm.
 *   head_forward (lib.rs:1698-1765): type_emb of the row's qtype, pre-norm TransformerEncoderLayers
 *     (biases, eps 1e-5, ReLU FFN, scale 1/sqrt(d / heads), lib.rs:576-578); the last layer computes
 *     queries, the output projection and the FFN only at the scorer rows [0, markers...]
 *     (lib.rs:1726-1760, ScorerRows lib.rs:872-889).
 *   score (lib.rs:1768-1800): pooled = row 0; scorer LN -> Linear -> erf GELU -> Linear at each
 *     marker; slots at or past marker_count hold -1e4 (lib.rs:1851-1857).
 *
 * Masked keys are left out of the softmax instead of receiving the additive -1e4: for any row with
 * at least one real key exp(-1e4 + ...) is 0 in fp32, so the two are the same.
 *
 * Build (x86-64-v3: AVX2 + FMA):  gcc -O3 -march=x86-64-v3 -fopenmp -shared -fPIC
 *                                 oracle/forward_ref.c -o oracle/_build/libforward_ref.so -lm
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  int d, heads, inter, n_layers, window;   /* encoder: hidden, heads (hd = d / heads), GeGLU width */
  int head_layers, head_heads, head_ffn;   /* decision head */
  int scorer_hidden;
  float eps, theta_global, theta_local;
  const int32_t* layer_is_local;           /* [n_layers] */
  const float* tok_emb;                    /* [vocab, d] */
  const float* emb_norm;                   /* [d] */
  const float* const* attn_norm;           /* [n_layers], entry 0 unused */
  const float* const* wqkv;                /* [n_layers] of [3d, d] */
  const float* const* wo;                  /* [n_layers] of [d, d] */
  const float* const* mlp_norm;            /* [n_layers] of [d] */
  const float* const* wi;                  /* [n_layers] of [2 * inter, d] (x rows, then gate rows) */
  const float* const* wo2;                 /* [n_layers] of [d, inter] */
  const float* final_norm;                 /* [d] */
  const float* type_emb;                   /* [3, d] */
  /* per head layer, 12 entries: norm1 w, b; in_proj w [3d, d], b; out_proj w [d, d], b;
   * norm2 w, b; linear1 w [ffn, d], b; linear2 w [d, ffn], b */
  const float* const* head;
  const float *sc0_w, *sc0_b, *sc1_w, *sc1_b, *sc3_w, *sc3_b; /* scorer.{0,1,3} */
} ofr_model;

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

static float hsum8(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
  lo = _mm_add_ps(lo, hi);
  lo = _mm_add_ps(lo, _mm_movehl_ps(lo, lo));
  lo = _mm_add_ss(lo, _mm_movehdup_ps(lo));
  return _mm_cvtss_f32(lo);
}

/* C[i, n] (+)= sum_k A[i, k] W[n, k] (+ bias[n]) for i < M, n < N: A row pitch lda, W [N, K]
 * row-major, C row pitch ldc. Blocks of 48 output columns are spread over the threads; inside a
 * block, 4 rows x 3 columns of accumulators per step of 8 along k. */
static void gemm_nt(const float* A, int lda, int M, int K, const float* W, int N, const float* bias, float* C,
                    int ldc, int accumulate) {
  const int NB = 48;
  const int nblocks = (N + NB - 1) / NB;
#pragma omp parallel for schedule(dynamic, 1)
  for (int b = 0; b < nblocks; ++b) {
    const int nlo = b * NB, nhi = imin(N, nlo + NB);
    for (int i0 = 0; i0 < M; i0 += 4) {
      const int mm = imin(4, M - i0);
      const float* a[4];
      for (int r = 0; r < 4; ++r) a[r] = A + (size_t)(i0 + imin(r, mm - 1)) * lda;
      for (int n0 = nlo; n0 < nhi; n0 += 3) {
        const int nn = imin(3, nhi - n0);
        const float* w[3];
        for (int j = 0; j < 3; ++j) w[j] = W + (size_t)(n0 + imin(j, nn - 1)) * K;
        __m256 acc[4][3];
        for (int r = 0; r < 4; ++r)
          for (int j = 0; j < 3; ++j) acc[r][j] = _mm256_setzero_ps();
        int k = 0;
        for (; k + 8 <= K; k += 8) {
          const __m256 w0 = _mm256_loadu_ps(w[0] + k), w1 = _mm256_loadu_ps(w[1] + k),
                       w2 = _mm256_loadu_ps(w[2] + k);
          for (int r = 0; r < 4; ++r) {
            const __m256 av = _mm256_loadu_ps(a[r] + k);
            acc[r][0] = _mm256_fmadd_ps(av, w0, acc[r][0]);
            acc[r][1] = _mm256_fmadd_ps(av, w1, acc[r][1]);
            acc[r][2] = _mm256_fmadd_ps(av, w2, acc[r][2]);
          }
        }
        for (int r = 0; r < mm; ++r)
          for (int j = 0; j < nn; ++j) {
            float v = hsum8(acc[r][j]);
            for (int kk = k; kk < K; ++kk) v += a[r][kk] * w[j][kk];
            if (bias) v += bias[n0 + j];
            float* c = C + (size_t)(i0 + r) * ldc + n0 + j;
            *c = accumulate ? *c + v : v;
          }
      }
    }
  }
}

/* LayerNorm of n rows of width d (mean and variance in double), weight w, optional bias b. */
static void layer_norm(const float* x, int ldx, int n, int d, const float* w, const float* b, float eps, float* y,
                       int ldy) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    const float* xr = x + (size_t)i * ldx;
    double s = 0.0;
    for (int c = 0; c < d; ++c) s += xr[c];
    const float mu = (float)(s / d);
    double v = 0.0;
    for (int c = 0; c < d; ++c) v += (double)(xr[c] - mu) * (xr[c] - mu);
    const float rs = 1.0f / sqrtf((float)(v / d) + eps);
    float* yr = y + (size_t)i * ldy;
    for (int c = 0; c < d; ++c) yr[c] = (xr[c] - mu) * rs * w[c] + (b ? b[c] : 0.0f);
  }
}

static float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

/* Rotate-half RoPE in place on the q and k blocks of qkv rows [L, 3d] (positions 0..L-1). */
static void rope(float* qkv, int L, int d, int heads, float theta) {
  const int hd = d / heads, half = hd / 2;
  const float lb = log2f(theta);
#pragma omp parallel for schedule(static)
  for (int p = 0; p < L; ++p) {
    float* row = qkv + (size_t)p * 3 * d;
    for (int i = 0; i < half; ++i) {
      const float inv = exp2f(-((float)i / (float)half) * lb);
      const float ang = (float)p * inv;
      const float c = cosf(ang), s = sinf(ang);
      for (int part = 0; part < 2; ++part)
        for (int h = 0; h < heads; ++h) {
          float* x = row + part * d + h * hd;
          const float x1 = x[i], x2 = x[i + half];
          x[i] = x1 * c - x2 * s;
          x[i + half] = x1 * s + x2 * c;
        }
    }
  }
}

/* Attention of queries qrows[0..nq) (row indices into q) over the keys of one row: for each head,
 * softmax(q k^T * scale) v with keys j in [0, L) (window < 0) or |i - j| <= window, where i is
 * the query's position. q/k/v row pitch ld; output [nq, d] with pitch ldo. */
static void attention(const float* q, const float* k, const float* v, int ld, int L, const int* qrows, int nq,
                      int d, int heads, int window, float* o, int ldo) {
  const int hd = d / heads;
  const float scale = 1.0f / sqrtf((float)hd);
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)L);
#pragma omp for schedule(dynamic, 4) collapse(2)
    for (int h = 0; h < heads; ++h)
      for (int t = 0; t < nq; ++t) {
        const int i = qrows ? qrows[t] : t;
        const int lo = window < 0 ? 0 : imax(0, i - window), hi = window < 0 ? L : imin(L, i + window + 1);
        const float* qi = q + (size_t)i * ld + h * hd;
        float m = -INFINITY;
        for (int j = lo; j < hi; ++j) {
          const float* kj = k + (size_t)j * ld + h * hd;
          float s = 0.0f;
          for (int c = 0; c < hd; ++c) s += qi[c] * kj[c];
          sc[j] = s * scale;
          if (sc[j] > m) m = sc[j];
        }
        float l = 0.0f;
        for (int j = lo; j < hi; ++j) {
          sc[j] = expf(sc[j] - m);
          l += sc[j];
        }
        float* oi = o + (size_t)t * ldo + h * hd;
        for (int c = 0; c < hd; ++c) oi[c] = 0.0f;
        for (int j = lo; j < hi; ++j) {
          const float p = sc[j] / l;
          const float* vj = v + (size_t)j * ld + h * hd;
          for (int c = 0; c < hd; ++c) oi[c] += p * vj[c];
        }
      }
    free(sc);
  }
}

/* One row: ids [L], marker positions [kmax] (the first marker_count are used), qtype 0..2.
 * Writes logits [kmax] (masked slots -1e4) and pooled [d]. Returns 0, or -1 when out of memory. */
int ofr_forward_row(const ofr_model* m, const uint32_t* ids, int L, const uint32_t* marker_pos, int kmax,
                    int marker_count, int qtype, float* logits, float* pooled) {
  const int d = m->d, I = m->inter, F = m->head_ffn;
  const int wide = imax(imax(3 * d, imax(2 * I, F)), m->scorer_hidden);
  /* the pruned layer keeps 1 + marker_count rows, which may be more than L (repeated positions) */
  const int R = imax(L, 1 + imin(imax(marker_count, 0), kmax));
  float* h = (float*)malloc(sizeof(float) * (size_t)R * d);
  float* x = (float*)malloc(sizeof(float) * (size_t)R * d);
  float* big = (float*)malloc(sizeof(float) * (size_t)R * wide);
  float* act = (float*)malloc(sizeof(float) * (size_t)R * imax(d, I));
  int* rows = (int*)malloc(sizeof(int) * (size_t)(1 + kmax));
  if (!h || !x || !big || !act || !rows) {
    free(h); free(x); free(big); free(act); free(rows);
    return -1;
  }
  /* encoder */
  for (int p = 0; p < L; ++p) memcpy(x + (size_t)p * d, m->tok_emb + (size_t)ids[p] * d, sizeof(float) * d);
  layer_norm(x, d, L, d, m->emb_norm, NULL, m->eps, h, d);
  for (int li = 0; li < m->n_layers; ++li) {
    const int local = m->layer_is_local[li];
    const float* a = h;
    if (li > 0) {
      layer_norm(h, d, L, d, m->attn_norm[li], NULL, m->eps, x, d);
      a = x;
    }
    gemm_nt(a, d, L, d, m->wqkv[li], 3 * d, NULL, big, 3 * d, 0);
    rope(big, L, d, m->heads, local ? m->theta_local : m->theta_global);
    attention(big, big + d, big + 2 * d, 3 * d, L, NULL, L, d, m->heads, local ? m->window : -1, act, d);
    gemm_nt(act, d, L, d, m->wo[li], d, NULL, h, d, 1);
    layer_norm(h, d, L, d, m->mlp_norm[li], NULL, m->eps, x, d);
    gemm_nt(x, d, L, d, m->wi[li], 2 * I, NULL, big, 2 * I, 0);
#pragma omp parallel for schedule(static)
    for (int p = 0; p < L; ++p)
      for (int c = 0; c < I; ++c)
        act[(size_t)p * I + c] = gelu_erf(big[(size_t)p * 2 * I + c]) * big[(size_t)p * 2 * I + I + c];
    gemm_nt(act, I, L, I, m->wo2[li], d, NULL, h, d, 1);
  }
  layer_norm(h, d, L, d, m->final_norm, NULL, m->eps, x, d);
  /* head: type embedding, then the layers; the last one only at the scorer rows */
  const float* te = m->type_emb + (size_t)qtype * d;
  for (int p = 0; p < L; ++p)
    for (int c = 0; c < d; ++c) h[(size_t)p * d + c] = x[(size_t)p * d + c] + te[c];
  const int nr = 1 + imin(imax(marker_count, 0), kmax);
  rows[0] = 0;
  for (int k = 0; k + 1 < nr; ++k) rows[1 + k] = (int)marker_pos[k];
  for (int j = 0; j < m->head_layers; ++j) {
    const float* const* P = m->head + 12 * j;
    const int last = j == m->head_layers - 1;
    const int nq = last ? nr : L;
    layer_norm(h, d, L, d, P[0], P[1], 1e-5f, x, d);
    /* keys and values at every position, queries at the rows this layer keeps */
    gemm_nt(x, d, L, d, P[2] + (size_t)d * d, 2 * d, P[3] + d, big + d, 3 * d, 0);
    if (last) {
      for (int t = 0; t < nq; ++t) gemm_nt(x + (size_t)rows[t] * d, d, 1, d, P[2], d, P[3], big + (size_t)rows[t] * 3 * d, 3 * d, 0);
    } else {
      gemm_nt(x, d, L, d, P[2], d, P[3], big, 3 * d, 0);
    }
    attention(big, big + d, big + 2 * d, 3 * d, L, last ? rows : NULL, nq, d, m->head_heads, -1, act, d);
    if (last) {
      /* the kept rows move to the front: h[t] = h[rows[t]] (+ out_proj) */
      for (int t = 0; t < nq; ++t) memcpy(x + (size_t)t * d, h + (size_t)rows[t] * d, sizeof(float) * d);
      memcpy(h, x, sizeof(float) * (size_t)nq * d);
    }
    gemm_nt(act, d, nq, d, P[4], d, P[5], h, d, 1);
    layer_norm(h, d, nq, d, P[6], P[7], 1e-5f, x, d);
    gemm_nt(x, d, nq, d, P[8], F, P[9], big, F, 0);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < nq; ++t)
      for (int c = 0; c < F; ++c) big[(size_t)t * F + c] = fmaxf(big[(size_t)t * F + c], 0.0f);
    gemm_nt(big, F, nq, F, P[10], d, P[11], h, d, 1);
    if (!last) continue;
    /* scorer at the marker rows (now rows 1..nr-1 of h), pooled = row 0 */
    memcpy(pooled, h, sizeof(float) * d);
    const int S = m->scorer_hidden;
    for (int k = 0; k < kmax; ++k) logits[k] = -1e4f;
    if (nr > 1) {
      layer_norm(h + d, d, nr - 1, d, m->sc0_w, m->sc0_b, 1e-5f, x, d);
      gemm_nt(x, d, nr - 1, d, m->sc1_w, S, m->sc1_b, big, S, 0);
      for (int t = 0; t < (nr - 1) * S; ++t) big[t] = gelu_erf(big[t]);
      gemm_nt(big, S, nr - 1, S, m->sc3_w, 1, m->sc3_b, logits, 1, 0);
    }
  }
  if (m->head_layers == 0) { /* no head layers: pooled and scorer read the type-embedded rows */
    memcpy(pooled, h, sizeof(float) * d);
    for (int k = 0; k < kmax; ++k) logits[k] = -1e4f;
    const int S = m->scorer_hidden;
    for (int t = 1; t < nr; ++t) {
      layer_norm(h + (size_t)rows[t] * d, d, 1, d, m->sc0_w, m->sc0_b, 1e-5f, x, d);
      gemm_nt(x, d, 1, d, m->sc1_w, S, m->sc1_b, big, S, 0);
      for (int c = 0; c < S; ++c) big[c] = gelu_erf(big[c]);
      gemm_nt(big, S, 1, S, m->sc3_w, 1, m->sc3_b, logits + t - 1, 1, 0);
    }
  }
  free(h); free(x); free(big); free(act); free(rows);
  return 0;
}
