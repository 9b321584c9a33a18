/* wasr_oracle.c -- CPU restatement of the reference CPU path (TEST INFRASTRUCTURE ONLY).
 *
 * Parity checker and timed CPU baseline; see wasr_oracle.h for who may use it.  Each
 * function cites the Rust it restates.  Build with -ffp-contract=off and without
 * -ffast-math: every float expression below is evaluated exactly in the written order,
 * like rustc does.  OpenMP stands in for rayon (same work split: 32-column N tiles for the
 * GEMM, rows for the row-wise ops, frames for fbank and the conv frontend).
 */
#include "wasr_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#define D WASR_D
#define HEADS WASR_HEADS
#define HD WASR_HD
#define FF WASR_FF
#define DIM WASR_DIM
#define F1 WASR_C1
#define F2 WASR_C2
#define F3 WASR_C3
#define K2 (F1 * 49)
#define K3 (F2 * 9)
#define W2 WASR_W2
#define FLAT WASR_FLAT

static int g_threads = 0;

void wo_set_threads(int n) {
  g_threads = n;
  if (n > 0) omp_set_num_threads(n);
}
int wo_get_threads(void) { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

/* ------------------------------------------------------------------ quant
 * src/kernels.rs:11-25.  Rust `f32::round` rounds half away from zero == C roundf. */
void wo_quant(const float* x, int64_t t, int k, int8_t* q, float* s) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < t; i++) {
    const float* r = x + i * (int64_t)k;
    float m = 0.0f;
    for (int j = 0; j < k; j++) m = fmaxf(m, fabsf(r[j]));
    float sc = m > 0.0f ? m / 127.0f : 1.0f;
    float inv = 1.0f / sc;
    int8_t* qr = q + i * (int64_t)k;
    for (int j = 0; j < k; j++) {
      float v = roundf(r[j] * inv);
      if (v > 127.0f) v = 127.0f;
      if (v < -127.0f) v = -127.0f;
      qr[j] = v != v ? 0 : (int8_t)v;  /* Rust: NaN.clamp(..) is NaN, and NaN as i8 is 0 */
    }
    s[i] = sc;
  }
}

/* src/kernels.rs:87-97 */
int32_t wo_dot1(const int8_t* a, const int8_t* b, int k) {
  int32_t acc[16] = {0};
  int c = k / 16;
  for (int i = 0; i < c; i++)
    for (int l = 0; l < 16; l++) acc[l] += (int32_t)a[i * 16 + l] * (int32_t)b[i * 16 + l];
  int32_t s = 0;
  for (int l = 0; l < 16; l++) s += acc[l];
  int32_t r = 0;
  for (int j = c * 16; j < k; j++) r += (int32_t)a[j] * (int32_t)b[j];
  return s + r;
}

/* src/kernels.rs:136-141 */
__attribute__((target("avx2"))) static inline int32_t hsum(__m256i v) {
  __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E)); /* 0b01_00_11_10 */
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1)); /* 0b10_11_00_01 */
  return _mm_cvtsi128_si32(s);
}

/* src/kernels.rs:143-168: |x| (u8) x sign(w, x) (i8) via maddubs into i16 pairs, then madd
 * to i32.  Exact for weights in [-127, 127]; a weight of -128 against a negative activation
 * flips sign there (sign_epi8 cannot negate -128), the same as the reference. */
__attribute__((target("avx2"))) static void dot2x4(const int8_t* x0p, const int8_t* x1p,
                                                   const int8_t* const w[4], int k,
                                                   int32_t r[2][4]) {
  const __m256i ones = _mm256_set1_epi16(1);
  __m256i a[8];
  for (int i = 0; i < 8; i++) a[i] = _mm256_setzero_si256();
  for (int i = 0; i < k; i += 32) {
    __m256i x0 = _mm256_loadu_si256((const __m256i*)(x0p + i));
    __m256i x1 = _mm256_loadu_si256((const __m256i*)(x1p + i));
    __m256i u0 = _mm256_sign_epi8(x0, x0), u1 = _mm256_sign_epi8(x1, x1);
    for (int b = 0; b < 4; b++) {
      __m256i wv = _mm256_loadu_si256((const __m256i*)(w[b] + i));
      __m256i p0 = _mm256_madd_epi16(_mm256_maddubs_epi16(u0, _mm256_sign_epi8(wv, x0)), ones);
      __m256i p1 = _mm256_madd_epi16(_mm256_maddubs_epi16(u1, _mm256_sign_epi8(wv, x1)), ones);
      a[b] = _mm256_add_epi32(a[b], p0);
      a[4 + b] = _mm256_add_epi32(a[4 + b], p1);
    }
  }
  for (int b = 0; b < 4; b++) {
    r[0][b] = hsum(a[b]);
    r[1][b] = hsum(a[4 + b]);
  }
}

static int have_avx2(void) {
  static int v = -1;
  if (v < 0) v = __builtin_cpu_supports("avx2") ? 1 : 0;
  return v;
}

/* src/kernels.rs:65-85: xr rows (<=2) x wr rows (<=4); missing rows repeat the last one */
static void dot_tile(const int8_t* x, int xr, const int8_t* w, int wr, int k, int32_t r[2][4]) {
  const int8_t* xp0 = x;
  const int8_t* xp1 = x + (int64_t)(xr - 1) * k;
  const int8_t* wp[4];
  for (int b = 0; b < 4; b++) wp[b] = w + (int64_t)(b < wr ? b : wr - 1) * k;
  if (k % 32 == 0 && have_avx2()) {
    dot2x4(xp0, xp1, wp, k, r);
    return;
  }
  memset(r, 0, sizeof(int32_t) * 8);
  for (int a = 0; a < xr; a++)
    for (int b = 0; b < wr; b++) r[a][b] = wo_dot1(x + (int64_t)a * k, w + (int64_t)b * k, k);
}

/* src/kernels.rs:33-63: 32-column N tiles in parallel, 4 weight rows x 2 activation rows per
 * register tile; epilogue `acc as f32 * x.s[i] * ws + bias` left to right (bias 0.0 when
 * absent, as `bias.map_or(0.0, ..)`). */
void wo_qgemm(const int8_t* xq, const float* xs, int64_t t, int k, const int8_t* w, int n, float ws,
              const float* ws_vec, const float* bias, float* out) {
  const int TILE = 32;
  int ntiles = (n + TILE - 1) / TILE;
#pragma omp parallel for schedule(dynamic)
  for (int ti = 0; ti < ntiles; ti++) {
    int n0 = ti * TILE, n1 = n0 + TILE < n ? n0 + TILE : n;
    int j = n0;
    while (j < n1) {
      int rows = n1 - j < 4 ? n1 - j : 4;
      int64_t i = 0;
      while (i < t) {
        int r2 = t - i < 2 ? (int)(t - i) : 2;
        int32_t acc[2][4];
        dot_tile(xq + i * k, r2, w + (int64_t)j * k, rows, k, acc);
        for (int a = 0; a < r2; a++)
          for (int b = 0; b < rows; b++) {
            float sc = ws_vec ? ws_vec[j + b] : ws;
            float v = (float)acc[a][b] * xs[i + a] * sc + (bias ? bias[j + b] : 0.0f);
            out[(i + a) * n + j + b] = v;
          }
        i += r2;
      }
      j += rows;
    }
  }
}

void wo_qgemm_acc(const int8_t* xq, int64_t t, int k, const int8_t* w, int n, int32_t* acc) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < t; i++)
    for (int j = 0; j < n; j++) acc[i * n + j] = wo_dot1(xq + i * k, w + (int64_t)j * k, k);
}

/* src/kernels.rs:172-183: 8 lane accumulators over whole chunks, lanes summed in order,
 * then the tail summed on its own and added. */
float wo_dotf(const float* a, const float* b, int n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int c = n / 8;
  for (int i = 0; i < c; i++)
    for (int l = 0; l < 8; l++) acc[l] += a[i * 8 + l] * b[i * 8 + l];
  float s = 0.0f;
  for (int l = 0; l < 8; l++) s += acc[l];
  float r = 0.0f;
  for (int j = c * 8; j < n; j++) r += a[j] * b[j];
  return s + r;
}

/* src/model.rs:693-704: sequential sums (Rust iter().sum() is a left fold). */
void wo_norm(const float* x, int64_t t, int d, const float* g, const float* b, float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < t; i++) {
    const float* r = x + i * d;
    float* o = y + i * d;
    float sum = 0.0f;
    for (int j = 0; j < d; j++) sum += r[j];
    float m = sum / (float)d;
    float s2 = 0.0f;
    for (int j = 0; j < d; j++) s2 += (r[j] - m) * (r[j] - m);
    float v = s2 / (float)d;
    float inv = 1.0f / sqrtf(v + 1e-6f);
    for (int j = 0; j < d; j++) o[j] = (r[j] - m) * inv * g[j] + b[j];
  }
}

/* src/model.rs:710-712 */
float wo_gelu(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978846f * (x + 0.044715f * x * x * x)));
}

void wo_libm_tanhf(const float* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) y[i] = tanhf(x[i]);
}
void wo_libm_expf(const float* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) y[i] = expf(x[i]);
}
void wo_gelu_array(const float* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) y[i] = wo_gelu(x[i]);
}

/* src/model.rs:714-739 */
void wo_attention(const float* q, const float* k, const float* v, int t, float* out) {
  memset(out, 0, sizeof(float) * (size_t)t * D);
#pragma omp parallel
  {
    float* s = (float*)malloc(sizeof(float) * (size_t)(t > 0 ? t : 1));
#pragma omp for schedule(static)
    for (int i = 0; i < t; i++) {
      float* o = out + (int64_t)i * D;
      for (int h = 0; h < HEADS; h++) {
        const float* qi = q + (int64_t)i * D + h * HD;
        for (int j = 0; j < t; j++) s[j] = wo_dotf(qi, k + (int64_t)j * D + h * HD, HD) * 0.125f;
        float m = -3.40282347e+38f; /* f32::MIN */
        for (int j = 0; j < t; j++) m = fmaxf(m, s[j]);
        float z = 0.0f;
        for (int j = 0; j < t; j++) {
          s[j] = expf(s[j] - m);
          z += s[j];
        }
        float* oh = o + h * HD;
        for (int j = 0; j < t; j++) {
          const float* vj = v + (int64_t)j * D + h * HD;
          float a = s[j];
          for (int dd = 0; dd < HD; dd++) oh[dd] += a / z * vj[dd];
        }
      }
    }
    free(s);
  }
}

/* src/model.rs:398-418: conv 5x5, 1->32, pad 2 in time and frequency, of one window's
 * x [t][40] -> y1 [t][32][40] (im2col + dotf + ReLU) */
void wo_conv1(const float* x, int t, const float* c1, float* y1) {
#pragma omp parallel for schedule(static)
  for (int ti = 0; ti < t; ti++) {
    float p[DIM][25];
    memset(p, 0, sizeof(p));
    for (int f = 0; f < DIM; f++)
      for (int i = 0; i < 5; i++) {
        int tt = ti + i - 2;
        if (tt < 0 || tt >= t) continue;
        for (int j = 0; j < 5; j++) {
          int ff = f + j - 2;
          if (ff >= 0 && ff < DIM) p[f][i * 5 + j] = x[(int64_t)tt * DIM + ff];
        }
      }
    float* y = y1 + (int64_t)ti * F1 * DIM;
    for (int o = 0; o < F1; o++)
      for (int f = 0; f < DIM; f++) y[o * DIM + f] = fmaxf(wo_dotf(c1 + o * 25, p[f], 25), 0.0f);
  }
}

/* src/model.rs:420-444: conv 7x7, 32->64, time stride 5 (pad 1), frequency pad 3 of one
 * window's y1 [t][32][40] -> y2 [t1][64][41], t1 = (t - 5) / 5 + 1; column 40 is 0 */
void wo_conv2(const float* y1, int t, const float* c2, float* y2) {
  if (t < 5) return;
  int t1 = (t - 5) / 5 + 1;
#pragma omp parallel
  {
    float* p = (float*)malloc(sizeof(float) * DIM * K2);
#pragma omp for schedule(static)
    for (int ti = 0; ti < t1; ti++) {
      memset(p, 0, sizeof(float) * DIM * K2);
      for (int i = 0; i < 7; i++) {
        int tt = ti * 5 + i - 1;
        if (tt < 0 || tt >= t) continue;
        const float* row = y1 + (int64_t)tt * F1 * DIM;
        for (int c = 0; c < F1; c++)
          for (int f = 0; f < DIM; f++)
            for (int j = 0; j < 7; j++) {
              int ff = f + j - 3;
              if (ff >= 0 && ff < DIM) p[f * K2 + c * 49 + i * 7 + j] = row[c * DIM + ff];
            }
      }
      float* y = y2 + (int64_t)ti * F2 * W2;
      for (int o = 0; o < F2; o++) {
        for (int f = 0; f < DIM; f++) y[o * W2 + f] = fmaxf(wo_dotf(c2 + (int64_t)o * K2, p + f * K2, K2), 0.0f);
        y[o * W2 + DIM] = 0.0f;
      }
    }
    free(p);
  }
}

/* src/model.rs:446-468: conv 3x3, 64->192, frequency stride 2, time pad 1 of one window's
 * y2 [t1][64][41] -> y3 [t1][192*20] (im2col + dotf + ReLU) */
void wo_conv3(const float* y2, int t1, const float* c3, float* y3) {
#pragma omp parallel
  {
    float* p = (float*)malloc(sizeof(float) * 20 * K3);
#pragma omp for schedule(static)
    for (int ti = 0; ti < t1; ti++) {
      memset(p, 0, sizeof(float) * 20 * K3);
      for (int i = 0; i < 3; i++) {
        int tt = ti + i - 1;
        if (tt < 0 || tt >= t1) continue;
        const float* row = y2 + (int64_t)tt * F2 * W2;
        for (int c = 0; c < F2; c++)
          for (int f = 0; f < 20; f++)
            for (int j = 0; j < 3; j++) p[f * K3 + c * 9 + i * 3 + j] = row[c * W2 + 2 * f + j];
      }
      float* y = y3 + (int64_t)ti * FLAT;
      for (int o = 0; o < F3; o++)
        for (int f = 0; f < 20; f++)
          y[o * 20 + f] = fmaxf(wo_dotf(c3 + (int64_t)o * K3, p + f * K3, K3), 0.0f);
    }
    free(p);
  }
}

/* src/model.rs:389-478 (im2col + dotf + ReLU) */
int wo_frontend(const float* x, int t, const float* c1, const float* c2, const float* c3,
                float* y3) {
  if (t < 5) return 0;
  int t1 = (t - 5) / 5 + 1;
  float* y1 = (float*)calloc((size_t)t * F1 * DIM, sizeof(float));
  float* y2 = (float*)calloc((size_t)t1 * F2 * W2, sizeof(float));
  wo_conv1(x, t, c1, y1);
  wo_conv2(y1, t, c2, y2);
  wo_conv3(y2, t1, c3, y3);
  free(y1);
  free(y2);
  return t1;
}

/* src/model.rs:499-500: fold from (0, f32::MIN), strictly greater replaces -> first max */
uint32_t wo_argmax(const float* row, int n) {
  uint32_t bi = 0;
  float bv = -3.40282347e+38f;
  for (int j = 0; j < n; j++)
    if (row[j] > bv) {
      bv = row[j];
      bi = (uint32_t)j;
    }
  return bi;
}

/* Model::mm (src/model.rs:361-365) with the optional per-channel scale extension */
static void mm(const uint8_t* blob, const int8_t* xq, const float* xs, int64_t t, int k,
               const WasrMat* q, int n, uint64_t bias_off, float* out) {
  const float* ws_vec = q->scale_off == WASR_NONE ? NULL : (const float*)(blob + q->scale_off);
  const float* bias = bias_off == WASR_NONE ? NULL : (const float*)(blob + bias_off);
  wo_qgemm(xq, xs, t, k, (const int8_t*)(blob + q->off), n, q->s, ws_vec, bias, out);
}

static void add_inplace(float* h, const float* o, int64_t n) {
  for (int64_t i = 0; i < n; i++) h[i] += o[i];
}

/* src/model.rs:488-502 */
int wo_run_post(const uint8_t* blob, const WasrPlan* plan, int t1, const float* y3, uint32_t* ids,
                float* logits) {
  int64_t T = t1;
  int vocab = plan->vocab;
  float* h = (float*)malloc(sizeof(float) * T * D);
  float* y = (float*)malloc(sizeof(float) * T * D);
  float* q = (float*)malloc(sizeof(float) * T * D);
  float* k = (float*)malloc(sizeof(float) * T * D);
  float* v = (float*)malloc(sizeof(float) * T * D);
  float* a = (float*)malloc(sizeof(float) * T * D);
  float* o = (float*)malloc(sizeof(float) * T * D);
  float* f = (float*)malloc(sizeof(float) * T * FF);
  int8_t* xq = (int8_t*)malloc((size_t)T * FLAT);
  float* xs = (float*)malloc(sizeof(float) * T);
  float* lo = logits ? logits : (float*)malloc(sizeof(float) * T * vocab);

  wo_quant(y3, T, FLAT, xq, xs);
  mm(blob, xq, xs, T, FLAT, &plan->lin, D, plan->lin_b, h);
  for (int l = 0; l < plan->n_layers; l++) {
    const WasrLayer* L = &plan->layers[l];
    wo_norm(h, T, D, (const float*)(blob + L->pn_g), (const float*)(blob + L->pn_b), y);
    wo_quant(y, T, D, xq, xs);
    mm(blob, xq, xs, T, D, &L->q, D, L->qb, q);
    mm(blob, xq, xs, T, D, &L->k, D, L->kb, k);
    mm(blob, xq, xs, T, D, &L->v, D, L->vb, v);
    wo_attention(q, k, v, t1, a);
    wo_quant(a, T, D, xq, xs);
    mm(blob, xq, xs, T, D, &L->o, D, L->ob, o);
    add_inplace(h, o, T * D);
    wo_norm(h, T, D, (const float*)(blob + L->mn_g), (const float*)(blob + L->mn_b), y);
    wo_quant(y, T, D, xq, xs);
    mm(blob, xq, xs, T, D, &L->f1, FF, L->f1b, f);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < T * FF; i++) f[i] = wo_gelu(f[i]);
    wo_quant(f, T, FF, xq, xs);
    mm(blob, xq, xs, T, FF, &L->f2, D, L->f2b, o);
    add_inplace(h, o, T * D);
  }
  wo_quant(h, T, D, xq, xs);
  /* the CPU path multiplies by the unpadded vocab rows (Q out.n = vocab, src/model.rs:301) */
  mm(blob, xq, xs, T, D, &plan->out, vocab, plan->out_b, lo);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < T; i++) ids[i] = wo_argmax(lo + i * vocab, vocab);
  if (!logits) free(lo);
  free(h); free(y); free(q); free(k); free(v); free(a); free(o); free(f); free(xq); free(xs);
  return t1;
}

/* src/model.rs:368-386 (CPU branch: frontend then run_post) */
int wo_forward(const uint8_t* blob, const WasrPlan* plan, const float* x, int t, uint32_t* ids,
               float* logits) {
  if (t < 5) return 0;
  int t1 = (t - 5) / 5 + 1;
  float* y3 = (float*)malloc(sizeof(float) * (size_t)t1 * FLAT);
  wo_frontend(x, t, (const float*)(blob + plan->c1), (const float*)(blob + plan->c2),
              (const float*)(blob + plan->c3), y3);
  wo_run_post(blob, plan, t1, y3, ids, logits);
  free(y3);
  return t1;
}

/* src/model.rs:622-642 (token ids only) */
int64_t wo_ctc(const uint32_t* ids, int64_t n, uint32_t* out) {
  int64_t m = 0;
  uint32_t prev = 0xFFFFFFFFu;
  for (int64_t i = 0; i < n; i++) {
    if (ids[i] != prev && ids[i] != 0) out[m++] = ids[i];
    prev = ids[i];
  }
  return m;
}

/* ------------------------------------------------------------------ fbank
 * src/fbank.rs (f64 throughout; same table construction and FFT butterfly order). */
#define WIN 400
#define HOP 160
#define NFFT 512
#define NCH 39
#define CMS_WIN 50

typedef struct {
  double ham[WIN];
  double twr[NFFT / 2], twi[NFFT / 2];
  int lo[NFFT / 2], hi[NFFT / 2];
  double wl[NFFT / 2], wh[NFFT / 2];
} FbTables;

static double mel(double f) { return 1127.0 * log(1.0 + f / 700.0); }

/* src/fbank.rs:21-44 */
static const FbTables* fb_tables(void) {
  static FbTables T;
  static int init = 0;
#pragma omp critical(wo_fb_tables)
  if (!init) {
    const double pi = 3.14159265358979323846;
    for (int n = 0; n < WIN; n++) T.ham[n] = 0.54 - 0.46 * cos(2.0 * pi * (double)n / (double)(WIN - 1));
    for (int i = 0; i < NFFT / 2; i++) {
      double a = -2.0 * pi * (double)i / (double)NFFT;
      T.twr[i] = cos(a);
      T.twi[i] = sin(a);
    }
    double hi = mel(8000.0);
    double cf[NCH + 1];
    for (int i = 1; i <= NCH + 1; i++) cf[i - 1] = hi * (double)i / (double)(NCH + 1);
    for (int k = 1; k <= NFFT / 2; k++) {
      double m = mel((double)k * 16000.0 / (double)NFFT);
      int c = 0;
      while (c < NCH + 1 && cf[c] < m) c++;
      int idx = k - 1;
      if (c == 0) {
        T.lo[idx] = 0; T.wl[idx] = m / cf[0]; T.hi[idx] = 0; T.wh[idx] = 0.0;
      } else if (c < NCH) {
        double w = (cf[c] - m) / (cf[c] - cf[c - 1]);
        T.lo[idx] = c - 1; T.wl[idx] = w; T.hi[idx] = c; T.wh[idx] = 1.0 - w;
      } else if (c == NCH) {
        T.lo[idx] = NCH - 1; T.wl[idx] = (cf[NCH] - m) / (cf[NCH] - cf[NCH - 1]);
        T.hi[idx] = 0; T.wh[idx] = 0.0;
      } else {
        T.lo[idx] = 0; T.wl[idx] = 0.0; T.hi[idx] = 0; T.wh[idx] = 0.0;
      }
    }
    init = 1;
  }
  return &T;
}

/* src/fbank.rs:46-77: in-place radix-2, bit-reversal permutation then butterflies */
static void fft(double* re, double* im, const FbTables* T) {
  int j = 0;
  for (int i = 1; i < NFFT; i++) {
    int b = NFFT >> 1;
    while (j & b) {
      j ^= b;
      b >>= 1;
    }
    j |= b;
    if (i < j) {
      double x = re[i]; re[i] = re[j]; re[j] = x;
      x = im[i]; im[i] = im[j]; im[j] = x;
    }
  }
  for (int len = 2; len <= NFFT; len <<= 1) {
    int step = NFFT / len;
    for (int s = 0; s < NFFT; s += len)
      for (int k = 0; k < len / 2; k++) {
        double wr = T->twr[k * step], wi = T->twi[k * step];
        int a = s + k, b = s + k + len / 2;
        double tr = re[b] * wr - im[b] * wi;
        double ti = re[b] * wi + im[b] * wr;
        re[b] = re[a] - tr;
        im[b] = im[a] - ti;
        re[a] += tr;
        im[a] += ti;
      }
  }
}

/* src/fbank.rs:79-102 */
void wo_fbank_frame(const int16_t* x, double* out) {
  const FbTables* T = fb_tables();
  double re[NFFT], im[NFFT];
  memset(re, 0, sizeof(re));
  memset(im, 0, sizeof(im));
  double e = 0.0;
  for (int n = 0; n < WIN; n++) {
    double v = (double)x[n];
    e += v * v;
    double pe = n == 0 ? v * (1.0 - 0.97) : v - 0.97 * (double)x[n - 1];
    re[n] = pe * T->ham[n];
  }
  fft(re, im, T);
  for (int i = 0; i < DIM; i++) out[i] = 0.0;
  for (int k = 0; k < NFFT / 2; k++) {
    double p = re[k + 1] * re[k + 1] + im[k + 1] * im[k + 1];
    out[T->lo[k]] += p * T->wl[k];
    out[T->hi[k]] += p * T->wh[k];
  }
  for (int i = 0; i < NCH; i++) out[i] = log(out[i] > 1.0 ? out[i] : 1.0);
  out[NCH] = log(e > 1e-10 ? e : 1e-10);
}

/* src/fbank.rs:111-161: frames in parallel, then the CMS running mean in frame order. */
int64_t wo_fbank(const int16_t* pcm, int64_t n, float* feats, int64_t cap, float* sil) {
  int64_t nfr = n >= WIN ? (n - WIN) / HOP + 1 : 0;
  if (!feats) return nfr;
  if (nfr > cap) return -1;
  double* raw = (double*)malloc(sizeof(double) * (size_t)(nfr > 0 ? nfr : 1) * DIM);
  (void)fb_tables();
#pragma omp parallel for schedule(static)
  for (int64_t k = 0; k < nfr; k++) wo_fbank_frame(pcm + k * HOP, raw + k * DIM);
  double sum[DIM];
  for (int i = 0; i < DIM; i++) sum[i] = 0.0;
  int64_t hn = 0;   /* hist.len() */
  for (int64_t k = 0; k < nfr; k++) {
    const double* f = raw + k * DIM;
    if (hn == CMS_WIN) {
      const double* o = raw + (k - CMS_WIN) * DIM;
      for (int i = 0; i < DIM; i++) sum[i] -= o[i];
      hn--;
    }
    hn++;
    for (int i = 0; i < DIM; i++) sum[i] += f[i];
    double nn = (double)(hn > 0 ? hn : 1);
    for (int i = 0; i < DIM; i++) feats[k * DIM + i] = (float)(f[i] - sum[i] / nn);
  }
  if (sil) {
    double s[DIM];
    for (int i = 0; i < DIM; i++) s[i] = 0.0;
    s[NCH] = log(1e-10);
    double nn = (double)(hn > 0 ? hn : 1);
    for (int i = 0; i < DIM; i++) sil[i] = (float)(s[i] - sum[i] / nn);
  }
  free(raw);
  return nfr;
}

/* ------------------------------------------------------------------ stream schedule
 * src/stream.rs:128-134 decode(): window [s - prev, end) + pad silence frames, keep the
 * output frames from s on. */
static int64_t decode(const uint8_t* blob, const WasrPlan* plan, const float* feats,
                      const float* sil, int64_t s, int prev, int64_t end, int pad, uint32_t* out,
                      int* n_fwd) {
  int64_t a = s > prev ? s - prev : 0;
  int64_t t = end - a + pad;
  float* x = (float*)malloc(sizeof(float) * (size_t)(t > 0 ? t : 1) * DIM);
  memcpy(x, feats + a * DIM, sizeof(float) * (size_t)(end - a) * DIM);
  for (int64_t i = end - a; i < t; i++) memcpy(x + i * DIM, sil, sizeof(float) * DIM);
  int64_t t1 = t >= 5 ? (t - 5) / 5 + 1 : 0;
  uint32_t* ids = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(t1 > 0 ? t1 : 1));
  if (t1 > 0) wo_forward(blob, plan, x, (int)t, ids, NULL);
  if (n_fwd) (*n_fwd)++;
  int64_t from = (s - a) / 5;
  int64_t m = t1 > from ? t1 - from : 0;
  if (m > 0) memcpy(out, ids + from, sizeof(uint32_t) * (size_t)m);
  free(x);
  free(ids);
  return m;
}

/* src/stream.rs:58-70 (push of the whole utterance), 136-147 (commit), 159-168 (finish) */
int64_t wo_transcribe(const uint8_t* blob, const WasrPlan* plan, const float* feats, int64_t n,
                      const float* sil, int prev, int blk, int post, uint32_t* ids, int64_t ids_cap,
                      int* n_fwd) {
  if (n_fwd) *n_fwd = 0;
  int64_t len = 0, s = 0;
  /* Stream::push runs commit() while feats >= s + blk + post; the whole-utterance branch
   * of finish() (n <= WHOLE_MAX) only discards those commits, so it is taken first. */
  if (n <= WASR_WHOLE_MAX) {
    if (n < 5) return 0;
    int64_t t1 = (n - 5) / 5 + 1;
    if (t1 > ids_cap) return -1;
    wo_forward(blob, plan, feats, (int)n, ids, NULL);
    if (n_fwd) (*n_fwd)++;
    return t1;
  }
  uint32_t* buf = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n / 5 + 64));
  while (n >= s + blk + post) {
    int64_t m = decode(blob, plan, feats, sil, s, prev, s + blk + post, WASR_PAD, buf, n_fwd);
    if (m > blk / 5) m = blk / 5;
    for (int64_t c = m - 1; c >= m / 2 && c >= 1; c--)
      if (buf[c] == 0 && buf[c - 1] == 0) {
        m = c;
        break;
      }
    if (len + m > ids_cap) { free(buf); return -1; }
    memcpy(ids + len, buf, sizeof(uint32_t) * (size_t)m);
    len += m;
    s += m * 5;
  }
  if (n > s) {
    int64_t m = decode(blob, plan, feats, sil, s, prev, n, WASR_PAD, buf, n_fwd);
    if (len + m > ids_cap) { free(buf); return -1; }
    memcpy(ids + len, buf, sizeof(uint32_t) * (size_t)m);
    len += m;
  }
  free(buf);
  return len;
}

/* ---- streaming schedule (src/stream.rs:128-168) over features that arrive in pieces.  The
 * caller keeps every frame so far (feats, n), the silence frame as the stream's fbank gives it
 * now (sil), and the stream state: the commit position *s and the committed ids (ids, *n_ids). */

/* push's loop (src/stream.rs:67-69): commit() while n >= s + blk + post (136-147) */
int wo_stream_commit(const uint8_t* blob, const WasrPlan* plan, const float* feats, int64_t n,
                     const float* sil, int prev, int blk, int post, int64_t* s, uint32_t* ids,
                     int64_t* n_ids, int64_t cap, int* n_fwd) {
  uint32_t* buf = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n / 5 + 64));
  while (n >= *s + blk + post) {
    int64_t m = decode(blob, plan, feats, sil, *s, prev, *s + blk + post, WASR_PAD, buf, n_fwd);
    if (m > blk / 5) m = blk / 5;
    for (int64_t c = m - 1; c >= m / 2 && c >= 1; c--)
      if (buf[c] == 0 && buf[c - 1] == 0) {
        m = c;
        break;
      }
    if (*n_ids + m > cap) { free(buf); return -1; }
    memcpy(ids + *n_ids, buf, sizeof(uint32_t) * (size_t)m);
    *n_ids += m;
    *s += m * 5;
  }
  free(buf);
  return 0;
}

/* partial() ids (src/stream.rs:150-157): the committed ids, then the open tail decoded with
 * half the left context; finish() ids (159-168): the whole utterance at once when it is at most
 * WHOLE_MAX frames, else the committed ids and the tail with the full left context.  Returns the
 * id count written to out, or -1. */
int64_t wo_stream_tail(const uint8_t* blob, const WasrPlan* plan, const float* feats, int64_t n,
                       const float* sil, int prev, int64_t s, const uint32_t* ids, int64_t n_ids,
                       int finish, uint32_t* out, int64_t cap, int* n_fwd) {
  if (finish && n <= WASR_WHOLE_MAX) {
    const int64_t t1 = n >= 5 ? (n - 5) / 5 + 1 : 0;
    if (t1 > cap) return -1;
    if (t1 > 0) {
      wo_forward(blob, plan, feats, (int)n, out, NULL);
      if (n_fwd) (*n_fwd)++;
    }
    return t1;
  }
  if (n_ids > cap) return -1;
  memcpy(out, ids, sizeof(uint32_t) * (size_t)n_ids);
  int64_t len = n_ids;
  if (n > s) {
    uint32_t* buf = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n / 5 + 64));
    const int64_t m = decode(blob, plan, feats, sil, s, finish ? prev : prev / 2, n, WASR_PAD, buf, n_fwd);
    if (len + m > cap) { free(buf); return -1; }
    memcpy(out + len, buf, sizeof(uint32_t) * (size_t)m);
    len += m;
    free(buf);
  }
  return len;
}

/* ---- text output: Model::text (src/model.rs:620-642) and tidy (src/stream.rs:203-210) */

/* UTF-8 helpers: length of the sequence starting at p, and its code point */
static int u8len(const unsigned char* p) {
  return p[0] < 0x80 ? 1 : (p[0] >> 5) == 6 ? 2 : (p[0] >> 4) == 14 ? 3 : 4;
}
static uint32_t u8cp(const unsigned char* p) {
  const int l = u8len(p);
  if (l == 1) return p[0];
  if (l == 2) return ((uint32_t)(p[0] & 31) << 6) | (p[1] & 63);
  if (l == 3) return ((uint32_t)(p[0] & 15) << 12) | ((uint32_t)(p[1] & 63) << 6) | (p[2] & 63);
  return ((uint32_t)(p[0] & 7) << 18) | ((uint32_t)(p[1] & 63) << 12) | ((uint32_t)(p[2] & 63) << 6) | (p[3] & 63);
}
/* PUNCT of src/stream.rs:173: ，。？！、,.?! */
static int is_punct(uint32_t c) {
  return c == 0xFF0C || c == 0x3002 || c == 0xFF1F || c == 0xFF01 || c == 0x3001 || c == ',' || c == '.' ||
         c == '?' || c == '!';
}

/* ids -> UTF-8 text: repeats and blank 0 dropped, "<UNK>" skipped, "<SPACE>" a space, "|w"
 * starts an English word (a space first when the text ends in an ASCII letter or digit).
 * vocab: n_vocab NUL-terminated UTF-8 tokens.  Returns the byte length (out is NUL-terminated),
 * or -1 if cap is short or an id is outside the vocabulary. */
int64_t wo_text(const uint32_t* ids, int64_t n, const char* const* vocab, int64_t n_vocab, char* out, int64_t cap) {
  int64_t len = 0;
  uint32_t prevt = 0xFFFFFFFFu;
  if (cap < 1) return -1;
  for (int64_t k = 0; k < n; k++) {
    const uint32_t i = ids[k];
    if (i != prevt && i != 0) {
      if ((int64_t)i >= n_vocab) return -1;
      const char* t = vocab[i];
      const size_t tl = strlen(t);
      if (strcmp(t, "<UNK>") == 0) {
      } else if (strcmp(t, "<SPACE>") == 0) {
        if (len + 2 > cap) return -1;
        out[len++] = ' ';
      } else if (tl > 1 && t[0] == '|') {
        const char last = len > 0 ? out[len - 1] : 0;
        const int alnum = (last >= '0' && last <= '9') || (last >= 'a' && last <= 'z') || (last >= 'A' && last <= 'Z');
        if (len + (alnum ? 1 : 0) + (int64_t)tl > cap) return -1;
        if (alnum) out[len++] = ' ';
        memcpy(out + len, t + 1, tl - 1);
        len += (int64_t)tl - 1;
      } else {
        if (len + (int64_t)tl + 1 > cap) return -1;
        memcpy(out + len, t, tl);
        len += (int64_t)tl;
      }
    }
    prevt = i;
  }
  out[len] = 0;
  return len;
}

/* tidy: leading punctuation removed; of a run of punctuation marks only the last kept.
 * trim_end: also remove trailing punctuation (partial()).  In place; returns the new length. */
int64_t wo_tidy(char* s, int trim_end) {
  const unsigned char* p = (const unsigned char*)s;
  int64_t n = (int64_t)strlen(s), i = 0, o = 0;
  while (i < n && is_punct(u8cp(p + i))) i += u8len(p + i);
  char* w = s;
  while (i < n) {
    const int l = u8len(p + i);
    const int pc = is_punct(u8cp(p + i));
    const int next_pc = i + l < n && is_punct(u8cp(p + i + l));
    if (!(pc && next_pc)) {
      memmove(w + o, s + i, (size_t)l);
      o += l;
    }
    i += l;
  }
  w[o] = 0;
  if (trim_end) {
    /* strip trailing punctuation: find the last non-punctuation character */
    int64_t j = 0, keep = 0;
    while (j < o) {
      const int l = u8len((const unsigned char*)w + j);
      if (!is_punct(u8cp((const unsigned char*)w + j))) keep = j + l;
      j += l;
    }
    o = keep;
    w[o] = 0;
  }
  return o;
}
