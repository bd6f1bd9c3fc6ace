/*
 * CPU ORACLE -- test infrastructure only.
 *
 * Plain-C restatement of the reference W4A4 arithmetic, used by tests/ as the
 * parity checker and by bench.py's CPU-baseline leg. Nothing in the product
 * (dscquant_b200/) links or calls this file.
 *
 *   orc_quant_rows   per-row int4 quantizers:
 *                    ACT_SYM     scale = max(absmax*clip/7, 1e-8), clamp(rn(y/s), -8, 7)
 *                    WEIGHT_SYM  core/quantization.py:7-11 (bound 7)
 *                    ACT_ASYM    kernel/w4a4.cu:20-63 as nvcc compiles it: scale = (max*clip -
 *                                min*clip)/15 with the subtraction fused into one fma
 *                                (fmaf(max, clip, -(min*clip))), q = rn(y/s + zero), packed (q-8)&15
 *                    ACT_ASYM_T  core/quantization.py:13-21 (rn(y/s + zero))
 *   orc_rotate       y = x (H_a (x) H_b) / sqrt(K) in double precision
 *   orc_gemm_s4      raw[m,n] = sum_k a_s4[m,k] b_s4[n,k]  (kernel/w4a4.cu:123-148)
 *   orc_epilogue     ((raw + (8-zx) sums) * sx) * sw (+bias) (+residual)  (kernel/w4a4.cu:70-78)
 *   orc_w4a4_linear  rotate -> quantize -> gemm -> epilogue (bf16 out), pthreads
 *
 * Built with -ffp-contract=off and without -ffast-math so that every float
 * operation is one IEEE-754 binary32 operation with round-to-nearest-even,
 * like the reference's torch ops and __fdiv_rn / __float2int_rn.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---- minimal parallel-for over [0, n) with pthreads (ORC_THREADS or all cores) */
typedef void (*orc_range_fn)(int64_t begin, int64_t end, void* ctx);
typedef struct { orc_range_fn fn; void* ctx; int64_t b, e; } orc_job;
static void* orc_run(void* p) { orc_job* j = (orc_job*)p; j->fn(j->b, j->e, j->ctx); return NULL; }
static int g_threads = 0;
int orc_num_threads(void) {
  if (!g_threads) {
    const char* env = getenv("ORC_THREADS");
    g_threads = env ? atoi(env) : (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (g_threads < 1) g_threads = 1;
    if (g_threads > 256) g_threads = 256;
  }
  return g_threads;
}
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
static void par_for(int64_t n, orc_range_fn fn, void* ctx) {
  int t = orc_num_threads();
  if (t > n) t = (int)(n > 0 ? n : 1);
  if (t <= 1) { fn(0, n, ctx); return; }
  pthread_t th[256];
  orc_job jobs[256];
  for (int i = 0; i < t; ++i) {
    jobs[i].fn = fn; jobs[i].ctx = ctx;
    jobs[i].b = n * i / t; jobs[i].e = n * (i + 1) / t;
    if (i) pthread_create(&th[i], NULL, orc_run, &jobs[i]);
  }
  orc_run(&jobs[0]);
  for (int i = 1; i < t; ++i) pthread_join(th[i], NULL);
}

#define ORC_ACT_SYM 0
#define ORC_WEIGHT_SYM 1
#define ORC_ACT_ASYM 2
#define ORC_ACT_ASYM_T 3

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* round half to even for the magnitudes used here */
static inline int rn(float v) { return (int)lrintf(v); }

static inline int code_of(float y, float scale, int zero, int mode) {
  float q = y / scale;
  switch (mode) {
    case ORC_ACT_SYM: return clampi(rn(q), -8, 7);
    case ORC_WEIGHT_SYM: return clampi(rn(q), -7, 7);
    default: {  /* both asymmetric modes: kernel/w4a4.cu:50 and core/quantization.py:20 round y/s + zero */
      float t = q + (float)zero;
      return clampi(rn(t), 0, 15);
    }
  }
}

/* y [M, K] fp32 (row stride K). Outputs rows_out rows, KP columns (even). */
typedef struct {
  const float* y; int64_t M, K, KP; int mode; float clip;
  uint8_t* packed; float* scales; int32_t* zeros; int32_t* sums; int8_t* codes;
} quant_ctx;

static void quant_range(int64_t r0, int64_t r1, void* vctx) {
  const quant_ctx* q = (const quant_ctx*)vctx;
  const float* y = q->y; const int64_t M = q->M, K = q->K, KP = q->KP; const int mode = q->mode;
  const float clip = q->clip; uint8_t* packed = q->packed; float* scales = q->scales;
  int32_t* zeros = q->zeros; int32_t* sums = q->sums; int8_t* codes = q->codes;
  const int asym = mode == ORC_ACT_ASYM || mode == ORC_ACT_ASYM_T;
  for (int64_t r = r0; r < r1; ++r) {
    const float* row = y + r * K;
    const int live = r < M;
    float amax = 0.f, amin = 0.f;
    if (live)
      for (int64_t k = 0; k < K; ++k) {
        float v = row[k];
        if (asym) {
          if (v > amax) amax = v;
          if (v < amin) amin = v;
        } else {
          float a = fabsf(v);
          if (a > amax) amax = a;
        }
      }
    float scale;
    int zero = 0;
    if (asym) {
      float lo = amin * clip, hi = amax * clip;
      /* kernel/w4a4.cu:42-43: nvcc contracts maximum - minimum into fma(upper, clip, -minimum) */
      scale = (mode == ORC_ACT_ASYM ? fmaf(amax, clip, -lo) : hi - lo) / 15.f;
      if (!(scale > 1e-8f)) scale = 1e-8f;
      zero = clampi(rn(-lo / scale), 0, 15);
    } else {
      scale = (amax * clip) / 7.f;
      if (!(scale > 1e-8f)) scale = 1e-8f;
    }
    int32_t s = 0;
    const int pad = asym ? zero : 0;
    for (int64_t p = 0; p < KP / 2; ++p) {
      int64_t k = 2 * p;
      int c0 = (live && k < K) ? code_of(row[k], scale, zero, mode) : pad;
      int c1 = (live && k + 1 < K) ? code_of(row[k + 1], scale, zero, mode) : pad;
      if (k < K) s += c0;
      if (k + 1 < K) s += c1;
      int n0 = (asym ? c0 - 8 : c0) & 15, n1 = (asym ? c1 - 8 : c1) & 15;
      packed[r * (KP / 2) + p] = (uint8_t)(n0 | (n1 << 4));
      if (codes) {
        codes[r * KP + k] = (int8_t)c0;
        codes[r * KP + k + 1] = (int8_t)c1;
      }
    }
    scales[r] = scale;
    if (zeros) zeros[r] = zero;
    if (sums) sums[r] = s;
  }
}

void orc_quant_rows(const float* y, int64_t M, int64_t K, int64_t rows_out, int64_t KP, int mode, float clip,
                    uint8_t* packed, float* scales, int32_t* zeros, int32_t* sums, int8_t* codes) {
  quant_ctx q = {y, M, K, KP, mode, clip, packed, scales, zeros, sums, codes};
  par_for(rows_out, quant_range, &q);
}

/* In-place Walsh-Hadamard transform (unnormalised) of n = 2^j doubles. */
static void fwht(double* v, int64_t n) {
  for (int64_t h = 1; h < n; h <<= 1)
    for (int64_t i = 0; i < n; i += 2 * h)
      for (int64_t j = i; j < i + h; ++j) {
        double a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
}

/* y = x (H_a (x) H_b) / sqrt(K), K = a*b, index k = i*b + c. h_a: a*a +-1 (row-major) or NULL for a == 1. */
typedef struct { const float* x; int64_t K; int a; const int8_t* h_a; float* y; } rot_ctx;

static void rot_range(int64_t m0, int64_t m1, void* vctx) {
  const rot_ctx* r = (const rot_ctx*)vctx;
  const int64_t K = r->K, a = r->a, b = K / a;
  const double norm = 1.0 / sqrt((double)K);
  double* z = (double*)malloc(sizeof(double) * K);
  double* w = (double*)malloc(sizeof(double) * K);
  for (int64_t m = m0; m < m1; ++m) {
    for (int64_t k = 0; k < K; ++k) z[k] = r->x[m * K + k];
    for (int64_t i = 0; i < a; ++i) fwht(z + i * b, b);
    if (a > 1) {
      for (int64_t i2 = 0; i2 < a; ++i2)
        for (int64_t c = 0; c < b; ++c) {
          double acc = 0.0;
          for (int64_t i = 0; i < a; ++i) acc += r->h_a[i * a + i2] * z[i * b + c];
          w[i2 * b + c] = acc;
        }
      for (int64_t k = 0; k < K; ++k) r->y[m * K + k] = (float)(w[k] * norm);
    } else {
      for (int64_t k = 0; k < K; ++k) r->y[m * K + k] = (float)(z[k] * norm);
    }
  }
  free(z);
  free(w);
}

void orc_rotate(const float* x, int64_t M, int64_t K, int a, const int8_t* h_a, float* y) {
  rot_ctx r = {x, K, a, h_a, y};
  par_for(M, rot_range, &r);
}

static void unpack_rows(const uint8_t* p, int64_t rows, int64_t KP, int8_t* out) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t k = 0; k < KP; ++k) {
      int b = p[r * (KP / 2) + k / 2];
      int v = (k & 1) ? (b >> 4) : (b & 15);
      out[r * KP + k] = (int8_t)(v >= 8 ? v - 16 : v);
    }
}

typedef struct { const int8_t *A, *B; int64_t M, N, KP; int32_t* raw; } gemm_ctx;

static void gemm_range(int64_t t0, int64_t t1, void* vctx) {
  const gemm_ctx* g = (const gemm_ctx*)vctx;
  const int64_t NB = 64, nblk = (g->N + NB - 1) / NB;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t m0 = (t / nblk) * 8, n0 = (t % nblk) * NB;
    const int64_t m1 = m0 + 8 < g->M ? m0 + 8 : g->M, n1 = n0 + NB < g->N ? n0 + NB : g->N;
    for (int64_t m = m0; m < m1; ++m) {
      const int8_t* ar = g->A + m * g->KP;
      for (int64_t n = n0; n < n1; ++n) {
        const int8_t* br = g->B + n * g->KP;
        int32_t acc = 0;
        for (int64_t k = 0; k < g->KP; ++k) acc += (int32_t)ar[k] * (int32_t)br[k];
        g->raw[m * g->N + n] = acc;
      }
    }
  }
}

/* raw [M, N] = A_s4 [M, KP] . B_s4 [N, KP]^T, packed rows of KP/2 bytes. */
void orc_gemm_s4(const uint8_t* a, const uint8_t* b, int64_t M, int64_t N, int64_t KP, int32_t* raw) {
  int8_t* A = (int8_t*)malloc((size_t)(M * KP));
  int8_t* B = (int8_t*)malloc((size_t)(N * KP));
  unpack_rows(a, M, KP, A);
  unpack_rows(b, N, KP, B);
  gemm_ctx g = {A, B, M, N, KP, raw};
  par_for(((M + 7) / 8) * ((N + 63) / 64), gemm_range, &g);
  free(A);
  free(B);
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)((u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u));
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* out_f32 [M, N]: ((raw + (8 - zx[m]) sums[n]) * sx[m]) * sw[n] (+ bias[n]) (+ residual[m,n]).
 * bias / residual are fp32 here (callers convert from bf16 exactly). */
void orc_epilogue(const int32_t* raw, const float* sx, const int32_t* zx, const float* sw, const int32_t* sums,
                  const float* bias, const float* residual, int64_t M, int64_t N, float* out_f32,
                  uint16_t* out_bf16) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      int32_t c = raw[m * N + n];
      if (zx) c += (8 - zx[m]) * sums[n];
      float f = ((float)c * sx[m]) * sw[n];
      if (bias) f = f + bias[n];
      if (residual) f = f + residual[m * N + n];
      if (out_f32) out_f32[m * N + n] = f;
      if (out_bf16) out_bf16[m * N + n] = f32_to_bf16(f);
    }
}

/* Whole W4A4 linear on the CPU (the baseline bench.py times): x bf16 [M, K]
 * -> rotate (a, h_a; a == 0 means no rotation) -> symmetric per-token codes ->
 * int32 GEMM against pre-packed weights -> epilogue -> bf16 [M, N]. */
void orc_w4a4_linear(const uint16_t* x_bf16, int64_t M, int64_t K, int a, const int8_t* h_a,
                     const uint8_t* w_packed, const float* sw, int64_t N, float clip, uint16_t* out_bf16) {
  const int64_t KP = (K + 63) / 64 * 64;
  float* xf = (float*)malloc(sizeof(float) * M * K);
  float* y = (float*)malloc(sizeof(float) * M * K);
  uint8_t* ap = (uint8_t*)malloc((size_t)(M * KP / 2));
  float* sx = (float*)malloc(sizeof(float) * M);
  int32_t* raw = (int32_t*)malloc(sizeof(int32_t) * M * N);
  for (int64_t i = 0; i < M * K; ++i) xf[i] = bf16_to_f32(x_bf16[i]);
  if (a > 0)
    orc_rotate(xf, M, K, a, h_a, y);
  else
    memcpy(y, xf, sizeof(float) * M * K);
  orc_quant_rows(y, M, K, M, KP, ORC_ACT_SYM, clip, ap, sx, NULL, NULL, NULL);
  orc_gemm_s4(ap, w_packed, M, N, KP, raw);
  orc_epilogue(raw, sx, NULL, sw, NULL, NULL, NULL, M, N, NULL, out_bf16);
  free(xf);
  free(y);
  free(ap);
  free(sx);
  free(raw);
}

