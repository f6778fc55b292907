/* The reference's expert products as a native CPU program over the packed MXFP4 pools: the fastest form of the
 * timed CPU baseline.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by oracle/cpu_path.py for bench.py's cpu_baseline leg and --impl reference
 * arm, never by the library.  Built by oracle/cpu_port_build.py into oracle/libmimo_cpu_port.so.
 *
 * Restates, per expert and for R <= 8 token rows:
 *   kernel A (engine/mimo_stream/kernels.py:33-85): g, u = float32 dot products of x with the e2m1 weights
 *     (sign bit 3, magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, element k = nibble k % 8 of word k / 8, low nibble
 *     first) times the e8m0 scale of each 32-value group (kernels.py:19-30); gt = bf16(g), ut = bf16(u);
 *     h = bf16(bf16(gt * sigmoid_bf16(gt)) * ut), the sigmoid rounded once to bf16 (kernels.py:138-146);
 *   kernel B (kernels.py:88-123): d = float32 dot product of h with the down weights, rounded to bf16 when the
 *     caller asks for the gather_qmm pair path's bf16 expert outputs (model.py:173-182, 221-228).
 * The caller weights and combines the rows (kernels.py:194-199, model.py:266-271).
 * It reads the 13.4 MB of packed bytes per expert a CPU implementation streams (the float32 variants of
 * oracle/cpu_path.py stream 100 MB of dequantised weights).  Every output row runs on one thread (OpenMP
 * over output rows).  Dot products, per 32-value group and lane j < 8 (elements j, j + 8, j + 16, j + 24):
 * the four products rounded to float32, summed as (p0 + p1) + (p2 + p3), then one fused multiply-add of that
 * sum and the group's scale into the lane's running total; the eight lanes are summed pairwise at the end.
 * The AVX2 path and the scalar path take the same steps (built with -ffp-contract=off), so their results
 * are bit-identical.  The summation order differs from the Metal kernel's lane sums, so results match the
 * checker within its tolerance, not bit for bit. */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

static const float kE2m1[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
static int g_force_scalar = 0;

static inline float bf16r(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return f;
  u += 0x7FFFu + ((u >> 16) & 1u);
  u &= 0xFFFF0000u;
  memcpy(&f, &u, 4);
  return f;
}

/* 2^(s - 127) from its bits: the byte is the float32 exponent field; s = 0 -> 2^-127 (subnormal), 255 -> NaN. */
static inline float e8m0(uint8_t s) {
  const uint32_t b = s == 0 ? 0x00400000u : (s == 255 ? 0x7FC00000u : (uint32_t)s << 23);
  float f;
  memcpy(&f, &b, 4);
  return f;
}

static inline float lanes_sum(const float* l) {
  return ((l[0] + l[1]) + (l[2] + l[3])) + ((l[4] + l[5]) + (l[6] + l[7]));
}

/* out[r] = sum_k x[r*K + k] * w_k, one weight row of K values (K / 8 words, K / 32 scales), R rows of x. */
static void rows_dot_scalar(const float* x, int R, int K, const uint32_t* w, const uint8_t* s, float* out) {
  float acc[8][8];
  memset(acc, 0, sizeof(acc));
  for (int g = 0; g < K / 32; ++g) {
    float v[4][8];
    for (int q = 0; q < 4; ++q) {
      const uint32_t word = w[g * 4 + q];
      for (int j = 0; j < 8; ++j) {
        const uint32_t nib = (word >> (4 * j)) & 0xFu;
        v[q][j] = (nib & 8u) ? -kE2m1[nib & 7u] : kE2m1[nib & 7u];
      }
    }
    const float sc = e8m0(s[g]);
    for (int r = 0; r < R; ++r) {
      const float* xr = x + (size_t)r * K + g * 32;
      for (int j = 0; j < 8; ++j) {
        const float p0 = v[0][j] * xr[j], p1 = v[1][j] * xr[8 + j];
        const float p2 = v[2][j] * xr[16 + j], p3 = v[3][j] * xr[24 + j];
        acc[r][j] = fmaf((p0 + p1) + (p2 + p3), sc, acc[r][j]);
      }
    }
  }
  for (int r = 0; r < R; ++r) out[r] = lanes_sum(acc[r]);
}

#if defined(__x86_64__)
__attribute__((always_inline, target("avx2,fma"))) static inline __m256 decode8(uint32_t word, __m256 mag,
                                                                                __m256i shifts) {
  const __m256i nib = _mm256_and_si256(_mm256_srlv_epi32(_mm256_set1_epi32((int)word), shifts),
                                       _mm256_set1_epi32(15));
  const __m256 m = _mm256_permutevar8x32_ps(mag, _mm256_and_si256(nib, _mm256_set1_epi32(7)));
  const __m256 sign = _mm256_castsi256_ps(_mm256_slli_epi32(_mm256_and_si256(nib, _mm256_set1_epi32(8)), 28));
  return _mm256_xor_ps(m, sign);
}

/* R known at compile time in each instantiation below, so the R accumulators stay in registers. */
__attribute__((always_inline, target("avx2,fma"))) static inline void dot_rows_avx2(const float* x, const int R,
                                                                                    int K, const uint32_t* w,
                                                                                    const uint8_t* s, float* out) {
  const __m256 mag = _mm256_loadu_ps(kE2m1);
  const __m256i shifts = _mm256_setr_epi32(0, 4, 8, 12, 16, 20, 24, 28);
  __m256 acc[8];
  for (int r = 0; r < R; ++r) acc[r] = _mm256_setzero_ps();
  for (int g = 0; g < K / 32; ++g) {
    const __m256 v0 = decode8(w[g * 4], mag, shifts), v1 = decode8(w[g * 4 + 1], mag, shifts);
    const __m256 v2 = decode8(w[g * 4 + 2], mag, shifts), v3 = decode8(w[g * 4 + 3], mag, shifts);
    const __m256 sc = _mm256_set1_ps(e8m0(s[g]));
    for (int r = 0; r < R; ++r) {
      const float* xr = x + (size_t)r * K + g * 32;
      const __m256 p0 = _mm256_mul_ps(v0, _mm256_loadu_ps(xr)), p1 = _mm256_mul_ps(v1, _mm256_loadu_ps(xr + 8));
      const __m256 p2 = _mm256_mul_ps(v2, _mm256_loadu_ps(xr + 16)), p3 = _mm256_mul_ps(v3, _mm256_loadu_ps(xr + 24));
      acc[r] = _mm256_fmadd_ps(_mm256_add_ps(_mm256_add_ps(p0, p1), _mm256_add_ps(p2, p3)), sc, acc[r]);
    }
  }
  for (int r = 0; r < R; ++r) {
    float l[8];
    _mm256_storeu_ps(l, acc[r]);
    out[r] = lanes_sum(l);
  }
}

__attribute__((target("avx2,fma"))) static void rows_dot_avx2(const float* x, int R, int K, const uint32_t* w,
                                                             const uint8_t* s, float* out) {
  switch (R) {
    case 1: dot_rows_avx2(x, 1, K, w, s, out); break;
    case 2: dot_rows_avx2(x, 2, K, w, s, out); break;
    case 3: dot_rows_avx2(x, 3, K, w, s, out); break;
    case 4: dot_rows_avx2(x, 4, K, w, s, out); break;
    case 5: dot_rows_avx2(x, 5, K, w, s, out); break;
    case 6: dot_rows_avx2(x, 6, K, w, s, out); break;
    case 7: dot_rows_avx2(x, 7, K, w, s, out); break;
    default: dot_rows_avx2(x, 8, K, w, s, out); break;
  }
}
#endif

typedef void (*dot_fn)(const float*, int, int, const uint32_t*, const uint8_t*, float*);

static dot_fn pick(void) {
#if defined(__x86_64__)
  if (!g_force_scalar && __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return rows_dot_avx2;
#endif
  return rows_dot_scalar;
}

/* 2 when the AVX2 path runs, 1 for the scalar path. */
int mimo_cpu_port_isa(void) { return pick() == rows_dot_scalar ? 1 : 2; }

/* force != 0: the scalar path even where AVX2 is present (tests compare the two). */
void mimo_cpu_port_force_scalar(int force) { g_force_scalar = force; }

/* Threads of the calls made from this thread (the timed baseline reports the count it used). */
void mimo_cpu_port_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
int mimo_cpu_port_threads(void) { return omp_get_max_threads(); }

/* One expert on R token rows: x [R][H] float32 (bf16 values); gate/up words [I][H/8], scales [I][H/32];
 * down words [H][I/8], scales [H][I/32]; hbuf [R][I] scratch (receives h); out [R][H] = the expert's
 * down products (bf16-rounded when pairs != 0).  Returns 0, or 1 for bad sizes. */
int mimo_cpu_port_expert(const float* x, int R, int H, int I, const uint32_t* gw, const uint8_t* gs,
                         const uint32_t* uw, const uint8_t* us, const uint32_t* dw, const uint8_t* ds, int pairs,
                         float* hbuf, float* out) {
  if (R < 1 || R > 8 || H < 32 || H % 32 || I < 32 || I % 32) return 1;
  const dot_fn dot = pick();
#pragma omp parallel for schedule(static)
  for (int n = 0; n < I; ++n) {
    float g[8], u[8];
    dot(x, R, H, gw + (size_t)n * (H / 8), gs + (size_t)n * (H / 32), g);
    dot(x, R, H, uw + (size_t)n * (H / 8), us + (size_t)n * (H / 32), u);
    for (int r = 0; r < R; ++r) {
      const float gt = bf16r(g[r]), ut = bf16r(u[r]);
      const float sig = bf16r((float)(1.0 / (1.0 + exp(-(double)gt))));
      hbuf[(size_t)r * I + n] = bf16r(bf16r(gt * sig) * ut);
    }
  }
#pragma omp parallel for schedule(static)
  for (int m = 0; m < H; ++m) {
    float d[8];
    dot(hbuf, R, I, dw + (size_t)m * (I / 8), ds + (size_t)m * (I / 32), d);
    for (int r = 0; r < R; ++r) out[(size_t)r * H + m] = pairs ? bf16r(d[r]) : d[r];
  }
  return 0;
}
