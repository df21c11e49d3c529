/*
 * simd_x86.c -- TEST INFRASTRUCTURE (oracle).  Restatement of the AVX2+FMA
 * and AVX-VNNI dot-product tier of crates/prana-kernels/src/simd_x86.rs, with
 * runtime CPU detection and per-function target attributes (the file itself is
 * compiled for baseline x86-64, like the Rust crate).
 */
#include <immintrin.h>
#include <stdint.h>

#include "prana_oracle.h"

float or_dot_f32_scalar(const float *a, const float *b, size_t n);
float or_dot_q8_q8_scalar(const int8_t *aq, const float *as, size_t k, const int8_t *wq, const float *ws);
float or_dot_q40_q8_scalar(const int8_t *aq, const float *as, const int32_t *asum, size_t k,
                           const uint8_t *row, const float *ds);
float or_dot_q4k_q8_scalar(const int8_t *aq, const float *as, const int32_t *asum, size_t k,
                           const uint8_t *row, const float *ds);

/* simd_x86.rs:18-29: detected once (the reference caches in a OnceLock) */
static int simd_cached = -1, vnni_cached = -1;

int or_simd_available(void) {
  if (simd_cached < 0) {
    __builtin_cpu_init();
    simd_cached = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  }
  return simd_cached;
}
int or_vnni_available(void) {
  if (vnni_cached < 0) {
    __builtin_cpu_init();
    vnni_cached = or_simd_available() && __builtin_cpu_supports("avxvnni");
  }
  return vnni_cached;
}
int or_default_tier(void) {
  if (or_vnni_available()) return OR_TIER_VNNI;
  if (or_simd_available()) return OR_TIER_AVX2;
  return OR_TIER_SCALAR;
}

#define T_AVX2 __attribute__((target("avx2,fma")))
#define T_VNNI __attribute__((target("avx2,fma,avxvnni")))

/* simd_x86.rs:36-44: (lo+hi) -> pairwise -> final lane add */
T_AVX2 static inline float hsum8(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 1));
  return _mm_cvtss_f32(s);
}

/* simd_x86.rs:52-72: two 8-lane FMA accumulators over 16-wide chunks */
T_AVX2 static float dot_f32_avx2(const float *a, const float *b, size_t n) {
  __m256 s0 = _mm256_setzero_ps(), s1 = _mm256_setzero_ps();
  size_t c = n / 16;
  for (size_t i = 0; i < c; i++) {
    s0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + 16 * i), _mm256_loadu_ps(b + 16 * i), s0);
    s1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + 16 * i + 8), _mm256_loadu_ps(b + 16 * i + 8), s1);
  }
  float r = hsum8(_mm256_add_ps(s0, s1));
  for (size_t i = c * 16; i < n; i++) r += a[i] * b[i];
  return r;
}

/* simd_x86.rs:82-88: signed i8 x i8 -> 8 i32 lanes via the sign trick */
T_AVX2 static inline __m256i i8_pairs(__m256i x, __m256i y) {
  __m256i p16 = _mm256_maddubs_epi16(_mm256_sign_epi8(x, x), _mm256_sign_epi8(y, x));
  return _mm256_madd_epi16(p16, _mm256_set1_epi16(1));
}

/* simd_x86.rs:163-180 */
T_AVX2 static float dot_q8_q8_avx2(const int8_t *aq, const float *as, size_t k, const int8_t *wq,
                                   const float *ws) {
  __m256 acc = _mm256_setzero_ps();
  for (size_t g = 0; g < k / 32; g++) {
    __m256i a = _mm256_loadu_si256((const __m256i *)(aq + 32 * g));
    __m256i w = _mm256_loadu_si256((const __m256i *)(wq + 32 * g));
    acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(i8_pairs(w, a)), _mm256_set1_ps(ws[g] * as[g]), acc);
  }
  return hsum8(acc);
}

/* simd_x86.rs:97-115 */
T_VNNI static float dot_q8_q8_vnni(const int8_t *aq, const float *as, size_t k, const int8_t *wq,
                                   const float *ws) {
  __m256 acc = _mm256_setzero_ps();
  for (size_t g = 0; g < k / 32; g++) {
    __m256i a = _mm256_loadu_si256((const __m256i *)(aq + 32 * g));
    __m256i w = _mm256_loadu_si256((const __m256i *)(wq + 32 * g));
    __m256i p = _mm256_dpbusd_avx_epi32(_mm256_setzero_si256(), _mm256_sign_epi8(w, w),
                                        _mm256_sign_epi8(a, w));
    acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p), _mm256_set1_ps(ws[g] * as[g]), acc);
  }
  return hsum8(acc);
}

/* simd_x86.rs:189-199: 16 packed bytes -> 32 centred lanes (q-8), low nibbles first */
T_AVX2 static inline __m256i q40_lanes(const uint8_t *qs) {
  __m128i raw = _mm_loadu_si128((const __m128i *)qs);
  __m128i m = _mm_set1_epi8(0x0F);
  __m128i lo = _mm_and_si128(raw, m), hi = _mm_and_si128(_mm_srli_epi16(raw, 4), m);
  return _mm256_sub_epi8(_mm256_set_m128i(hi, lo), _mm256_set1_epi8(8));
}

/* simd_x86.rs:210-244: blocks in pairs on two accumulators */
T_AVX2 static float dot_q40_q8_avx2(const int8_t *aq, const float *as, size_t k,
                                    const uint8_t *row, const float *ds) {
  size_t nb = k / 32, i = 0;
  __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
  for (; i + 2 <= nb; i += 2) {
    __m256i w0 = q40_lanes(row + i * 18 + 2), w1 = q40_lanes(row + (i + 1) * 18 + 2);
    __m256i x0 = _mm256_loadu_si256((const __m256i *)(aq + i * 32));
    __m256i x1 = _mm256_loadu_si256((const __m256i *)(aq + i * 32 + 32));
    a0 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(i8_pairs(w0, x0)), _mm256_set1_ps(ds[i] * as[i]), a0);
    a1 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(i8_pairs(w1, x1)), _mm256_set1_ps(ds[i + 1] * as[i + 1]), a1);
  }
  if (i < nb) {
    __m256i w = q40_lanes(row + i * 18 + 2);
    __m256i x = _mm256_loadu_si256((const __m256i *)(aq + i * 32));
    a0 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(i8_pairs(w, x)), _mm256_set1_ps(ds[i] * as[i]), a0);
  }
  return hsum8(_mm256_add_ps(a0, a1));
}

/* simd_x86.rs:123-156 */
T_VNNI static float dot_q40_q8_vnni(const int8_t *aq, const float *as, size_t k,
                                    const uint8_t *row, const float *ds) {
  size_t nb = k / 32, i = 0;
  __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
  __m256i z = _mm256_setzero_si256();
  for (; i + 2 <= nb; i += 2) {
    __m256i w0 = q40_lanes(row + i * 18 + 2), w1 = q40_lanes(row + (i + 1) * 18 + 2);
    __m256i x0 = _mm256_loadu_si256((const __m256i *)(aq + i * 32));
    __m256i x1 = _mm256_loadu_si256((const __m256i *)(aq + i * 32 + 32));
    __m256i p0 = _mm256_dpbusd_avx_epi32(z, _mm256_sign_epi8(w0, w0), _mm256_sign_epi8(x0, w0));
    __m256i p1 = _mm256_dpbusd_avx_epi32(z, _mm256_sign_epi8(w1, w1), _mm256_sign_epi8(x1, w1));
    a0 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p0), _mm256_set1_ps(ds[i] * as[i]), a0);
    a1 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p1), _mm256_set1_ps(ds[i + 1] * as[i + 1]), a1);
  }
  if (i < nb) {
    __m256i w = q40_lanes(row + i * 18 + 2);
    __m256i x = _mm256_loadu_si256((const __m256i *)(aq + i * 32));
    __m256i p = _mm256_dpbusd_avx_epi32(z, _mm256_sign_epi8(w, w), _mm256_sign_epi8(x, w));
    a0 = _mm256_fmadd_ps(_mm256_cvtepi32_ps(p), _mm256_set1_ps(ds[i] * as[i]), a0);
  }
  return hsum8(_mm256_add_ps(a0, a1));
}

/* simd_x86.rs:252-299: nibble planes x activations, hsum per group, scalar scale math */
T_AVX2 static float dot_q4k_q8_avx2(const int8_t *aq, const float *as, const int32_t *asum,
                                    size_t k, const uint8_t *row, const float *ds) {
  float total = 0.0f;
  __m256i nib = _mm256_set1_epi8(0x0F), ones = _mm256_set1_epi16(1);
  for (size_t bi = 0; bi < k / 256; bi++) {
    const uint8_t *b = row + bi * 144;
    float d = ds[bi * 2], dmin = ds[bi * 2 + 1];
    const int8_t *pa = aq + bi * 256;
    for (int pair = 0; pair < 4; pair++) {
      __m256i bytes = _mm256_loadu_si256((const __m256i *)(b + 16 + pair * 32));
      __m256i lo = _mm256_and_si256(bytes, nib);
      __m256i hi = _mm256_and_si256(_mm256_srli_epi16(bytes, 4), nib);
      __m256i xl = _mm256_loadu_si256((const __m256i *)(pa + pair * 64));
      __m256i xh = _mm256_loadu_si256((const __m256i *)(pa + pair * 64 + 32));
      float s1 = hsum8(_mm256_cvtepi32_ps(_mm256_madd_epi16(_mm256_maddubs_epi16(lo, xl), ones)));
      float s2 = hsum8(_mm256_cvtepi32_ps(_mm256_madd_epi16(_mm256_maddubs_epi16(hi, xh), ones)));
      size_t g_lo = bi * 8 + pair * 2, g_hi = g_lo + 1;
      float sc1, m1, sc2, m2;
      or_q4k_scale_min(pair * 2, b + 4, &sc1, &m1);
      or_q4k_scale_min(pair * 2 + 1, b + 4, &sc2, &m2);
      total += as[g_lo] * (d * sc1 * s1 - dmin * m1 * (float)asum[g_lo]);
      total += as[g_hi] * (d * sc2 * s2 - dmin * m2 * (float)asum[g_hi]);
    }
  }
  return total;
}

static int resolve(int tier) { return tier == OR_TIER_AUTO ? or_default_tier() : tier; }

/* matmul.rs:353-360 dispatch */
float or_dot_f32(int tier, const float *a, const float *b, size_t n) {
  tier = resolve(tier);
  if (tier >= OR_TIER_AVX2 && or_simd_available()) return dot_f32_avx2(a, b, n);
  return or_dot_f32_scalar(a, b, n);
}

/* matmul.rs:364-374 dispatch */
float or_dot_q8_q8(int tier, const int8_t *aq, const float *as, size_t k, const int8_t *wq,
                   const float *ws) {
  tier = resolve(tier);
  if (tier == OR_TIER_VNNI && or_vnni_available()) return dot_q8_q8_vnni(aq, as, k, wq, ws);
  if (tier >= OR_TIER_AVX2 && or_simd_available()) return dot_q8_q8_avx2(aq, as, k, wq, ws);
  return or_dot_q8_q8_scalar(aq, as, k, wq, ws);
}

/* kquant.rs:338-363 dispatch (Q4_0 arm) */
float or_dot_q40_q8(int tier, const int8_t *aq, const float *as, const int32_t *asum, size_t k,
                    const uint8_t *row, const float *ds) {
  tier = resolve(tier);
  if (tier == OR_TIER_VNNI && or_vnni_available()) return dot_q40_q8_vnni(aq, as, k, row, ds);
  if (tier >= OR_TIER_AVX2 && or_simd_available()) return dot_q40_q8_avx2(aq, as, k, row, ds);
  return or_dot_q40_q8_scalar(aq, as, asum, k, row, ds);
}

/* kquant.rs:338-363 dispatch (Q4_K arm: AVX2 only, no VNNI form) */
float or_dot_q4k_q8(int tier, const int8_t *aq, const float *as, const int32_t *asum, size_t k,
                    const uint8_t *row, const float *ds) {
  tier = resolve(tier);
  if (tier >= OR_TIER_AVX2 && or_simd_available()) return dot_q4k_q8_avx2(aq, as, asum, k, row, ds);
  return or_dot_q4k_q8_scalar(aq, as, asum, k, row, ds);
}
