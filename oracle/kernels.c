/*
 * kernels.c -- TEST INFRASTRUCTURE (oracle).  Scalar restatement of the
 * `prana-kernels` crate: f16 conversion, activation/weight quantization,
 * block dequantization, scalar integer dots, norms, RoPE, attention, argmax.
 * Built with -ffp-contract=off so every a*b+c rounds twice, as in Rust.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "prana_oracle.h"

/* crates/prana-kernels/src/lib.rs:57-73 (inline body in prana_oracle.h) */
float or_f16_to_f32(uint16_t h) { return or_f16_to_f32_inline(h); }

/* crates/prana-kernels/src/lib.rs:78-113 (round-to-nearest-even) */
uint16_t or_f32_to_f16(float x) {
  uint32_t bits;
  memcpy(&bits, &x, 4);
  uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  int32_t exp = (int32_t)((bits >> 23) & 0xffu);
  uint32_t frac = bits & 0x7fffffu;
  if (exp == 0xff) return sign | 0x7c00u | (frac ? 0x0200u : 0u);
  int32_t e = exp - 127 + 15;
  if (e >= 0x1f) return sign | 0x7c00u;
  if (e <= 0) {
    if (e < -10) return sign;
    uint32_t m = frac | 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    uint16_t half = (uint16_t)(m >> shift);
    uint32_t round_bit = 1u << (shift - 1);
    uint32_t rem = m & (round_bit * 2 - 1);
    int round = rem > round_bit || (rem == round_bit && (half & 1));
    return sign | (uint16_t)(half + round);
  }
  uint16_t half = (uint16_t)(((uint32_t)e << 10) | (frac >> 13));
  uint32_t rem = frac & 0x1fffu;
  int round = rem > 0x1000u || (rem == 0x1000u && (half & 1));
  return sign | (uint16_t)(half + round);
}

/* Rust `f32::max` / fold(0, max(|x|)): NaN-ignoring like fmaxf. */
static float amax32(const float *x) {
  float m = 0.0f;
  for (int i = 0; i < 32; i++) m = fmaxf(m, fabsf(x[i]));
  return m;
}

/* Rust `v.round().clamp(-127.0, 127.0) as i32` (saturating cast, NaN -> 0). */
static int32_t round_clamp127(float v) {
  float r = roundf(v);
  if (r < -127.0f) r = -127.0f;
  if (r > 127.0f) r = 127.0f;
  if (r != r) return 0;
  return (int32_t)r;
}

/* crates/prana-kernels/src/matmul.rs:105-127 */
void or_quantize_acts(const float *a, size_t k, int8_t *q, float *scales, int32_t *sums) {
  size_t groups = k / OR_Q8_BLOCK;
  for (size_t g = 0; g < groups; g++) {
    const float *blk = a + g * OR_Q8_BLOCK;
    float amax = amax32(blk);
    float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
    float inv = 1.0f / scale;
    int32_t sum = 0;
    for (int i = 0; i < OR_Q8_BLOCK; i++) {
      int32_t v = round_clamp127(blk[i] * inv);
      q[g * OR_Q8_BLOCK + i] = (int8_t)v;
      sum += v;
    }
    scales[g] = scale;
    sums[g] = sum;
  }
}

/* crates/prana-kernels/src/matmul.rs:61-84 */
void or_quantize_q8(size_t rows, size_t cols, const float *w, int8_t *q, float *scales) {
  size_t gpr = cols / OR_Q8_BLOCK;
  for (size_t r = 0; r < rows; r++)
    for (size_t g = 0; g < gpr; g++) {
      size_t base = r * cols + g * OR_Q8_BLOCK;
      float amax = amax32(w + base);
      float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
      float inv = 1.0f / scale;
      for (int i = 0; i < OR_Q8_BLOCK; i++) q[base + i] = (int8_t)round_clamp127(w[base + i] * inv);
      scales[r * gpr + g] = scale;
    }
}

static float rd_f16(const uint8_t *b) { return or_f16_to_f32((uint16_t)(b[0] | (b[1] << 8))); }

/* crates/prana-kernels/src/kquant.rs:39-47 */
void or_dequant_q40_block(const uint8_t *b, float *out) {
  float d = rd_f16(b);
  for (int j = 0; j < 16; j++) out[j] = d * ((float)(b[2 + j] & 0xF) - 8.0f);
  for (int j = 0; j < 16; j++) out[16 + j] = d * ((float)(b[2 + j] >> 4) - 8.0f);
}

/* crates/prana-kernels/src/kquant.rs:52-61 */
void or_q4k_scale_min(int j, const uint8_t *s, float *sc, float *m) {
  if (j < 4) {
    *sc = (float)(s[j] & 63);
    *m = (float)(s[j + 4] & 63);
  } else {
    *sc = (float)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (float)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

/* crates/prana-kernels/src/kquant.rs:66-83 */
void or_dequant_q4k_block(const uint8_t *b, float *out) {
  float d = rd_f16(b), dmin = rd_f16(b + 2);
  const uint8_t *scales = b + 4, *qs = b + 16;
  for (int pair = 0; pair < 4; pair++) {
    const uint8_t *q = qs + pair * 32;
    float sc1, m1, sc2, m2;
    or_q4k_scale_min(pair * 2, scales, &sc1, &m1);
    or_q4k_scale_min(pair * 2 + 1, scales, &sc2, &m2);
    float d1 = d * sc1, min1 = dmin * m1, d2 = d * sc2, min2 = dmin * m2;
    for (int l = 0; l < 32; l++) out[pair * 64 + l] = d1 * (float)(q[l] & 0xF) - min1;
    for (int l = 0; l < 32; l++) out[pair * 64 + 32 + l] = d2 * (float)(q[l] >> 4) - min2;
  }
}

/* crates/prana-kernels/src/kquant.rs:88-112 */
void or_dequant_q6k_block(const uint8_t *b, float *y) {
  const uint8_t *ql0 = b, *qh0 = b + 128;
  const int8_t *sc = (const int8_t *)(b + 192);
  float d = rd_f16(b + 208);
  for (int half = 0; half < 2; half++) {
    const uint8_t *ql = ql0 + half * 64, *qh = qh0 + half * 32;
    int s0 = half * 8, yo = half * 128;
    for (int l = 0; l < 32; l++) {
      int is = s0 + l / 16;
      float q1 = (float)((int8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32);
      float q2 = (float)((int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
      float q3 = (float)((int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
      float q4 = (float)((int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
      y[yo + l] = (d * (float)sc[is]) * q1;
      y[yo + l + 32] = (d * (float)sc[is + 2]) * q2;
      y[yo + l + 64] = (d * (float)sc[is + 4]) * q3;
      y[yo + l + 96] = (d * (float)sc[is + 6]) * q4;
    }
  }
}

/* ---- scalar tier dots ---- */

/* crates/prana-kernels/src/matmul.rs:377-391 */
float or_dot_f32_scalar(const float *a, const float *b, size_t n) {
  float acc[4] = {0, 0, 0, 0};
  size_t c = n / 4;
  for (size_t i = 0; i < c; i++)
    for (int l = 0; l < 4; l++) acc[l] += a[i * 4 + l] * b[i * 4 + l];
  float sum = acc[0] + acc[1] + acc[2] + acc[3];
  for (size_t i = c * 4; i < n; i++) sum += a[i] * b[i];
  return sum;
}

/* crates/prana-kernels/src/matmul.rs:395-406 */
float or_dot_q8_q8_scalar(const int8_t *aq, const float *as, size_t k, const int8_t *wq,
                          const float *ws) {
  float sum = 0.0f;
  for (size_t g = 0; g < k / 32; g++) {
    int32_t acc = 0;
    for (int l = 0; l < 32; l++) acc += (int32_t)aq[g * 32 + l] * (int32_t)wq[g * 32 + l];
    sum += ws[g] * as[g] * (float)acc;
  }
  return sum;
}

/* crates/prana-kernels/src/kquant.rs:240-252 */
float or_dot_q40_q8_scalar(const int8_t *aq, const float *as, const int32_t *asum, size_t k,
                           const uint8_t *row, const float *ds) {
  float total = 0.0f;
  for (size_t i = 0; i < k / 32; i++) {
    const uint8_t *b = row + i * OR_Q4_0_BLOCK_BYTES;
    const int8_t *qa = aq + i * 32;
    int32_t s = 0;
    for (int l = 0; l < 16; l++)
      s += (int32_t)qa[l] * (b[2 + l] & 0xF) + (int32_t)qa[16 + l] * (b[2 + l] >> 4);
    total += ds[i] * as[i] * (float)(s - 8 * asum[i]);
  }
  return total;
}

/* crates/prana-kernels/src/kquant.rs:257-282 */
float or_dot_q4k_q8_scalar(const int8_t *aq, const float *as, const int32_t *asum, size_t k,
                           const uint8_t *row, const float *ds) {
  float total = 0.0f;
  for (size_t bi = 0; bi < k / OR_QK_K; bi++) {
    const uint8_t *b = row + bi * OR_Q4_K_BLOCK_BYTES;
    float d = ds[bi * 2], dmin = ds[bi * 2 + 1];
    const uint8_t *scales = b + 4, *qs = b + 16;
    for (int pair = 0; pair < 4; pair++) {
      const uint8_t *q = qs + pair * 32;
      size_t g_lo = bi * 8 + pair * 2, g_hi = g_lo + 1;
      const int8_t *qa_lo = aq + g_lo * 32, *qa_hi = aq + g_hi * 32;
      float sc1, m1, sc2, m2;
      or_q4k_scale_min(pair * 2, scales, &sc1, &m1);
      or_q4k_scale_min(pair * 2 + 1, scales, &sc2, &m2);
      int32_t s1 = 0, s2 = 0;
      for (int l = 0; l < 32; l++) {
        s1 += (int32_t)qa_lo[l] * (q[l] & 0xF);
        s2 += (int32_t)qa_hi[l] * (q[l] >> 4);
      }
      total += as[g_lo] * (d * sc1 * (float)s1 - dmin * m1 * (float)asum[g_lo]);
      total += as[g_hi] * (d * sc2 * (float)s2 - dmin * m2 * (float)asum[g_hi]);
    }
  }
  return total;
}

/* Q6_K 6-bit unpack shared by the dot and the block-dot dump (kquant.rs:294-303). */
static void q6k_quads(const uint8_t *ql, const uint8_t *qh, int l, int32_t q[4]) {
  q[0] = (int32_t)(int8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
  q[1] = (int32_t)(int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
  q[2] = (int32_t)(int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
  q[3] = (int32_t)(int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
}

/* crates/prana-kernels/src/kquant.rs:287-318 */
float or_dot_q6k_q8(const int8_t *aq, const float *as, size_t k, const uint8_t *row,
                    const float *ds) {
  float total = 0.0f;
  for (size_t bi = 0; bi < k / OR_QK_K; bi++) {
    const uint8_t *b = row + bi * OR_Q6_K_BLOCK_BYTES;
    const int8_t *sc = (const int8_t *)(b + 192);
    float d = ds[bi];
    const int8_t *qa = aq + bi * OR_QK_K;
    for (int half = 0; half < 2; half++) {
      const uint8_t *ql = b + half * 64, *qh = b + 128 + half * 32;
      int s0 = half * 8, ao = half * 128;
      int32_t sums[8] = {0};
      for (int l = 0; l < 32; l++) {
        int sub = l / 16;
        int32_t q[4];
        q6k_quads(ql, qh, l, q);
        sums[sub] += (int32_t)qa[ao + l] * q[0];
        sums[2 + sub] += (int32_t)qa[ao + l + 32] * q[1];
        sums[4 + sub] += (int32_t)qa[ao + l + 64] * q[2];
        sums[6 + sub] += (int32_t)qa[ao + l + 96] * q[3];
      }
      for (int g = 0; g < 4; g++) {
        float sa = as[bi * 8 + half * 4 + g];
        total += d * sa * (float)sc[s0 + g * 2] * (float)sums[g * 2];
        total += d * sa * (float)sc[s0 + g * 2 + 1] * (float)sums[g * 2 + 1];
      }
    }
  }
  return total;
}

/*
 * Per-block integer dots for one packed row: the quantities BASELINE requires
 * to be bit-exact.  Q8_0: Σ qa·qw per 32-group.  Q4_0: Σ qa·(q−8) per block
 * (== `s - 8*sums` of kquant.rs:249).  Q4_K: Σ qa·q (raw nibble) per 32-group
 * (s1/s2 of kquant.rs:272-276).  Q6_K: Σ qa·(q6−32) per 16-element sub-block
 * in sc[] order (sums[] of kquant.rs:300-307, re-indexed to sub-block id).
 * For Q8_0 `row` is the int8 plane of the row.
 */
void or_block_dots(int type, const int8_t *aq, size_t k, const uint8_t *row, int32_t *out) {
  if (type == OR_GGML_Q8_0) {
    const int8_t *w = (const int8_t *)row;
    for (size_t g = 0; g < k / 32; g++) {
      int32_t acc = 0;
      for (int l = 0; l < 32; l++) acc += (int32_t)aq[g * 32 + l] * w[g * 32 + l];
      out[g] = acc;
    }
  } else if (type == OR_GGML_Q4_0) {
    for (size_t i = 0; i < k / 32; i++) {
      const uint8_t *b = row + i * 18;
      int32_t s = 0, sum = 0;
      for (int l = 0; l < 16; l++) {
        s += (int32_t)aq[i * 32 + l] * (b[2 + l] & 0xF) + (int32_t)aq[i * 32 + 16 + l] * (b[2 + l] >> 4);
      }
      for (int l = 0; l < 32; l++) sum += aq[i * 32 + l];
      out[i] = s - 8 * sum;
    }
  } else if (type == OR_GGML_Q4_K) {
    for (size_t bi = 0; bi < k / 256; bi++) {
      const uint8_t *qs = row + bi * 144 + 16;
      for (int pair = 0; pair < 4; pair++) {
        int32_t s1 = 0, s2 = 0;
        const int8_t *lo = aq + bi * 256 + pair * 64, *hi = lo + 32;
        for (int l = 0; l < 32; l++) {
          s1 += (int32_t)lo[l] * (qs[pair * 32 + l] & 0xF);
          s2 += (int32_t)hi[l] * (qs[pair * 32 + l] >> 4);
        }
        out[bi * 8 + pair * 2] = s1;
        out[bi * 8 + pair * 2 + 1] = s2;
      }
    }
  } else if (type == OR_GGML_Q6_K) {
    for (size_t bi = 0; bi < k / 256; bi++) {
      const uint8_t *b = row + bi * 210;
      const int8_t *qa = aq + bi * 256;
      for (int half = 0; half < 2; half++) {
        const uint8_t *ql = b + half * 64, *qh = b + 128 + half * 32;
        int32_t sums[8] = {0};
        for (int l = 0; l < 32; l++) {
          int sub = l / 16;
          int32_t q[4];
          q6k_quads(ql, qh, l, q);
          sums[sub] += (int32_t)qa[half * 128 + l] * q[0];
          sums[2 + sub] += (int32_t)qa[half * 128 + l + 32] * q[1];
          sums[4 + sub] += (int32_t)qa[half * 128 + l + 64] * q[2];
          sums[6 + sub] += (int32_t)qa[half * 128 + l + 96] * q[3];
        }
        /* sums[g*2+s] pairs with sc[half*8 + g*2 + s] */
        for (int i = 0; i < 8; i++) out[bi * 16 + half * 8 + i] = sums[i];
      }
    }
  }
}

/* ---- norms (norms.rs:9-56) ---- */

void or_rmsnorm(const float *x, const float *w, size_t rows, size_t dim, float eps, float *out) {
  for (size_t r = 0; r < rows; r++) {
    const float *row = x + r * dim;
    float ss = 0.0f;
    for (size_t i = 0; i < dim; i++) ss += row[i] * row[i];
    float mean_sq = ss / (float)dim;
    float inv = 1.0f / sqrtf(mean_sq + eps);
    for (size_t i = 0; i < dim; i++) out[r * dim + i] = row[i] * inv * w[i];
  }
}

void or_silu(float *x, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] *= 1.0f / (1.0f + expf(-x[i]));
}

void or_softmax(const float *x, size_t n, float *out) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; i++) mx = fmaxf(mx, x[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    out[i] = expf(x[i] - mx);
  }
  for (size_t i = 0; i < n; i++) sum += out[i];
  float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
  for (size_t i = 0; i < n; i++) out[i] *= inv;
}

/* ---- sampler (sampler.rs) ---- */

/* XorShift::next_u64 (sampler.rs:59-66): xorshift64* */
uint64_t or_xorshift_next(uint64_t *state) {
  uint64_t x = *state;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  *state = x;
  return x * 0x2545F4914F6CDD1DULL;
}

/* XorShift::next_f32 (sampler.rs:67-70): the top 24 bits over 2^24 */
float or_xorshift_f32(uint64_t *state) { return (float)(or_xorshift_next(state) >> 40) / (float)(1ULL << 24); }

/* Sampler::sample (sampler.rs:22-37): greedy (argmax) when temp <= 0, else
 * softmax(logits / temp), one draw r, and the first i whose running
 * r -= p[i] reaches <= 0 (the last index when round-off never gets there).
 * probs (may be NULL) receives the softmax; *r_out (may be NULL) the draw. */
uint32_t or_sample(const float *logits, size_t n, float temp, uint64_t *state, float *probs, float *r_out) {
  if (temp <= 0.0f) return or_argmax(logits, n); /* a NaN temperature samples */
  float *p = malloc(sizeof(float) * n);
  for (size_t i = 0; i < n; i++) p[i] = logits[i] / temp;
  or_softmax(p, n, p);
  float r = or_xorshift_f32(state);
  if (r_out) *r_out = r;
  if (probs) memcpy(probs, p, sizeof(float) * n);
  uint32_t tok = (uint32_t)(n - 1);
  for (size_t i = 0; i < n; i++) {
    r -= p[i];
    if (r <= 0.0f) {
      tok = (uint32_t)i;
      break;
    }
  }
  free(p);
  return tok;
}

/* ---- RoPE (attention.rs:59-121) ---- */

void or_rope_interleaved(float *x, size_t n, size_t pos, size_t hd, float theta) {
  for (size_t i = 0; i < n; i += 2) {
    size_t j = i % hd;
    float freq = powf(theta, -((float)j) / (float)hd);
    float ang = (float)pos * freq;
    float s = sinf(ang), c = cosf(ang);
    float x0 = x[i], x1 = x[i + 1];
    x[i] = x0 * c - x1 * s;
    x[i + 1] = x0 * s + x1 * c;
  }
}

void or_rope_neox(float *x, size_t n, size_t pos, size_t hd, float theta) {
  size_t half = hd / 2;
  for (size_t h = 0; h < n / hd; h++) {
    size_t base = h * hd;
    for (size_t j = 0; j < half; j++) {
      float freq = powf(theta, -(2.0f * (float)j) / (float)hd);
      float ang = (float)pos * freq;
      float s = sinf(ang), c = cosf(ang);
      float x1 = x[base + j], x2 = x[base + j + half];
      x[base + j] = x1 * c - x2 * s;
      x[base + j + half] = x1 * s + x2 * c;
    }
  }
}

void or_rope_batch(float *x, size_t seq, size_t n_heads, size_t hd, float theta) {
  for (size_t p = 0; p < seq; p++) or_rope_neox(x + p * n_heads * hd, n_heads * hd, p, hd, theta);
}

/*
 * The (cos, sin) pairs the two RoPE forms use, tabulated with this host's
 * libm: entry [pos][i] is the rotation of pair i (interleaved: dims 2i,2i+1
 * with freq θ^(−2i/hd); NeoX: dims i, i+hd/2 with freq θ^(−2i/hd)).  Both
 * forms compute the exponent exactly as their loops do, so the table is
 * bit-identical to the values the loops above produce.
 */
void or_rope_table(size_t positions, size_t hd, float theta, int neox, float *co, float *si) {
  size_t half = hd / 2;
  for (size_t p = 0; p < positions; p++)
    for (size_t i = 0; i < half; i++) {
      float freq = neox ? powf(theta, -(2.0f * (float)i) / (float)hd)
                        : powf(theta, -((float)(2 * i)) / (float)hd);
      float ang = (float)p * freq;
      co[p * half + i] = cosf(ang);
      si[p * half + i] = sinf(ang);
    }
}

/* attention.rs:47-52 */
void or_f16_kv_write(uint16_t *cache, size_t first_row, size_t kv_stride, const float *src, size_t n) {
  for (size_t i = 0; i < n; i++) cache[first_row * kv_stride + i] = or_f32_to_f16(src[i]);
}

/* attention.rs:165-195 */
static void decode_one_head(const float *q, const uint16_t *kc, const uint16_t *vc, size_t pos,
                            size_t h, size_t group, size_t kv_stride, size_t hd, float *dst,
                            float *scores, float *probs, float *tmp) {
  float scale = 1.0f / sqrtf((float)hd);
  size_t kv_h = h / group;
  const float *qv = q + h * hd;
  for (size_t t = 0; t <= pos; t++) {
    const uint16_t *kr = kc + t * kv_stride + kv_h * hd;
    for (size_t d = 0; d < hd; d++) tmp[d] = or_f16_to_f32_inline(kr[d]);
    float dot = 0.0f;
    for (size_t d = 0; d < hd; d++) dot += qv[d] * tmp[d];
    scores[t] = dot * scale;
  }
  or_softmax(scores, pos + 1, probs);
  for (size_t d = 0; d < hd; d++) dst[d] = 0.0f;
  for (size_t t = 0; t <= pos; t++) {
    const uint16_t *vr = vc + t * kv_stride + kv_h * hd;
    float p = probs[t];
    for (size_t d = 0; d < hd; d++) dst[d] += p * or_f16_to_f32_inline(vr[d]);
  }
}

/* attention.rs:129-160 */
void or_attention_decode(const float *q, const uint16_t *kc, const uint16_t *vc, size_t pos,
                         size_t n_heads, size_t n_kv_heads, size_t hd, float *out) {
  size_t kv_stride = n_kv_heads * hd, group = n_heads / n_kv_heads;
  float *scores = malloc(sizeof(float) * (pos + 1) * 2 + sizeof(float) * hd);
  for (size_t h = 0; h < n_heads; h++)
    decode_one_head(q, kc, vc, pos, h, group, kv_stride, hd, out + h * hd, scores,
                    scores + pos + 1, scores + 2 * (pos + 1));
  free(scores);
}

/* attention.rs:296-333 */
void or_attention_verify(const float *q, const uint16_t *kc, const uint16_t *vc, size_t pos0,
                         size_t seq, size_t n_heads, size_t n_kv_heads, size_t hd, float *out) {
  size_t q_stride = n_heads * hd;
  for (size_t i = 0; i < seq; i++)
    or_attention_decode(q + i * q_stride, kc, vc, pos0 + i, n_heads, n_kv_heads, hd, out + i * q_stride);
}

/* attention.rs:236-284: causal f32 attention over the prompt window */
void or_attention(const float *q, const float *k, const float *v, size_t seq, size_t n_heads,
                  size_t n_kv_heads, size_t hd, float *out) {
  size_t group = n_heads / n_kv_heads, q_stride = n_heads * hd, kv_stride = n_kv_heads * hd;
  float scale = 1.0f / sqrtf((float)hd);
  float *scores = malloc(sizeof(float) * seq * 2);
  float *probs = scores + seq;
  memset(out, 0, sizeof(float) * seq * q_stride);
  for (size_t i = 0; i < seq; i++)
    for (size_t h = 0; h < n_heads; h++) {
      size_t kv_h = h / group;
      const float *qv = q + i * q_stride + h * hd;
      for (size_t t = 0; t <= i; t++) {
        const float *kv = k + t * kv_stride + kv_h * hd;
        float dot = 0.0f;
        for (size_t d = 0; d < hd; d++) dot += qv[d] * kv[d];
        scores[t] = dot * scale;
      }
      or_softmax(scores, i + 1, probs);
      float *dst = out + i * q_stride + h * hd;
      for (size_t t = 0; t <= i; t++) {
        const float *vv = v + t * kv_stride + kv_h * hd;
        for (size_t d = 0; d < hd; d++) dst[d] += probs[t] * vv[d];
      }
    }
  free(scores);
}

/* infer.rs:560-568: first index of the maximum (strict >) */
uint32_t or_argmax(const float *x, size_t n) {
  size_t best = 0;
  for (size_t i = 0; i < n; i++)
    if (x[i] > x[best]) best = i;
  return (uint32_t)best;
}
