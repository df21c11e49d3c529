/*
 * synth.c -- seeded random-init model and matrix generator (host only).
 *
 * Writes GGUF v3 files with the tensor names and metadata keys Prana's loader
 * reads (crates/prana-model/src/gguf.rs:338-460), filled with N(0, std)
 * weights, unit norm weights and the quantized block formats the decode path
 * consumes.  There is no network for real checkpoints, so every benchmark and
 * parity model is built here from a seed.
 *
 * Encoders:
 *  - Q4_K, Q6_K: the reference's own quantizers, restated from
 *    scripts/convert-to-gguf.py:29-89 (float64 math, round-half-even `round`,
 *    f16 packing with round-half-even from double).  Byte-identical output is
 *    pinned by fixtures generated with the reference script itself.
 *  - Q8_0, Q4_0: the reference has no writer; these follow llama.cpp's
 *    published quantize_row_q8_0 / quantize_row_q4_0 algorithms
 *    (d = amax/127, q = round(x/d); d = signed-max / -8, q = min(15, x/d + 8.5)).
 *
 * Normals: Marsaglia's polar method in double precision over a per-row
 * splitmix64-seeded xoshiro256** stream, so tensors are identical for any
 * thread count.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "synth.h"

/* ---------------- RNG ---------------- */

static uint64_t splitmix64(uint64_t *s) {
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

typedef struct {
  uint64_t s[4];
  int have;
  double spare;
} rng_t;

static void rng_seed(rng_t *r, uint64_t seed, uint64_t tensor, uint64_t row) {
  uint64_t sm = seed ^ (tensor * 0xD1B54A32D192ED03ull) ^ (row * 0x8CB92BA72F3D8DD7ull);
  for (int i = 0; i < 4; i++) r->s[i] = splitmix64(&sm);
  r->have = 0;
}

static inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

static uint64_t xoshiro(rng_t *r) {
  uint64_t *s = r->s;
  uint64_t res = rotl(s[1] * 5, 7) * 9, t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl(s[3], 45);
  return res;
}

/* uniform in (-1, 1) with 53 random bits */
static double unif_pm1(rng_t *r) { return ((double)(xoshiro(r) >> 11) * 0x1.0p-53) * 2.0 - 1.0; }

static double normal(rng_t *r) {
  if (r->have) {
    r->have = 0;
    return r->spare;
  }
  double u, v, s;
  do {
    u = unif_pm1(r);
    v = unif_pm1(r);
    s = u * u + v * v;
  } while (s >= 1.0 || s == 0.0);
  double m = sqrt(-2.0 * log(s) / s);
  r->spare = v * m;
  r->have = 1;
  return u * m;
}

void synth_normal_row(uint64_t seed, uint64_t tensor, uint64_t row, size_t n, float std, float *out) {
  rng_t r;
  rng_seed(&r, seed, tensor, row);
  for (size_t i = 0; i < n; i++) out[i] = (float)(normal(&r) * (double)std);
}

/* ---------------- f16 ---------------- */

/* f32 -> f16, round to nearest even (IEEE) */
static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  int32_t e = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t m = x & 0x7fffffu;
  if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (m ? 0x200u : 0u));
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    m |= 0x800000u;
    uint32_t sh = (uint32_t)(14 - e), h = m >> sh, rem = m & ((1u << sh) - 1), half = 1u << (sh - 1);
    if (rem > half || (rem == half && (h & 1))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (m >> 13), rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
  return (uint16_t)(sign | h);
}

/* double -> f16, round to nearest even directly from double (CPython's
 * PyFloat_Pack2, used by struct 'e').  |x| must be < 65520. */
static uint16_t f64_to_f16(double x) {
  uint16_t sign = signbit(x) ? 0x8000u : 0;
  double a = fabs(x);
  if (a == 0.0) return sign;
  if (isnan(x)) return 0x7e00u;
  int e;
  double fr = frexp(a, &e); /* a = fr * 2^e, fr in [0.5, 1) */
  if (e < -13) {
    /* subnormal half: units of 2^-24 */
    double q = rint(a * 0x1.0p24);
    return (uint16_t)(sign | (uint16_t)q); /* q == 1024 carries into the exponent field */
  }
  /* normal: a = (1 + m/1024) * 2^(e-1) */
  double mant = rint((fr * 2.0 - 1.0) * 1024.0);
  int be = e - 1 + 15;
  if (mant >= 1024.0) {
    mant = 0.0;
    be++;
  }
  if (be >= 31) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | (uint16_t)(be << 10) | (uint16_t)mant);
}

static void put16(uint8_t *p, uint16_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
}

/* ---------------- block encoders ---------------- */

/* llama.cpp quantize_row_q8_0: d = amax/127, q = round(x/d) */
static void enc_q8_0(const float *x, uint8_t *b) {
  float amax = 0.0f;
  for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
  float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  for (int i = 0; i < 32; i++) {
    float v = roundf(x[i] * id);
    if (v > 127.0f) v = 127.0f;
    if (v < -127.0f) v = -127.0f;
    b[2 + i] = (uint8_t)(int8_t)v;
  }
}

/* llama.cpp quantize_row_q4_0: signed max-magnitude value m, d = m / -8,
 * q = min(15, (int)(x/d + 8.5)); byte j holds elements j (low) and j+16 (high). */
static void enc_q4_0(const float *x, uint8_t *b) {
  float amax = 0.0f, mx = 0.0f;
  for (int i = 0; i < 32; i++)
    if (fabsf(x[i]) > amax) {
      amax = fabsf(x[i]);
      mx = x[i];
    }
  float d = mx / -8.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
  put16(b, f32_to_f16(d));
  for (int j = 0; j < 16; j++) {
    int q0 = (int)(x[j] * id + 8.5f), q1 = (int)(x[j + 16] * id + 8.5f);
    if (q0 > 15) q0 = 15;
    if (q1 > 15) q1 = 15;
    if (q0 < 0) q0 = 0;
    if (q1 < 0) q1 = 0;
    b[2 + j] = (uint8_t)(q0 | (q1 << 4));
  }
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* scripts/convert-to-gguf.py:29-60 q4k_encode_block */
static void enc_q4_k(const float *xf, uint8_t *b) {
  double vals[256], scs[8], ms[8];
  for (int i = 0; i < 256; i++) vals[i] = (double)xf[i];
  for (int g = 0; g < 8; g++) {
    double vmin = vals[g * 32], vmax = vals[g * 32];
    for (int l = 1; l < 32; l++) {
      double v = vals[g * 32 + l];
      if (v < vmin) vmin = v;
      if (v > vmax) vmax = v;
    }
    double m = -vmin > 0.0 ? -vmin : 0.0;
    double sc = (vmax + m) / 15.0;
    scs[g] = sc > 0.0 ? sc : 0.0;
    ms[g] = m;
  }
  double mxs = scs[0], mxm = ms[0];
  for (int g = 1; g < 8; g++) {
    if (scs[g] > mxs) mxs = scs[g];
    if (ms[g] > mxm) mxm = ms[g];
  }
  double d = mxs / 63.0, dmin = mxm / 63.0;
  if (d == 0.0) d = 1e-12;
  if (dmin == 0.0) dmin = 1e-12;
  int ls[8], lm[8];
  for (int g = 0; g < 8; g++) {
    ls[g] = clampi((int)rint(scs[g] / d), 0, 63);
    lm[g] = clampi((int)rint(ms[g] / dmin), 0, 63);
  }
  put16(b, f64_to_f16(d));
  put16(b + 2, f64_to_f16(dmin));
  uint8_t *scales = b + 4;
  for (int j = 0; j < 4; j++) {
    scales[j] = (uint8_t)((ls[j] & 63) | ((ls[j + 4] >> 4) << 6));
    scales[j + 4] = (uint8_t)((lm[j] & 63) | ((lm[j + 4] >> 4) << 6));
    scales[j + 8] = (uint8_t)((ls[j + 4] & 0xF) | ((lm[j + 4] & 0xF) << 4));
  }
  uint8_t *qs = b + 16;
  memset(qs, 0, 128);
  for (int pair = 0; pair < 4; pair++)
    for (int kind = 0; kind < 2; kind++) {
      int g = pair * 2 + kind;
      double d1 = d * ls[g], m1 = dmin * lm[g];
      for (int l = 0; l < 32; l++) {
        int q = d1 > 0.0 ? clampi((int)rint((vals[g * 32 + l] + m1) / d1), 0, 15) : 0;
        qs[pair * 32 + l] |= (uint8_t)(q << (4 * kind));
      }
    }
}

/* scripts/convert-to-gguf.py:63-89 q6k_encode_block */
static void enc_q6_k(const float *xf, uint8_t *b) {
  double vals[256], s16[16];
  for (int i = 0; i < 256; i++) vals[i] = (double)xf[i];
  for (int s = 0; s < 16; s++) {
    int half = s / 8, w = s % 8, base = half * 128 + (w / 2) * 32 + (w % 2) * 16;
    double mx = 0.0;
    for (int i = 0; i < 16; i++) {
      double a = fabs(vals[base + i]);
      if (a > mx) mx = a;
    }
    s16[s] = mx / 31.0;
  }
  double mxs = s16[0];
  for (int s = 1; s < 16; s++)
    if (s16[s] > mxs) mxs = s16[s];
  double d = mxs / 127.0;
  if (d == 0.0) d = 1e-12;
  int ls[16];
  for (int s = 0; s < 16; s++) ls[s] = clampi((int)rint(s16[s] / d), 1, 127);
  uint8_t *ql = b, *qh = b + 128;
  memset(b, 0, 210);
  for (int half = 0; half < 2; half++)
    for (int l = 0; l < 32; l++) {
      int sub = half * 8 + l / 16, qs[4];
      for (int g = 0; g < 4; g++) {
        double eff = d * ls[sub + g * 2];
        qs[g] = eff > 0.0 ? clampi((int)rint(vals[half * 128 + g * 32 + l] / eff) + 32, 0, 63) : 32;
      }
      ql[half * 64 + l] = (uint8_t)((qs[0] & 0xF) | ((qs[2] & 0xF) << 4));
      ql[half * 64 + l + 32] = (uint8_t)((qs[1] & 0xF) | ((qs[3] & 0xF) << 4));
      qh[half * 32 + l] = (uint8_t)((qs[0] >> 4) | ((qs[1] >> 4) << 2) | ((qs[2] >> 4) << 4) | ((qs[3] >> 4) << 6));
    }
  for (int s = 0; s < 16; s++) b[192 + s] = (uint8_t)(int8_t)ls[s];
  put16(b + 208, f64_to_f16(d));
}

size_t synth_row_bytes(int type, size_t cols) {
  switch (type) {
    case SYNTH_F32: return cols * 4;
    case SYNTH_F16: return cols * 2;
    case SYNTH_Q4_0: return cols / 32 * 18;
    case SYNTH_Q8_0: return cols / 32 * 34;
    case SYNTH_Q4_K: return cols / 256 * 144;
    case SYNTH_Q6_K: return cols / 256 * 210;
  }
  return 0;
}

int synth_encode_row(int type, const float *x, size_t cols, uint8_t *out) {
  switch (type) {
    case SYNTH_F32: memcpy(out, x, cols * 4); return 0;
    case SYNTH_F16:
      for (size_t i = 0; i < cols; i++) put16(out + 2 * i, f32_to_f16(x[i]));
      return 0;
    case SYNTH_Q8_0:
      if (cols % 32) return -1;
      for (size_t i = 0; i < cols / 32; i++) enc_q8_0(x + 32 * i, out + 34 * i);
      return 0;
    case SYNTH_Q4_0:
      if (cols % 32) return -1;
      for (size_t i = 0; i < cols / 32; i++) enc_q4_0(x + 32 * i, out + 18 * i);
      return 0;
    case SYNTH_Q4_K:
      if (cols % 256) return -1;
      for (size_t i = 0; i < cols / 256; i++) enc_q4_k(x + 256 * i, out + 144 * i);
      return 0;
    case SYNTH_Q6_K:
      if (cols % 256) return -1;
      for (size_t i = 0; i < cols / 256; i++) enc_q6_k(x + 256 * i, out + 210 * i);
      return 0;
  }
  return -1;
}

/* ---------------- parallel tensor generation ---------------- */

typedef struct {
  int code;          /* 0: plain; 1: embedding rows P c_t; 2: head rows P c_{s(j)} (synth_model.code_rank) */
  int rank;
  uint64_t code_seed;
  float noise;
  const float *proj; /* [cols][rank] */
} code_spec;

typedef struct {
  int type;
  size_t rows, cols;
  uint64_t seed, tid;
  float std;
  float constant; /* used when std == 0 */
  uint8_t *out;
  size_t r0, r1;
  int rc;
  const code_spec *cs;
} gen_job;

#define CODE_TID 0xC0DEull
#define PROJ_TID 0x9E07ull
#define SUCC_A 48271u
#define SUCC_B 12345u

/* s(j): the token whose successor is j, succ(t) = (A t + B) mod V */
static uint64_t succ_inverse(uint64_t j, uint64_t v) {
  /* A^-1 mod V by the extended Euclid algorithm */
  int64_t t0 = 0, t1 = 1, r0 = (int64_t)v, r1 = (int64_t)(SUCC_A % v);
  while (r1) {
    int64_t q = r0 / r1, tt = t0 - q * t1, rr = r0 - q * r1;
    t0 = t1;
    t1 = tt;
    r0 = r1;
    r1 = rr;
  }
  uint64_t inv = (uint64_t)((t0 % (int64_t)v + (int64_t)v) % (int64_t)v);
  uint64_t d = (j + v - (SUCC_B % v)) % v;
  return (uint64_t)(((unsigned __int128)inv * d) % v);
}

/* row r of a shared-code table: P c_t (+ noise) */
static void code_row(const code_spec *cs, uint64_t seed, uint64_t tid, uint64_t r, size_t rows, size_t cols,
                     float *row, float *code) {
  const uint64_t t = cs->code == 1 ? r : succ_inverse(r, rows);
  synth_normal_row(cs->code_seed, CODE_TID, t, (size_t)cs->rank, 1.0f, code);
  synth_normal_row(seed, tid, r, cols, cs->noise, row);
  for (size_t d = 0; d < cols; d++) {
    double acc = 0.0;
    for (int k = 0; k < cs->rank; k++) acc += (double)cs->proj[d * cs->rank + k] * code[k];
    row[d] += (float)acc;
  }
}

static void *gen_rows(void *arg) {
  gen_job *j = arg;
  float *row = malloc(sizeof(float) * j->cols);
  float *code = j->cs ? malloc(sizeof(float) * (size_t)j->cs->rank) : NULL;
  size_t rb = synth_row_bytes(j->type, j->cols);
  for (size_t r = j->r0; r < j->r1; r++) {
    if (j->cs)
      code_row(j->cs, j->seed, j->tid, r, j->rows, j->cols, row, code);
    else if (j->std == 0.0f)
      for (size_t i = 0; i < j->cols; i++) row[i] = j->constant;
    else synth_normal_row(j->seed, j->tid, r, j->cols, j->std, row);
    if (synth_encode_row(j->type, row, j->cols, j->out + r * rb)) j->rc = -1;
  }
  free(row);
  free(code);
  return NULL;
}

static int gen_tensor(int type, size_t rows, size_t cols, uint64_t seed, uint64_t tid, float std, float constant,
                      int threads, uint8_t *out, const code_spec *cs);

int synth_tensor(int type, size_t rows, size_t cols, uint64_t seed, uint64_t tid, float std,
                 float constant, int threads, uint8_t *out) {
  return gen_tensor(type, rows, cols, seed, tid, std, constant, threads, out, NULL);
}

static int gen_tensor(int type, size_t rows, size_t cols, uint64_t seed, uint64_t tid, float std, float constant,
                      int threads, uint8_t *out, const code_spec *cs) {
  if (!synth_row_bytes(type, cols)) return -1;
  if (threads < 1) threads = 1;
  if ((size_t)threads > rows) threads = (int)(rows ? rows : 1);
  gen_job *jobs = calloc((size_t)threads, sizeof(gen_job));
  pthread_t *th = calloc((size_t)threads, sizeof(pthread_t));
  size_t per = (rows + threads - 1) / threads;
  int rc = 0;
  for (int t = 0; t < threads; t++) {
    jobs[t] = (gen_job){type, rows, cols, seed, tid, std, constant, out, t * per, (t + 1) * per, 0, cs};
    if (jobs[t].r1 > rows) jobs[t].r1 = rows;
    if (jobs[t].r0 > rows) jobs[t].r0 = rows;
    pthread_create(&th[t], NULL, gen_rows, &jobs[t]);
  }
  for (int t = 0; t < threads; t++) {
    pthread_join(th[t], NULL);
    rc |= jobs[t].rc;
  }
  free(jobs);
  free(th);
  return rc;
}

/* ---------------- GGUF writer ---------------- */

typedef struct {
  uint8_t *p;
  size_t len, cap;
} buf_t;

static void bput(buf_t *b, const void *src, size_t n) {
  if (b->len + n > b->cap) {
    size_t nc = b->cap ? b->cap * 2 : 1 << 16;
    while (nc < b->len + n) nc *= 2;
    b->p = realloc(b->p, nc);
    b->cap = nc;
  }
  memcpy(b->p + b->len, src, n);
  b->len += n;
}
static void bu32(buf_t *b, uint32_t v) { bput(b, &v, 4); }
static void bu64(buf_t *b, uint64_t v) { bput(b, &v, 8); }
static void bstr(buf_t *b, const char *s) {
  bu64(b, strlen(s));
  bput(b, s, strlen(s));
}
static void kv_u32(buf_t *b, const char *k, uint32_t v) {
  bstr(b, k);
  bu32(b, 4);
  bu32(b, v);
}
static void kv_f32(buf_t *b, const char *k, float v) {
  bstr(b, k);
  bu32(b, 6);
  bput(b, &v, 4);
}
static void kv_str(buf_t *b, const char *k, const char *v) {
  bstr(b, k);
  bu32(b, 8);
  bstr(b, v);
}

typedef struct {
  char name[64];
  int type;
  size_t rows, cols; /* 1-D tensors: rows = 1 */
  int one_d;
  float std, constant;
  uint64_t tid;
  size_t bytes, offset;
  int code; /* shared-code table: 1 embedding, 2 head */
} tdesc;

#define ALIGN 32

int synth_write_gguf(const synth_model *c, const char *path, int threads) {
  if (!c || !path) return -1;
  int n_t = 0;
  size_t cap = 16 + (size_t)c->n_layers * 12;
  tdesc *T = calloc(cap, sizeof(tdesc));
  size_t q_dim = (size_t)c->n_heads * c->head_dim, kv_dim = (size_t)c->n_kv_heads * c->head_dim;
  uint64_t tid = 1;
#define ADD(nm_, ty_, rows_, cols_, oned_, std_, const_)                     \
  do {                                                                        \
    tdesc *d_ = &T[n_t++];                                                    \
    snprintf(d_->name, sizeof(d_->name), "%s", nm_);                          \
    d_->type = (ty_);                                                         \
    d_->rows = (rows_);                                                       \
    d_->cols = (cols_);                                                       \
    d_->one_d = (oned_);                                                      \
    d_->std = (std_);                                                         \
    d_->constant = (const_);                                                  \
    d_->tid = tid++;                                                          \
    d_->bytes = synth_row_bytes(d_->type, d_->cols) * d_->rows;               \
  } while (0)
  char nm[64];
  float s = c->std;
  ADD("token_embd.weight", c->type_embd, (size_t)c->vocab, (size_t)c->dim, 0, s * c->embd_std_mult, 0.0f);
  if (c->code_rank > 0) T[n_t - 1].code = 1;
  for (int i = 0; i < c->n_layers; i++) {
    snprintf(nm, sizeof nm, "blk.%d.attn_norm.weight", i);
    ADD(nm, SYNTH_F32, 1, (size_t)c->dim, 1, 0.0f, 1.0f);
    snprintf(nm, sizeof nm, "blk.%d.attn_q.weight", i);
    ADD(nm, c->type_q, q_dim, (size_t)c->dim, 0, s, 0.0f);
    snprintf(nm, sizeof nm, "blk.%d.attn_k.weight", i);
    ADD(nm, c->type_k, kv_dim, (size_t)c->dim, 0, s, 0.0f);
    snprintf(nm, sizeof nm, "blk.%d.attn_v.weight", i);
    ADD(nm, c->type_v, kv_dim, (size_t)c->dim, 0, s, 0.0f);
    snprintf(nm, sizeof nm, "blk.%d.attn_output.weight", i);
    ADD(nm, c->type_o, (size_t)c->dim, q_dim, 0, s * c->out_proj_mult, 0.0f);
    if (c->has_bias) {
      snprintf(nm, sizeof nm, "blk.%d.attn_q.bias", i);
      ADD(nm, SYNTH_F32, 1, q_dim, 1, s, 0.0f);
      snprintf(nm, sizeof nm, "blk.%d.attn_k.bias", i);
      ADD(nm, SYNTH_F32, 1, kv_dim, 1, s, 0.0f);
      snprintf(nm, sizeof nm, "blk.%d.attn_v.bias", i);
      ADD(nm, SYNTH_F32, 1, kv_dim, 1, s, 0.0f);
    }
    snprintf(nm, sizeof nm, "blk.%d.ffn_norm.weight", i);
    ADD(nm, SYNTH_F32, 1, (size_t)c->dim, 1, 0.0f, 1.0f);
    snprintf(nm, sizeof nm, "blk.%d.ffn_gate.weight", i);
    ADD(nm, c->type_gate, (size_t)c->hidden, (size_t)c->dim, 0, s, 0.0f);
    snprintf(nm, sizeof nm, "blk.%d.ffn_down.weight", i);
    ADD(nm, c->type_down, (size_t)c->dim, (size_t)c->hidden, 0, s * c->out_proj_mult, 0.0f);
    snprintf(nm, sizeof nm, "blk.%d.ffn_up.weight", i);
    ADD(nm, c->type_up, (size_t)c->hidden, (size_t)c->dim, 0, s, 0.0f);
  }
  ADD("output_norm.weight", SYNTH_F32, 1, (size_t)c->dim, 1, 0.0f, 1.0f);
  if (!c->tied || c->code_rank > 0) {
    ADD("output.weight", c->type_output, (size_t)c->vocab, (size_t)c->dim, 0, s * c->head_std_mult, 0.0f);
    if (c->code_rank > 0) T[n_t - 1].code = 2;
  }
#undef ADD
  for (int i = 0; i < n_t; i++)
    if (!T[i].bytes) {
      fprintf(stderr, "synth: tensor %s: type %d cannot hold %zu columns\n", T[i].name, T[i].type, T[i].cols);
      free(T);
      return -2;
    }

  buf_t h = {0};
  bu32(&h, 0x46554747u);
  bu32(&h, 3);
  bu64(&h, (uint64_t)n_t);
  int n_kv = 14 + (c->eps > 0.0f ? 1 : 0);
  bu64(&h, (uint64_t)n_kv);
  const char *a = c->arch;
  char key[128];
  kv_str(&h, "general.architecture", a);
  kv_u32(&h, "general.alignment", ALIGN);
#define KU(suf, v) (snprintf(key, sizeof key, "%s." suf, a), kv_u32(&h, key, (uint32_t)(v)))
  KU("embedding_length", c->dim);
  KU("block_count", c->n_layers);
  KU("attention.head_count", c->n_heads);
  KU("attention.head_count_kv", c->n_kv_heads);
  KU("feed_forward_length", c->hidden);
  KU("context_length", c->ctx);
  KU("attention.key_length", c->head_dim);
#undef KU
  snprintf(key, sizeof key, "%s.rope.freq_base", a);
  kv_f32(&h, key, c->rope_theta);
  if (c->eps > 0.0f) {
    snprintf(key, sizeof key, "%s.attention.layer_norm_rms_epsilon", a);
    kv_f32(&h, key, c->eps);
  }
  kv_str(&h, "tokenizer.ggml.model", "llama");
  /* vocabulary: one distinct piece per id, so the reference's tokenizer loads */
  bstr(&h, "tokenizer.ggml.tokens");
  bu32(&h, 9);
  bu32(&h, 8);
  bu64(&h, (uint64_t)c->vocab);
  char piece[32];
  for (int i = 0; i < c->vocab; i++) {
    snprintf(piece, sizeof piece, "<t%d>", i);
    bstr(&h, piece);
  }
  bstr(&h, "tokenizer.ggml.scores");
  bu32(&h, 9);
  bu32(&h, 6);
  bu64(&h, (uint64_t)c->vocab);
  for (int i = 0; i < c->vocab; i++) {
    float sc = -1.0f;
    bput(&h, &sc, 4);
  }
  /* tokenizer.ggml.eos_token_id: outside the vocab, so greedy runs never stop early */
  bstr(&h, "tokenizer.ggml.eos_token_id");
  bu32(&h, 4);
  bu32(&h, (uint32_t)c->vocab);
  /* tensor directory */
  size_t off = 0;
  for (int i = 0; i < n_t; i++) {
    bstr(&h, T[i].name);
    if (T[i].one_d) {
      bu32(&h, 1);
      bu64(&h, T[i].cols);
    } else {
      bu32(&h, 2);
      bu64(&h, T[i].cols);
      bu64(&h, T[i].rows);
    }
    bu32(&h, (uint32_t)T[i].type);
    bu64(&h, off);
    T[i].offset = off;
    off = (off + T[i].bytes + ALIGN - 1) / ALIGN * ALIGN;
  }
  while (h.len % ALIGN) {
    uint8_t z = 0;
    bput(&h, &z, 1);
  }
  FILE *f = fopen(path, "wb");
  if (!f) {
    free(h.p);
    free(T);
    return -3;
  }
  int rc = fwrite(h.p, 1, h.len, f) == h.len ? 0 : -4;
  /* the shared-code projection of this model: [dim][code_rank], N(0, 1/code_rank) */
  float *proj = NULL;
  code_spec cs = {0, c->code_rank, c->code_seed, c->code_noise, NULL};
  if (c->code_rank > 0) {
    proj = malloc(sizeof(float) * (size_t)c->dim * (size_t)c->code_rank);
    for (int d = 0; d < c->dim; d++)
      synth_normal_row(c->seed, PROJ_TID, (uint64_t)d, (size_t)c->code_rank, 1.0f / sqrtf((float)c->code_rank),
                       proj + (size_t)d * c->code_rank);
    cs.proj = proj;
  }
  size_t written = 0;
  for (int i = 0; i < n_t && !rc; i++) {
    while (written < T[i].offset) {
      uint8_t z = 0;
      fwrite(&z, 1, 1, f);
      written++;
    }
    uint8_t *data = malloc(T[i].bytes);
    code_spec csi = cs;
    csi.code = T[i].code;
    if (gen_tensor(T[i].type, T[i].rows, T[i].cols, c->seed, T[i].tid, T[i].std, T[i].constant, threads, data,
                   T[i].code ? &csi : NULL))
      rc = -5;
    if (!rc && fwrite(data, 1, T[i].bytes, f) != T[i].bytes) rc = -4;
    written += T[i].bytes;
    free(data);
  }
  fclose(f);
  free(proj);
  free(h.p);
  free(T);
  return rc;
}
