/*
 * model.c -- TEST INFRASTRUCTURE (oracle).  GGUF subset reader and model
 * construction (crates/prana-model/src/gguf.rs:87-460, checkpoint.rs:32-265)
 * and the KV-cached forward / prefill / verify / generate / speculative loops
 * (crates/prana-model/src/infer.rs:25-79,142-374,560-771).  Token ids in,
 * token ids out: the tokenizer is outside the decode path.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "prana_oracle.h"

/* ---------------- matrices ---------------- */

static float rd_f16(const uint8_t *b) { return or_f16_to_f32((uint16_t)(b[0] | (b[1] << 8))); }

/* gguf.rs:271-305 (Linear) and kquant.rs:166-183 (dscales hoisting) */
int or_matrix_from_gguf(or_matrix *m, int type, size_t rows, size_t cols, const uint8_t *raw) {
  memset(m, 0, sizeof(*m));
  m->rows = rows;
  m->cols = cols;
  size_t n = rows * cols;
  if (type == OR_GGML_Q8_0 && cols % 32 == 0) {
    m->kind = OR_GGML_Q8_0;
    m->q = malloc(n);
    m->scales = malloc(sizeof(float) * (n / 32));
    for (size_t b = 0; b < n / 32; b++) {
      m->scales[b] = rd_f16(raw + b * 34);
      memcpy(m->q + b * 32, raw + b * 34 + 2, 32);
    }
    return 0;
  }
  if ((type == OR_GGML_Q4_0 && cols % 32 == 0) || ((type == OR_GGML_Q4_K || type == OR_GGML_Q6_K) && cols % 256 == 0)) {
    m->kind = type;
    size_t bv = type == OR_GGML_Q4_0 ? 32 : 256;
    size_t bb = type == OR_GGML_Q4_0 ? 18 : (type == OR_GGML_Q4_K ? 144 : 210);
    size_t nb = n / bv;
    m->blocks = malloc(nb * bb);
    memcpy(m->blocks, raw, nb * bb);
    size_t spb = type == OR_GGML_Q4_K ? 2 : 1;
    m->scales = malloc(sizeof(float) * nb * spb);
    for (size_t b = 0; b < nb; b++) {
      const uint8_t *blk = raw + b * bb;
      if (type == OR_GGML_Q4_0) m->scales[b] = rd_f16(blk);
      else if (type == OR_GGML_Q4_K) {
        m->scales[2 * b] = rd_f16(blk);
        m->scales[2 * b + 1] = rd_f16(blk + 2);
      } else m->scales[b] = rd_f16(blk + 208);
    }
    return 0;
  }
  /* everything else densifies (gguf.rs:208-267 tensor_f32) */
  m->kind = OR_GGML_F32;
  m->f32 = malloc(sizeof(float) * n);
  if (type == OR_GGML_F32) memcpy(m->f32, raw, n * 4);
  else if (type == OR_GGML_F16)
    for (size_t i = 0; i < n; i++) m->f32[i] = rd_f16(raw + 2 * i);
  else if (type == OR_GGML_Q8_0)
    for (size_t b = 0; b < n / 32; b++) {
      float s = rd_f16(raw + b * 34);
      for (int i = 0; i < 32; i++) m->f32[b * 32 + i] = (float)(int8_t)raw[b * 34 + 2 + i] * s;
    }
  else if (type == OR_GGML_Q4_0)
    for (size_t b = 0; b < n / 32; b++) or_dequant_q40_block(raw + b * 18, m->f32 + b * 32);
  else if (type == OR_GGML_Q4_K)
    for (size_t b = 0; b < n / 256; b++) or_dequant_q4k_block(raw + b * 144, m->f32 + b * 256);
  else if (type == OR_GGML_Q6_K)
    for (size_t b = 0; b < n / 256; b++) or_dequant_q6k_block(raw + b * 210, m->f32 + b * 256);
  else return -1;
  return 0;
}

void or_matrix_free(or_matrix *m) {
  free(m->f32);
  free(m->q);
  free(m->scales);
  free(m->blocks);
  memset(m, 0, sizeof(*m));
}

void or_matrix_dequant_row(const or_matrix *m, size_t r, float *out) {
  size_t k = m->cols;
  switch (m->kind) {
    case OR_GGML_F32:
      memcpy(out, m->f32 + r * k, k * 4);
      break;
    case OR_GGML_Q8_0:
      for (size_t i = 0; i < k; i++) out[i] = (float)m->q[r * k + i] * m->scales[(r * k + i) / 32];
      break;
    case OR_GGML_Q4_0:
      for (size_t b = 0; b < k / 32; b++) or_dequant_q40_block(m->blocks + (r * k / 32 + b) * 18, out + b * 32);
      break;
    case OR_GGML_Q4_K:
      for (size_t b = 0; b < k / 256; b++) or_dequant_q4k_block(m->blocks + (r * k / 256 + b) * 144, out + b * 256);
      break;
    case OR_GGML_Q6_K:
      for (size_t b = 0; b < k / 256; b++) or_dequant_q6k_block(m->blocks + (r * k / 256 + b) * 210, out + b * 256);
      break;
  }
}

void or_matrix_dequant(const or_matrix *m, float *out) {
  for (size_t r = 0; r < m->rows; r++) or_matrix_dequant_row(m, r, out + r * m->cols);
}

/* ---------------- GGUF ---------------- */

typedef struct {
  char *name;
  size_t dims[4];
  uint32_t n_dims, type;
  uint64_t offset;
} tinfo;

typedef struct {
  uint8_t *data;
  size_t len, off, data_start;
  size_t n_tensors;
  tinfo *t;
  /* the few metadata values the loader reads (gguf.rs:338-376) */
  char arch[32];
  int64_t dim, n_layers, n_heads, n_kv_heads, hidden, ctx, key_length, alignment, vocab;
  double rope_theta, eps;
  int has_rope_theta, has_eps;
} gguf;

static int rd(gguf *g, void *dst, size_t n) {
  if (g->off + n > g->len) return -1;
  memcpy(dst, g->data + g->off, n);
  g->off += n;
  return 0;
}
static uint32_t ru32(gguf *g, int *e) {
  uint32_t v = 0;
  *e |= rd(g, &v, 4);
  return v;
}
static uint64_t ru64(gguf *g, int *e) {
  uint64_t v = 0;
  *e |= rd(g, &v, 8);
  return v;
}

/* gguf.rs:110-134 value reader; returns integer/float view when scalar */
static int rvalue(gguf *g, uint32_t ty, int64_t *iv, double *fv, char *sv, size_t svlen, uint64_t *arr_count) {
  int e = 0;
  *iv = -1;
  *fv = NAN;
  switch (ty) {
    case 0: { uint8_t v = 0; e |= rd(g, &v, 1); *iv = v; break; }
    case 1: { int8_t v = 0; e |= rd(g, &v, 1); *iv = v; break; }
    case 2: { uint16_t v = 0; e |= rd(g, &v, 2); *iv = v; break; }
    case 3: { int16_t v = 0; e |= rd(g, &v, 2); *iv = v; break; }
    case 4: { uint32_t v = ru32(g, &e); *iv = v; break; }
    case 5: { int32_t v = (int32_t)ru32(g, &e); *iv = v; break; }
    case 6: { float v = 0; e |= rd(g, &v, 4); *fv = v; break; }
    case 7: { uint8_t v = 0; e |= rd(g, &v, 1); *iv = v; break; }
    case 8: {
      uint64_t n = ru64(g, &e);
      if (e || g->off + n > g->len) return -1;
      if (sv) {
        size_t c = n < svlen - 1 ? n : svlen - 1;
        memcpy(sv, g->data + g->off, c);
        sv[c] = 0;
      }
      g->off += n;
      break;
    }
    case 9: {
      uint32_t et = ru32(g, &e);
      uint64_t n = ru64(g, &e);
      if (e) return -1;
      if (arr_count) *arr_count = n;
      int64_t i2;
      double f2;
      for (uint64_t i = 0; i < n; i++)
        if (rvalue(g, et, &i2, &f2, NULL, 0, NULL)) return -1;
      break;
    }
    case 10: { uint64_t v = ru64(g, &e); *iv = (int64_t)v; break; }
    case 11: { int64_t v = (int64_t)ru64(g, &e); *iv = v; break; }
    case 12: { double v = 0; e |= rd(g, &v, 8); *fv = v; break; }
    default: return -1;
  }
  return e;
}

static int ends_with(const char *k, const char *arch, const char *suffix) {
  size_t la = strlen(arch);
  return strncmp(k, arch, la) == 0 && k[la] == '.' && strcmp(k + la + 1, suffix) == 0;
}

/* gguf.rs:157-196 Gguf::from_bytes */
static int gguf_parse(gguf *g, char *err, size_t errlen) {
  int e = 0;
  if (ru32(g, &e) != 0x46554747u || e) { snprintf(err, errlen, "not a GGUF file (bad magic)"); return -1; }
  uint32_t ver = ru32(g, &e);
  if (ver < 2 || ver > 3) { snprintf(err, errlen, "unsupported GGUF version %u", ver); return -1; }
  g->n_tensors = ru64(g, &e);
  uint64_t n_kv = ru64(g, &e);
  g->dim = g->n_layers = g->n_heads = g->n_kv_heads = g->hidden = g->ctx = g->key_length = -1;
  g->alignment = 32;
  g->vocab = -1;
  char key[256], sv[64];
  for (uint64_t i = 0; i < n_kv && !e; i++) {
    uint64_t kl = ru64(g, &e);
    if (e || g->off + kl > g->len) { e = 1; break; }
    size_t c = kl < sizeof(key) - 1 ? kl : sizeof(key) - 1;
    memcpy(key, g->data + g->off, c);
    key[c] = 0;
    g->off += kl;
    uint32_t ty = ru32(g, &e);
    int64_t iv;
    double fv;
    uint64_t cnt = 0;
    sv[0] = 0;
    if (rvalue(g, ty, &iv, &fv, sv, sizeof(sv), &cnt)) { e = 1; break; }
    if (!strcmp(key, "general.architecture")) snprintf(g->arch, sizeof(g->arch), "%s", sv);
    else if (!strcmp(key, "general.alignment")) g->alignment = iv;
    else if (!strcmp(key, "tokenizer.ggml.tokens")) g->vocab = (int64_t)cnt;
    else if (g->arch[0]) {
      const char *a = g->arch;
      if (ends_with(key, a, "embedding_length")) g->dim = iv;
      else if (ends_with(key, a, "block_count")) g->n_layers = iv;
      else if (ends_with(key, a, "attention.head_count")) g->n_heads = iv;
      else if (ends_with(key, a, "attention.head_count_kv")) g->n_kv_heads = iv;
      else if (ends_with(key, a, "feed_forward_length")) g->hidden = iv;
      else if (ends_with(key, a, "context_length")) g->ctx = iv;
      else if (ends_with(key, a, "attention.key_length")) g->key_length = iv;
      else if (ends_with(key, a, "rope.freq_base") && fv == fv) { g->rope_theta = fv; g->has_rope_theta = 1; }
      else if (ends_with(key, a, "attention.layer_norm_rms_epsilon") && fv == fv) { g->eps = fv; g->has_eps = 1; }
    }
  }
  if (e) { snprintf(err, errlen, "gguf truncated"); return -1; }
  g->t = calloc(g->n_tensors ? g->n_tensors : 1, sizeof(tinfo));
  for (size_t i = 0; i < g->n_tensors && !e; i++) {
    uint64_t nl = ru64(g, &e);
    if (e || g->off + nl > g->len) { e = 1; break; }
    g->t[i].name = malloc(nl + 1);
    memcpy(g->t[i].name, g->data + g->off, nl);
    g->t[i].name[nl] = 0;
    g->off += nl;
    g->t[i].n_dims = ru32(g, &e);
    if (g->t[i].n_dims > 4) { e = 1; break; }
    for (uint32_t d = 0; d < g->t[i].n_dims; d++) g->t[i].dims[d] = ru64(g, &e);
    g->t[i].type = ru32(g, &e);
    g->t[i].offset = ru64(g, &e);
  }
  if (e) { snprintf(err, errlen, "gguf truncated"); return -1; }
  size_t al = (g->alignment > 0 && (g->alignment & (g->alignment - 1)) == 0) ? (size_t)g->alignment : 32;
  g->data_start = (g->off + al - 1) / al * al;
  return 0;
}

static tinfo *gguf_find(gguf *g, const char *name) {
  for (size_t i = 0; i < g->n_tensors; i++)
    if (!strcmp(g->t[i].name, name)) return &g->t[i];
  return NULL;
}

static size_t type_bytes(uint32_t type, size_t n) {
  switch (type) {
    case OR_GGML_F32: return n * 4;
    case OR_GGML_F16: return n * 2;
    case OR_GGML_Q4_0: return n / 32 * 18;
    case OR_GGML_Q8_0: return n / 32 * 34;
    case OR_GGML_Q4_K: return n / 256 * 144;
    case OR_GGML_Q6_K: return n / 256 * 210;
  }
  return 0;
}

static const uint8_t *gguf_raw(gguf *g, tinfo *t) {
  size_t n = 1;
  for (uint32_t d = 0; d < t->n_dims; d++) n *= t->dims[d];
  size_t bytes = type_bytes(t->type, n);
  if (!bytes || g->data_start + t->offset + bytes > g->len) return NULL;
  return g->data + g->data_start + t->offset;
}

/* ---------------- model ---------------- */

typedef struct {
  float *rms_att, *rms_ffn, *bq, *bk, *bv;
  or_matrix wq, wk, wv, wo, w1, w2, w3;
} layer;

struct or_model {
  or_config c;
  int tier;
  or_matrix emb; /* F32 table or packed K-quant (checkpoint.rs:162-189) */
  layer *layers;
  float *rms_final;
  or_matrix wcls;
  int has_wcls;
};

/* gguf.rs:208-267 tensor_f32: any supported type, densified */
static float *vec_f32(gguf *g, const char *name, size_t n, int *e) {
  tinfo *t = gguf_find(g, name);
  const uint8_t *raw = t ? gguf_raw(g, t) : NULL;
  size_t cnt = 1;
  if (t)
    for (uint32_t d = 0; d < t->n_dims; d++) cnt *= t->dims[d];
  if (!raw || cnt != n) {
    *e = 1;
    return NULL;
  }
  float *out = malloc(sizeof(float) * n);
  const uint8_t *b = raw;
  switch (t->type) {
    case OR_GGML_F32: memcpy(out, raw, n * 4); break;
    case OR_GGML_F16: for (size_t i = 0; i < n; i++) out[i] = rd_f16(raw + 2 * i); break;
    case OR_GGML_Q8_0:
      for (size_t i = 0; i < n / 32; i++, b += 34)
        for (int j = 0; j < 32; j++) out[i * 32 + j] = (float)(int8_t)b[2 + j] * rd_f16(b);
      break;
    case OR_GGML_Q4_0: for (size_t i = 0; i < n / 32; i++) or_dequant_q40_block(raw + i * 18, out + i * 32); break;
    case OR_GGML_Q4_K: for (size_t i = 0; i < n / 256; i++) or_dequant_q4k_block(raw + i * 144, out + i * 256); break;
    case OR_GGML_Q6_K: for (size_t i = 0; i < n / 256; i++) or_dequant_q6k_block(raw + i * 210, out + i * 256); break;
    default: free(out); *e = 1; return NULL;
  }
  return out;
}

static int load_linear(gguf *g, const char *name, or_matrix *m) {
  tinfo *t = gguf_find(g, name);
  if (!t || t->n_dims != 2) return -1;
  const uint8_t *raw = gguf_raw(g, t);
  if (!raw) return -1;
  return or_matrix_from_gguf(m, (int)t->type, t->dims[1], t->dims[0], raw);
}

/* Linear::new(w, Precision::Q8) (checkpoint.rs): a dense matrix becomes
 * quantize_q8 of it (matmul.rs:61-84), int8 plus f32 scales */
static void requantize_q8(or_matrix *m) {
  if (m->kind != OR_GGML_F32 || m->cols % 32) return;
  size_t n = m->rows * m->cols;
  int8_t *q = malloc(n);
  float *sc = malloc(sizeof(float) * (n / 32));
  or_quantize_q8(m->rows, m->cols, m->f32, q, sc);
  free(m->f32);
  m->f32 = NULL;
  m->q = q;
  m->scales = sc;
  m->kind = OR_GGML_Q8_0;
}

or_model *or_model_load(const char *path, int tier, char *err, size_t errlen) {
  return or_model_load_ex(path, tier, 0, err, errlen);
}

/* gguf::load(path, precision) (gguf.rs:338-460): precision 1 (Q8) turns every
 * dense tensor the model multiplies -- projections, and a tied classifier over
 * a densified (F32 / F16 / Q8_0) embedding table (gguf.rs:425-437) -- into
 * quantize_q8 of it; precision 0 (F32) keeps them dense */
or_model *or_model_load_ex(const char *path, int tier, int precision, char *err, size_t errlen) {
  FILE *f = fopen(path, "rb");
  if (!f) { snprintf(err, errlen, "cannot open %s", path); return NULL; }
  fseek(f, 0, SEEK_END);
  long len = ftell(f);
  fseek(f, 0, SEEK_SET);
  gguf g = {0};
  g.data = malloc((size_t)len);
  g.len = (size_t)len;
  if (fread(g.data, 1, g.len, f) != g.len) { fclose(f); free(g.data); snprintf(err, errlen, "short read"); return NULL; }
  fclose(f);
  or_model *m = NULL;
  if (gguf_parse(&g, err, errlen)) goto done;
  if (strcmp(g.arch, "llama") && strcmp(g.arch, "qwen2")) {
    snprintf(err, errlen, "unsupported architecture '%s'", g.arch);
    goto done;
  }
  if (g.dim <= 0 || g.n_layers <= 0 || g.n_heads <= 0 || g.hidden <= 0 || g.ctx <= 0 || g.vocab <= 0) {
    snprintf(err, errlen, "missing metadata");
    goto done;
  }
  m = calloc(1, sizeof(*m));
  m->tier = tier;
  or_config *c = &m->c;
  c->dim = (size_t)g.dim;
  c->n_layers = (size_t)g.n_layers;
  c->n_heads = (size_t)g.n_heads;
  c->n_kv_heads = g.n_kv_heads > 0 ? (size_t)g.n_kv_heads : c->n_heads;
  c->hidden_dim = (size_t)g.hidden;
  c->seq_len = (size_t)g.ctx;
  c->rope_theta = g.has_rope_theta ? (float)g.rope_theta : 10000.0f;
  c->head_dim = g.key_length > 0 ? (size_t)g.key_length : c->dim / c->n_heads;
  c->norm_eps = g.has_eps ? (float)g.eps : 1e-5f;
  c->vocab_size = (size_t)g.vocab;
  c->rope_neox = strcmp(g.arch, "llama") != 0;
  int e = 0;
  /* token embedding: packed K-quants stay packed, others densify (gguf.rs:309-326) */
  {
    tinfo *t = gguf_find(&g, "token_embd.weight");
    const uint8_t *raw = t ? gguf_raw(&g, t) : NULL;
    if (!raw || t->n_dims != 2) { snprintf(err, errlen, "missing tensor 'token_embd.weight'"); goto fail; }
    int ty = (int)t->type;
    if (ty == OR_GGML_Q8_0) {
      /* Q8_0 tables go through tensor_f32 -> dense f32 */
      or_matrix tmp;
      or_matrix_from_gguf(&tmp, ty, t->dims[1], t->dims[0], raw);
      m->emb.kind = OR_GGML_F32;
      m->emb.rows = tmp.rows;
      m->emb.cols = tmp.cols;
      m->emb.f32 = malloc(sizeof(float) * tmp.rows * tmp.cols);
      or_matrix_dequant(&tmp, m->emb.f32);
      or_matrix_free(&tmp);
    } else if (or_matrix_from_gguf(&m->emb, ty, t->dims[1], t->dims[0], raw)) {
      snprintf(err, errlen, "bad token_embd");
      goto fail;
    }
    if (m->emb.rows * m->emb.cols != c->vocab_size * c->dim) { snprintf(err, errlen, "token_embd.weight size mismatch with vocab"); goto fail; }
  }
  m->layers = calloc(c->n_layers, sizeof(layer));
  size_t q_dim = c->n_heads * c->head_dim, kv_dim = c->n_kv_heads * c->head_dim;
  char nm[128];
  for (size_t i = 0; i < c->n_layers; i++) {
    layer *L = &m->layers[i];
#define NM(s) (snprintf(nm, sizeof(nm), "blk.%zu." s, i), nm)
    L->rms_att = vec_f32(&g, NM("attn_norm.weight"), c->dim, &e);
    L->rms_ffn = vec_f32(&g, NM("ffn_norm.weight"), c->dim, &e);
    if (e) { snprintf(err, errlen, "missing norm tensor in layer %zu", i); goto fail; }
    if (load_linear(&g, NM("attn_q.weight"), &L->wq) || load_linear(&g, NM("attn_k.weight"), &L->wk) ||
        load_linear(&g, NM("attn_v.weight"), &L->wv) || load_linear(&g, NM("attn_output.weight"), &L->wo) ||
        load_linear(&g, NM("ffn_gate.weight"), &L->w1) || load_linear(&g, NM("ffn_down.weight"), &L->w2) ||
        load_linear(&g, NM("ffn_up.weight"), &L->w3)) {
      snprintf(err, errlen, "missing/bad projection in layer %zu", i);
      goto fail;
    }
    /* gguf.rs:388-394: each bias independently optional */
    if (gguf_find(&g, NM("attn_q.bias"))) L->bq = vec_f32(&g, nm, q_dim, &e);
    if (gguf_find(&g, NM("attn_k.bias"))) L->bk = vec_f32(&g, nm, kv_dim, &e);
    if (gguf_find(&g, NM("attn_v.bias"))) L->bv = vec_f32(&g, nm, kv_dim, &e);
    if (e) { snprintf(err, errlen, "bad bias in layer %zu", i); goto fail; }
    if (L->bq || L->bk || L->bv) c->has_bias = 1;
#undef NM
  }
  m->rms_final = vec_f32(&g, "output_norm.weight", c->dim, &e);
  if (e) { snprintf(err, errlen, "missing output_norm.weight"); goto fail; }
  if (gguf_find(&g, "output.weight")) {
    if (load_linear(&g, "output.weight", &m->wcls)) { snprintf(err, errlen, "bad output.weight"); goto fail; }
    m->has_wcls = 1;
  } else {
    c->shared_classifier = 1;
    if (precision == 1 && m->emb.kind == OR_GGML_F32 && c->dim % 32 == 0) {
      m->wcls.kind = OR_GGML_F32;
      m->wcls.rows = m->emb.rows;
      m->wcls.cols = m->emb.cols;
      m->wcls.f32 = malloc(sizeof(float) * m->emb.rows * m->emb.cols);
      memcpy(m->wcls.f32, m->emb.f32, sizeof(float) * m->emb.rows * m->emb.cols);
      requantize_q8(&m->wcls);
      m->has_wcls = 1;
    }
  }
  if (precision == 1)
    for (size_t i = 0; i < c->n_layers; i++) {
      layer *L = &m->layers[i];
      requantize_q8(&L->wq); requantize_q8(&L->wk); requantize_q8(&L->wv); requantize_q8(&L->wo);
      requantize_q8(&L->w1); requantize_q8(&L->w2); requantize_q8(&L->w3);
    }
  if (precision == 1 && m->has_wcls) requantize_q8(&m->wcls);
  goto done;
fail:
  or_model_free(m);
  m = NULL;
done:
  for (size_t i = 0; i < g.n_tensors && g.t; i++) free(g.t[i].name);
  free(g.t);
  free(g.data);
  return m;
}

void or_model_free(or_model *m) {
  if (!m) return;
  if (m->layers)
    for (size_t i = 0; i < m->c.n_layers; i++) {
      layer *L = &m->layers[i];
      free(L->rms_att); free(L->rms_ffn); free(L->bq); free(L->bk); free(L->bv);
      or_matrix_free(&L->wq); or_matrix_free(&L->wk); or_matrix_free(&L->wv); or_matrix_free(&L->wo);
      or_matrix_free(&L->w1); or_matrix_free(&L->w2); or_matrix_free(&L->w3);
    }
  free(m->layers);
  free(m->rms_final);
  or_matrix_free(&m->emb);
  or_matrix_free(&m->wcls);
  free(m);
}

void or_model_config(const or_model *m, or_config *c) { *c = m->c; }

const or_matrix *or_model_matrix(const or_model *m, int l, const char *w) {
  if (!strcmp(w, "output")) return m->has_wcls ? &m->wcls : NULL;
  if (!strcmp(w, "token_embd")) return &m->emb;
  if (l < 0 || (size_t)l >= m->c.n_layers) return NULL;
  layer *L = &m->layers[l];
  if (!strcmp(w, "wq")) return &L->wq;
  if (!strcmp(w, "wk")) return &L->wk;
  if (!strcmp(w, "wv")) return &L->wv;
  if (!strcmp(w, "wo")) return &L->wo;
  if (!strcmp(w, "w1")) return &L->w1;
  if (!strcmp(w, "w2")) return &L->w2;
  if (!strcmp(w, "w3")) return &L->w3;
  return NULL;
}

/* ---------------- KV cache (infer.rs:25-45) ---------------- */

struct or_kv {
  size_t positions, kv_dim, n_layers;
  uint16_t *k, *v;
};

or_kv *or_kv_create(const or_model *m, size_t positions) {
  or_kv *kv = calloc(1, sizeof(*kv));
  if (positions > m->c.seq_len) positions = m->c.seq_len;
  kv->positions = positions;
  kv->kv_dim = m->c.n_kv_heads * m->c.head_dim;
  kv->n_layers = m->c.n_layers;
  kv->k = calloc(positions * kv->kv_dim * kv->n_layers, 2);
  kv->v = calloc(positions * kv->kv_dim * kv->n_layers, 2);
  return kv;
}
void or_kv_free(or_kv *kv) {
  if (!kv) return;
  free(kv->k);
  free(kv->v);
  free(kv);
}
uint16_t *or_kv_layer(or_kv *kv, int l, int is_v) {
  return (is_v ? kv->v : kv->k) + (size_t)l * kv->positions * kv->kv_dim;
}

/* ---------------- forward ---------------- */

static void add_bias(float *x, const float *b, size_t n) {
  if (b)
    for (size_t i = 0; i < n; i++) x[i] += b[i];
}

static void rope_row(const or_config *c, float *x, size_t n, size_t pos) {
  if (c->rope_neox) or_rope_neox(x, n, pos, c->head_dim, c->rope_theta);
  else or_rope_interleaved(x, n, pos, c->head_dim, c->rope_theta);
}

/* Embedding::row (checkpoint.rs:169-174) */
static void emb_row(const or_model *m, uint32_t tok, float *x) { or_matrix_dequant_row(&m->emb, tok, x); }

/* Linear::apply (checkpoint.rs:94-100); in forced trace mode a quantized
 * matrix takes the current site's given row through matmul_q8_prefill /
 * matmul_kquant_prefill, whose per-element dot is the decode GEMV's. */
static int forced_rows(size_t n, size_t k, const int8_t **q, const float **s, int32_t **sums);
static void apply(const or_model *m, const or_matrix *w, const float *x, float *y) {
  const int8_t *fq;
  const float *fs;
  int32_t *fsum;
  if (w->kind != OR_GGML_F32 && forced_rows(1, w->cols, &fq, &fs, &fsum)) {
    or_matmul_prefill(m->tier, w, fq, fs, fsum, 1, y);
    free(fsum);
    return;
  }
  or_matmul(m->tier, w, x, 1, y);
}

/* Model::logits (checkpoint.rs:239-248) */
static void logits(const or_model *m, const float *x, float *out) {
  if (m->has_wcls) apply(m, &m->wcls, x, out);
  else apply(m, &m->emb, x, out);
}

/* Diagnostic trace of the quantized activation rows a forward pass feeds its
 * integer dots (the same quantize_acts the matmuls run internally).
 *
 * Forced mode (test instrumentation): when tr_fq is set, the rows quantized at
 * each site are recorded as usual, but the matmuls that consume the site take
 * the given rows (tr_fq / tr_fs at the same offsets) instead.  A comparison
 * that first proves every difference between the given rows and the recorded
 * ones is a rounding tie can then follow the given rows through the rest of
 * the pass: the next site's values differ from the other side's only by f32
 * summation order. */
static __thread int8_t *tr_q;
static __thread float *tr_s, *tr_v;
static __thread size_t tr_nq, tr_cap;
static __thread const int8_t *tr_fq;
static __thread const float *tr_fs;
static __thread size_t tr_site_off;
static __thread int tr_site_forced;
/* K/V rows: the f16 rows this pass computed (and their f32 values) are
 * recorded per layer [K rows][V rows]; with tr_fkv set, the cache then holds
 * the given rows instead (the f16 write is a rounding point like the int8
 * sites). */
static __thread uint16_t *tr_kv_own;
static __thread float *tr_kv_val;
static __thread const uint16_t *tr_fkv;
static __thread size_t tr_kv_off, tr_kv_cap;

/* n rows of kv_dim K (or V) values just written at cache row `first` */
static void trace_kv(uint16_t *cache, size_t first, size_t kv_dim, const float *vals, size_t n) {
  if (!tr_kv_own || tr_kv_off + n * kv_dim > tr_kv_cap) return;
  memcpy(tr_kv_own + tr_kv_off, cache + first * kv_dim, n * kv_dim * sizeof(uint16_t));
  memcpy(tr_kv_val + tr_kv_off, vals, n * kv_dim * sizeof(float));
  if (tr_fkv) memcpy(cache + first * kv_dim, tr_fkv + tr_kv_off, n * kv_dim * sizeof(uint16_t));
  tr_kv_off += n * kv_dim;
}

static void trace_site(const float *x, size_t n) {
  tr_site_forced = 0;
  if (!tr_q || tr_nq + n > tr_cap) return;
  int32_t *sums = malloc(sizeof(int32_t) * (n / 32));
  or_quantize_acts(x, n, tr_q + tr_nq, tr_s + tr_nq / 32, sums);
  if (tr_v) memcpy(tr_v + tr_nq, x, n * sizeof(float));
  free(sums);
  tr_site_off = tr_nq;
  tr_site_forced = tr_fq != NULL;
  tr_nq += n;
}

/* n rows of k quantized values of the current site, taken from the forced rows */
static int forced_rows(size_t n, size_t k, const int8_t **q, const float **s, int32_t **sums) {
  if (!tr_site_forced) return 0;
  *q = tr_fq + tr_site_off;
  *s = tr_fs + tr_site_off / 32;
  size_t g = n * k / 32;
  *sums = malloc(sizeof(int32_t) * g);
  for (size_t i = 0; i < g; i++) {
    int32_t t = 0;
    for (int j = 0; j < 32; j++) t += (*q)[i * 32 + j];
    (*sums)[i] = t;
  }
  return 1;
}

/* infer.rs:142-211 forward_impl */
void or_forward(const or_model *m, or_kv *kv, uint32_t token, size_t pos, float *out_logits) {
  const or_config *c = &m->c;
  size_t dim = c->dim, hd = c->head_dim, q_dim = c->n_heads * hd, kv_dim = c->n_kv_heads * hd,
         hid = c->hidden_dim;
  float *x = malloc(sizeof(float) * dim), *xb = malloc(sizeof(float) * dim);
  float *q = malloc(sizeof(float) * q_dim), *k = malloc(sizeof(float) * kv_dim),
        *v = malloc(sizeof(float) * kv_dim), *att = malloc(sizeof(float) * q_dim),
        *o = malloc(sizeof(float) * dim), *g = malloc(sizeof(float) * hid),
        *u = malloc(sizeof(float) * hid), *dn = malloc(sizeof(float) * dim);
  emb_row(m, token, x);
  for (size_t l = 0; l < c->n_layers; l++) {
    layer *L = &m->layers[l];
    or_rmsnorm(x, L->rms_att, 1, dim, c->norm_eps, xb);
    trace_site(xb, dim);
    apply(m, &L->wq, xb, q);
    apply(m, &L->wk, xb, k);
    apply(m, &L->wv, xb, v);
    add_bias(q, L->bq, q_dim);
    add_bias(k, L->bk, kv_dim);
    add_bias(v, L->bv, kv_dim);
    rope_row(c, q, q_dim, pos);
    rope_row(c, k, kv_dim, pos);
    or_f16_kv_write(or_kv_layer(kv, (int)l, 0), pos, kv_dim, k, kv_dim);
    or_f16_kv_write(or_kv_layer(kv, (int)l, 1), pos, kv_dim, v, kv_dim);
    trace_kv(or_kv_layer(kv, (int)l, 0), pos, kv_dim, k, 1);
    trace_kv(or_kv_layer(kv, (int)l, 1), pos, kv_dim, v, 1);
    or_attention_decode(q, or_kv_layer(kv, (int)l, 0), or_kv_layer(kv, (int)l, 1), pos, c->n_heads,
                        c->n_kv_heads, hd, att);
    trace_site(att, q_dim);
    apply(m, &L->wo, att, o);
    for (size_t i = 0; i < dim; i++) x[i] += o[i];
    or_rmsnorm(x, L->rms_ffn, 1, dim, c->norm_eps, xb);
    trace_site(xb, dim);
    apply(m, &L->w1, xb, g);
    apply(m, &L->w3, xb, u);
    or_silu(g, hid);
    for (size_t i = 0; i < hid; i++) g[i] *= u[i];
    trace_site(g, hid);
    apply(m, &L->w2, g, dn);
    for (size_t i = 0; i < dim; i++) x[i] += dn[i];
  }
  if (out_logits) {
    or_rmsnorm(x, m->rms_final, 1, dim, c->norm_eps, xb);
    trace_site(xb, dim);
    logits(m, xb, out_logits);
  }
  free(x); free(xb); free(q); free(k); free(v); free(att); free(o); free(g); free(u); free(dn);
}

static void trace_kv_begin(uint16_t *own, float *val, const uint16_t *fkv, size_t cap) {
  tr_kv_own = own;
  tr_kv_val = val;
  tr_fkv = fkv;
  tr_kv_off = 0;
  tr_kv_cap = cap;
}
static void trace_begin(int8_t *q, float *s, float *vals, size_t cap, const int8_t *fq, const float *fs) {
  tr_q = q;
  tr_s = s;
  tr_v = vals;
  tr_nq = 0;
  tr_cap = cap;
  tr_fq = fq;
  tr_fs = fs;
  tr_site_forced = 0;
}
static size_t trace_end(void) {
  size_t n = tr_nq;
  tr_kv_own = NULL;
  tr_kv_val = NULL;
  tr_fkv = NULL;
  tr_q = NULL;
  tr_s = NULL;
  tr_v = NULL;
  tr_fq = NULL;
  tr_fs = NULL;
  tr_site_forced = 0;
  return n;
}

size_t or_forward_trace(const or_model *m, or_kv *kv, uint32_t token, size_t pos, float *logits, int8_t *q,
                        float *s, float *vals, size_t cap) {
  trace_begin(q, s, vals, cap, NULL, NULL);
  or_forward(m, kv, token, pos, logits);
  return trace_end();
}

size_t or_forward_trace_forced(const or_model *m, or_kv *kv, uint32_t token, size_t pos, float *logits,
                               int8_t *q, float *s, float *vals, size_t cap, const int8_t *fq, const float *fs,
                               uint16_t *kv_own, float *kv_val, const uint16_t *fkv, size_t kv_cap) {
  trace_begin(q, s, vals, cap, fq, fs);
  trace_kv_begin(kv_own, kv_val, fkv, kv_cap);
  or_forward(m, kv, token, pos, logits);
  return trace_end();
}

/* Linear::apply_prefill (checkpoint.rs:140-146) for n rows */
static void apply_prefill(const or_model *m, const or_matrix *w, const float *xs, size_t n, float *y) {
  if (w->kind == OR_GGML_F32) {
    or_matmul(m->tier, w, xs, n, y);
    return;
  }
  const int8_t *fq;
  const float *fs;
  int32_t *fsum;
  if (forced_rows(n, w->cols, &fq, &fs, &fsum)) {
    or_matmul_prefill(m->tier, w, fq, fs, fsum, n, y);
    free(fsum);
    return;
  }
  size_t k = w->cols, g = k / 32;
  int8_t *aq = malloc(n * k);
  float *as = malloc(sizeof(float) * n * g);
  int32_t *asum = malloc(sizeof(int32_t) * n * g);
  for (size_t t = 0; t < n; t++) or_quantize_acts(xs + t * k, k, aq + t * k, as + t * g, asum + t * g);
  or_matmul_prefill(m->tier, w, aq, as, asum, n, y);
  free(aq);
  free(as);
  free(asum);
}

/* Shared body of prefill (infer.rs:220-286) and forward_batch (:296-374).
 * verify == 0: positions 0..n, f32 in-window attention, no logits.
 * verify == 1: positions pos0.., attention over the f16 cache, logits [n][vocab]. */
static void batch_body(const or_model *m, or_kv *kv, const uint32_t *toks, size_t n, size_t pos0,
                       int verify, float *out_logits) {
  const or_config *c = &m->c;
  size_t dim = c->dim, hd = c->head_dim, q_dim = c->n_heads * hd, kv_dim = c->n_kv_heads * hd,
         hid = c->hidden_dim;
  float *x = malloc(sizeof(float) * n * dim), *xb = malloc(sizeof(float) * n * dim);
  float *q = malloc(sizeof(float) * n * q_dim), *k = malloc(sizeof(float) * n * kv_dim),
        *v = malloc(sizeof(float) * n * kv_dim), *att = malloc(sizeof(float) * n * q_dim),
        *o = malloc(sizeof(float) * n * dim), *g = malloc(sizeof(float) * n * hid),
        *u = malloc(sizeof(float) * n * hid), *dn = malloc(sizeof(float) * n * dim);
  for (size_t t = 0; t < n; t++) emb_row(m, toks[t], x + t * dim);
  for (size_t l = 0; l < c->n_layers; l++) {
    layer *L = &m->layers[l];
    or_rmsnorm(x, L->rms_att, n, dim, c->norm_eps, xb);
    trace_site(xb, n * dim);
    apply_prefill(m, &L->wq, xb, n, q);
    apply_prefill(m, &L->wk, xb, n, k);
    apply_prefill(m, &L->wv, xb, n, v);
    for (size_t t = 0; t < n; t++) {
      add_bias(q + t * q_dim, L->bq, q_dim);
      add_bias(k + t * kv_dim, L->bk, kv_dim);
      add_bias(v + t * kv_dim, L->bv, kv_dim);
      rope_row(c, q + t * q_dim, q_dim, pos0 + t);
      rope_row(c, k + t * kv_dim, kv_dim, pos0 + t);
    }
    uint16_t *kc = or_kv_layer(kv, (int)l, 0), *vc = or_kv_layer(kv, (int)l, 1);
    or_f16_kv_write(kc, pos0, kv_dim, k, n * kv_dim);
    or_f16_kv_write(vc, pos0, kv_dim, v, n * kv_dim);
    trace_kv(kc, pos0, kv_dim, k, n);
    trace_kv(vc, pos0, kv_dim, v, n);
    if (verify) or_attention_verify(q, kc, vc, pos0, n, c->n_heads, c->n_kv_heads, hd, att);
    else or_attention(q, k, v, n, c->n_heads, c->n_kv_heads, hd, att);
    trace_site(att, n * q_dim);
    apply_prefill(m, &L->wo, att, n, o);
    for (size_t i = 0; i < n * dim; i++) x[i] += o[i];
    or_rmsnorm(x, L->rms_ffn, n, dim, c->norm_eps, xb);
    trace_site(xb, n * dim);
    apply_prefill(m, &L->w1, xb, n, g);
    apply_prefill(m, &L->w3, xb, n, u);
    or_silu(g, n * hid);
    for (size_t i = 0; i < n * hid; i++) g[i] *= u[i];
    trace_site(g, n * hid);
    apply_prefill(m, &L->w2, g, n, dn);
    for (size_t i = 0; i < n * dim; i++) x[i] += dn[i];
  }
  if (verify && out_logits) {
    /* Model::logits_batch (checkpoint.rs:256-265) */
    or_rmsnorm(x, m->rms_final, n, dim, c->norm_eps, xb);
    trace_site(xb, n * dim);
    apply_prefill(m, m->has_wcls ? &m->wcls : &m->emb, xb, n, out_logits);
  }
  free(x); free(xb); free(q); free(k); free(v); free(att); free(o); free(g); free(u); free(dn);
}

void or_prefill(const or_model *m, or_kv *kv, const uint32_t *tokens, size_t n) {
  batch_body(m, kv, tokens, n, 0, 0, NULL);
}

void or_forward_batch(const or_model *m, or_kv *kv, const uint32_t *tokens, size_t n, size_t pos0,
                      float *logits_out) {
  batch_body(m, kv, tokens, n, pos0, 1, logits_out);
}

/* prefill (verify == 0, positions 0..n) or forward_batch (verify == 1) with
 * the activation trace of or_forward_trace_forced: per layer the n rows of
 * each site, then the final-norm rows (verify only); fq / fs (or NULL) force
 * the rows the matmuls take. */
size_t or_batch_trace(const or_model *m, or_kv *kv, const uint32_t *tokens, size_t n, size_t pos0, int verify,
                      float *logits_out, int8_t *q, float *s, float *vals, size_t cap, const int8_t *fq,
                      const float *fs, uint16_t *kv_own, float *kv_val, const uint16_t *fkv, size_t kv_cap) {
  trace_begin(q, s, vals, cap, fq, fs);
  trace_kv_begin(kv_own, kv_val, fkv, kv_cap);
  batch_body(m, kv, tokens, n, verify ? pos0 : 0, verify, logits_out);
  return trace_end();
}

/* infer.rs:696-771 generate, greedy, over ids */
size_t or_generate_sampled(const or_model *m, const uint32_t *prompt, size_t p, size_t steps, int64_t stop_id,
                           float temp, uint64_t *state, uint32_t *out) {
  if (p == 0) return 0;
  if (*state == 0) *state = 1; /* XorShift::new: seed.max(1) */
  size_t max_pos = m->c.seq_len < p + steps ? m->c.seq_len : p + steps;
  or_kv *kv = or_kv_create(m, max_pos);
  float *lg = malloc(sizeof(float) * m->c.vocab_size);
  uint32_t token = prompt[0];
  size_t generated = 0, start = 0;
  if (p > 1 && p <= max_pos) {
    or_prefill(m, kv, prompt, p - 1);
    start = p - 1;
    token = prompt[p - 1];
  }
  for (size_t pos = start; pos < max_pos; pos++) {
    int need = pos + 1 >= p && pos + 1 < max_pos;
    or_forward(m, kv, token, pos, need ? lg : NULL);
    if (pos + 1 >= max_pos) break;
    uint32_t next = pos + 1 < p ? prompt[pos + 1] : or_sample(lg, m->c.vocab_size, temp, state, NULL, NULL);
    if (pos + 1 >= p) {
      if (stop_id >= 0 && next == (uint32_t)stop_id) break;
      out[generated++] = next;
    }
    token = next;
  }
  free(lg);
  or_kv_free(kv);
  return generated;
}

size_t or_generate(const or_model *m, const uint32_t *prompt, size_t p, size_t steps, int64_t stop_id,
                   uint32_t *out) {
  uint64_t state = 1;
  return or_generate_sampled(m, prompt, p, steps, stop_id, 0.0f, &state, out);
}

/* infer.rs:581-690 generate_speculative */
size_t or_generate_speculative(const or_model *target, const or_model *draft, const uint32_t *prompt,
                               size_t p, size_t steps, size_t k, int64_t stop_id, uint32_t *out,
                               size_t *stats) {
  if (p == 0 || k == 0 || target->c.vocab_size != draft->c.vocab_size) return 0;
  size_t V = target->c.vocab_size;
  size_t max_pos = target->c.seq_len < p + steps ? target->c.seq_len : p + steps;
  or_kv *tc = or_kv_create(target, max_pos), *dc = or_kv_create(draft, max_pos);
  if (p > 1) {
    or_prefill(target, tc, prompt, p - 1);
    or_prefill(draft, dc, prompt, p - 1);
  }
  size_t pos = p - 1, generated = 0, proposed = 0, accepted = 0;
  uint32_t last = prompt[p - 1];
  float *dl = malloc(sizeof(float) * V);
  float *tl = malloc(sizeof(float) * V * (k + 1));
  uint32_t *drafts = malloc(sizeof(uint32_t) * k), *inputs = malloc(sizeof(uint32_t) * (k + 1));
  while (pos + 1 < max_pos) {
    size_t budget = max_pos - 1 - pos < k ? max_pos - 1 - pos : k;
    uint32_t d = last;
    for (size_t j = 0; j < budget; j++) {
      or_forward(draft, dc, d, pos + j, dl);
      d = or_argmax(dl, V);
      drafts[j] = d;
    }
    proposed += budget;
    inputs[0] = last;
    memcpy(inputs + 1, drafts, budget * sizeof(uint32_t));
    or_forward_batch(target, tc, inputs, budget + 1, pos, tl);
    int stop = 0;
    for (size_t i = 0; i <= budget; i++) {
      uint32_t tn = or_argmax(tl + i * V, V);
      if (i < budget && tn == drafts[i]) accepted++;
      if (stop_id >= 0 && tn == (uint32_t)stop_id) { stop = 1; break; }
      out[generated++] = tn;
      pos++;
      last = tn;
      if (generated >= steps || pos + 1 >= max_pos) { stop = 1; break; }
      if (i == budget || tn != drafts[i]) break;
    }
    if (stop) break;
  }
  if (stats) {
    stats[0] = proposed;
    stats[1] = accepted;
  }
  free(dl); free(tl); free(drafts); free(inputs);
  or_kv_free(tc);
  or_kv_free(dc);
  return generated;
}
