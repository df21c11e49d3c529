/*
 * prana_oracle.h -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A plain-C restatement of Prana's CPU decode path (the `prana-kernels` and
 * `prana-model` Rust crates).  It is the parity checker for the CUDA library
 * and the timed CPU baseline.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it; the product (prana_b200/) never
 * links, imports or calls anything here.
 *
 * Every function cites the reference file:line it restates (paths relative
 * to the Prana workspace root).  Numerics follow the reference exactly:
 * no FMA contraction (built with -ffp-contract=off), sequential f32 sums in
 * the scalar tier, Rust `round` == C `roundf` (half away from zero), IEEE
 * divides, argmax ties to the lowest index.
 */
#ifndef PRANA_ORACLE_H
#define PRANA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- block-format constants: crates/prana-kernels/src/kquant.rs:25-36, matmul.rs:12 ---- */
#define OR_Q8_BLOCK 32
#define OR_QK_K 256
#define OR_Q4_0_BLOCK_BYTES 18
#define OR_Q4_K_BLOCK_BYTES 144
#define OR_Q6_K_BLOCK_BYTES 210
#define OR_Q8_0_BLOCK_BYTES 34

/* ggml type ids: crates/prana-model/src/gguf.rs:33-38 */
#define OR_GGML_F32 0
#define OR_GGML_F16 1
#define OR_GGML_Q4_0 2
#define OR_GGML_Q8_0 8
#define OR_GGML_Q4_K 12
#define OR_GGML_Q6_K 14

/* SIMD tier selection for the dot products (simd_x86.rs:18-29). */
enum { OR_TIER_AUTO = 0, OR_TIER_SCALAR = 1, OR_TIER_AVX2 = 2, OR_TIER_VNNI = 3 };

/* ---- f16 (lib.rs:57-113) ---- */
float or_f16_to_f32(uint16_t h);
/* inline form used by the attention loops (the Rust version inlines too) */
static inline float or_f16_to_f32_inline(uint16_t h) {
  uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1fu, frac = h & 0x3ffu, bits;
  if (exp == 0 && frac == 0) {
    bits = sign << 31;
  } else if (exp == 0) {
    float v = (float)frac * 5.9604644775390625e-08f; /* frac * 2^-24, exact */
    return sign ? -v : v;
  } else if (exp == 0x1f) {
    bits = (sign << 31) | 0x7f800000u | (frac << 13);
  } else {
    bits = (sign << 31) | ((exp + 127 - 15) << 23) | (frac << 13);
  }
  union { uint32_t u; float f; } cv = {bits};
  return cv.f;
}
uint16_t or_f32_to_f16(float x);

/* ---- activation / weight quantization (matmul.rs:61-127) ---- */
void or_quantize_acts(const float *a, size_t k, int8_t *q, float *scales, int32_t *sums);
void or_quantize_q8(size_t rows, size_t cols, const float *w, int8_t *q, float *scales);

/* ---- block dequant (kquant.rs:39-112) ---- */
void or_dequant_q40_block(const uint8_t *b, float *out32);
void or_q4k_scale_min(int j, const uint8_t *s, float *sc, float *m);
void or_dequant_q4k_block(const uint8_t *b, float *out256);
void or_dequant_q6k_block(const uint8_t *b, float *out256);

/* ---- row dots; `tier` as above (matmul.rs:364-406, kquant.rs:240-363, simd_x86.rs) ---- */
float or_dot_q8_q8(int tier, const int8_t *aq, const float *as, size_t k,
                   const int8_t *wq, const float *ws);
float or_dot_q40_q8(int tier, const int8_t *aq, const float *as, const int32_t *asum,
                    size_t k, const uint8_t *row, const float *ds);
float or_dot_q4k_q8(int tier, const int8_t *aq, const float *as, const int32_t *asum,
                    size_t k, const uint8_t *row, const float *ds);
float or_dot_q6k_q8(const int8_t *aq, const float *as, size_t k,
                    const uint8_t *row, const float *ds);
float or_dot_f32(int tier, const float *a, const float *b, size_t n);
/* per-block integer dots (the bit-exact part) for one packed row */
void or_block_dots(int ggml_type, const int8_t *aq, size_t k, const uint8_t *row,
                   int32_t *out /* one per 32-group, or per 16-sub for Q6_K */);

int or_simd_available(void);
int or_vnni_available(void);
int or_default_tier(void);

/* ---- pool (pool.rs, threading.rs:46-53) ---- */
int or_pool_threads(void);
void or_pool_set_threads(int n); /* must be called before first use */

/* ---- matrices (matmul.rs:21-57, kquant.rs:116-233) ---- */
typedef struct or_matrix {
  int kind;          /* OR_GGML_F32, OR_GGML_Q8_0 (int8 + f32 scales), Q4_0, Q4_K, Q6_K */
  size_t rows, cols;
  float *f32;        /* F32: rows*cols */
  int8_t *q;         /* Q8: rows*cols */
  float *scales;     /* Q8: rows*cols/32 (f32) ; K-quants: hoisted dscales */
  uint8_t *blocks;   /* K-quants: raw GGUF blocks */
} or_matrix;

/* raw GGUF bytes -> matrix (gguf.rs:271-305 mapping) */
int or_matrix_from_gguf(or_matrix *m, int ggml_type, size_t rows, size_t cols, const uint8_t *raw);
void or_matrix_free(or_matrix *m);
/* dense f32 dequantization of the whole matrix (tests) */
void or_matrix_dequant(const or_matrix *m, float *out);
void or_matrix_dequant_row(const or_matrix *m, size_t r, float *out);

/* y[t, r] for n_tokens rows of f32 activations (matmul_q8_f32 / matmul_kquant_f32 /
 * matmul_f32): activations quantized per token (matmul.rs:162-178, kquant.rs:323-333). */
void or_matmul(int tier, const or_matrix *m, const float *a, size_t n_tokens, float *out);
/* row-outer batched variant over already-quantized activation rows
 * (matmul_q8_prefill / matmul_kquant_prefill, matmul.rs:185-232, kquant.rs:368-370). */
void or_matmul_prefill(int tier, const or_matrix *m, const int8_t *aq, const float *as,
                       const int32_t *asum, size_t n_tokens, float *out);

/* ---- norms / activations (norms.rs:9-56) ---- */
void or_rmsnorm(const float *x, const float *w, size_t rows, size_t dim, float eps, float *out);
void or_silu(float *x, size_t n);
void or_softmax(const float *x, size_t n, float *out);

/* ---- rope / kv / attention (attention.rs) ---- */
void or_rope_interleaved(float *x, size_t n, size_t pos, size_t head_dim, float theta);
void or_rope_neox(float *x, size_t n, size_t pos, size_t head_dim, float theta);
void or_rope_batch(float *x, size_t seq, size_t n_heads, size_t head_dim, float theta);
void or_rope_table(size_t positions, size_t head_dim, float theta, int neox,
                   float *cos_out, float *sin_out); /* [positions][head_dim/2] */
void or_f16_kv_write(uint16_t *cache, size_t first_row, size_t kv_stride, const float *src, size_t n);
void or_attention_decode(const float *q, const uint16_t *kc, const uint16_t *vc, size_t pos,
                         size_t n_heads, size_t n_kv_heads, size_t head_dim, float *out);
void or_attention_verify(const float *q, const uint16_t *kc, const uint16_t *vc, size_t pos0,
                         size_t seq, size_t n_heads, size_t n_kv_heads, size_t head_dim, float *out);
void or_attention(const float *q, const float *k, const float *v, size_t seq, size_t n_heads,
                  size_t n_kv_heads, size_t head_dim, float *out);
uint32_t or_argmax(const float *x, size_t n);

/* ---- sampler (sampler.rs) ---- */
uint64_t or_xorshift_next(uint64_t *state);
float or_xorshift_f32(uint64_t *state);
/* Sampler::sample: argmax when temp <= 0; probs / r_out (may be NULL) receive
 * the softmax and the draw */
uint32_t or_sample(const float *logits, size_t n, float temp, uint64_t *state, float *probs, float *r_out);

/* ---- model (checkpoint.rs, gguf.rs:338-460, infer.rs) ---- */
typedef struct or_model or_model;
typedef struct or_config {
  size_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, head_dim;
  float rope_theta, norm_eps;
  int rope_neox, has_bias, shared_classifier;
} or_config;

or_model *or_model_load(const char *path, int tier, char *err, size_t errlen);
or_model *or_model_load_ex(const char *path, int tier, int precision, char *err, size_t errlen);
void or_model_free(or_model *m);
void or_model_config(const or_model *m, or_config *c);
const or_matrix *or_model_matrix(const or_model *m, int layer, const char *which);

typedef struct or_kv or_kv;
or_kv *or_kv_create(const or_model *m, size_t positions);
void or_kv_free(or_kv *kv);
uint16_t *or_kv_layer(or_kv *kv, int layer, int is_v); /* [positions][kv_dim] f16 bits */

/* forward one token; logits may be NULL (need_logits = false) (infer.rs:142-211) */
void or_forward(const or_model *m, or_kv *kv, uint32_t token, size_t pos, float *logits);
/* or_forward that also records every quantized activation row (per layer: attn-norm
 * input, attention output, ffn-norm input, silu(g)*u; then the final-norm input) */
size_t or_forward_trace(const or_model *m, or_kv *kv, uint32_t token, size_t pos, float *logits, int8_t *q,
                        float *s, float *vals /* f32 values quantized, may be NULL */, size_t cap);
/* Test instrumentation: or_forward_trace whose matmuls take the given rows
 * (fq / fs, may be NULL) and whose K/V cache rows become the given f16 rows
 * (fkv, may be NULL) after the pass's own rows and their f32 values are
 * recorded in kv_own / kv_val (per layer: K rows, then V rows). */
size_t or_forward_trace_forced(const or_model *m, or_kv *kv, uint32_t token, size_t pos, float *logits,
                               int8_t *q, float *s, float *vals, size_t cap, const int8_t *fq, const float *fs,
                               uint16_t *kv_own, float *kv_val, const uint16_t *fkv, size_t kv_cap);
/* prefill (verify == 0) or forward_batch (verify == 1) with the same trace and forcing */
size_t or_batch_trace(const or_model *m, or_kv *kv, const uint32_t *tokens, size_t n, size_t pos0, int verify,
                      float *logits_out, int8_t *q, float *s, float *vals, size_t cap, const int8_t *fq,
                      const float *fs, uint16_t *kv_own, float *kv_val, const uint16_t *fkv, size_t kv_cap);
/* batched prompt, no logits (infer.rs:220-286) */
void or_prefill(const or_model *m, or_kv *kv, const uint32_t *tokens, size_t n);
/* verify pass: logits [n][vocab] (infer.rs:296-374) */
void or_forward_batch(const or_model *m, or_kv *kv, const uint32_t *tokens, size_t n,
                      size_t pos0, float *logits);
/* greedy generate over token ids (infer.rs:696-771); returns generated count.
 * stop_id < 0 disables the stop check. */
size_t or_generate(const or_model *m, const uint32_t *prompt, size_t p, size_t steps,
                   int64_t stop_id, uint32_t *out_tokens);
/* generate with Sampler::new(temp, seed) (infer.rs:696-771, sampler.rs:13-37):
 * *state is the xorshift state (a zero seed reads as 1) and is left where the
 * last draw put it */
size_t or_generate_sampled(const or_model *m, const uint32_t *prompt, size_t p, size_t steps,
                           int64_t stop_id, float temp, uint64_t *state, uint32_t *out_tokens);
/* greedy speculative decode (infer.rs:581-690); stats[0]=proposed, stats[1]=accepted */
size_t or_generate_speculative(const or_model *target, const or_model *draft,
                               const uint32_t *prompt, size_t p, size_t steps, size_t k,
                               int64_t stop_id, uint32_t *out_tokens, size_t *stats);

#ifdef __cplusplus
}
#endif
#endif
