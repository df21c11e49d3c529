/*
 * synth.h -- seeded random-init GGUF model / quantized-matrix generator.
 * Host-only C; see synth.c for the distributions and encoders.
 */
#ifndef PRANA_SYNTH_H
#define PRANA_SYNTH_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ggml tensor types (same ids as GGUF) */
enum { SYNTH_F32 = 0, SYNTH_F16 = 1, SYNTH_Q4_0 = 2, SYNTH_Q8_0 = 8, SYNTH_Q4_K = 12, SYNTH_Q6_K = 14 };

typedef struct synth_model {
  char arch[16]; /* "llama" (interleaved RoPE) or "qwen2" (NeoX RoPE, biases) */
  int dim, hidden, n_layers, n_heads, n_kv_heads, head_dim, vocab, ctx;
  float rope_theta;
  float eps; /* <= 0: key omitted (loader default 1e-5) */
  int has_bias, tied;
  int type_embd, type_q, type_k, type_v, type_o, type_gate, type_up, type_down, type_output;
  uint64_t seed;
  float std;           /* weight standard deviation (0.02) */
  float out_proj_mult; /* std multiplier for attn_output / ffn_down (1.0) */
  float embd_std_mult; /* std multiplier for token_embd (1.0) */
  float head_std_mult; /* std multiplier for output.weight (1.0) */
  /* Shared-code construction (code_rank > 0): every model built with the same
   * code_seed and vocab shares a token code c_t ~ N(0, 1)^code_rank.  Row t of
   * token_embd is P c_t and row j of output.weight is P c_{s(j)}, with P a
   * [dim, code_rank] N(0, 1/code_rank) projection of this model's own seed and
   * s the inverse of the successor map succ(t) = (48271 t + 12345) mod vocab:
   * head . norm(emb(t)) then peaks at succ(t) in every such model.  On top,
   * this model's own N(0, code_noise) noise on both tables decides how often
   * two models pick different tokens.  The output table is written even when
   * `tied` is set (the tables then stay separate). */
  int code_rank;
  uint64_t code_seed;
  float code_noise;
} synth_model;

/* N(0, std) f32 values of row `row` of tensor `tensor` under `seed` */
void synth_normal_row(uint64_t seed, uint64_t tensor, uint64_t row, size_t n, float std, float *out);
/* bytes of one encoded row; 0 if `cols` does not fit the block size */
size_t synth_row_bytes(int type, size_t cols);
/* encode one f32 row into GGUF block bytes */
int synth_encode_row(int type, const float *x, size_t cols, uint8_t *out);
/* generate + encode a whole [rows, cols] tensor (std == 0: every value = constant) */
int synth_tensor(int type, size_t rows, size_t cols, uint64_t seed, uint64_t tensor, float std,
                 float constant, int threads, uint8_t *out);
/* write a complete GGUF v3 model file */
int synth_write_gguf(const synth_model *cfg, const char *path, int threads);

#ifdef __cplusplus
}
#endif
#endif
