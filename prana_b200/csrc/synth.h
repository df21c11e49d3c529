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
