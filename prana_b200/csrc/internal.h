// internal.h -- argument blocks and launcher entry points shared between the
// kernel translation units and the host engine.  Not part of the public ABI.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace prana {

// GEMV prologues: how the activation rows reach shared memory.
enum : int { PRO_Q = 0, PRO_F32 = 1, PRO_NORM = 2 };
// GEMV epilogues.
enum : int { EPI_STORE = 0, EPI_RESID = 1, EPI_ARGMAX = 2 };

struct GemvArgs {
  DevWeight w;
  int m;  // activation rows, 1..8
  // PRO_Q: pre-quantized rows
  const int8_t* aq;
  const float* as;
  const int32_t* asum;
  // PRO_F32 / PRO_NORM: f32 rows [m][K]; PRO_NORM adds the rmsnorm weight
  const float* x;
  const float* norm_w;
  float eps;
  // EPI_STORE/RESID: out [m][N]; EPI_ARGMAX: logits [m][N] (nullable)
  float* out;
  const float* bias;
  // EPI_ARGMAX scratch: per-CTA partials [m][n_parts], a zeroed ticket counter,
  // the argmax per row, and (optionally) the next-step token slot
  float* part_val;
  int* part_idx;
  unsigned* counter;
  int n_parts;
  uint32_t* token_out;
  int* token_next;
  // diagnostic trace: when set, CTA 0 copies the staged activation rows here
  int8_t* trace_q;  // [m][K]
  float* trace_s;   // [m][K/32]
};

struct QkvArgs {
  GemvArgs a;          // prologue inputs (m, x, norm_w, eps or aq/as/asum)
  DevWeight w[3];
  int kind[3];         // 0 = q, 1 = k, 2 = v
  const float* bias[3];
  int nseg;
  int pair_start[4];   // prefix sums of row-pairs per segment
  int hd, neox, q_dim, kv_dim;
  const float* cos_t;  // [positions][hd/2]
  const float* sin_t;
  int pos0;            // first position (used when pos_dev is null)
  const int* pos_dev;
  int cap;             // cache rows; positions >= cap are not written
  float* q_out;        // [m][q_dim]
  __half* kc;          // layer K cache [positions][kv_dim]
  __half* vc;
  float* k_f32;        // optional in-window f32 copies [m][kv_dim] (prefill attention)
  float* v_f32;
};

struct SwigluArgs {
  GemvArgs a;
  DevWeight w1, w3;  // gate, up: [hidden][dim]
  int8_t* hq;        // quantized silu(gate)*up [m][hidden]
  float* hs;         // [m][hidden/32]
  int32_t* hsum;
  float* h_f32;      // optional f32 copy [m][hidden]
};

struct AttnArgs {
  const float* q;        // [m][n_heads*hd]
  const __half* kc;      // [positions][n_kv*hd]
  const __half* vc;
  int m;                 // query rows; row i sits at position pos0 + i
  int pos0;
  const int* pos_dev;    // overrides pos0 when non-null
  int n_heads, n_kv, hd;
  int n_splits;
  float* part_ml;        // [n_kv][n_splits][m*group][2]
  float* part_o;         // [n_kv][n_splits][m*group][hd]
  unsigned* counters;    // [n_kv], zero between launches
  float* out;            // [m][n_heads*hd]
};

struct PrefillAttnArgs {
  const float* q;  // [n][n_heads*hd]
  const float* k;  // [n][n_kv*hd]
  const float* v;
  int n, n_heads, n_kv, hd;
  float* out;
};

cudaError_t launch_gemv(const GemvArgs& g, int pro, int epi, cudaStream_t st, bool pdl);
cudaError_t launch_qkv(const QkvArgs& g, int pro, cudaStream_t st, bool pdl);
cudaError_t launch_swiglu(const SwigluArgs& g, int pro, cudaStream_t st, bool pdl);
cudaError_t launch_quantize_acts(const float* x, int rows, int k, int8_t* q, float* s, int32_t* sum, cudaStream_t st);
cudaError_t launch_rmsnorm(const float* x, const float* w, int rows, int dim, float eps, float* out, cudaStream_t st);
cudaError_t launch_rope(float* x, int rows, int n, int pos0, int hd, int neox, const float* c, const float* s,
                        cudaStream_t st);
cudaError_t launch_silu(float* x, size_t n, cudaStream_t st);
cudaError_t launch_silu_mul(float* g, const float* u, size_t n, cudaStream_t st);
cudaError_t launch_softmax(const float* x, int rows, int n, float* out, cudaStream_t st);
cudaError_t launch_kv_write(__half* cache, size_t start, const float* src, size_t n, cudaStream_t st);
cudaError_t launch_embed(const DevWeight& w, const uint32_t* toks, const int* tok_single, int m, float* x,
                         cudaStream_t st, bool pdl);
cudaError_t launch_argmax(const float* x, int rows, int n, uint32_t* out, cudaStream_t st);
cudaError_t launch_block_dots(const DevWeight& w, int row, const int8_t* aq, const int32_t* asum, int32_t* out,
                              cudaStream_t st);
cudaError_t launch_advance(int* tok, int* pos, uint32_t* ring, int ring_cap, int* ring_n, cudaStream_t st, bool pdl);

// attention.cu
int attn_max_rows_per_cta(int hd);
cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl);
cudaError_t launch_attn_prefill(const PrefillAttnArgs& a, cudaStream_t st);

}  // namespace prana
