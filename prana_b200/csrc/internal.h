// internal.h -- argument blocks and launcher entry points shared between the
// kernel translation units and the host engine.  Not part of the public ABI.
#pragma once
#include <cuda.h>
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

// One sequence of a decode-attention launch over several independent
// sequences (blockIdx.z): its cache views, position and split scratch.
struct AttnSeq {
  CUtensorMap tm_k;  // first: 64-byte aligned in the device array
  CUtensorMap tm_v;
  const __half* kc;
  const __half* vc;
  float* part_ml;
  float* part_o;
  unsigned* counters;
  int pos0;
};

struct AttnArgs {
  // TMA views of this layer's K and V cache ({hd, n_kv, positions}, 128-byte
  // swizzled boxes of 64 x 1 x 128); has_tm = 0 when they could not be made
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  int has_tm;
  const float* q;        // [m][n_heads*hd]
  const __half* kc;      // [positions][n_kv*hd]
  const __half* vc;
  int m;                 // query rows; row i sits at position pos0 + i
  int pos0;
  const int* pos_dev;    // overrides pos0 when non-null
  int n_heads, n_kv, hd;
  int n_splits;
  float* part_ml;        // [n_kv][n_splits][m*group][2]
  float* part_o;         // [n_kv][n_splits][m*group][hd], 16-byte aligned
  unsigned* counters;    // [n_kv], zero between launches
  float* out;            // [m][n_heads*hd]
  unsigned* err;         // device error flag for bounded waits (nullable)
  int cap;               // positions the cache holds (0: pos0 + m); sizes the launch, not the work
  int tail_merge;        // tcgen05 attention: the last split CTA merges (else a merge kernel follows)
  // non-null: gridDim.z sequences, sequence z = seqs[z] (one query row each,
  // at q / out row z); seqs replaces tm_*, kc, vc, pos0, part_*, counters
  const AttnSeq* seqs;
};

struct PrefillAttnArgs {
  const float* q;  // [n][n_heads*hd]
  const float* k;  // [n][n_kv*hd]
  const float* v;
  int n, n_heads, n_kv, hd;
  float* out;
};

// ---------------------------------------------------------------- streaming GEMV (decode.cu)
enum : int { EPI_QKV = 3, EPI_SWIGLU = 4 };

// Q|K|V epilogue: the stored matrix concatenates projections of one weight
// type; RoPE partners are adjacent stored rows (NeoX rows permuted at upload).
// One independent sequence of a multi-sequence decode pass: its KV cache
// (layer-0 base and per-layer stride, in halves), capacity and position.
struct SeqRow {
  __half* k;
  __half* v;
  size_t lstride;
  int pos;
  int cap;
};

struct QkvMap {
  int nseg;
  int seg_start[4];  // stored-row offsets of each projection (+ end)
  int kind[3];       // 0 = q, 1 = k, 2 = v
  const float* bias[3];
  int hd, neox, q_dim, kv_dim;
  const float* cos_t;
  const float* sin_t;
  int pos0;
  const int* pos_dev;
  int cap;
  float* q_out;
  __half* kc;
  __half* vc;
  float* k_f32;
  float* v_f32;
  const SeqRow* rows;  // non-null: activation row m belongs to sequence rows[m] (cache, position)
  int layer;           // with rows: the layer whose cache rows are written
};

struct StreamArgs {
  DevWeight w;
  int K, N, m;
  int ks;  // warps per row group (K split), set by the launcher
  const int8_t* aq;  // PRO_Q: quantized activation rows [m][K] (+ scales, sums [m][K/32])
  const float* as;
  const int32_t* asum;
  const float* x;       // PRO_F32 / PRO_NORM: f32 rows [m][K]
  const float* norm_w;  // PRO_NORM: rmsnorm weight [K]
  float eps;
  int8_t* trace_q;      // diagnostic: CTA 0 copies the staged rows here
  float* trace_s;
  float* out;          // STORE / RESID / ARGMAX logits [m][N]; SWIGLU h [m][N/2]
  const float* bias;   // STORE
  unsigned* err;       // device error flag
  // ARGMAX
  float* part_val;
  int* part_idx;
  int n_parts;
  uint32_t* token_out;
  int* token_next;
  // last-CTA argmax merge; the counter is zero between launches
  unsigned* counter;
  int idx_offset;      // ARGMAX: global index of this matrix's row 0 (vocab shard start)
  float* best_val;     // ARGMAX: the maximum itself per activation row (nullable)
  QkvMap qkv;
  // rows [0, pf_rows) of the next kernel's weights are prefetched toward L2 by
  // warps that have finished their own rows (pf_rows == 0: none)
  DevWeight pf_w;
  int pf_rows;
};

cudaError_t launch_stream(const StreamArgs& g, int epi, int pro, cudaStream_t st, bool pdl);
// Batch path around the tensor-core GEMM: rows (rmsnorm'd when w is set, then)
// quantized once per projection; the EPI_QKV / EPI_SWIGLU arithmetic over
// rows the GEMM stored ([n][N] f32).
cudaError_t launch_norm_quant(const float* x, const float* w, float eps, int rows, int K, int8_t* q, float* s,
                              int32_t* sum, cudaStream_t st);
cudaError_t launch_qkv_finish(const float* y, int n, int N, const QkvMap& qm, cudaStream_t st);
cudaError_t launch_swiglu_finish(const float* y, int n, int N, float* h, cudaStream_t st);
int gemv_split_k(int type, int K, int N, int sm_count);
size_t gemv_smem_bytes(int M, int K, int pro);

cudaError_t launch_gemv(const GemvArgs& g, int pro, int epi, cudaStream_t st, bool pdl);
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
// Sampler state the device advances: the xorshift64* word and the temperature
struct SampleState {
  unsigned long long rng;
  float temp;
  int pad;
};
// Sampler::sample over one row of n logits (temperature > 0 or NaN): one draw
// from *state (advanced), the token to tok_out[0] and, when set, *tok_next
cudaError_t launch_sample(const float* logits, int n, SampleState* state, uint32_t* tok_out, int* tok_next,
                          cudaStream_t st);
int sample_max_vocab();
cudaError_t launch_block_dots(const DevWeight& w, int row, const int8_t* aq, const int32_t* asum, int32_t* out,
                              cudaStream_t st);
cudaError_t launch_advance(int* tok, int* pos, uint32_t* ring, int ring_cap, int* ring_n, cudaStream_t st, bool pdl);
// diagnostic: one bounded mbarrier wait that nothing completes (raises *err)
cudaError_t launch_wait_never(unsigned polls, unsigned* err, cudaStream_t st);
// first maximum over ranks: all = [world][16] (8 best values, then 8 index bit patterns)
cudaError_t launch_tp_argmax(const float* all, int world, int m, uint32_t* tok_out, int* tok_next, cudaStream_t st);

// ---------------------------------------------------------------- tensor-core GEMM (qgemm.cu)
struct QgemmArgs {
  DevWeight w;
  int N, K, M;          // weight rows, columns; activation rows
  int m_pad;            // set by the launcher
  float* out;           // [M][N] (null with dots)
  const float* bias;    // [N] added to every row (nullable)
  int resid;            // 1: out += result
  int32_t* dots;        // diagnostic: per-block int32 [M][N][K/32 (x2 for Q6_K)] instead of out
  unsigned* err;        // device error flag
  int splits;           // set by the launcher: K splits (partials in `part`, summed in split order)
  float* part;
};
// out = W . rows (q [M][K] int8, s / sums [M][K/32]); scratch >= qgemm_scratch_bytes
cudaError_t launch_qgemm(QgemmArgs g, const int8_t* q, const float* s, const int32_t* sums, void* scratch,
                         cudaStream_t st);
size_t qgemm_scratch_bytes(int m, int k);
int qgemm_tokens_per_tile(int m);

// attention.cu
int attn_max_rows_per_cta(int hd);
// attention splits for a cache of `positions` rows (scratch is sized by it)
int attn_splits(int positions, int n_kv, int hd, int sm_count);
// Fill a.tm_k / a.tm_v for caches of `positions` rows (a.kc, a.vc, a.n_kv,
// a.hd set); leaves has_tm = 0 for head sizes the TMA kernel does not take.
void attn_make_maps(AttnArgs& a, int positions);
cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl);
// a.seqs set, a.m == 1: n_seq sequences in one launch (head dims 64 / 128 with
// tensor maps); cudaErrorNotSupported when the shape needs per-sequence launches
cudaError_t launch_attn_decode_seqs(const AttnArgs& a, int n_seq, cudaStream_t st, bool pdl);
cudaError_t launch_attn_prefill(const PrefillAttnArgs& a, cudaStream_t st);

}  // namespace prana
