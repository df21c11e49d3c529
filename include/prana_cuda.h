/*
 * prana_cuda.h -- C ABI of the B200 (sm_100a) decode path for Prana.
 *
 * Plain pointers and sizes only.  Kernel-level entry points take DEVICE
 * pointers and run on the context's stream; model-level entry points take HOST
 * buffers for token ids and logits.  Every function returns 0 on success or a
 * negative PRANA_E_* code; prana_last_error() gives a message for the calling
 * thread (the null-on-failure / last-error convention of Prana's FFI layer,
 * crates/prana-cactus/src/mock.rs:8-12).  No exception crosses the ABI.
 *
 * Each kernel entry point names the prana-kernels / prana-model function it
 * replaces (file:line in the Prana workspace).  Calls on one context are not
 * thread-safe; calls on different contexts are.
 */
#ifndef PRANA_CUDA_H
#define PRANA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PRANA_OK 0
#define PRANA_E_INVALID -1     /* bad argument, shape or layout (the reference asserts) */
#define PRANA_E_CUDA -2        /* CUDA runtime / launch failure */
#define PRANA_E_OOM -3         /* device or host allocation failed */
#define PRANA_E_FORMAT -4      /* malformed GGUF (gguf.rs io::Error cases) */
#define PRANA_E_UNSUPPORTED -5 /* valid input outside what this build implements */
#define PRANA_E_TIMEOUT -6     /* a bounded device-side wait expired */
#define PRANA_E_COMM -7        /* collective / peer setup failed */

/* ggml tensor type ids (crates/prana-model/src/gguf.rs:33-38) */
#define PRANA_TYPE_F32 0
#define PRANA_TYPE_F16 1
#define PRANA_TYPE_Q4_0 2
#define PRANA_TYPE_Q8_0 8
#define PRANA_TYPE_Q4_K 12
#define PRANA_TYPE_Q6_K 14

typedef struct prana_ctx prana_ctx;
typedef struct prana_weight prana_weight;
typedef struct prana_model prana_model;
typedef struct prana_kv prana_kv;

const char *prana_last_error(void);
int prana_version(void);

/* ---------------------------------------------------------------- context */
int prana_ctx_create(int device, prana_ctx **out);
int prana_ctx_destroy(prana_ctx *ctx); /* idempotent on NULL */
/* run kernel-level calls on a caller-owned cudaStream_t (NULL = the context's own
 * stream; pass cudaStreamLegacy, 0x1, for the legacy default stream) */
int prana_ctx_set_stream(prana_ctx *ctx, void *cuda_stream);
/* Wait for the context's kernel-level calls; a bounded device wait that gave
 * up in one of them (including prana_attention_decode_noalloc on this device)
 * returns PRANA_E_TIMEOUT here, once, and the context stays usable. */
int prana_ctx_synchronize(prana_ctx *ctx);
/* the context's own stream (model-level work always runs there), for event timing */
int prana_ctx_stream(prana_ctx *ctx, void **cuda_stream);

/* Diagnostic, no reference counterpart: make one bounded device wait run out
 * on data that never arrives, and report it the way the kernel-level calls do.
 * which = 0: an mbarrier wait that no copy completes; which = 1: the peer
 * exchange's receive wait, run on this GPU alone with a second local buffer
 * standing in for a rank that never stores.  polls bounds the wait.  Returns
 * PRANA_E_TIMEOUT when the wait gave up (the expected outcome); no fault is
 * raised and the context stays usable. */
int prana_debug_wait_timeout(prana_ctx *ctx, int which, unsigned polls);

/* ---------------------------------------------------------------- device arena / buffer pool
 * BufferPool (crates/prana-tensor/src/pool.rs:13-103) with its storage in one
 * reservation: prana_pool_create makes the only allocator call (cudaMalloc of
 * `capacity` bytes on the context's device; ctx NULL: host memory, for
 * bookkeeping tests).  acquire rounds a request up to the reference's bucket
 * (a power of two, at least 1 KiB; requests above 64 MiB are carved at their
 * own 256-byte-aligned size), reuses a released buffer of that bucket or carves
 * a new one, and returns it zeroed (a device pool clears it on the context's
 * stream).  release returns a buffer to its bucket's list; clear hands every
 * listed buffer back to the arena (coalesced).  active / pooled / peak are the
 * reference's counters; carved is the arena space in use (checked out or
 * listed).  A full arena returns PRANA_E_OOM. */
typedef struct prana_pool prana_pool;
int prana_pool_create(prana_ctx *ctx, size_t capacity, prana_pool **out);
int prana_pool_destroy(prana_pool *pool); /* idempotent on NULL; the arena's buffers die with it */
int prana_pool_acquire(prana_pool *pool, size_t bytes, void **ptr, size_t *bucket_bytes);
int prana_pool_release(prana_pool *pool, void *ptr);
int prana_pool_clear(prana_pool *pool);
int prana_pool_stats(prana_pool *pool, size_t *active, size_t *pooled, size_t *peak, size_t *carved);
/* Every later device allocation of the context -- weights, models, KV caches,
 * activation buffers, kernel scratch -- comes from the pool (NULL: back to
 * cudaMalloc).  Switching first waits for the context's streams and returns
 * its kernel scratch and RoPE tables to where they came from.  Weights,
 * models and caches made while a pool was attached must be freed before it is
 * detached or destroyed. */
int prana_ctx_use_pool(prana_ctx *ctx, prana_pool *pool);

/* ---------------------------------------------------------------- weights
 * Upload one [rows, cols] tensor given in its GGUF byte layout and repack it
 * for 128-bit loads (replaces QuantMatrix::from_parts, matmul.rs:34-39, and
 * KQuantMatrix::from_raw, kquant.rs:166-183).  F16 tensors are widened to F32
 * (gguf.rs:208-267).  Q8_0/Q4_0 need cols % 32 == 0, Q4_K/Q6_K cols % 256 == 0. */
int prana_weight_upload(prana_ctx *ctx, int ggml_type, size_t rows, size_t cols, const void *host_bytes,
                        prana_weight **out);
/* quantize_q8 (matmul.rs:61-84), on the host: [rows, cols] f32 into int8 q
 * [rows * cols] and one f32 scale per 32 values (amax / 127, round half away
 * from zero, clamp to +-127).  No device is touched. */
int prana_quantize_q8(size_t rows, size_t cols, const float *w, int8_t *q, float *scales);
/* Linear::new(w, Precision::Q8) (checkpoint.rs): quantize_q8 of a host f32
 * [rows, cols] matrix, resident in HBM (int8 plane and f32 scales); it takes
 * prana_matmul_q8_f32 / prana_matmul_q8_prefill like a GGUF Q8_0 weight. */
int prana_weight_upload_q8(prana_ctx *ctx, size_t rows, size_t cols, const float *w, prana_weight **out);
int prana_weight_free(prana_weight *w);
/* device bytes the packed matrix occupies */
int prana_weight_bytes(const prana_weight *w, size_t *bytes);

/* ---------------------------------------------------------------- kernels (device pointers)
 * quantize_acts (matmul.rs:105-127): per 32-group int8, f32 scale, i32 sum; rows of k values. */
int prana_quantize_acts(prana_ctx *ctx, const float *x, size_t rows, size_t k, int8_t *q, float *scales,
                        int32_t *sums);
/* matmul_q8_f32 (matmul.rs:162-178) and matmul_kquant_f32 (kquant.rs:323-333):
 * out[t, r] = row r of W . quantize_acts(a[t]); a is [n_tokens, cols]. */
int prana_matmul_q8_f32(prana_ctx *ctx, const float *a, const prana_weight *w, size_t n_tokens, float *out);
int prana_matmul_kquant_f32(prana_ctx *ctx, const float *a, const prana_weight *w, size_t n_tokens, float *out);
/* matmul_q8_prefill (matmul.rs:185-187) / matmul_kquant_prefill (kquant.rs:368-370):
 * already-quantized activation rows; out [n_tokens, rows]. */
int prana_matmul_q8_prefill(prana_ctx *ctx, const int8_t *q, const float *scales, const int32_t *sums,
                            size_t n_tokens, const prana_weight *w, float *out);
int prana_matmul_kquant_prefill(prana_ctx *ctx, const int8_t *q, const float *scales, const int32_t *sums,
                                size_t n_tokens, const prana_weight *w, float *out);
/* The same products on the tensor cores (tcgen05 kind::i8, one MMA per
 * 32-value block -- 16 for Q6_K -- into a fresh TMEM accumulator, per-block
 * scales applied in f32): the path matmul_*_prefill takes above 8 rows,
 * callable at any row count.  q must be 16-byte aligned. */
int prana_qgemm(prana_ctx *ctx, const int8_t *q, const float *scales, const int32_t *sums, size_t n_tokens,
                const prana_weight *w, float *out);
/* Diagnostic: the per-block int32 dots the tensor cores produced, out
 * [n_tokens][rows][blocks] (blocks = cols/32, or cols/16 for Q6_K) -- the
 * quantities of dot_q8_q8_scalar / dot_q40_q8_scalar / dot_q4k_q8_scalar /
 * dot_q6k_q8_scalar (matmul.rs:395-406, kquant.rs:240-318). */
int prana_qgemm_block_dots(prana_ctx *ctx, const int8_t *q, const float *scales, const int32_t *sums,
                           size_t n_tokens, const prana_weight *w, int32_t *out);
/* matmul_f32 (matmul.rs:150-156) for F32 weights */
int prana_matmul_f32(prana_ctx *ctx, const float *a, const prana_weight *w, size_t n_tokens, float *out);
/* Per-block int32 dots of weight row `row` against one quantized activation row:
 * the bit-exact quantities of dot_q8_q8_scalar (matmul.rs:395-406), dot_q40_q8_scalar
 * (kquant.rs:240-252, value s - 8*sum), dot_q4k_q8_scalar (kquant.rs:257-282, s1/s2 per
 * 32-group) and dot_q6k_q8_scalar (kquant.rs:287-318, one per 16-element sub-block). */
int prana_block_dots(prana_ctx *ctx, const prana_weight *w, size_t row, const int8_t *q, const int32_t *sums,
                     int32_t *out);

/* rmsnorm (norms.rs:9-23) */
int prana_rmsnorm(prana_ctx *ctx, const float *x, const float *weight, size_t rows, size_t dim, float eps,
                  float *out);
/* silu in place (norms.rs:27-31) and the SwiGLU gate product g = silu(g) * u (infer.rs:193-199) */
int prana_silu(prana_ctx *ctx, float *x, size_t n);
int prana_silu_mul(prana_ctx *ctx, float *gate, const float *up, size_t n);
/* softmax over each of `rows` rows of n (norms.rs:44-56) */
int prana_softmax(prana_ctx *ctx, const float *x, size_t rows, size_t n, float *out);
/* rope_interleaved (attention.rs:90-101) / rope_neox (attention.rs:107-121) in place on
 * `rows` rows of n values; row i is at position pos + i. */
int prana_rope_interleaved(prana_ctx *ctx, float *x, size_t rows, size_t n, size_t pos, size_t head_dim,
                           float theta);
int prana_rope_neox(prana_ctx *ctx, float *x, size_t rows, size_t n, size_t pos, size_t head_dim, float theta);
/* f16_kv_write (attention.rs:47-52): cache is f16 bits [capacity, kv_stride] */
int prana_f16_kv_write(prana_ctx *ctx, uint16_t *cache, size_t first_row, size_t kv_stride, const float *src,
                       size_t n);
/* attention_decode (attention.rs:129-160) */
int prana_attention_decode(prana_ctx *ctx, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                           size_t pos, size_t n_heads, size_t n_kv_heads, size_t head_dim, float *out);
/* attention_decode without allocation.  No counterpart in the reference: it
 * is for callers that cannot allocate device memory on the call path (a host
 * that reserved all device memory for its own pool, a loop that must never
 * block on cudaMalloc/cudaFree).  Same kernels and results as
 * prana_attention_decode, but the split partials live in a fixed 4 MiB static
 * device array (1,048,576 floats; at most 1024 kv heads); a shape that needs
 * more returns PRANA_E_INVALID and names the limit.  It never allocates.
 * The first call on a device looks up the array's address (set-up); make that
 * first call before any stream capture.  The array is shared by every context
 * of the process on that device: calls that overlap in time (other streams,
 * other threads) race on it and must be serialized by the caller.  Its ticket
 * counters must be zero between calls; they start at zero and every call
 * leaves them at zero. */
int prana_attention_decode_noalloc(prana_ctx *ctx, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                                   size_t pos, size_t n_heads, size_t n_kv_heads, size_t head_dim, float *out);
/* attention_verify (attention.rs:296-333) */
int prana_attention_verify(prana_ctx *ctx, const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                           size_t pos0, size_t seq, size_t n_heads, size_t n_kv_heads, size_t head_dim,
                           float *out);
/* attention (attention.rs:236-284): causal over f32 in-window K/V; q, k, v and out 16-byte aligned */
int prana_attention(prana_ctx *ctx, const float *q, const float *k, const float *v, size_t seq, size_t n_heads,
                    size_t n_kv_heads, size_t head_dim, float *out);
/* first index of the row maximum (infer.rs:560-568, sampler.rs:40-48) */
int prana_argmax(prana_ctx *ctx, const float *x, size_t rows, size_t n, uint32_t *out);

/* ---------------------------------------------------------------- model (host buffers) */
typedef struct prana_model_config {
  int64_t dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len, head_dim;
  float rope_theta, norm_eps;
  int32_t rope_neox, has_bias, shared_classifier;
  int64_t weight_bytes; /* device bytes of all packed projection/embedding weights */
} prana_model_config;

/* gguf::load (gguf.rs:338-460) for llama / qwen2 into the device arena, at F32
 * precision (the reference's default) */
int prana_model_load_gguf(prana_ctx *ctx, const char *path, prana_model **out);
/* gguf::load with an explicit Precision: PRANA_PRECISION_Q8 (`--q8`) turns
 * every dense (F32 / F16) tensor the model multiplies -- projections and a tied
 * classifier over an F32 / F16 / Q8_0 embedding table -- into quantize_q8 of it
 * (gguf.rs:425-437, matmul.rs:61-84); PRANA_PRECISION_F32 keeps a tied dense
 * table as the f32 classifier (matmul_f32) and rejects dense projections. */
#define PRANA_PRECISION_F32 0
#define PRANA_PRECISION_Q8 1
int prana_model_load_gguf_ex(prana_ctx *ctx, const char *path, int precision, prana_model **out);
/* Tensor parallelism over `world` GPUs, one process (or context) per rank
 * (the Megatron-style split of the survey: column-split Q/K/V by heads and
 * gate/up by FFN rows, row-split wo and ffn_down by input columns, vocabulary
 * split LM head; one all-reduce after wo and one after ffn_down).  Rank 0 calls
 * prana_tp_unique_id and hands the NCCL_UNIQUE_ID_BYTES (128) id to every
 * rank, which loads its shard with prana_model_load_gguf_tp; from there every
 * model-level call runs on all ranks together (same tokens, same order) and
 * returns the full result on each.  KV caches hold the rank's kv heads
 * (prana_kv_read/write move [rows, n_kv_heads / world * head_dim]). */
int prana_tp_unique_id(void *id_out);
int prana_model_load_gguf_tp(prana_ctx *ctx, const char *path, int world, int rank, const void *nccl_id,
                             prana_model **out);
/* peer_exchange (may be NULL): 1 when the decode-sized all-reduces and the argmax
   all-gather run over mapped peer memory, 0 when NCCL carries every exchange */
int prana_model_tp_get(const prana_model *m, int *world, int *rank, int *peer_exchange);
int prana_model_free(prana_model *m); /* also frees the model's remaining KV caches */
int prana_model_config_get(const prana_model *m, prana_model_config *out);
/* KvCache::with_len (infer.rs:37-45): f16 K/V for `positions` rows per layer */
int prana_kv_create(prana_model *m, size_t positions, prana_kv **out);
int prana_kv_free(prana_kv *kv); /* only while its model is alive */
/* copy one layer's K or V cache rows [0, rows) to host (f16 bits) */
int prana_kv_read(prana_kv *kv, size_t layer, int is_v, size_t rows, uint16_t *host_out);
/* copy rows [first, first + rows) of one layer's K or V cache to host */
int prana_kv_read_rows(prana_kv *kv, size_t layer, int is_v, size_t first, size_t rows, uint16_t *host_out);

/* overwrite one layer's K or V cache rows [0, rows) from host f16 bits */
int prana_kv_write(prana_kv *kv, size_t layer, int is_v, size_t rows, const uint16_t *host_in);

/* forward / forward_impl (infer.rs:134-211): one token at `pos`; writes the logits
 * (host, may be NULL) and their argmax (may be NULL).  Runs as one CUDA graph whose
 * only host traffic is the (token, pos) pair in and the sampled id out. */
int prana_forward(prana_model *m, prana_kv *kv, uint32_t token, size_t pos, float *logits, uint32_t *next_token);
/* Diagnostic form of prana_forward (the role PRANA_TIMING plays in infer.rs:83-130):
 * one token, run eagerly, additionally returning every int8 activation row the pass
 * quantized, in CPU-path order -- per layer the attention-norm input (dim), the
 * attention output (n_heads*head_dim), the ffn-norm input (dim) and silu(gate)*up
 * (hidden); then the final-norm input (dim) -- with their per-32 scales. */
int prana_forward_trace(prana_model *m, prana_kv *kv, uint32_t token, size_t pos, float *logits, int8_t *q_out,
                        float *scales_out, size_t capacity, size_t *n_out);
/* Diagnostic batch form of prana_forward_trace: prefill (prefill = 1; positions
 * 0..n, pos0 ignored) or forward_batch (prefill = 0; positions pos0..) of n
 * tokens, run eagerly, additionally returning the quantized activation rows of
 * every site in CPU-path order -- per layer the n rows of the attention-norm
 * input, the attention output, the ffn-norm input and silu(gate)*up; then the
 * n final-norm rows (forward_batch only) -- with their per-32 scales.
 * logits [n, vocab] (forward_batch only; may be NULL). */
int prana_forward_batch_trace(prana_model *m, prana_kv *kv, const uint32_t *tokens, size_t n, size_t pos0,
                              int prefill, float *logits, int8_t *q_out, float *scales_out, size_t capacity,
                              size_t *n_out);
/* prefill (infer.rs:220-286): tokens at positions 0..n, no logits */
int prana_prefill(prana_model *m, prana_kv *kv, const uint32_t *tokens, size_t n);
/* forward_batch (infer.rs:296-374): n tokens at pos0.., logits [n, vocab] (may be NULL)
 * and per-row argmax (may be NULL) */
int prana_forward_batch(prana_model *m, prana_kv *kv, const uint32_t *tokens, size_t n, size_t pos0,
                        float *logits, uint32_t *argmax);
/* n independent sequences, one token each: row i is forward_impl (infer.rs:142-211)
 * for tokens[i] at positions[i] over caches[i] (n distinct caches of this model),
 * with the weights streamed once per 8 rows.  The reference has no such batch:
 * its equivalent is n forward calls.  logits [n, vocab] and argmax [n] may be NULL.
 * Single-GPU models only. */
int prana_forward_multi(prana_model *m, prana_kv *const *caches, size_t n, const uint32_t *tokens,
                        const size_t *positions, float *logits, uint32_t *argmax);
/* Diagnostic form of prana_forward_multi (eager, no logits gather shortcut):
 * additionally returns the quantized activation rows in the layout of
 * prana_forward_batch_trace (per layer the n rows of each site, then the n
 * final-norm rows). */
int prana_forward_multi_trace(prana_model *m, prana_kv *const *caches, size_t n, const uint32_t *tokens,
                              const size_t *positions, float *logits, int8_t *q_out, float *scales_out,
                              size_t capacity, size_t *n_out);
/* generate (infer.rs:696-771), greedy, over token ids; stop_id < 0 disables stopping.
 * out must hold `steps` ids; *n_out receives the count. */
int prana_generate(prana_model *m, const uint32_t *prompt, size_t p, size_t steps, int64_t stop_id,
                   uint32_t *out, size_t *n_out);
/* generate_speculative (infer.rs:581-690), greedy; stats[0] = proposed, stats[1] = accepted */
int prana_generate_speculative(prana_model *target, prana_model *draft, const uint32_t *prompt, size_t p,
                               size_t steps, size_t k, int64_t stop_id, uint32_t *out, size_t *n_out,
                               size_t *stats);

/* Device-resident decode loop for throughput measurement: after
 * prana_decode_begin(token, pos), each prana_decode_run(n) replays the per-token
 * graph n times back to back (token fed back on device, no host round trip) and
 * prana_decode_tokens copies the ids produced so far. */
int prana_decode_begin(prana_model *m, prana_kv *kv, uint32_t token, size_t pos);
int prana_decode_run(prana_model *m, prana_kv *kv, size_t n_steps);
int prana_decode_tokens(prana_model *m, prana_kv *kv, uint32_t *out, size_t max, size_t *n_out);

/* ---- tokenizers (host only; no device is touched) ----
 * Text is bytes; invalid UTF-8 is first replaced as Rust's String::from_utf8_lossy
 * does.  Calls that fill a caller buffer set *n_out to the size needed and return
 * PRANA_E_INVALID when cap is smaller. */
typedef struct prana_tokenizer prana_tokenizer;
/* load_tokenizer (gguf.rs:462-537): "llama" (SentencePiece pieces, U+2581 read as
 * a space) or "gpt2" (byte-level BPE with tokenizer.ggml.merges; token types 3 and
 * 4 encode verbatim) from a GGUF file's tokenizer.ggml.* metadata */
int prana_tokenizer_load_gguf(const char *path, prana_tokenizer **out);
/* Tokenizer::from_parts + with_special (tokenizer.rs:51-67): n pieces of lens[i] bytes */
int prana_tokenizer_spm(size_t n, const char *const *pieces, const size_t *lens, const float *scores,
                        uint32_t bos, uint32_t eos, int add_bos, prana_tokenizer **out);
/* BpeTokenizer::new + with_specials (bpe.rs:57-84): merges are "left right" strings
 * in rank order; bos / eos < 0: none */
int prana_tokenizer_bpe(size_t n, const char *const *pieces, const size_t *lens, size_t n_merges,
                        const char *const *merges, const size_t *merge_lens, size_t n_specials,
                        const uint32_t *special_ids, int64_t bos, int64_t eos, int add_bos,
                        prana_tokenizer **out);
int prana_tokenizer_free(prana_tokenizer *t);
int prana_tokenizer_vocab_size(const prana_tokenizer *t, size_t *out);
/* encode_prompt (Tokenize::encode_prompt, tokenizer.rs / bpe.rs:166-192) with bos = -1
 * and eos = 0; SentencePiece also takes Tokenizer::encode's explicit bos / eos (0 or 1,
 * tokenizer.rs:89-140) */
int prana_tokenize(const prana_tokenizer *t, const char *text, size_t len, int bos, int eos, uint32_t *ids,
                   size_t cap, size_t *n_out);
/* Tokenize::decode (tokenizer.rs:144-160, bpe.rs:194-199): the bytes of one token
 * given the previous one */
int prana_detokenize(const prana_tokenizer *t, uint32_t prev, uint32_t token, char *out, size_t cap,
                     size_t *n_out);
/* Tokenize::is_stop: the EOS or BOS id */
int prana_tokenizer_is_stop(const prana_tokenizer *t, uint32_t token, int *out);

/* ---- sampling ----
 * Sampler::new (sampler.rs:13-20): greedy when temperature <= 0, else temperature
 * sampling driven by xorshift64* from seed (0 reads as 1) */
typedef struct prana_sampler prana_sampler;
int prana_sampler_create(float temperature, uint64_t seed, prana_sampler **out);
int prana_sampler_free(prana_sampler *s);
/* Sampler::sample (sampler.rs:22-37) over n host logits: softmax(logits / temperature)
 * (norms.rs:44-56), then the first id where the running draw drops to <= 0 */
int prana_sample(prana_sampler *s, const float *logits, size_t n, uint32_t *token);
/* XorShift::next_f32 (sampler.rs:67-70): the stream's next uniform draw in [0, 1) */
int prana_sampler_next_f32(prana_sampler *s, float *out);
/* Sampler::sample on the device over n device logits (n <= 393216), writing the
 * token to device memory on the context stream: a greedy sampler takes the first
 * maximum; otherwise the kernel takes the sampler's next draw, which the host
 * stream skips over.  The cumulative probabilities are summed in f64, so the id
 * is prana_sample's except where the draw lies within the reference's
 * sequential f32 rounding of a bucket boundary. */
int prana_sample_logits(prana_ctx *ctx, const float *logits, size_t n, prana_sampler *s, uint32_t *token);
/* prana_forward whose next token is Sampler::sample on the device over the
 * step's logits (which stay in HBM); a greedy sampler is prana_forward's argmax.
 * s moves past the draw taken. */
int prana_forward_sampled(prana_model *m, prana_kv *kv, uint32_t token, size_t pos, prana_sampler *s,
                          uint32_t *next);
/* prana_decode_begin whose loop samples each next token on the device with the
 * sampler's temperature and stream (the sampler itself is not advanced; greedy
 * or NULL: prana_decode_begin) */
int prana_decode_begin_sampled(prana_model *m, prana_kv *kv, uint32_t token, size_t pos, const prana_sampler *s);
/* generate (infer.rs:696-771) with a Sampler: every sampled position draws on the
 * device, and s is left advanced by the draws the reference's loop makes (one
 * per sampled position, up to and including a stop token) */
int prana_generate_sampled(prana_model *m, const uint32_t *prompt, size_t p, size_t steps, int64_t stop_id,
                           prana_sampler *s, uint32_t *out, size_t *n_out);

#ifdef __cplusplus
}
#endif
#endif
