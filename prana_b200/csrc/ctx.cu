// ctx.cu -- context, error reporting, weight upload/repack and the
// kernel-level C-ABI entry points (the prana-kernels function surface).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>

#include "comm.h"
#include "host.h"
#include "sampler.h"

namespace prana {

static thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ctx_scratch(prana_ctx* ctx, size_t bytes, void** out) {
  bytes = (bytes + 255) & ~(size_t)255;
  if (ctx->scratch.bytes < bytes) {
    if (ctx->scratch.base) {
      PRANA_CK(cudaStreamSynchronize(ctx->stream));
      dev_free(ctx, ctx->scratch.base);
      ctx->scratch.base = nullptr;
      ctx->scratch.bytes = 0;
    }
    size_t want = bytes < ((size_t)16 << 20) ? ((size_t)16 << 20) : bytes;
    if (int rc = dev_alloc(ctx, want, &ctx->scratch.base)) return rc;
    ctx->scratch.bytes = want;
  }
  *out = ctx->scratch.base;
  return PRANA_OK;
}

static uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

int ctx_rope(prana_ctx* ctx, int hd, float theta, int neox, int positions, const RopeTable** out) {
  auto key = std::make_tuple(hd, f32_bits(theta), neox);
  RopeTable& t = ctx->rope[key];
  if (t.positions < positions) {
    const int n = positions < 256 ? 256 : positions;
    const int half = hd / 2;
    std::vector<float> c((size_t)n * half), s((size_t)n * half);
    for (int p = 0; p < n; p++)
      for (int i = 0; i < half; i++) {
        // interleaved: pair (2i, 2i+1), freq = theta^(-(2i)/hd)   (attention.rs:96)
        // neox:        pair (i, i+hd/2), freq = theta^(-(2*i)/hd) (attention.rs:114)
        const float freq = neox ? powf(theta, -(2.0f * (float)i) / (float)hd)
                                : powf(theta, -((float)(2 * i)) / (float)hd);
        const float ang = (float)p * freq;
        c[(size_t)p * half + i] = cosf(ang);
        s[(size_t)p * half + i] = sinf(ang);
      }
    if (t.cos) {
      ctx->retired.push_back(t.cos);
      ctx->retired.push_back(t.sin);
      t.cos = t.sin = nullptr;
      t.positions = 0;
    }
    void *pc = nullptr, *ps = nullptr;
    if (int rc = dev_alloc(ctx, c.size() * 4, &pc)) return rc;
    if (int rc = dev_alloc(ctx, s.size() * 4, &ps)) {
      dev_free(ctx, pc);
      return rc;
    }
    t.cos = static_cast<float*>(pc);
    t.sin = static_cast<float*>(ps);
    PRANA_CK(cudaMemcpy(t.cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    PRANA_CK(cudaMemcpy(t.sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
    t.positions = n;
  }
  *out = &t;
  return PRANA_OK;
}

static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// One tensor through a streamer whose chunk holds it whole (at most 64 MiB).
int upload_weight(prana_ctx* ctx, int type, size_t rows, size_t cols, const void* host, prana_weight* w) {
  const uint8_t* src = static_cast<const uint8_t*>(host);
  const size_t rb = gguf_bytes_per_row(type, cols);
  WeightStreamer ws(ctx, std::max<size_t>(std::min(rows * rb, size_t(64) << 20), std::max<size_t>(rb, 1)));
  int rc = ws.upload(type, rows, cols, [src, rb](size_t r) { return src + r * rb; }, w);
  if (!rc) rc = ws.finish();
  if (rc && w->mem) free_weight(w);
  return rc;
}

// quantize_q8 (matmul.rs:61-84): per 32 values amax (f32::max fold from 0),
// scale = amax / 127 (1 when amax is 0), q = round(x * (1 / scale)) clamped
// to +-127, round half away from zero; NaN becomes 0 as Rust's `as i8` does.
void quantize_q8_host(size_t rows, size_t cols, const float* w, int8_t* q, float* scales) {
  const size_t groups = cols / 32;
  for (size_t r = 0; r < rows; r++)
    for (size_t g = 0; g < groups; g++) {
      const float* blk = w + r * cols + g * 32;
      float amax = 0.0f;
      for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(blk[i]));
      const float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
      const float inv = 1.0f / scale;
      for (int i = 0; i < 32; i++) {
        const float v = roundf(blk[i] * inv);  // a NaN survives clamp and becomes 0
        q[r * cols + g * 32 + i] = (v != v) ? 0 : (int8_t)fminf(fmaxf(v, -127.0f), 127.0f);
      }
      scales[r * groups + g] = scale;
    }
}

int upload_q8s(prana_ctx* ctx, size_t rows, size_t cols, const float* host, prana_weight* w) {
  if (!rows || !cols) return fail(PRANA_E_INVALID, "empty weight [%zu, %zu]", rows, cols);
  if (cols % 32) return fail(PRANA_E_INVALID, "quantize_q8 needs cols %% 32 == 0 (cols=%zu)", cols);
  if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX) return fail(PRANA_E_INVALID, "weight too large");
  const size_t n = rows * cols, off = al256(n), total = off + al256(n / 32 * 4);
  std::vector<uint8_t> buf(total);
  quantize_q8_host(rows, cols, host, reinterpret_cast<int8_t*>(buf.data()), reinterpret_cast<float*>(buf.data() + off));
  void* mem = nullptr;
  if (int rc = dev_alloc(ctx, total, &mem)) return rc;
  if (cudaMemcpy(mem, buf.data(), total, cudaMemcpyHostToDevice) != cudaSuccess) {
    dev_free(ctx, mem);
    return fail(PRANA_E_CUDA, "weight upload failed");
  }
  DevWeight dw{};
  dw.type = T_Q8S;
  dw.rows = (int)rows;
  dw.cols = (int)cols;
  dw.qs = static_cast<uint8_t*>(mem);
  dw.ds = reinterpret_cast<const float*>(static_cast<uint8_t*>(mem) + off);
  w->ctx = ctx;
  w->dw = dw;
  w->mem = mem;
  w->bytes = total;
  return PRANA_OK;
}

void free_weight(prana_weight* w) {
  if (w && w->mem) {
    dev_free(w->ctx, w->mem);
    w->mem = nullptr;
  }
}

}  // namespace prana

using namespace prana;

#define API_BEGIN try {
#define API_END                                                    \
  }                                                                \
  catch (const std::bad_alloc&) {                                  \
    return fail(PRANA_E_OOM, "host allocation failed");            \
  }                                                                \
  catch (...) {                                                    \
    return fail(PRANA_E_INVALID, "unexpected host exception");     \
  }

#define NEED(cond, ...) \
  if (!(cond)) return fail(PRANA_E_INVALID, __VA_ARGS__)

extern "C" {

const char* prana_last_error(void) { return g_last_error.c_str(); }
int prana_version(void) { return 1; }

int prana_ctx_create(int device, prana_ctx** out) {
  API_BEGIN
  NEED(out, "out is null");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(PRANA_E_CUDA, "no CUDA device available");
  }
  NEED(device >= 0 && device < n, "device %d out of range (%d devices)", device, n);
  DevScope ds(device);
  PRANA_CK(cudaSetDevice(device));
  cudaDeviceProp prop;
  PRANA_CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(PRANA_E_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", prop.major, prop.minor);
  prana_ctx* c = new prana_ctx();
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->counters, (4096 + 64) * sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(c->counters, 0, (4096 + 64) * sizeof(unsigned)) != cudaSuccess) {
    cudaGetLastError();
    delete c;
    return fail(PRANA_E_CUDA, "context setup failed");
  }
  c->stream = c->own;
  c->err = c->counters + 4096;  // past every kv head's counter, on its own 256-byte line
  *out = c;
  return PRANA_OK;
  API_END
}

int prana_ctx_destroy(prana_ctx* c) {
  if (!c) return PRANA_OK;
  DevScope ds(c->device);
  cudaStreamSynchronize(c->stream);
  for (auto& kv : c->rope) {
    dev_free(c, kv.second.cos);
    dev_free(c, kv.second.sin);
  }
  for (void* p : c->retired) dev_free(c, p);
  dev_free(c, c->scratch.base);
  cudaFree(c->counters);
  cudaStreamDestroy(c->own);
  delete c;
  return PRANA_OK;
}

int prana_ctx_set_stream(prana_ctx* c, void* stream) {
  NEED(c, "ctx is null");
  c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own;
  return PRANA_OK;
}

int prana_ctx_stream(prana_ctx* c, void** stream) {
  NEED(c && stream, "null argument");
  *stream = c->own;
  return PRANA_OK;
}

// Waits for the kernel-level calls on the context's stream, then reports a
// bounded device wait that gave up in any of them (the context's own error
// word, and the no-allocation attention word of this device) as
// PRANA_E_TIMEOUT, clearing the word so the context stays usable.
int prana_ctx_synchronize(prana_ctx* c) {
  NEED(c, "ctx is null");
  DevScope ds(c->device);
  PRANA_CK(cudaStreamSynchronize(c->stream));
  unsigned e = 0, e2 = 0;
  PRANA_CK(cudaMemcpy(&e, c->err, sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (e) PRANA_CK(cudaMemset(c->err, 0, sizeof(unsigned)));
  if (int rc = noalloc_take_error(c->device, &e2)) return rc;
  if (e || e2)
    return fail(PRANA_E_TIMEOUT, "a bounded device-side wait expired in a kernel-level call (%s)",
                e ? "context" : "no-allocation attention");
  return PRANA_OK;
}

int prana_debug_wait_timeout(prana_ctx* c, int which, unsigned polls) {
  NEED(c, "ctx is null");
  NEED(which == 0 || which == 1, "which must be 0 (mbarrier) or 1 (peer exchange)");
  NEED(polls > 0, "polls must be positive");
  DevScope ds(c->device);
  if (int rc = prana_ctx_synchronize(c)) return rc;  // start from a clear error word
  if (which == 0) {
    PRANA_CK(launch_wait_never(polls, c->err, c->stream));
    return prana_ctx_synchronize(c);
  }
  // rank 0 of two, both receive areas on this GPU: rank 1's slot in rank 0's
  // area is never stored to, so the receive wait runs out
  constexpr size_t cap = 64;
  const size_t area = 2 * 2 * cap * sizeof(uint64_t);
  void* mem = nullptr;
  PRANA_CK(cudaMalloc(&mem, 2 * area + 64 * sizeof(unsigned) + cap * sizeof(float)));
  struct Free {
    void* p;
    ~Free() { cudaFree(p); }
  } fr{mem};
  PRANA_CK(cudaMemset(mem, 0, 2 * area + 64 * sizeof(unsigned) + cap * sizeof(float)));
  TpPeers p;
  p.world = 2;
  p.rank = 0;
  p.cap = cap;
  p.buf[0] = static_cast<uint64_t*>(mem);
  p.buf[1] = reinterpret_cast<uint64_t*>(static_cast<char*>(mem) + area);
  p.epoch = reinterpret_cast<unsigned*>(static_cast<char*>(mem) + 2 * area);
  p.budget = polls;
  float* x = reinterpret_cast<float*>(p.epoch + 64);
  PRANA_CK(launch_tp_allreduce(p, x, (int)cap, c->err, c->stream, false));
  return prana_ctx_synchronize(c);
}

int prana_weight_upload(prana_ctx* c, int type, size_t rows, size_t cols, const void* host, prana_weight** out) {
  API_BEGIN
  NEED(c && host && out, "null argument");
  *out = nullptr;
  DevScope ds(c->device);
  prana_weight* w = new prana_weight();
  int rc = upload_weight(c, type, rows, cols, host, w);
  if (rc) {
    delete w;
    return rc;
  }
  *out = w;
  return PRANA_OK;
  API_END
}

int prana_quantize_q8(size_t rows, size_t cols, const float* w, int8_t* q, float* scales) {
  API_BEGIN
  NEED(w && q && scales, "null argument");
  NEED(cols % 32 == 0, "cols must be a multiple of 32 (cols=%zu)", cols);
  quantize_q8_host(rows, cols, w, q, scales);
  return PRANA_OK;
  API_END
}

int prana_weight_upload_q8(prana_ctx* c, size_t rows, size_t cols, const float* host, prana_weight** out) {
  API_BEGIN
  NEED(c && host && out, "null argument");
  *out = nullptr;
  DevScope ds(c->device);
  prana_weight* w = new prana_weight();
  int rc = upload_q8s(c, rows, cols, host, w);
  if (rc) {
    delete w;
    return rc;
  }
  *out = w;
  return PRANA_OK;
  API_END
}

int prana_weight_free(prana_weight* w) {
  if (!w) return PRANA_OK;
  DevScope ds(w->ctx->device);
  free_weight(w);
  delete w;
  return PRANA_OK;
}

int prana_weight_bytes(const prana_weight* w, size_t* bytes) {
  NEED(w && bytes, "null argument");
  *bytes = w->bytes;
  return PRANA_OK;
}

int prana_quantize_acts(prana_ctx* c, const float* x, size_t rows, size_t k, int8_t* q, float* s, int32_t* sum) {
  NEED(c && x && q && s && sum, "null argument");
  NEED(k % 32 == 0, "k must be a multiple of 32 (k=%zu)", k);
  if (!rows || !k) return PRANA_OK;
  DevScope ds(c->device);
  PRANA_CK(launch_quantize_acts(x, (int)rows, (int)k, q, s, sum, c->stream));
  return PRANA_OK;
}

// out[t] = W . quantize_acts(a[t]) (or the given quantized rows), 8 rows per
// launch of the streaming GEMV (decode.cu); dense F32 weights use the f32 GEMV.
static int matmul_common(prana_ctx* c, const prana_weight* w, const float* a, const int8_t* q, const float* s,
                         const int32_t* sum, size_t n_tokens, float* out) {
  DevScope ds(c->device);
  const size_t K = (size_t)w->dw.cols, G = K / 32;
  if (w->dw.type == T_F32) {
    for (size_t t0 = 0; t0 < n_tokens; t0 += 8) {
      GemvArgs g{};
      g.w = w->dw;
      g.m = (int)(n_tokens - t0 < 8 ? n_tokens - t0 : 8);
      g.x = a + t0 * K;
      g.out = out + t0 * w->dw.rows;
      PRANA_CK(launch_gemv(g, PRO_F32, EPI_STORE, c->stream, false));
    }
    return PRANA_OK;
  }
  // Rows go to the tensor cores above 8, and from 6 on for tall weights: the
  // dp4a GEMV repeats its per-block dots for every row (issue-bound from about
  // 5 rows) while the GEMM's cost is flat up to 16 (8 rows on [14336 x 4096]:
  // Q8_0 48 -> 26 us, Q4_0 45 -> 28, Q4_K 73 -> 34; no gain at 4096 rows, nor
  // for Q6_K, whose GEMM issues two MMAs per block).
  const bool tc = n_tokens > 8 || (n_tokens >= 6 && w->dw.rows >= 8192 && w->dw.type != T_Q6_K);
  // scratch: the quantized rows when given f32 rows (quantize_acts first,
  // matmul.rs:169, kquant.rs:329), then the tensor-core GEMM's scale tables
  const size_t qb = (n_tokens * K + 255) & ~(size_t)255;
  const size_t act = a ? qb + ((n_tokens * G * 8 + 255) & ~(size_t)255) : 0;
  const size_t gemm = tc ? qgemm_scratch_bytes((int)n_tokens, (int)K) : 0;
  void* sp = nullptr;
  if (act + gemm) {
    int rc = ctx_scratch(c, act + gemm, &sp);
    if (rc) return rc;
  }
  if (a) {
    int8_t* qq = static_cast<int8_t*>(sp);
    float* ss = reinterpret_cast<float*>(qq + qb);
    int32_t* mm = reinterpret_cast<int32_t*>(ss + n_tokens * G);
    PRANA_CK(launch_quantize_acts(a, (int)n_tokens, (int)K, qq, ss, mm, c->stream));
    q = qq;
    s = ss;
    sum = mm;
  }
  if (tc) {  // the tensor cores (qgemm.cu)
    QgemmArgs g{};
    g.w = w->dw;
    g.N = w->dw.rows;
    g.K = (int)K;
    g.M = (int)n_tokens;
    g.out = out;
    g.err = c->err;
    const cudaError_t e = launch_qgemm(g, q, s, sum, static_cast<uint8_t*>(sp) + act, c->stream);
    if (e == cudaErrorNotSupported) return fail(PRANA_E_UNSUPPORTED, "tensor map for this weight could not be made");
    PRANA_CK(e);
    return PRANA_OK;
  }
  // Consecutive calls chain by programmatic dependent launch, as the decode
  // step's GEMVs do: the only reads a GEMV issues before its wait on the
  // previous kernel are of its weights, which no kernel writes (uploads
  // synchronize before they return), so its first weight loads overlap the
  // previous kernel's tail while activations and outputs wait for it.
  for (size_t t0 = 0; t0 < n_tokens; t0 += 8) {
    const int m = (int)(n_tokens - t0 < 8 ? n_tokens - t0 : 8);
    StreamArgs sa{};
    sa.w = w->dw;
    sa.K = (int)K;
    sa.N = w->dw.rows;
    sa.m = m;
    sa.aq = q + t0 * K;
    sa.as = s + t0 * G;
    sa.asum = sum + t0 * G;
    sa.out = out + t0 * w->dw.rows;
    sa.err = c->err;
    PRANA_CK(launch_stream(sa, EPI_STORE, PRO_Q, c->stream, true));
  }
  return PRANA_OK;
}

int prana_matmul_q8_f32(prana_ctx* c, const float* a, const prana_weight* w, size_t n_tokens, float* out) {
  NEED(c && a && w && out, "null argument");
  NEED(w->dw.type == T_Q8_0 || w->dw.type == T_Q8S, "matmul_q8_f32 needs a Q8 weight (type %d)", w->dw.type);
  return matmul_common(c, w, a, nullptr, nullptr, nullptr, n_tokens, out);
}

int prana_matmul_kquant_f32(prana_ctx* c, const float* a, const prana_weight* w, size_t n_tokens, float* out) {
  NEED(c && a && w && out, "null argument");
  NEED(w->dw.type == T_Q4_0 || w->dw.type == T_Q4_K || w->dw.type == T_Q6_K,
       "matmul_kquant_f32 needs a Q4_0/Q4_K/Q6_K weight (type %d)", w->dw.type);
  return matmul_common(c, w, a, nullptr, nullptr, nullptr, n_tokens, out);
}

int prana_matmul_q8_prefill(prana_ctx* c, const int8_t* q, const float* s, const int32_t* sum, size_t n_tokens,
                            const prana_weight* w, float* out) {
  NEED(c && q && s && sum && w && out, "null argument");
  NEED(w->dw.type == T_Q8_0 || w->dw.type == T_Q8S, "matmul_q8_prefill needs a Q8 weight");
  return matmul_common(c, w, nullptr, q, s, sum, n_tokens, out);
}

int prana_matmul_kquant_prefill(prana_ctx* c, const int8_t* q, const float* s, const int32_t* sum, size_t n_tokens,
                                const prana_weight* w, float* out) {
  NEED(c && q && s && sum && w && out, "null argument");
  NEED(w->dw.type == T_Q4_0 || w->dw.type == T_Q4_K || w->dw.type == T_Q6_K,
       "matmul_kquant_prefill needs a Q4_0/Q4_K/Q6_K weight");
  return matmul_common(c, w, nullptr, q, s, sum, n_tokens, out);
}

int prana_matmul_f32(prana_ctx* c, const float* a, const prana_weight* w, size_t n_tokens, float* out) {
  NEED(c && a && w && out, "null argument");
  NEED(w->dw.type == T_F32, "matmul_f32 needs an F32 weight");
  NEED((size_t)w->dw.cols * 8 * 4 <= 200 * 1024, "matmul_f32: cols too large for shared staging");
  return matmul_common(c, w, a, nullptr, nullptr, nullptr, n_tokens, out);
}

int prana_block_dots(prana_ctx* c, const prana_weight* w, size_t row, const int8_t* q, const int32_t* sum,
                     int32_t* out) {
  NEED(c && w && q && sum && out, "null argument");
  NEED(row < (size_t)w->dw.rows, "row %zu out of range", row);
  NEED(w->dw.type != T_F32, "block dots need a quantized weight");
  DevScope ds(c->device);
  PRANA_CK(launch_block_dots(w->dw, (int)row, q, sum, out, c->stream));
  return PRANA_OK;
}

int prana_rmsnorm(prana_ctx* c, const float* x, const float* w, size_t rows, size_t dim, float eps, float* out) {
  NEED(c && x && w && out, "null argument");
  if (!rows) return PRANA_OK;
  DevScope ds(c->device);
  PRANA_CK(launch_rmsnorm(x, w, (int)rows, (int)dim, eps, out, c->stream));
  return PRANA_OK;
}

int prana_silu(prana_ctx* c, float* x, size_t n) {
  NEED(c && x, "null argument");
  if (!n) return PRANA_OK;
  DevScope ds(c->device);
  PRANA_CK(launch_silu(x, n, c->stream));
  return PRANA_OK;
}

int prana_silu_mul(prana_ctx* c, float* g, const float* u, size_t n) {
  NEED(c && g && u, "null argument");
  if (!n) return PRANA_OK;
  DevScope ds(c->device);
  PRANA_CK(launch_silu_mul(g, u, n, c->stream));
  return PRANA_OK;
}

int prana_softmax(prana_ctx* c, const float* x, size_t rows, size_t n, float* out) {
  NEED(c && x && out, "null argument");
  if (!rows || !n) return PRANA_OK;
  DevScope ds(c->device);
  PRANA_CK(launch_softmax(x, (int)rows, (int)n, out, c->stream));
  return PRANA_OK;
}

static int rope_common(prana_ctx* c, float* x, size_t rows, size_t n, size_t pos, size_t hd, float theta, int neox) {
  NEED(c && x, "null argument");
  NEED(hd % 2 == 0, "head_dim must be even for RoPE");
  NEED(hd && n % hd == 0, "row must be a whole number of heads");
  if (!rows || !n) return PRANA_OK;
  DevScope ds(c->device);
  const RopeTable* t;
  int rc = ctx_rope(c, (int)hd, theta, neox, (int)(pos + rows), &t);
  if (rc) return rc;
  PRANA_CK(launch_rope(x, (int)rows, (int)n, (int)pos, (int)hd, neox, t->cos, t->sin, c->stream));
  return PRANA_OK;
}

int prana_rope_interleaved(prana_ctx* c, float* x, size_t rows, size_t n, size_t pos, size_t hd, float theta) {
  return rope_common(c, x, rows, n, pos, hd, theta, 0);
}
int prana_rope_neox(prana_ctx* c, float* x, size_t rows, size_t n, size_t pos, size_t hd, float theta) {
  return rope_common(c, x, rows, n, pos, hd, theta, 1);
}

int prana_f16_kv_write(prana_ctx* c, uint16_t* cache, size_t first_row, size_t kv_stride, const float* src, size_t n) {
  NEED(c && cache && src, "null argument");
  if (!n) return PRANA_OK;
  DevScope ds(c->device);
  PRANA_CK(launch_kv_write(reinterpret_cast<__half*>(cache), first_row * kv_stride, src, n, c->stream));
  return PRANA_OK;
}

// Splits for one attention launch: enough CTAs to cover the SMs twice,
// at least 32 positions each.

static int attn_common(prana_ctx* c, const float* q, const uint16_t* kc, const uint16_t* vc, size_t pos0, size_t m,
                       size_t nh, size_t nkv, size_t hd, float* out) {
  NEED(c && q && kc && vc && out, "null argument");
  NEED(nkv > 0 && nh % nkv == 0, "n_heads must be a multiple of n_kv_heads");
  NEED(hd <= 256, "head_dim %zu exceeds 256", hd);
  NEED(hd * (nh / nkv) <= 4096, "head_dim x group exceeds 4096");
  NEED(nkv <= 4096, "too many kv heads");
  if (!m) return PRANA_OK;
  DevScope ds(c->device);
  const int splits = attn_splits((int)(pos0 + m), (int)nkv, (int)hd, c->sm_count);
  const int group = (int)(nh / nkv);
  const int rows_per_cta = 4096 / (int)(hd * group);
  const size_t vh = (size_t)(rows_per_cta < (int)m ? rows_per_cta : (int)m) * group;
  const size_t ml = (nkv * splits * vh * 2 + 3) / 4 * 4, po = nkv * splits * vh * hd;  // part_o 16-byte aligned
  void* sp;
  int rc = ctx_scratch(c, (ml + po) * 4, &sp);
  if (rc) return rc;
  AttnArgs a{};
  a.q = q;
  a.kc = reinterpret_cast<const __half*>(kc);
  a.vc = reinterpret_cast<const __half*>(vc);
  a.m = (int)m;
  a.pos0 = (int)pos0;
  a.n_heads = (int)nh;
  a.n_kv = (int)nkv;
  a.hd = (int)hd;
  a.n_splits = splits;
  a.part_ml = static_cast<float*>(sp);
  a.part_o = static_cast<float*>(sp) + ml;
  a.counters = c->counters;
  a.out = out;
  a.err = c->err;
  attn_make_maps(a, (int)(pos0 + m));
  cudaError_t e = launch_attn_decode(a, c->stream, false);
  if (e == cudaErrorInvalidValue) return fail(PRANA_E_UNSUPPORTED, "attention: head_dim %zu not built", hd);
  PRANA_CK(e);
  return PRANA_OK;
}

int prana_attention_decode(prana_ctx* c, const float* q, const uint16_t* kc, const uint16_t* vc, size_t pos,
                           size_t nh, size_t nkv, size_t hd, float* out) {
  return attn_common(c, q, kc, vc, pos, 1, nh, nkv, hd, out);
}

int prana_attention_verify(prana_ctx* c, const float* q, const uint16_t* kc, const uint16_t* vc, size_t pos0,
                           size_t seq, size_t nh, size_t nkv, size_t hd, float* out) {
  return attn_common(c, q, kc, vc, pos0, seq, nh, nkv, hd, out);
}

int prana_attention(prana_ctx* c, const float* q, const float* k, const float* v, size_t seq, size_t nh, size_t nkv,
                    size_t hd, float* out) {
  NEED(c && q && k && v && out, "null argument");
  NEED(nkv > 0 && nh % nkv == 0, "n_heads must be a multiple of n_kv_heads");
  NEED(hd * (nh / nkv) <= 4096, "head_dim x group exceeds 4096");
  NEED(!((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
          reinterpret_cast<uintptr_t>(out)) & 15),
       "attention: q, k, v and out must be 16-byte aligned");
  if (!seq) return PRANA_OK;
  DevScope ds(c->device);
  PrefillAttnArgs a{q, k, v, (int)seq, (int)nh, (int)nkv, (int)hd, out};
  cudaError_t e = launch_attn_prefill(a, c->stream);
  if (e == cudaErrorInvalidValue) return fail(PRANA_E_UNSUPPORTED, "attention: head_dim %zu not built", hd);
  PRANA_CK(e);
  return PRANA_OK;
}

int prana_argmax(prana_ctx* c, const float* x, size_t rows, size_t n, uint32_t* out) {
  NEED(c && x && out, "null argument");
  NEED(n > 0, "argmax of an empty row");
  if (!rows) return PRANA_OK;
  DevScope ds(c->device);
  PRANA_CK(launch_argmax(x, (int)rows, (int)n, out, c->stream));
  return PRANA_OK;
}

int prana_sample_logits(prana_ctx* c, const float* logits, size_t n, prana_sampler* s, uint32_t* token) {
  NEED(c && logits && s && token, "null argument");
  NEED(n > 0, "sampling from empty logits");
  NEED(n <= (size_t)sample_max_vocab(), "%zu logits exceed the device sampler's %d", n, sample_max_vocab());
  DevScope ds(c->device);
  if (s->greedy) {
    PRANA_CK(launch_argmax(logits, 1, (int)n, token, c->stream));
    return PRANA_OK;
  }
  void* p = nullptr;
  if (int rc = ctx_scratch(c, sizeof(SampleState), &p)) return rc;
  const SampleState h{s->state, s->temp, 0};
  PRANA_CK(cudaMemcpyAsync(p, &h, sizeof h, cudaMemcpyHostToDevice, c->stream));
  PRANA_CK(launch_sample(logits, (int)n, static_cast<SampleState*>(p), token, nullptr, c->stream));
  s->next_u64();  // the kernel took one draw of the stream
  return PRANA_OK;
}

}  // extern "C"
