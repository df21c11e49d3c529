// model.cu -- the device-resident model: GGUF load into HBM
// (crates/prana-model/src/gguf.rs:157-460), the KV cache (infer.rs:25-45) and
// the forward paths (infer.rs:142-374) as one stream of fused kernels per
// token, captured once into a CUDA graph whose only host traffic is the token
// id in and the sampled id out.  generate / generate_speculative
// (infer.rs:581-771) run on top.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <new>

#include "comm.h"
#include "host.h"
#include "sampler.h"

namespace prana {

// ------------------------------------------------------------------ GGUF (subset)

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;  // dims[0] is the contiguous (column) dimension
  uint32_t type = 0;
  uint64_t offset = 0;
};

struct Gguf {
  const uint8_t* data = nullptr;
  size_t len = 0;
  size_t off = 0;
  size_t data_start = 0;
  std::map<std::string, int64_t> ints;
  std::map<std::string, double> floats;
  std::map<std::string, std::string> strs;
  std::map<std::string, uint64_t> arr_len;
  std::map<std::string, GgufTensor> tensors;

  bool rd(void* dst, size_t n) {
    if (off + n > len) return false;
    memcpy(dst, data + off, n);
    off += n;
    return true;
  }
  template <typename T>
  bool get(T& v) {
    return rd(&v, sizeof(T));
  }
  bool str(std::string* out) {
    uint64_t n;
    if (!get(n) || off + n > len) return false;
    if (out) out->assign(reinterpret_cast<const char*>(data + off), n);
    off += n;
    return true;
  }
  // gguf.rs:110-134 value types 0..12
  bool value(uint32_t ty, const std::string* key) {
    switch (ty) {
      case 0: case 1: case 7: { uint8_t v; if (!get(v)) return false; if (key) ints[*key] = ty == 1 ? (int8_t)v : v; return true; }
      case 2: case 3: { uint16_t v; if (!get(v)) return false; if (key) ints[*key] = ty == 3 ? (int16_t)v : v; return true; }
      case 4: case 5: { uint32_t v; if (!get(v)) return false; if (key) ints[*key] = ty == 5 ? (int64_t)(int32_t)v : v; return true; }
      case 6: { float v; if (!get(v)) return false; if (key) floats[*key] = v; return true; }
      case 8: { std::string s; if (!str(key ? &s : nullptr)) return false; if (key) strs[*key] = s; return true; }
      case 9: {
        uint32_t et;
        uint64_t n;
        if (!get(et) || !get(n)) return false;
        if (key) arr_len[*key] = n;
        for (uint64_t i = 0; i < n; i++)
          if (!value(et, nullptr)) return false;
        return true;
      }
      case 10: case 11: { uint64_t v; if (!get(v)) return false; if (key) ints[*key] = (int64_t)v; return true; }
      case 12: { double v; if (!get(v)) return false; if (key) floats[*key] = v; return true; }
    }
    return false;
  }
};

static size_t type_size(uint32_t t, uint64_t n) {
  switch (t) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q4_0: return n / 32 * 18;
    case T_Q8_0: return n / 32 * 34;
    case T_Q4_K: return n / 256 * 144;
    case T_Q6_K: return n / 256 * 210;
  }
  return 0;
}

// gguf.rs:157-196 Gguf::from_bytes
static int gguf_parse(Gguf& g) {
  uint32_t magic, ver;
  uint64_t nt, nkv;
  if (!g.get(magic) || magic != 0x46554747u) return fail(PRANA_E_FORMAT, "not a GGUF file (bad magic)");
  if (!g.get(ver) || ver < 2 || ver > 3) return fail(PRANA_E_FORMAT, "unsupported GGUF version %u", ver);
  if (!g.get(nt) || !g.get(nkv)) return fail(PRANA_E_FORMAT, "gguf truncated");
  for (uint64_t i = 0; i < nkv; i++) {
    std::string key;
    uint32_t ty;
    if (!g.str(&key) || !g.get(ty) || !g.value(ty, &key)) return fail(PRANA_E_FORMAT, "gguf truncated");
  }
  for (uint64_t i = 0; i < nt; i++) {
    GgufTensor t;
    uint32_t nd;
    if (!g.str(&t.name) || !g.get(nd) || nd > 4) return fail(PRANA_E_FORMAT, "gguf truncated");
    t.dims.resize(nd);
    for (uint32_t d = 0; d < nd; d++)
      if (!g.get(t.dims[d])) return fail(PRANA_E_FORMAT, "gguf truncated");
    if (!g.get(t.type) || !g.get(t.offset)) return fail(PRANA_E_FORMAT, "gguf truncated");
    g.tensors[t.name] = t;
  }
  int64_t al = 32;
  auto it = g.ints.find("general.alignment");
  if (it != g.ints.end() && it->second > 0 && (it->second & (it->second - 1)) == 0) al = it->second;
  g.data_start = (g.off + al - 1) / al * al;
  return PRANA_OK;
}

static int tensor_raw(const Gguf& g, const std::string& name, const GgufTensor** t, const uint8_t** raw) {
  auto it = g.tensors.find(name);
  if (it == g.tensors.end()) return fail(PRANA_E_FORMAT, "missing tensor '%s'", name.c_str());
  uint64_t n = 1;
  for (auto d : it->second.dims) n *= d;
  const size_t bytes = type_size(it->second.type, n);
  if (!bytes) return fail(PRANA_E_UNSUPPORTED, "tensor '%s': unsupported ggml type %u", name.c_str(), it->second.type);
  if (g.data_start + it->second.offset + bytes > g.len)
    return fail(PRANA_E_FORMAT, "tensor '%s' data out of range", name.c_str());
  *t = &it->second;
  *raw = g.data + g.data_start + it->second.offset;
  return PRANA_OK;
}

static float f16_host(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1fu, frac = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0 && frac == 0) bits = sign << 31;
  else if (exp == 0) {
    const float v = (float)frac * 5.9604644775390625e-08f;
    return sign ? -v : v;
  } else if (exp == 0x1f) bits = (sign << 31) | 0x7f800000u | (frac << 13);
  else bits = (sign << 31) | ((exp + 112u) << 23) | (frac << 13);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// tensor_f32 for the 1-D tensors the model reads (norms, biases)
static int vec_f32(const Gguf& g, const std::string& name, size_t n, std::vector<float>& out) {
  const GgufTensor* t;
  const uint8_t* raw;
  int rc = tensor_raw(g, name, &t, &raw);
  if (rc) return rc;
  uint64_t cnt = 1;
  for (auto d : t->dims) cnt *= d;
  if (cnt != n) return fail(PRANA_E_FORMAT, "tensor '%s' has %llu values, expected %zu", name.c_str(), (unsigned long long)cnt, n);
  out.resize(n);
  if (t->type == T_F32) memcpy(out.data(), raw, n * 4);
  else if (t->type == T_F16)
    for (size_t i = 0; i < n; i++) {
      uint16_t h;
      memcpy(&h, raw + 2 * i, 2);
      out[i] = f16_host(h);
    }
  else return fail(PRANA_E_UNSUPPORTED, "tensor '%s': only F32/F16 vectors supported", name.c_str());
  return PRANA_OK;
}

}  // namespace prana

using namespace prana;

// ------------------------------------------------------------------ model objects

namespace {

// A weight that streams through stream_gemv (the head may alias the embedding).
struct StreamW {
  prana_weight w;
  bool owns = true;
};

struct QkvPart {
  StreamW sw;
  int nseg = 0;
  int seg_start[4] = {0, 0, 0, 0};
  int kind[3] = {0, 0, 0};
};

struct LayerW {
  std::vector<QkvPart> qkv;
  StreamW wo, gu, w1, w3, w2;  // gu: gate/up rows interleaved; w1/w3 when their types differ
  bool fused_gu = false;
  float *rms_att = nullptr, *rms_ffn = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
};

// Activation buffers for `rows` rows (decode: 8; prefill: the prompt length).
struct Bufs {
  size_t rows = 0;
  float *x = nullptr, *q = nullptr, *att = nullptr, *kf = nullptr, *vf = nullptr, *h = nullptr, *u = nullptr;
  float* logits = nullptr;
  float* logits_l = nullptr;  // tensor parallel: this rank's vocabulary slice
  uint32_t* toks = nullptr;     // input ids [rows]
  uint32_t* tok_out = nullptr;  // argmax per row [rows]
  // dense f32 classifier: the final-norm rows and (for a trace) their group sums
  float* xn = nullptr;
  int32_t* xsum = nullptr;
  // batch path (rows > 8): quantized rows, GEMM outputs, GEMM scratch
  int8_t* bq = nullptr;
  float* bs = nullptr;
  int32_t* bsum = nullptr;
  float* y = nullptr;
  void* qg = nullptr;
  std::vector<void*> owned;
  prana_ctx* ctx = nullptr;  // device memory from its pool when one is attached
  explicit Bufs(prana_ctx* c) : ctx(c) {}
  ~Bufs() {
    for (void* p : owned) dev_free(ctx, p);
  }
  template <typename T>
  int alloc(T*& p, size_t n) {
    void* v = nullptr;
    if (int rc = dev_alloc(ctx, std::max<size_t>(n, 1) * sizeof(T), &v)) return rc;
    owned.push_back(v);
    p = static_cast<T*>(v);
    return PRANA_OK;
  }
};

// A captured multi-sequence step for one ordered set of caches: its own row
// buffers and per-sequence device views; a call copies the tokens and the
// positions in, replays the graph (whose first kernel writes the positions
// into the views) and reads the ids back.
struct MultiPlan {
  std::vector<prana_kv*> kvs;
  std::unique_ptr<Bufs> bufs;
  SeqRow* rows_dev = nullptr;
  AttnSeq* att_dev = nullptr;
  int* pos_dev = nullptr;
  uint32_t* h_stage = nullptr;  // pinned: tokens [n], then positions [n]
  cudaGraphExec_t graph = nullptr;
  explicit MultiPlan(prana_ctx* c) : bufs(new Bufs(c)) {}
  ~MultiPlan() {
    if (graph) cudaGraphExecDestroy(graph);
    if (h_stage) cudaFreeHost(h_stage);
  }
};

__global__ void multi_positions_kernel(const int* pos, int n, int n_att, SeqRow* rows, AttnSeq* att) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) rows[i].pos = pos[i];
  for (int j = i; j < n_att; j += gridDim.x * blockDim.x) att[j].pos0 = pos[j % n];
}

}  // namespace

struct prana_model {
  prana_ctx* ctx = nullptr;
  prana_model_config cfg{};
  prana_weight emb;
  std::vector<LayerW> layers;
  float* rms_final = nullptr;
  StreamW head;
  const RopeTable* rope = nullptr;
  std::vector<void*> owned;  // norms / biases / scratch
  std::unique_ptr<Bufs> dec;
  float* part_val = nullptr;  // LM-head argmax partials [8][n_parts]
  int* part_idx = nullptr;
  int n_parts = 0;
  unsigned* ctr = nullptr;    // ticket counter of the streaming kernels
  unsigned* err = nullptr;    // device error flag
  int* d_tokpos = nullptr;    // [token, pos] of the graph-driven step
  SampleState* d_sample = nullptr;  // sampler state of the sampled decode loop
  int* h_io = nullptr;        // pinned mirror
  uint32_t* h_tok = nullptr;
  bool pdl = true;
  int precision = 0;  // PRANA_PRECISION_F32 / _Q8 (gguf::load's precision, gguf.rs:338-460)
  std::vector<prana_kv*> caches;  // live KV caches (freed with the model)
  // tensor parallelism: this rank's share of heads, FFN rows and vocabulary
  // (the whole model when tp_world == 1)
  int tp_world = 1, tp_rank = 0;
  ncclComm_t comm = nullptr;
  int64_t heads_l = 0, kv_heads_l = 0, hid_l = 0, vocab_l = 0, vocab_off = 0;
  float* tp_local = nullptr;  // [16]: per row the best logit, then its index bits
  float* tp_all = nullptr;    // [world][16]
  prana::TpPeers peers;       // one-shot all-reduce over peer memory (world == 1: unused)
  void* peers_mem = nullptr;
  bool peers_ok = false;
  std::unique_ptr<MultiPlan> multi;  // the last captured multi-sequence step
};

struct prana_kv {
  prana_model* m = nullptr;
  size_t positions = 0;
  __half* k = nullptr;
  __half* v = nullptr;
  std::vector<prana::AttnArgs> maps;  // per layer: the K / V tensor maps (tm_k, tm_v, has_tm)
  int n_splits = 1;
  float* part_ml = nullptr;
  float* part_o = nullptr;
  unsigned* counters = nullptr;
  uint32_t* ring = nullptr;
  int* ring_n = nullptr;
  cudaGraphExec_t g_step = nullptr;
  cudaGraphExec_t g_loop = nullptr;
  cudaGraphExec_t g_loop_s = nullptr;  // the loop with Sampler::sample on the device
  size_t loop_pos = 0;  // host mirror of the device-loop position
  bool loop_active = false;
  bool loop_sampled = false;
};

namespace {

int dev_vec(prana_model* m, const std::vector<float>& h, float** out) {
  void* p = nullptr;
  if (int rc = dev_alloc(m->ctx, h.size() * 4, &p)) return rc;
  m->owned.push_back(p);
  if (cudaMemcpy(p, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(PRANA_E_CUDA, "upload failed");
  *out = static_cast<float*>(p);
  return PRANA_OK;
}

// The linear loading rule of gguf.rs:271-305: Q8_0 (cols%32), Q4_0 (cols%32),
// Q4_K/Q6_K (cols%256) stay quantized.  Dense projections are not built.
int linear_raw(const Gguf& g, const std::string& name, size_t rows, size_t cols, uint32_t* type, const uint8_t** raw,
               int precision) {
  const GgufTensor* t;
  int rc = tensor_raw(g, name, &t, raw);
  if (rc) return rc;
  if (t->dims.size() != 2) return fail(PRANA_E_FORMAT, "tensor '%s' is not 2-D", name.c_str());
  if (t->dims[0] != cols || t->dims[1] != rows)
    return fail(PRANA_E_FORMAT, "tensor '%s' is [%llu, %llu], expected [%zu, %zu]", name.c_str(),
                (unsigned long long)t->dims[1], (unsigned long long)t->dims[0], rows, cols);
  const uint32_t ty = t->type;
  const bool packed = (ty == T_Q8_0 && cols % 32 == 0) || (ty == T_Q4_0 && cols % 32 == 0) ||
                      ((ty == T_Q4_K || ty == T_Q6_K) && cols % 256 == 0);
  // dense tensors (F32, F16) become Linear::new(w, precision): quantize_q8 under
  // Q8 precision (matmul.rs:61-84); the dense f32 matmul for projections is not built
  const bool dense_q8 = (ty == T_F32 || ty == T_F16) && precision == PRANA_PRECISION_Q8 && cols % 32 == 0;
  if (!packed && !dense_q8)
    return fail(PRANA_E_UNSUPPORTED,
                "tensor '%s': type %u with %zu cols would run the dense f32 matmul for a projection, not built "
                "(load with Q8 precision to quantize it)",
                name.c_str(), ty, cols);
  *type = ty;
  return PRANA_OK;
}

size_t gguf_row_bytes(uint32_t type, size_t cols) { return type_size(type, cols); }

// Rows of a GGUF tensor stored one after another from `raw`.
RowSrc linear_rows(const uint8_t* raw, size_t rb) {
  return [raw, rb](size_t r) { return raw + r * rb; };
}

// Columns [c0, c1) of every row of a [rows, cols] GGUF tensor (whole blocks),
// as rows of a [rows, c1 - c0] tensor.
int col_rows(uint32_t type, size_t cols, const uint8_t* raw, size_t c0, size_t c1, RowSrc* out) {
  const size_t blk = (type == T_Q4_K || type == T_Q6_K) ? 256 : (type == T_Q8_0 || type == T_Q4_0) ? 32 : 1;
  if (c0 % blk || c1 % blk || c1 > cols || c0 >= c1)
    return fail(PRANA_E_UNSUPPORTED, "column shard [%zu, %zu) does not fall on %zu-value blocks", c0, c1, blk);
  const size_t rb = gguf_row_bytes(type, cols), off = gguf_row_bytes(type, c0);
  *out = [raw, rb, off](size_t r) { return raw + r * rb + off; };
  return PRANA_OK;
}

// f32 values of `rows` rows of a dense (F32 / F16) or Q8_0 GGUF tensor, as the
// reference's tensor_f32 densifies them (gguf.rs:208-267)
std::vector<float> densify(uint32_t type, size_t rows, size_t cols, const uint8_t* raw) {
  std::vector<float> out(rows * cols);
  const size_t n = rows * cols;
  if (type == T_F32) {
    memcpy(out.data(), raw, n * 4);
  } else if (type == T_F16) {
    for (size_t i = 0; i < n; i++) {
      uint16_t h;
      memcpy(&h, raw + 2 * i, 2);
      out[i] = f16_host(h);
    }
  } else {  // Q8_0: q * d in f32
    for (size_t b = 0; b < n / 32; b++) {
      uint16_t h;
      memcpy(&h, raw + b * 34, 2);
      const float d = f16_host(h);
      for (int i = 0; i < 32; i++) out[b * 32 + i] = (float)(int8_t)raw[b * 34 + 2 + i] * d;
    }
  }
  return out;
}

int upload_stream(prana_model* m, WeightStreamer& ws, uint32_t type, size_t rows, size_t cols, const RowSrc& src,
                  StreamW* sw) {
  if (type == T_F32 || type == T_F16) {  // Q8 precision: quantize_q8 of the dense rows
    const size_t rb = gguf_row_bytes(type, cols);
    std::vector<uint8_t> raw(rows * rb);
    for (size_t r = 0; r < rows; r++) memcpy(&raw[r * rb], src(r), rb);
    const std::vector<float> f = densify(type, rows, cols, raw.data());
    return upload_q8s(m->ctx, rows, cols, f.data(), &sw->w);
  }
  return ws.upload((int)type, rows, cols, src, &sw->w);
}

void free_stream(StreamW& s) {
  if (s.owns) free_weight(&s.w);
}

void destroy_kv(prana_kv* kv);

void free_model(prana_model* m) {
  if (!m) return;
  DevScope ds(m->ctx->device);
  cudaStreamSynchronize(m->ctx->own);
  m->multi.reset();
  while (!m->caches.empty()) destroy_kv(m->caches.back());
  free_weight(&m->emb);
  free_stream(m->head);
  for (auto& L : m->layers) {
    for (auto& p : L.qkv) free_stream(p.sw);
    free_stream(L.wo);
    free_stream(L.gu);
    free_stream(L.w1);
    free_stream(L.w3);
    free_stream(L.w2);
  }
  for (void* p : m->owned) dev_free(m->ctx, p);
  m->dec.reset();
  if (m->peers_ok) tp_peers_release(&m->peers, m->peers_mem);
  if (m->comm) {
    const Nccl* api = nccl(nullptr);
    if (api) api->comm_destroy(m->comm);
  }
  if (m->h_io) cudaFreeHost(m->h_io);
  delete m;
}

int make_bufs(prana_model* m, size_t rows, bool window, Bufs& b) {
  const auto& c = m->cfg;
  const size_t q_dim = m->heads_l * c.head_dim, kv_dim = m->kv_heads_l * c.head_dim, dim = c.dim, hid = m->hid_l;
  b.rows = rows;
  int rc = 0;
  rc |= b.alloc(b.x, rows * dim);
  rc |= b.alloc(b.q, rows * q_dim);
  rc |= b.alloc(b.att, rows * q_dim);
  rc |= b.alloc(b.h, rows * hid);
  rc |= b.alloc(b.u, rows * hid);
  rc |= b.alloc(b.toks, rows);
  rc |= b.alloc(b.tok_out, rows);
  if (m->head.w.dw.type == T_F32) {
    rc |= b.alloc(b.xn, rows * dim);
    rc |= b.alloc(b.xsum, rows * dim / 32);
  }
  if (rows > 8 && m->tp_world == 1) {
    const size_t max_k = std::max(std::max(dim, q_dim), hid);
    const size_t max_n = std::max(q_dim + 2 * kv_dim, 2 * hid);
    rc |= b.alloc(b.bq, rows * max_k);
    rc |= b.alloc(b.bs, rows * max_k / 32);
    rc |= b.alloc(b.bsum, rows * max_k / 32);
    rc |= b.alloc(b.y, rows * max_n);
    uint8_t* qg = nullptr;
    rc |= b.alloc(qg, qgemm_scratch_bytes((int)rows, (int)max_k));
    b.qg = qg;
  }
  if (window) {
    rc |= b.alloc(b.kf, rows * kv_dim);
    rc |= b.alloc(b.vf, rows * kv_dim);
  } else {
    rc |= b.alloc(b.logits, rows * c.vocab_size);
    if (m->tp_world > 1) rc |= b.alloc(b.logits_l, rows * m->vocab_l);
  }
  return rc ? PRANA_E_OOM : PRANA_OK;
}

enum { MODE_CACHE = 0, MODE_WINDOW = 1 };

// Diagnostic trace of every quantized activation row of a one-token pass, in
// the order the CPU path quantizes them: per layer the attention-norm input,
// the attention output, the ffn-norm input and silu(g)*u; then the final norm.
// Each site is the int8 rows a streaming kernel staged (CTA 0 copies them out).
struct Trace {
  int8_t* q = nullptr;
  float* s = nullptr;
  size_t nq = 0, ns = 0;
  // a launch over a.m rows of k values each appends its rows [a.m][k]
  void site(StreamArgs& a, int k) {
    a.trace_q = q + nq;
    a.trace_s = s + ns;
    nq += (size_t)a.m * k;
    ns += (size_t)a.m * k / 32;
  }
};

StreamArgs stream_args(prana_model* m, StreamW& w, int mrows, const float* x, const float* norm_w) {
  StreamArgs a{};
  a.w = w.w.dw;
  a.K = w.w.dw.cols;
  a.N = w.w.dw.rows;
  a.m = mrows;
  a.x = x;
  a.norm_w = norm_w;
  a.eps = m->cfg.norm_eps;
  a.err = m->err;
  return a;
}

// The next matrix's first rows (up to kPrefetchBytes) for a kernel's tail:
// wo -> gate|up, gate|up -> down, down -> the next layer's Q|K|V (or the LM
// head).  Q|K|V prefetches nothing: attention follows it and streams the
// cache, and wo's rows fetched then measured slower.
constexpr size_t kPrefetchBytes = size_t(16) << 20;
void set_prefetch(StreamArgs& a, const StreamW* next) {
  if (!next || next->w.dw.rows <= 0) return;
  const DevWeight& w = next->w.dw;
  size_t row_bytes;
  switch (w.type) {
    case T_Q8_0: row_bytes = (size_t)w.cols * 34 / 32; break;
    case T_Q4_0: row_bytes = (size_t)w.cols * 18 / 32; break;
    case T_Q4_K: row_bytes = (size_t)w.cols / 256 * 144; break;
    case T_Q6_K: row_bytes = (size_t)w.cols / 256 * 210; break;
    default: return;
  }
  const size_t rows = kPrefetchBytes / (row_bytes ? row_bytes : 1);
  a.pf_w = w;
  a.pf_rows = (int)std::min<size_t>(rows, (size_t)w.rows);
}

int run_stream(prana_model* m, StreamArgs& a, int epi, int pro, bool pdl) {
  PRANA_CK(launch_stream(a, epi, pro, m->ctx->own, pdl));
  return PRANA_OK;
}

// Batch path: the n quantized rows in b.bq times w on the tensor cores.
int run_qgemm(prana_model* m, Bufs& b, const StreamW& w, int n, float* out, int resid) {
  QgemmArgs g{};
  g.w = w.w.dw;
  g.N = w.w.dw.rows;
  g.K = w.w.dw.cols;
  g.M = n;
  g.out = out;
  g.resid = resid;
  g.err = m->err;
  const cudaError_t e = launch_qgemm(g, b.bq, b.bs, b.bsum, b.qg, m->ctx->own);
  if (e == cudaErrorNotSupported) return fail(PRANA_E_UNSUPPORTED, "tensor map for a [%d x %d] weight could not be made", g.N, g.K);
  PRANA_CK(e);
  return PRANA_OK;
}

// Batch path: rows x [n][k] (rmsnorm'd by w when set) quantized into b.bq / b.bs / b.bsum.
int quantize_rows(prana_model* m, Bufs& b, const float* x, const float* w, int n, int k, Trace* tr) {
  PRANA_CK(launch_norm_quant(x, w, m->cfg.norm_eps, n, k, b.bq, b.bs, b.bsum, m->ctx->own));
  if (tr) {  // the site's rows, as the streaming kernels' CTA 0 copies them
    PRANA_CK(cudaMemcpyAsync(tr->q + tr->nq, b.bq, (size_t)n * k, cudaMemcpyDeviceToDevice, m->ctx->own));
    PRANA_CK(cudaMemcpyAsync(tr->s + tr->ns, b.bs, (size_t)n * k / 32 * 4, cudaMemcpyDeviceToDevice, m->ctx->own));
    tr->nq += (size_t)n * k;
    tr->ns += (size_t)n * k / 32;
  }
  return PRANA_OK;
}

// One pass of n rows through the model (infer.rs:142-211 for n = 1 and
// :296-374 / :220-286 for the batched forms).  Rows sit at positions pos0..
// (or *pos_dev.. when pos_dev is set, n == 1).  MODE_WINDOW attends over the
// f32 in-window K/V (prefill); MODE_CACHE over the f16 cache (decode, verify).
// Every projection's kernel normalizes / quantizes its own input rows in its
// prologue while its first weight tiles are already streaming in.
// Tensor parallel (tp_world > 1): each rank holds its heads, FFN rows and
// vocabulary slice.  wo and ffn_down are split by input columns: rank 0 adds
// its partial product to x (residual epilogue), the other ranks store theirs
// into x, and one in-place all-reduce (sum) leaves x + sum of partials on every
// rank.  The LM head reports each shard's (max, index); an all-gather and the
// first maximum over ranks give the token.  gather_logits also assembles the
// full logits rows.
int tp_sum_rows(prana_model* m, float* x, size_t n, cudaStream_t st, bool pdl) {
  if (m->peers_ok && n <= m->peers.cap) {  // small (decode / verify) rows: one-shot over peer memory
    PRANA_CK(launch_tp_allreduce(m->peers, x, (int)n, m->err, st, pdl));
    return PRANA_OK;
  }
  const char* why = nullptr;
  const Nccl* api = nccl(&why);
  if (!api) return fail(PRANA_E_COMM, "%s", why);
  const ncclResult_t r = api->all_reduce(x, x, n, ncclFloat, ncclSum, m->comm, st);
  if (r != ncclSuccess) return fail(PRANA_E_COMM, "ncclAllReduce: %s", api->error_string(r));
  return PRANA_OK;
}

int tp_gather(prana_model* m, const float* src, float* dst, size_t n, cudaStream_t st, bool pdl) {
  if (m->peers_ok && n <= m->peers.cap) {
    PRANA_CK(launch_tp_allgather(m->peers, src, (int)n, dst, m->err, st, pdl));
    return PRANA_OK;
  }
  const char* why = nullptr;
  const Nccl* api = nccl(&why);
  if (!api) return fail(PRANA_E_COMM, "%s", why);
  const ncclResult_t r = api->all_gather(src, dst, n, ncclFloat, m->comm, st);
  if (r != ncclSuccess) return fail(PRANA_E_COMM, "ncclAllGather: %s", api->error_string(r));
  return PRANA_OK;
}

// Rows of independent sequences (prana_forward_multi): row i decodes one token
// of sequence i at its own position with its own KV cache.
struct Multi {
  const SeqRow* rows_dev;    // [n] device: cache bases, strides, positions
  prana_kv* const* kvs;      // [n] the caches
  const size_t* pos;         // [n] host copy of the positions
  const AttnSeq* attn_dev;   // [layers][n] device: per-sequence attention views (one launch per layer)
  int min_splits;            // the smallest split scratch among the caches
  bool all_tm;               // every cache has tensor maps for every layer
};

int enqueue_rows(prana_model* m, prana_kv* kv, Bufs& b, int n, const uint32_t* toks_dev, const int* tok_dev, int pos0,
                 const int* pos_dev, int mode, bool head, bool pdl, Trace* tr = nullptr, bool gather_logits = true,
                 const Multi* mu = nullptr) {
  const auto& c = m->cfg;
  cudaStream_t st = m->ctx->own;
  const bool tp = m->tp_world > 1;
  const int dim = (int)c.dim, hd = (int)c.head_dim, hid = (int)m->hid_l;
  const int q_dim = (int)(m->heads_l * c.head_dim), kv_dim = (int)(m->kv_heads_l * c.head_dim);
  const size_t lstride = kv->positions * (size_t)kv_dim;
  int rc;
  // more than 8 rows on one GPU: every projection's rows are quantized once and
  // multiplied on the tensor cores (qgemm.cu); up to 8, the streaming GEMV
  const bool batch = n > 8 && b.bq != nullptr;
  PRANA_CK(launch_embed(m->emb.dw, toks_dev, tok_dev, n, b.x, st, pdl));
  for (size_t l = 0; l < m->layers.size(); l++) {
    LayerW& L = m->layers[l];
    __half* kc = kv->k + l * lstride;
    __half* vc = kv->v + l * lstride;
    // --- rmsnorm -> Q|K|V -> bias -> RoPE -> KV-cache write
    bool first_part = true;
    if (batch && (rc = quantize_rows(m, b, b.x, L.rms_att, n, dim, tr))) return rc;
    for (auto& part : L.qkv) {
      for (int c0 = 0; c0 < n; c0 += batch ? n : 8) {
        const int mc = batch ? n : std::min(8, n - c0);
        StreamArgs a = stream_args(m, part.sw, mc, b.x + (size_t)c0 * dim, L.rms_att);
        if (tr && first_part && !batch) tr->site(a, dim);
        QkvMap& q = a.qkv;
        q.nseg = part.nseg;
        for (int s = 0; s <= part.nseg; s++) q.seg_start[s] = part.seg_start[s];
        const float* biases[3] = {L.bq, L.bk, L.bv};
        for (int s = 0; s < part.nseg; s++) {
          q.kind[s] = part.kind[s];
          q.bias[s] = biases[part.kind[s]];
        }
        q.hd = hd;
        q.neox = c.rope_neox;
        q.q_dim = q_dim;
        q.kv_dim = kv_dim;
        q.cos_t = m->rope->cos;
        q.sin_t = m->rope->sin;
        q.pos0 = pos0 + c0;
        q.pos_dev = pos_dev;
        q.cap = (int)kv->positions;
        q.q_out = b.q + (size_t)c0 * q_dim;
        q.kc = kc;
        q.vc = vc;
        if (mode == MODE_WINDOW) {
          q.k_f32 = b.kf + (size_t)c0 * kv_dim;
          q.v_f32 = b.vf + (size_t)c0 * kv_dim;
        }
        if (mu) {
          q.rows = mu->rows_dev + c0;
          q.layer = (int)l;
        }
        if (batch) {
          if ((rc = run_qgemm(m, b, part.sw, n, b.y, 0))) return rc;
          PRANA_CK(launch_qkv_finish(b.y, n, part.sw.w.dw.rows, q, st));
        } else if ((rc = run_stream(m, a, EPI_QKV, PRO_NORM, pdl))) {
          return rc;
        }
      }
      first_part = false;
    }
    // --- attention
    if (mode == MODE_WINDOW) {
      PrefillAttnArgs a{b.q, b.kf, b.vf, n, (int)m->heads_l, (int)m->kv_heads_l, hd, b.att};
      PRANA_CK(launch_attn_prefill(a, st));
    } else {
      // one launch over the rows of one cache, over all sequences, or one per sequence
      cudaError_t es = cudaErrorNotSupported;
      if (mu) {
        AttnArgs a{};
        a.q = b.q;
        a.out = b.att;
        a.m = 1;
        a.n_heads = (int)m->heads_l;
        a.n_kv = (int)m->kv_heads_l;
        a.hd = hd;
        a.n_splits = mu->min_splits;
        a.has_tm = mu->all_tm ? 1 : 0;
        a.err = m->err;
        a.seqs = mu->attn_dev + l * (size_t)n;
        for (int s0 = 0; s0 < n; s0++) a.cap = std::max(a.cap, (int)mu->kvs[s0]->positions);
        es = launch_attn_decode_seqs(a, n, st, pdl);
        if (es != cudaErrorNotSupported) PRANA_CK(es);
      }
      for (int s0 = 0; es == cudaErrorNotSupported && s0 < (mu ? n : 1); s0++) {
        prana_kv* kq = mu ? mu->kvs[s0] : kv;
        const size_t ls = kq->positions * (size_t)kv_dim;
        AttnArgs a{};
        a.q = b.q + (size_t)s0 * q_dim;
        a.kc = mu ? kq->k + l * ls : kc;
        a.vc = mu ? kq->v + l * ls : vc;
        a.m = mu ? 1 : n;
        a.pos0 = mu ? (int)mu->pos[s0] : pos0;
        // a captured multi-sequence step reads each position from its row view
        a.pos_dev = mu ? &(mu->rows_dev + s0)->pos : pos_dev;
        a.n_heads = (int)m->heads_l;
        a.n_kv = (int)m->kv_heads_l;
        a.hd = hd;
        a.n_splits = kq->n_splits;
        a.cap = (int)kq->positions;
        a.part_ml = kq->part_ml;
        a.part_o = kq->part_o;
        a.counters = kq->counters;
        a.out = b.att + (size_t)s0 * q_dim;
        a.err = m->err;
        if ((size_t)l < kq->maps.size()) {
          a.tm_k = kq->maps[l].tm_k;
          a.tm_v = kq->maps[l].tm_v;
          a.has_tm = kq->maps[l].has_tm;
        }
        PRANA_CK(launch_attn_decode(a, st, pdl));
      }
    }
    // --- quantize(attn) -> wo -> residual
    if (batch) {
      if ((rc = quantize_rows(m, b, b.att, nullptr, n, q_dim, tr)) || (rc = run_qgemm(m, b, L.wo, n, b.x, 1)))
        return rc;
    }
    for (int c0 = 0; c0 < n && !batch; c0 += 8) {
      const int mc = std::min(8, n - c0);
      StreamArgs a = stream_args(m, L.wo, mc, b.att + (size_t)c0 * q_dim, nullptr);
      if (tr) tr->site(a, q_dim);
      a.out = b.x + (size_t)c0 * dim;
      if (n <= 8) set_prefetch(a, L.fused_gu ? &L.gu : &L.w1);
      if ((rc = run_stream(m, a, tp && m->tp_rank ? EPI_STORE : EPI_RESID, PRO_F32, pdl))) return rc;
    }
    if (tp && (rc = tp_sum_rows(m, b.x, (size_t)n * dim, st, pdl))) return rc;
    // --- rmsnorm -> gate|up -> silu(gate) * up
    if (batch) {
      if ((rc = quantize_rows(m, b, b.x, L.rms_ffn, n, dim, tr))) return rc;
      if (L.fused_gu) {
        if ((rc = run_qgemm(m, b, L.gu, n, b.y, 0))) return rc;
        PRANA_CK(launch_swiglu_finish(b.y, n, L.gu.w.dw.rows, b.h, st));
      } else {
        if ((rc = run_qgemm(m, b, L.w1, n, b.h, 0)) || (rc = run_qgemm(m, b, L.w3, n, b.u, 0))) return rc;
        PRANA_CK(launch_silu_mul(b.h, b.u, (size_t)n * hid, st));
      }
    }
    for (int c0 = 0; c0 < n && !batch; c0 += 8) {
      const int mc = std::min(8, n - c0);
      if (L.fused_gu) {
        StreamArgs a = stream_args(m, L.gu, mc, b.x + (size_t)c0 * dim, L.rms_ffn);
        if (tr) tr->site(a, dim);
        a.out = b.h + (size_t)c0 * hid;
        if (n <= 8) set_prefetch(a, &L.w2);
        if ((rc = run_stream(m, a, EPI_SWIGLU, PRO_NORM, pdl))) return rc;
      } else {
        StreamArgs a = stream_args(m, L.w1, mc, b.x + (size_t)c0 * dim, L.rms_ffn);
        if (tr) tr->site(a, dim);
        a.out = b.h + (size_t)c0 * hid;
        if ((rc = run_stream(m, a, EPI_STORE, PRO_NORM, pdl))) return rc;
        StreamArgs u = stream_args(m, L.w3, mc, b.x + (size_t)c0 * dim, L.rms_ffn);
        u.out = b.u + (size_t)c0 * hid;
        if ((rc = run_stream(m, u, EPI_STORE, PRO_NORM, pdl))) return rc;
        PRANA_CK(launch_silu_mul(b.h + (size_t)c0 * hid, b.u + (size_t)c0 * hid, (size_t)mc * hid, st));
      }
    }
    // --- quantize(h) -> w2 -> residual
    if (batch) {
      if ((rc = quantize_rows(m, b, b.h, nullptr, n, hid, tr)) || (rc = run_qgemm(m, b, L.w2, n, b.x, 1))) return rc;
    }
    for (int c0 = 0; c0 < n && !batch; c0 += 8) {
      const int mc = std::min(8, n - c0);
      StreamArgs a = stream_args(m, L.w2, mc, b.h + (size_t)c0 * hid, nullptr);
      if (tr) tr->site(a, hid);
      a.out = b.x + (size_t)c0 * dim;
      if (n <= 8) {
        if (l + 1 < m->layers.size())
          set_prefetch(a, &m->layers[l + 1].qkv.front().sw);
        else if (head)
          set_prefetch(a, &m->head);
      }
      if ((rc = run_stream(m, a, tp && m->tp_rank ? EPI_STORE : EPI_RESID, PRO_F32, pdl))) return rc;
    }
    if (tp && (rc = tp_sum_rows(m, b.x, (size_t)n * dim, st, pdl))) return rc;
  }
  if (!head) return PRANA_OK;
  // --- final rmsnorm -> LM head -> argmax (Model::logits, checkpoint.rs:239-248; infer.rs:560-568)
  if (m->head.w.dw.type == T_F32) {  // dense f32 tied classifier: matmul_f32 over the table
    PRANA_CK(launch_rmsnorm(b.x, m->rms_final, n, dim, c.norm_eps, b.xn, st));
    if (tr) {  // the site's rows as the CPU path quantizes them for its own record
      PRANA_CK(launch_quantize_acts(b.xn, n, dim, tr->q + tr->nq, tr->s + tr->ns, b.xsum, st));
      tr->nq += (size_t)n * dim;
      tr->ns += (size_t)n * dim / 32;
    }
    for (int c0 = 0; c0 < n; c0 += 8) {
      GemvArgs gv{};
      gv.w = m->head.w.dw;
      gv.m = std::min(8, n - c0);
      gv.x = b.xn + (size_t)c0 * dim;
      gv.out = b.logits + (size_t)c0 * c.vocab_size;
      PRANA_CK(launch_gemv(gv, PRO_F32, EPI_STORE, st, false));
    }
    PRANA_CK(launch_argmax(b.logits, n, (int)c.vocab_size, b.tok_out, st));
    if (n == 1 && tok_dev)
      PRANA_CK(cudaMemcpyAsync(const_cast<int*>(tok_dev), b.tok_out, 4, cudaMemcpyDeviceToDevice, st));
    return PRANA_OK;
  }
  if (batch) {  // logits_batch (checkpoint.rs:256-265): the head streams once for all rows
    if ((rc = quantize_rows(m, b, b.x, m->rms_final, n, dim, tr)) ||
        (rc = run_qgemm(m, b, m->head, n, b.logits, 0)))
      return rc;
    PRANA_CK(launch_argmax(b.logits, n, (int)c.vocab_size, b.tok_out, st));
    return PRANA_OK;
  }
  for (int c0 = 0; c0 < n; c0 += 8) {
    const int mc = std::min(8, n - c0);
    StreamArgs a = stream_args(m, m->head, mc, b.x + (size_t)c0 * dim, m->rms_final);
    if (tr) tr->site(a, dim);
    a.part_val = m->part_val;
    a.part_idx = m->part_idx;
    a.n_parts = m->n_parts;
    a.counter = m->ctr;
    if (!tp) {
      a.out = b.logits + (size_t)c0 * c.vocab_size;
      a.token_out = b.tok_out + c0;
      a.token_next = (n == 1 && tok_dev) ? const_cast<int*>(tok_dev) : nullptr;
      if ((rc = run_stream(m, a, EPI_ARGMAX, PRO_NORM, pdl))) return rc;
      continue;
    }
    a.out = b.logits_l + (size_t)c0 * m->vocab_l;
    a.idx_offset = (int)m->vocab_off;
    a.best_val = m->tp_local;
    a.token_out = reinterpret_cast<uint32_t*>(m->tp_local + 8);
    if ((rc = run_stream(m, a, EPI_ARGMAX, PRO_NORM, pdl))) return rc;
    if ((rc = tp_gather(m, m->tp_local, m->tp_all, 16, st, pdl))) return rc;
    PRANA_CK(launch_tp_argmax(m->tp_all, m->tp_world, mc, b.tok_out + c0,
                              (n == 1 && tok_dev) ? const_cast<int*>(tok_dev) : nullptr, st));
    if (gather_logits)
      for (int i = 0; i < mc; i++)
        if ((rc = tp_gather(m, b.logits_l + (size_t)(c0 + i) * m->vocab_l, b.logits + (size_t)(c0 + i) * c.vocab_size,
                            (size_t)m->vocab_l, st, false)))
          return rc;
  }
  return PRANA_OK;
}

int check_err(prana_model* m) {
  unsigned e = 0;
  PRANA_CK(cudaMemcpyAsync(&e, m->err, 4, cudaMemcpyDeviceToHost, m->ctx->own));
  PRANA_CK(cudaStreamSynchronize(m->ctx->own));
  if (e) {
    cudaMemsetAsync(m->err, 0, 4, m->ctx->own);
    return fail(PRANA_E_TIMEOUT, "a bounded device-side wait expired (error %u)", e);
  }
  return PRANA_OK;
}

// The error word read back beside a step's token (m->h_tok[1], pinned): one
// synchronization per token instead of check_err's second copy and wait.
static cudaError_t enqueue_err_read(prana_model* m, cudaStream_t st) {
  return cudaMemcpyAsync(m->h_tok + 1, m->err, 4, cudaMemcpyDeviceToHost, st);
}
static int err_after_sync(prana_model* m) {
  const unsigned e = m->h_tok[1];
  if (e) {
    cudaMemsetAsync(m->err, 0, 4, m->ctx->own);
    return fail(PRANA_E_TIMEOUT, "a bounded device-side wait expired (error %u)", e);
  }
  return PRANA_OK;
}

int capture(prana_model* m, prana_kv* kv, bool loop, bool sampled, cudaGraphExec_t* out) {
  cudaStream_t st = m->ctx->own;
  for (int attempt = 0; attempt < 2; attempt++) {
    const bool pdl = m->pdl && attempt == 0;
    cudaGraph_t graph = nullptr;
    PRANA_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
    int rc = enqueue_rows(m, kv, *m->dec, 1, nullptr, m->d_tokpos, 0, m->d_tokpos + 1, MODE_CACHE, true, pdl, nullptr,
                          !loop || sampled);
    if (!rc && sampled) {  // the draw replaces the argmax as the next token
      cudaError_t e = launch_sample(m->dec->logits, (int)m->cfg.vocab_size, m->d_sample, m->dec->tok_out, m->d_tokpos, st);
      if (e != cudaSuccess) rc = fail(PRANA_E_CUDA, "sample launch: %s", cudaGetErrorString(e));
    }
    if (!rc && loop) {
      cudaError_t e = launch_advance(m->d_tokpos, m->d_tokpos + 1, kv->ring, (int)kv->positions, kv->ring_n, st, pdl);
      if (e != cudaSuccess) rc = fail(PRANA_E_CUDA, "advance launch: %s", cudaGetErrorString(e));
    }
    cudaError_t ec = cudaStreamEndCapture(st, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      return rc;
    }
    if (ec == cudaSuccess) {
      cudaError_t ei = cudaGraphInstantiate(out, graph, 0);
      cudaGraphDestroy(graph);
      if (ei == cudaSuccess) return PRANA_OK;
    } else if (graph) {
      cudaGraphDestroy(graph);
    }
    cudaGetLastError();
    m->pdl = false;  // retry once without programmatic dependent launches
  }
  return fail(PRANA_E_CUDA, "decode graph capture failed");
}

int ensure_graphs(prana_model* m, prana_kv* kv, bool loop, bool sampled = false) {
  if (!kv->g_step) {
    int rc = capture(m, kv, false, false, &kv->g_step);
    if (rc) return rc;
  }
  if (loop && !sampled && !kv->g_loop) {
    int rc = capture(m, kv, true, false, &kv->g_loop);
    if (rc) return rc;
  }
  if (loop && sampled && !kv->g_loop_s) {
    int rc = capture(m, kv, true, true, &kv->g_loop_s);
    if (rc) return rc;
  }
  return PRANA_OK;
}

void destroy_kv(prana_kv* kv) {
  if (!kv) return;
  DevScope ds(kv->m->ctx->device);
  cudaStreamSynchronize(kv->m->ctx->own);
  if (kv->m->multi) {
    const auto& ks = kv->m->multi->kvs;
    if (std::find(ks.begin(), ks.end(), kv) != ks.end()) kv->m->multi.reset();
  }
  auto& cs = kv->m->caches;
  cs.erase(std::remove(cs.begin(), cs.end(), kv), cs.end());
  if (kv->g_step) cudaGraphExecDestroy(kv->g_step);
  if (kv->g_loop) cudaGraphExecDestroy(kv->g_loop);
  if (kv->g_loop_s) cudaGraphExecDestroy(kv->g_loop_s);
  prana_ctx* c = kv->m->ctx;
  dev_free(c, kv->k);
  dev_free(c, kv->v);
  dev_free(c, kv->part_ml);
  dev_free(c, kv->counters);
  dev_free(c, kv->ring);
  delete kv;
}

}  // namespace

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

// Load a GGUF model, or one tensor-parallel shard of it (world > 1): this
// rank's query / kv heads, FFN rows and vocabulary rows; wo and ffn_down keep
// this rank's input columns.  nccl_id (NCCL_UNIQUE_ID_BYTES) names the
// communicator every rank joins.
static int load_model(prana_ctx* ctx, const char* path, int world, int rank, const void* nccl_id, int precision,
                      prana_model** out) {
  API_BEGIN
  NEED(ctx && path && out, "null argument");
  NEED(precision == PRANA_PRECISION_F32 || precision == PRANA_PRECISION_Q8, "unknown precision %d", precision);
  NEED(world >= 1 && rank >= 0 && rank < world && (world == 1 || nccl_id), "bad tensor-parallel rank %d of %d", rank,
       world);
  *out = nullptr;
  DevScope ds(ctx->device);
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(PRANA_E_INVALID, "cannot open %s", path);
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
    close(fd);
    return fail(PRANA_E_FORMAT, "cannot stat %s", path);
  }
  void* map = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return fail(PRANA_E_FORMAT, "cannot map %s", path);
  struct Unmap {
    void* p;
    size_t n;
    ~Unmap() { munmap(p, n); }
  } unmap{map, (size_t)sb.st_size};
  Gguf g;
  g.data = static_cast<const uint8_t*>(map);
  g.len = (size_t)sb.st_size;
  int rc = gguf_parse(g);
  if (rc) return rc;

  auto arch_it = g.strs.find("general.architecture");
  if (arch_it == g.strs.end()) return fail(PRANA_E_FORMAT, "missing general.architecture");
  const std::string arch = arch_it->second;
  if (arch != "llama" && arch != "qwen2")
    return fail(PRANA_E_UNSUPPORTED, "unsupported architecture '%s' (llama, qwen2)", arch.c_str());
  auto meta_int = [&](const std::string& k, int64_t* v) -> bool {
    auto it = g.ints.find(arch + "." + k);
    if (it == g.ints.end() || it->second < 0) return false;
    *v = it->second;
    return true;
  };
  auto meta_f = [&](const std::string& k, float dflt) -> float {
    auto it = g.floats.find(arch + "." + k);
    return it == g.floats.end() ? dflt : (float)it->second;
  };
  std::unique_ptr<prana_model, void (*)(prana_model*)> m(new prana_model(), free_model);
  m->ctx = ctx;
  m->precision = precision;
  WeightStreamer ws(ctx, size_t(64) << 20);  // destroyed before m: its copies end first
  auto& c = m->cfg;
  if (!meta_int("embedding_length", &c.dim)) return fail(PRANA_E_FORMAT, "missing metadata '%s.embedding_length'", arch.c_str());
  if (!meta_int("block_count", &c.n_layers)) return fail(PRANA_E_FORMAT, "missing metadata '%s.block_count'", arch.c_str());
  if (!meta_int("attention.head_count", &c.n_heads)) return fail(PRANA_E_FORMAT, "missing metadata '%s.attention.head_count'", arch.c_str());
  if (!meta_int("attention.head_count_kv", &c.n_kv_heads)) c.n_kv_heads = c.n_heads;
  if (!meta_int("feed_forward_length", &c.hidden_dim)) return fail(PRANA_E_FORMAT, "missing metadata '%s.feed_forward_length'", arch.c_str());
  if (!meta_int("context_length", &c.seq_len)) return fail(PRANA_E_FORMAT, "missing metadata '%s.context_length'", arch.c_str());
  c.rope_theta = meta_f("rope.freq_base", 10000.0f);
  if (!meta_int("attention.key_length", &c.head_dim)) c.head_dim = c.n_heads ? c.dim / c.n_heads : 0;
  c.norm_eps = meta_f("attention.layer_norm_rms_epsilon", 1e-5f);
  c.rope_neox = arch != "llama";
  auto vt = g.arr_len.find("tokenizer.ggml.tokens");
  if (vt == g.arr_len.end()) return fail(PRANA_E_FORMAT, "missing tokenizer.ggml.tokens");
  c.vocab_size = (int64_t)vt->second;
  NEED(c.dim > 0 && c.n_layers > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.n_heads % c.n_kv_heads == 0,
       "inconsistent model metadata");
  NEED(c.head_dim > 0 && c.head_dim % 2 == 0 && c.head_dim <= 256, "head_dim %lld not supported", (long long)c.head_dim);
  NEED(c.dim % 32 == 0 && c.hidden_dim % 32 == 0, "dim and hidden must be multiples of 32");
  const size_t dim = (size_t)c.dim, hid = (size_t)c.hidden_dim, q_dim = (size_t)(c.n_heads * c.head_dim),
               kv_dim = (size_t)(c.n_kv_heads * c.head_dim);
  NEED(q_dim % 32 == 0, "q_dim must be a multiple of 32");
  NEED(world == 1 || (c.n_kv_heads % world == 0 && c.hidden_dim % world == 0 && c.vocab_size % world == 0),
       "tensor parallel over %d ranks needs kv heads, FFN width and vocabulary divisible by it", world);
  m->tp_world = world;
  m->tp_rank = rank;
  m->heads_l = c.n_heads / world;
  m->kv_heads_l = c.n_kv_heads / world;
  m->hid_l = c.hidden_dim / world;
  m->vocab_l = c.vocab_size / world;
  m->vocab_off = (int64_t)rank * m->vocab_l;
  const size_t q_dim_l = (size_t)(m->heads_l * c.head_dim), kv_dim_l = (size_t)(m->kv_heads_l * c.head_dim),
               hid_l = (size_t)m->hid_l;

  // token embedding (gguf.rs:309-326)
  {
    const GgufTensor* t;
    const uint8_t* raw;
    rc = tensor_raw(g, "token_embd.weight", &t, &raw);
    if (rc) return rc;
    uint64_t nv = 1;
    for (auto d : t->dims) nv *= d;
    if (nv != (uint64_t)c.vocab_size * dim) return fail(PRANA_E_FORMAT, "token_embd.weight size mismatch with vocab");
    rc = ws.upload((int)t->type, (size_t)c.vocab_size, dim, linear_rows(raw, gguf_row_bytes(t->type, dim)), &m->emb);
    if (rc) return rc;
  }
  m->layers.resize((size_t)c.n_layers);
  const size_t half = (size_t)c.head_dim / 2;
  for (size_t i = 0; i < m->layers.size(); i++) {
    LayerW& L = m->layers[i];
    const std::string p = "blk." + std::to_string(i) + ".";
    std::vector<float> v;
    if ((rc = vec_f32(g, p + "attn_norm.weight", dim, v)) || (rc = dev_vec(m.get(), v, &L.rms_att))) return rc;
    if ((rc = vec_f32(g, p + "ffn_norm.weight", dim, v)) || (rc = dev_vec(m.get(), v, &L.rms_ffn))) return rc;
    // Q|K|V: concatenate runs of one weight type; RoPE partners become adjacent rows
    const char* names[3] = {"attn_q.weight", "attn_k.weight", "attn_v.weight"};
    const size_t full_rows[3] = {q_dim, kv_dim, kv_dim};
    const size_t seg_rows[3] = {q_dim_l, kv_dim_l, kv_dim_l};  // this rank's heads
    uint32_t types[3];
    const uint8_t* raws[3];
    for (int s = 0; s < 3; s++) {
      if ((rc = linear_raw(g, p + names[s], full_rows[s], dim, &types[s], &raws[s], precision))) return rc;
      raws[s] += (size_t)rank * seg_rows[s] * gguf_row_bytes(types[s], dim);
    }
    for (int s0 = 0; s0 < 3;) {
      int s1 = s0 + 1;
      while (s1 < 3 && types[s1] == types[s0]) s1++;
      const size_t rb = gguf_row_bytes(types[s0], dim);
      std::vector<const uint8_t*> rows;  // stored row -> GGUF row
      QkvPart part;
      part.nseg = s1 - s0;
      for (int s = s0; s < s1; s++) {
        part.seg_start[s - s0] = (int)rows.size();
        part.kind[s - s0] = s;
        for (size_t pp = 0; pp < seg_rows[s] / 2; pp++) {
          size_t ra = 2 * pp, rbw = 2 * pp + 1;
          if (s != 2 && c.rope_neox) {
            ra = (pp / half) * (size_t)c.head_dim + pp % half;
            rbw = ra + half;
          }
          rows.push_back(raws[s] + ra * rb);
          rows.push_back(raws[s] + rbw * rb);
        }
      }
      part.seg_start[part.nseg] = (int)rows.size();
      L.qkv.push_back(part);
      if ((rc = upload_stream(m.get(), ws, types[s0], rows.size(), dim, [&rows](size_t r) { return rows[r]; },
                              &L.qkv.back().sw)))
        return rc;
      s0 = s1;
    }
    uint32_t ty;
    const uint8_t* raw;
    RowSrc cols;
    if ((rc = linear_raw(g, p + "attn_output.weight", dim, q_dim, &ty, &raw, precision)) ||
        (rc = col_rows(ty, q_dim, raw, rank * q_dim_l, (rank + 1) * q_dim_l, &cols)) ||
        (rc = upload_stream(m.get(), ws, ty, dim, q_dim_l, cols, &L.wo)))
      return rc;
    // gate|up: interleave rows (gate j, up j) when both have one type
    uint32_t t1, t3;
    const uint8_t *r1, *r3;
    if ((rc = linear_raw(g, p + "ffn_gate.weight", hid, dim, &t1, &r1, precision)) ||
        (rc = linear_raw(g, p + "ffn_up.weight", hid, dim, &t3, &r3, precision)))
      return rc;
    r1 += (size_t)rank * hid_l * gguf_row_bytes(t1, dim);  // this rank's FFN rows
    r3 += (size_t)rank * hid_l * gguf_row_bytes(t3, dim);
    if (t1 == t3) {
      const size_t rb = gguf_row_bytes(t1, dim);
      L.fused_gu = true;
      const RowSrc gu = [r1, r3, rb](size_t r) { return (r & 1 ? r3 : r1) + (r >> 1) * rb; };
      if ((rc = upload_stream(m.get(), ws, t1, 2 * hid_l, dim, gu, &L.gu))) return rc;
    } else {
      if ((rc = upload_stream(m.get(), ws, t1, hid_l, dim, linear_rows(r1, gguf_row_bytes(t1, dim)), &L.w1)) ||
          (rc = upload_stream(m.get(), ws, t3, hid_l, dim, linear_rows(r3, gguf_row_bytes(t3, dim)), &L.w3)))
        return rc;
    }
    if ((rc = linear_raw(g, p + "ffn_down.weight", dim, hid, &ty, &raw, precision)) ||
        (rc = col_rows(ty, hid, raw, rank * hid_l, (rank + 1) * hid_l, &cols)) ||
        (rc = upload_stream(m.get(), ws, ty, dim, hid_l, cols, &L.w2)))
      return rc;
    // gguf.rs:388-394: each bias optional
    const char* bn[3] = {"attn_q.bias", "attn_k.bias", "attn_v.bias"};
    float** bd[3] = {&L.bq, &L.bk, &L.bv};
    const size_t bl[3] = {q_dim, kv_dim, kv_dim}, bl_l[3] = {q_dim_l, kv_dim_l, kv_dim_l};
    for (int j = 0; j < 3; j++)
      if (g.tensors.count(p + bn[j])) {
        if ((rc = vec_f32(g, p + bn[j], bl[j], v))) return rc;
        std::vector<float> local(v.begin() + (size_t)rank * bl_l[j], v.begin() + (size_t)(rank + 1) * bl_l[j]);
        if ((rc = dev_vec(m.get(), local, bd[j]))) return rc;
        c.has_bias = 1;
      }
  }
  {
    std::vector<float> v;
    if ((rc = vec_f32(g, "output_norm.weight", dim, v)) || (rc = dev_vec(m.get(), v, &m->rms_final))) return rc;
  }
  if (g.tensors.count("output.weight")) {
    uint32_t ty;
    const uint8_t* raw;
    if ((rc = linear_raw(g, "output.weight", (size_t)c.vocab_size, dim, &ty, &raw, precision))) return rc;
    raw += (size_t)m->vocab_off * gguf_row_bytes(ty, dim);  // this rank's vocabulary rows
    if ((rc = upload_stream(m.get(), ws, ty, (size_t)m->vocab_l, dim, linear_rows(raw, gguf_row_bytes(ty, dim)),
                            &m->head)))
      return rc;
  } else {
    // tied classifier (gguf.rs:425-437, checkpoint.rs:239-248): a packed table
    // (Q4_0 / Q4_K / Q6_K) runs the quantized kernel over the table itself; a
    // table the reference densifies (F32, F16, Q8_0) becomes quantize_q8 of it
    // under Q8 precision, else the dense f32 head (matmul_f32)
    c.shared_classifier = 1;
    const int et = m->emb.dw.type;
    const GgufTensor* t;
    const uint8_t* raw;
    if ((rc = tensor_raw(g, "token_embd.weight", &t, &raw))) return rc;
    raw += (size_t)m->vocab_off * gguf_row_bytes(t->type, dim);
    if (et == T_Q4_0 || et == T_Q4_K || et == T_Q6_K) {
      if (world == 1) {
        m->head.w = m->emb;
        m->head.owns = false;
      } else if ((rc = upload_stream(m.get(), ws, t->type, (size_t)m->vocab_l, dim,
                                     linear_rows(raw, gguf_row_bytes(t->type, dim)), &m->head))) {
        return rc;
      }
    } else {
      const std::vector<float> f = densify(t->type, (size_t)m->vocab_l, dim, raw);
      if (precision == PRANA_PRECISION_Q8 && dim % 32 == 0) {
        if ((rc = upload_q8s(ctx, (size_t)m->vocab_l, dim, f.data(), &m->head.w))) return rc;
      } else {
        NEED(world == 1, "the dense f32 tied classifier runs on a single-GPU model");
        NEED(dim * 8 * 4 <= 200 * 1024, "dense f32 classifier: dim %zu too wide for the f32 GEMV", dim);
        if ((rc = ws.upload(T_F32, (size_t)m->vocab_l, dim, linear_rows(reinterpret_cast<const uint8_t*>(f.data()), dim * 4),
                            &m->head.w)))
          return rc;
      }
    }
  }
  if ((rc = ws.finish())) return rc;
  // weight bytes on the device
  size_t wb = m->emb.bytes + (m->head.owns ? m->head.w.bytes : 0);
  for (auto& L : m->layers) {
    for (auto& q : L.qkv) wb += q.sw.w.bytes;
    wb += L.wo.w.bytes + L.gu.w.bytes + L.w1.w.bytes + L.w3.w.bytes + L.w2.w.bytes;
  }
  c.weight_bytes = (int64_t)wb;
  // RoPE table over the whole context (never regrown: graphs hold its address)
  rc = ctx_rope(ctx, (int)c.head_dim, c.rope_theta, c.rope_neox, (int)c.seq_len + 8, &m->rope);
  if (rc) return rc;
  // decode buffers, argmax partials, counters, error flag
  m->dec.reset(new Bufs(ctx));
  if ((rc = make_bufs(m.get(), 8, false, *m->dec))) return rc;
  m->n_parts = 1024;
  void* p = nullptr;
  if ((rc = dev_alloc(ctx, (size_t)8 * m->n_parts * 8, &p))) return rc;
  m->owned.push_back(p);
  m->part_val = static_cast<float*>(p);
  m->part_idx = reinterpret_cast<int*>(static_cast<float*>(p) + (size_t)8 * m->n_parts);
  if ((rc = dev_alloc(ctx, 256, &p))) return rc;
  m->owned.push_back(p);
  PRANA_CK(cudaMemset(p, 0, 256));
  m->ctr = static_cast<unsigned*>(p);
  m->err = m->ctr + 4;
  m->d_tokpos = reinterpret_cast<int*>(static_cast<uint8_t*>(p) + 64);
  m->d_sample = reinterpret_cast<SampleState*>(static_cast<uint8_t*>(p) + 128);
  PRANA_CK(cudaHostAlloc((void**)&m->h_io, 64, cudaHostAllocDefault));
  m->h_tok = reinterpret_cast<uint32_t*>(m->h_io + 4);
  if (world > 1) {
    if ((rc = dev_alloc(ctx, (size_t)(world + 1) * 16 * 4, &p))) return rc;
    m->owned.push_back(p);
    m->tp_local = static_cast<float*>(p);
    m->tp_all = m->tp_local + 16;
    const char* why = nullptr;
    const Nccl* api = nccl(&why);
    if (!api) return fail(PRANA_E_COMM, "%s", why);
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    const ncclResult_t r = api->comm_init_rank(&m->comm, world, id, rank);
    if (r != ncclSuccess) return fail(PRANA_E_COMM, "ncclCommInitRank: %s", api->error_string(r));
    // peer-memory all-reduce for up to 8 rows of the residual stream (NCCL otherwise)
    const char* mode = getenv("PRANA_TP_ALLREDUCE");
    if (!(mode && !strcmp(mode, "nccl")))
      m->peers_ok = tp_peers_setup(m->comm, world, rank, 8 * dim, ctx->own, &m->peers, &m->peers_mem);
  }
  const char* e = getenv("PRANA_PDL");
  m->pdl = !(e && e[0] == '0');
  *out = m.release();
  return PRANA_OK;
  API_END
}

int prana_model_load_gguf(prana_ctx* ctx, const char* path, prana_model** out) {
  return load_model(ctx, path, 1, 0, nullptr, PRANA_PRECISION_F32, out);
}

int prana_model_load_gguf_ex(prana_ctx* ctx, const char* path, int precision, prana_model** out) {
  return load_model(ctx, path, 1, 0, nullptr, precision, out);
}

int prana_model_load_gguf_tp(prana_ctx* ctx, const char* path, int world, int rank, const void* nccl_id,
                             prana_model** out) {
  return load_model(ctx, path, world, rank, nccl_id, PRANA_PRECISION_F32, out);
}

int prana_tp_unique_id(void* out) {
  NEED(out, "null argument");
  const char* why = nullptr;
  const Nccl* api = nccl(&why);
  if (!api) return fail(PRANA_E_COMM, "%s", why);
  ncclUniqueId id;
  const ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return fail(PRANA_E_COMM, "ncclGetUniqueId: %s", api->error_string(r));
  memcpy(out, &id, sizeof(id));
  return PRANA_OK;
}

int prana_model_tp_get(const prana_model* m, int* world, int* rank, int* peer_exchange) {
  NEED(m && world && rank, "null argument");
  *world = m->tp_world;
  *rank = m->tp_rank;
  if (peer_exchange) *peer_exchange = m->peers_ok ? 1 : 0;
  return PRANA_OK;
}

int prana_model_free(prana_model* m) {
  free_model(m);
  return PRANA_OK;
}

int prana_model_config_get(const prana_model* m, prana_model_config* out) {
  NEED(m && out, "null argument");
  *out = m->cfg;
  return PRANA_OK;
}

int prana_kv_create(prana_model* m, size_t positions, prana_kv** out) {
  API_BEGIN
  NEED(m && out, "null argument");
  *out = nullptr;
  DevScope ds(m->ctx->device);
  const auto& c = m->cfg;
  if (positions > (size_t)c.seq_len) positions = (size_t)c.seq_len;
  NEED(positions > 0, "kv cache needs at least one position");
  std::unique_ptr<prana_kv, void (*)(prana_kv*)> kv(new prana_kv(), destroy_kv);
  kv->m = m;
  kv->positions = positions;
  const size_t kv_dim = (size_t)(m->kv_heads_l * c.head_dim);
  const size_t per = (size_t)c.n_layers * positions * kv_dim;
  {
    void *pk = nullptr, *pv = nullptr;
    int rc = dev_alloc(m->ctx, per * 2, &pk);
    kv->k = static_cast<__half*>(pk);
    if (!rc) rc = dev_alloc(m->ctx, per * 2, &pv);
    kv->v = static_cast<__half*>(pv);
    if (rc) return fail(PRANA_E_OOM, "kv cache allocation (%zu bytes) failed", per * 4);
  }
  PRANA_CK(cudaMemset(kv->k, 0, per * 2));
  PRANA_CK(cudaMemset(kv->v, 0, per * 2));
  // TMA views of every layer's K and V cache for the decode attention
  kv->maps.resize(c.n_layers);
  for (size_t l = 0; l < c.n_layers; l++) {
    AttnArgs& t = kv->maps[l];
    t.kc = kv->k + l * positions * kv_dim;
    t.vc = kv->v + l * positions * kv_dim;
    t.n_kv = (int)m->kv_heads_l;
    t.hd = (int)c.head_dim;
    attn_make_maps(t, (int)positions);
  }
  // attention splits for this capacity (the decode graph keeps them as the cache fills)
  kv->n_splits = attn_splits((int)positions, (int)m->kv_heads_l, (int)c.head_dim, m->ctx->sm_count);
  const int group = (int)(c.n_heads / c.n_kv_heads);
  const int rows_cta = std::max(1, 4096 / (int)(c.head_dim * group));
  const size_t vh = (size_t)rows_cta * group;  // largest row chunk one attention CTA takes
  const size_t ml = ((size_t)m->kv_heads_l * kv->n_splits * vh * 2 + 3) / 4 * 4;  // part_o 16-byte aligned
  const size_t po = (size_t)m->kv_heads_l * kv->n_splits * vh * c.head_dim;
  {
    void *pm = nullptr, *pc = nullptr, *pr = nullptr;
    int rc = dev_alloc(m->ctx, (ml + po) * 4, &pm);
    kv->part_ml = static_cast<float*>(pm);
    if (!rc) rc = dev_alloc(m->ctx, 1024 * sizeof(unsigned), &pc);
    kv->counters = static_cast<unsigned*>(pc);
    if (!rc) rc = dev_alloc(m->ctx, (positions + 64) * sizeof(uint32_t), &pr);
    kv->ring = static_cast<uint32_t*>(pr);
    if (rc) return rc;
  }
  kv->part_o = kv->part_ml + ml;
  PRANA_CK(cudaMemset(kv->counters, 0, 1024 * sizeof(unsigned)));
  kv->ring_n = reinterpret_cast<int*>(kv->ring + positions + 32);
  m->caches.push_back(kv.get());
  *out = kv.release();
  return PRANA_OK;
  API_END
}

int prana_kv_free(prana_kv* kv) {
  destroy_kv(kv);
  return PRANA_OK;
}

int prana_kv_read_rows(prana_kv* kv, size_t layer, int is_v, size_t first, size_t rows, uint16_t* host) {
  NEED(kv && host, "null argument");
  const auto& c = kv->m->cfg;
  NEED(layer < (size_t)c.n_layers && first <= kv->positions && rows <= kv->positions - first,
       "layer/rows out of range");
  DevScope ds(kv->m->ctx->device);
  const size_t kv_dim = (size_t)(kv->m->kv_heads_l * c.head_dim);  // this rank's kv heads
  const __half* base = (is_v ? kv->v : kv->k) + layer * kv->positions * kv_dim + first * kv_dim;
  PRANA_CK(cudaStreamSynchronize(kv->m->ctx->own));
  PRANA_CK(cudaMemcpy(host, base, rows * kv_dim * 2, cudaMemcpyDeviceToHost));
  return PRANA_OK;
}

int prana_kv_read(prana_kv* kv, size_t layer, int is_v, size_t rows, uint16_t* host) {
  return prana_kv_read_rows(kv, layer, is_v, 0, rows, host);
}

int prana_forward(prana_model* m, prana_kv* kv, uint32_t token, size_t pos, float* logits, uint32_t* next) {
  API_BEGIN
  NEED(m && kv && kv->m == m, "null or mismatched argument");
  NEED(pos < kv->positions, "position %zu beyond kv capacity %zu", pos, kv->positions);
  NEED(token < (uint64_t)m->cfg.vocab_size, "token %u out of vocabulary", token);
  DevScope ds(m->ctx->device);
  int rc = ensure_graphs(m, kv, false);
  if (rc) return rc;
  cudaStream_t st = m->ctx->own;
  m->h_io[0] = (int)token;
  m->h_io[1] = (int)pos;
  PRANA_CK(cudaMemcpyAsync(m->d_tokpos, m->h_io, 8, cudaMemcpyHostToDevice, st));
  PRANA_CK(cudaGraphLaunch(kv->g_step, st));
  PRANA_CK(cudaMemcpyAsync(m->h_tok, m->dec->tok_out, 4, cudaMemcpyDeviceToHost, st));
  PRANA_CK(enqueue_err_read(m, st));
  if (logits) PRANA_CK(cudaMemcpyAsync(logits, m->dec->logits, (size_t)m->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, st));
  PRANA_CK(cudaStreamSynchronize(st));
  if (next) *next = m->h_tok[0];
  kv->loop_active = false;
  return err_after_sync(m);
  API_END
}

int prana_forward_sampled(prana_model* m, prana_kv* kv, uint32_t token, size_t pos, prana_sampler* s,
                          uint32_t* next) {
  API_BEGIN
  NEED(m && kv && kv->m == m && s && next, "null or mismatched argument");
  if (s->greedy) return prana_forward(m, kv, token, pos, nullptr, next);
  NEED(pos < kv->positions, "position %zu beyond kv capacity %zu", pos, kv->positions);
  NEED(token < (uint64_t)m->cfg.vocab_size, "token %u out of vocabulary", token);
  NEED(m->cfg.vocab_size <= sample_max_vocab(), "vocabulary of %lld exceeds the device sampler's %d",
       (long long)m->cfg.vocab_size, sample_max_vocab());
  DevScope ds(m->ctx->device);
  int rc = ensure_graphs(m, kv, false);
  if (rc) return rc;
  cudaStream_t st = m->ctx->own;
  m->h_io[0] = (int)token;
  m->h_io[1] = (int)pos;
  SampleState* h = reinterpret_cast<SampleState*>(m->h_io + 8);
  *h = SampleState{s->state, s->temp, 0};
  PRANA_CK(cudaMemcpyAsync(m->d_tokpos, m->h_io, 8, cudaMemcpyHostToDevice, st));
  PRANA_CK(cudaMemcpyAsync(m->d_sample, h, sizeof(SampleState), cudaMemcpyHostToDevice, st));
  PRANA_CK(cudaGraphLaunch(kv->g_step, st));  // the step leaves the whole logits row in HBM
  PRANA_CK(launch_sample(m->dec->logits, (int)m->cfg.vocab_size, m->d_sample, m->dec->tok_out, nullptr, st));
  PRANA_CK(cudaMemcpyAsync(m->h_tok, m->dec->tok_out, 4, cudaMemcpyDeviceToHost, st));
  PRANA_CK(enqueue_err_read(m, st));
  PRANA_CK(cudaStreamSynchronize(st));
  *next = m->h_tok[0];
  s->next_u64();  // the draw the kernel took
  kv->loop_active = false;
  return err_after_sync(m);
  API_END
}

int prana_forward_trace(prana_model* m, prana_kv* kv, uint32_t token, size_t pos, float* logits, int8_t* q_host,
                        float* s_host, size_t cap, size_t* n_out) {
  API_BEGIN
  NEED(m && kv && kv->m == m && q_host && s_host && n_out, "null or mismatched argument");
  NEED(pos < kv->positions, "position %zu beyond kv capacity %zu", pos, kv->positions);
  NEED(token < (uint64_t)m->cfg.vocab_size, "token %u out of vocabulary", token);
  const auto& c = m->cfg;
  const size_t need = (size_t)c.n_layers * (2 * c.dim + c.n_heads * c.head_dim + c.hidden_dim) + c.dim;
  NEED(cap >= need, "trace buffer holds %zu values, %zu needed", cap, need);
  NEED(m->tp_world == 1, "forward_trace runs on a single-GPU model");
  DevScope ds(m->ctx->device);
  cudaStream_t st = m->ctx->own;
  Trace tr;
  PRANA_CK(cudaMalloc(&tr.q, need));
  PRANA_CK(cudaMalloc(&tr.s, need / 32 * 4 + 4));
  struct Free {
    Trace& t;
    ~Free() {
      cudaFree(t.q);
      cudaFree(t.s);
    }
  } fr{tr};
  uint32_t* tok_d = m->dec->toks;
  PRANA_CK(cudaMemcpyAsync(tok_d, &token, 4, cudaMemcpyHostToDevice, st));
  int rc = enqueue_rows(m, kv, *m->dec, 1, tok_d, nullptr, (int)pos, nullptr, MODE_CACHE, true, false, &tr);
  if (rc) return rc;
  PRANA_CK(cudaMemcpyAsync(q_host, tr.q, tr.nq, cudaMemcpyDeviceToHost, st));
  PRANA_CK(cudaMemcpyAsync(s_host, tr.s, tr.ns * 4, cudaMemcpyDeviceToHost, st));
  if (logits) PRANA_CK(cudaMemcpyAsync(logits, m->dec->logits, (size_t)c.vocab_size * 4, cudaMemcpyDeviceToHost, st));
  PRANA_CK(cudaStreamSynchronize(st));
  *n_out = tr.nq;
  kv->loop_active = false;
  return check_err(m);
  API_END
}

int prana_forward_batch_trace(prana_model* m, prana_kv* kv, const uint32_t* tokens, size_t n, size_t pos0,
                              int prefill, float* logits, int8_t* q_host, float* s_host, size_t cap, size_t* n_out) {
  API_BEGIN
  NEED(m && kv && kv->m == m && tokens && q_host && s_host && n_out, "null or mismatched argument");
  NEED(n > 0, "empty batch");
  NEED(m->tp_world == 1, "forward_batch_trace runs on a single-GPU model");
  if (prefill) pos0 = 0;
  NEED(pos0 + n <= kv->positions, "rows %zu..%zu beyond kv capacity %zu", pos0, pos0 + n, kv->positions);
  for (size_t i = 0; i < n; i++) NEED(tokens[i] < (uint64_t)m->cfg.vocab_size, "token out of vocabulary");
  const auto& c = m->cfg;
  const size_t need =
      n * ((size_t)c.n_layers * (2 * c.dim + c.n_heads * c.head_dim + c.hidden_dim) + (prefill ? 0 : c.dim));
  NEED(cap >= need, "trace buffer holds %zu values, %zu needed", cap, need);
  DevScope ds(m->ctx->device);
  cudaStream_t st = m->ctx->own;
  Bufs b(m->ctx);
  int rc = make_bufs(m, n, prefill != 0, b);
  if (rc) return rc;
  Trace tr;
  PRANA_CK(cudaMalloc(&tr.q, need));
  PRANA_CK(cudaMalloc(&tr.s, need / 32 * 4 + 4));
  struct Free {
    Trace& t;
    ~Free() {
      cudaFree(t.q);
      cudaFree(t.s);
    }
  } fr{tr};
  PRANA_CK(cudaMemcpyAsync(b.toks, tokens, n * 4, cudaMemcpyHostToDevice, st));
  rc = enqueue_rows(m, kv, b, (int)n, b.toks, nullptr, (int)pos0, nullptr, prefill ? MODE_WINDOW : MODE_CACHE,
                    !prefill, false, &tr);
  if (rc) return rc;
  if (tr.nq != need) return fail(PRANA_E_INVALID, "trace recorded %zu values, expected %zu", tr.nq, need);
  PRANA_CK(cudaMemcpyAsync(q_host, tr.q, tr.nq, cudaMemcpyDeviceToHost, st));
  PRANA_CK(cudaMemcpyAsync(s_host, tr.s, tr.ns * 4, cudaMemcpyDeviceToHost, st));
  if (logits && !prefill)
    PRANA_CK(cudaMemcpyAsync(logits, b.logits, n * (size_t)c.vocab_size * 4, cudaMemcpyDeviceToHost, st));
  PRANA_CK(cudaStreamSynchronize(st));
  *n_out = tr.nq;
  kv->loop_active = false;
  return check_err(m);
  API_END
}

int prana_kv_write(prana_kv* kv, size_t layer, int is_v, size_t rows, const uint16_t* host) {
  NEED(kv && host, "null argument");
  const auto& c = kv->m->cfg;
  NEED(layer < (size_t)c.n_layers && rows <= kv->positions, "layer/rows out of range");
  DevScope ds(kv->m->ctx->device);
  const size_t kv_dim = (size_t)(kv->m->kv_heads_l * c.head_dim);  // this rank's kv heads
  __half* base = (is_v ? kv->v : kv->k) + layer * kv->positions * kv_dim;
  PRANA_CK(cudaStreamSynchronize(kv->m->ctx->own));
  PRANA_CK(cudaMemcpy(base, host, rows * kv_dim * 2, cudaMemcpyHostToDevice));
  return PRANA_OK;
}

int prana_prefill(prana_model* m, prana_kv* kv, const uint32_t* tokens, size_t n) {
  API_BEGIN
  NEED(m && kv && kv->m == m && tokens, "null or mismatched argument");
  if (!n) return PRANA_OK;
  NEED(n <= kv->positions, "prefill of %zu tokens beyond kv capacity %zu", n, kv->positions);
  for (size_t i = 0; i < n; i++) NEED(tokens[i] < (uint64_t)m->cfg.vocab_size, "token out of vocabulary");
  DevScope ds(m->ctx->device);
  Bufs b(m->ctx);
  int rc = make_bufs(m, n, true, b);
  if (rc) return rc;
  cudaStream_t st = m->ctx->own;
  PRANA_CK(cudaMemcpyAsync(b.toks, tokens, n * 4, cudaMemcpyHostToDevice, st));
  rc = enqueue_rows(m, kv, b, (int)n, b.toks, nullptr, 0, nullptr, MODE_WINDOW, false, false);
  if (rc) return rc;
  PRANA_CK(cudaStreamSynchronize(st));
  kv->loop_active = false;
  return check_err(m);
  API_END
}

int prana_forward_batch(prana_model* m, prana_kv* kv, const uint32_t* tokens, size_t n, size_t pos0, float* logits,
                        uint32_t* argmax) {
  API_BEGIN
  NEED(m && kv && kv->m == m && tokens, "null or mismatched argument");
  if (!n) return PRANA_OK;
  NEED(pos0 + n <= kv->positions, "rows %zu..%zu beyond kv capacity %zu", pos0, pos0 + n, kv->positions);
  for (size_t i = 0; i < n; i++) NEED(tokens[i] < (uint64_t)m->cfg.vocab_size, "token out of vocabulary");
  DevScope ds(m->ctx->device);
  cudaStream_t st = m->ctx->own;
  std::unique_ptr<Bufs> tmp;
  Bufs* b = m->dec.get();
  if (n > b->rows) {
    tmp.reset(new Bufs(m->ctx));
    int rc = make_bufs(m, n, false, *tmp);
    if (rc) return rc;
    b = tmp.get();
  }
  PRANA_CK(cudaMemcpyAsync(b->toks, tokens, n * 4, cudaMemcpyHostToDevice, st));
  int rc = enqueue_rows(m, kv, *b, (int)n, b->toks, nullptr, (int)pos0, nullptr, MODE_CACHE, true, false, nullptr,
                        logits != nullptr);
  if (rc) return rc;
  if (logits) PRANA_CK(cudaMemcpyAsync(logits, b->logits, n * (size_t)m->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, st));
  if (argmax) PRANA_CK(cudaMemcpyAsync(argmax, b->tok_out, n * 4, cudaMemcpyDeviceToHost, st));
  PRANA_CK(cudaStreamSynchronize(st));
  kv->loop_active = false;
  return check_err(m);
  API_END
}

static int forward_multi_impl(prana_model* m, prana_kv* const* kvs, size_t n, const uint32_t* tokens,
                              const size_t* positions, float* logits, uint32_t* argmax, Trace* tr) {
  API_BEGIN
  NEED(m && kvs && tokens && positions, "null argument");
  if (!n) return PRANA_OK;
  NEED(m->tp_world == 1, "multi-sequence decode runs on a single-GPU model");
  const size_t kv_dim = (size_t)(m->kv_heads_l * m->cfg.head_dim);
  std::vector<SeqRow> rows(n);
  for (size_t i = 0; i < n; i++) {
    NEED(kvs[i] && kvs[i]->m == m, "cache %zu is null or of another model", i);
    NEED(positions[i] < kvs[i]->positions, "sequence %zu: position %zu beyond kv capacity %zu", i, positions[i],
         kvs[i]->positions);
    NEED(tokens[i] < (uint64_t)m->cfg.vocab_size, "token out of vocabulary");
    for (size_t j = 0; j < i; j++) NEED(kvs[j] != kvs[i], "sequences %zu and %zu share a cache", j, i);
    rows[i] = SeqRow{kvs[i]->k, kvs[i]->v, kvs[i]->positions * kv_dim, (int)positions[i], (int)kvs[i]->positions};
  }
  DevScope ds(m->ctx->device);
  cudaStream_t st = m->ctx->own;
  // per layer and sequence: the cache's tensor maps, scratch and position
  const size_t nl = m->layers.size();
  std::vector<AttnSeq> att(nl * n);
  int min_splits = INT_MAX;
  bool all_tm = true;
  for (size_t i = 0; i < n; i++) {
    prana_kv* kq = kvs[i];
    min_splits = std::min(min_splits, kq->n_splits);
    for (size_t l = 0; l < nl; l++) {
      AttnSeq& q = att[l * n + i];
      q = AttnSeq{};
      const size_t ls = kq->positions * kv_dim;
      q.kc = kq->k + l * ls;
      q.vc = kq->v + l * ls;
      q.part_ml = kq->part_ml;
      q.part_o = kq->part_o;
      q.counters = kq->counters;
      q.pos0 = (int)positions[i];
      if (l < kq->maps.size() && kq->maps[l].has_tm) {
        q.tm_k = kq->maps[l].tm_k;
        q.tm_v = kq->maps[l].tm_v;
      } else {
        all_tm = false;
      }
    }
  }
  if (!tr) {
    // ---- the captured step: build it once for this ordered set of caches
    MultiPlan* pl = m->multi.get();
    if (!pl || pl->kvs.size() != n || !std::equal(pl->kvs.begin(), pl->kvs.end(), kvs)) {
      m->multi.reset();
      std::unique_ptr<MultiPlan> np(new MultiPlan(m->ctx));
      np->kvs.assign(kvs, kvs + n);
      Bufs& nb = *np->bufs;
      int rc = make_bufs(m, std::max<size_t>(n, 8), false, nb);
      if (!rc) rc = nb.alloc(np->rows_dev, n);
      if (!rc) rc = nb.alloc(np->att_dev, att.size());
      if (!rc) rc = nb.alloc(np->pos_dev, n);
      if (rc) return rc;
      PRANA_CK(cudaHostAlloc((void**)&np->h_stage, 2 * n * sizeof(uint32_t), cudaHostAllocDefault));
      PRANA_CK(cudaMemcpyAsync(np->rows_dev, rows.data(), n * sizeof(SeqRow), cudaMemcpyHostToDevice, st));
      PRANA_CK(cudaMemcpyAsync(np->att_dev, att.data(), att.size() * sizeof(AttnSeq), cudaMemcpyHostToDevice, st));
      PRANA_CK(cudaStreamSynchronize(st));
      const Multi mu{np->rows_dev, np->kvs.data(), positions, np->att_dev, min_splits, all_tm};
      for (int attempt = 0; attempt < 2 && !np->graph; attempt++) {
        const bool pdl = m->pdl && attempt == 0;
        cudaGraph_t graph = nullptr;
        PRANA_CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
        multi_positions_kernel<<<1, 256, 0, st>>>(np->pos_dev, (int)n, (int)att.size(), np->rows_dev, np->att_dev);
        cudaError_t el = cudaGetLastError();
        rc = el == cudaSuccess ? enqueue_rows(m, kvs[0], nb, (int)n, nb.toks, nullptr, 0, nullptr, MODE_CACHE, true,
                                              pdl, nullptr, true, &mu)
                               : fail(PRANA_E_CUDA, "positions launch: %s", cudaGetErrorString(el));
        const cudaError_t ec = cudaStreamEndCapture(st, &graph);
        if (rc) {
          if (graph) cudaGraphDestroy(graph);
          cudaGetLastError();
          return rc;
        }
        if (ec == cudaSuccess) {
          const cudaError_t ei = cudaGraphInstantiate(&np->graph, graph, 0);
          if (ei != cudaSuccess) np->graph = nullptr;
        }
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
      }
      if (!np->graph) return fail(PRANA_E_CUDA, "multi-sequence graph capture failed");
      m->multi = std::move(np);
      pl = m->multi.get();
    }
    Bufs& b = *pl->bufs;
    memcpy(pl->h_stage, tokens, n * 4);
    for (size_t i = 0; i < n; i++) pl->h_stage[n + i] = (uint32_t)positions[i];
    PRANA_CK(cudaMemcpyAsync(b.toks, pl->h_stage, n * 4, cudaMemcpyHostToDevice, st));
    PRANA_CK(cudaMemcpyAsync(pl->pos_dev, pl->h_stage + n, n * 4, cudaMemcpyHostToDevice, st));
    PRANA_CK(cudaGraphLaunch(pl->graph, st));
    if (logits) PRANA_CK(cudaMemcpyAsync(logits, b.logits, n * (size_t)m->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, st));
    if (argmax) PRANA_CK(cudaMemcpyAsync(argmax, b.tok_out, n * 4, cudaMemcpyDeviceToHost, st));
    PRANA_CK(cudaStreamSynchronize(st));
    for (size_t i = 0; i < n; i++) kvs[i]->loop_active = false;
    return check_err(m);
  }
  // ---- the diagnostic trace: eager
  std::unique_ptr<Bufs> tmp;
  Bufs* b = m->dec.get();
  if (n > b->rows) {
    tmp.reset(new Bufs(m->ctx));
    int rc = make_bufs(m, n, false, *tmp);
    if (rc) return rc;
    b = tmp.get();
  }
  SeqRow* rows_dev = nullptr;
  AttnSeq* att_dev = nullptr;
  Bufs scratch(m->ctx);
  if (int rc = scratch.alloc(rows_dev, n)) return rc;
  if (int rc = scratch.alloc(att_dev, att.size())) return rc;
  PRANA_CK(cudaMemcpyAsync(b->toks, tokens, n * 4, cudaMemcpyHostToDevice, st));
  PRANA_CK(cudaMemcpyAsync(rows_dev, rows.data(), n * sizeof(SeqRow), cudaMemcpyHostToDevice, st));
  PRANA_CK(cudaMemcpyAsync(att_dev, att.data(), att.size() * sizeof(AttnSeq), cudaMemcpyHostToDevice, st));
  const Multi mu{rows_dev, kvs, positions, att_dev, min_splits, all_tm};
  int rc = enqueue_rows(m, kvs[0], *b, (int)n, b->toks, nullptr, 0, nullptr, MODE_CACHE, true, false, tr,
                        logits != nullptr, &mu);
  if (rc) return rc;
  if (logits) PRANA_CK(cudaMemcpyAsync(logits, b->logits, n * (size_t)m->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, st));
  PRANA_CK(cudaStreamSynchronize(st));
  for (size_t i = 0; i < n; i++) kvs[i]->loop_active = false;
  return check_err(m);
  API_END
}

int prana_forward_multi(prana_model* m, prana_kv* const* kvs, size_t n, const uint32_t* tokens,
                        const size_t* positions, float* logits, uint32_t* argmax) {
  return forward_multi_impl(m, kvs, n, tokens, positions, logits, argmax, nullptr);
}

int prana_forward_multi_trace(prana_model* m, prana_kv* const* kvs, size_t n, const uint32_t* tokens,
                              const size_t* positions, float* logits, int8_t* q_host, float* s_host, size_t cap,
                              size_t* n_out) {
  API_BEGIN
  NEED(m && q_host && s_host && n_out, "null argument");
  NEED(n > 0, "empty batch");
  const auto& c = m->cfg;
  const size_t need = n * ((size_t)c.n_layers * (2 * c.dim + c.n_heads * c.head_dim + c.hidden_dim) + c.dim);
  NEED(cap >= need, "trace buffer holds %zu values, %zu needed", cap, need);
  DevScope ds(m->ctx->device);
  Trace tr;
  PRANA_CK(cudaMalloc(&tr.q, need));
  PRANA_CK(cudaMalloc(&tr.s, need / 32 * 4 + 4));
  struct Free {
    Trace& t;
    ~Free() {
      cudaFree(t.q);
      cudaFree(t.s);
    }
  } fr{tr};
  int rc = forward_multi_impl(m, kvs, n, tokens, positions, logits, nullptr, &tr);
  if (rc) return rc;
  if (tr.nq != need) return fail(PRANA_E_INVALID, "trace recorded %zu values, expected %zu", tr.nq, need);
  PRANA_CK(cudaMemcpy(q_host, tr.q, tr.nq, cudaMemcpyDeviceToHost));
  PRANA_CK(cudaMemcpy(s_host, tr.s, tr.ns * 4, cudaMemcpyDeviceToHost));
  *n_out = tr.nq;
  return PRANA_OK;
  API_END
}

static int decode_begin(prana_model* m, prana_kv* kv, uint32_t token, size_t pos, const prana_sampler* smp) {
  API_BEGIN
  NEED(m && kv && kv->m == m, "null or mismatched argument");
  NEED(pos < kv->positions, "position beyond kv capacity");
  NEED(token < (uint64_t)m->cfg.vocab_size, "token out of vocabulary");
  const bool sampled = smp && !smp->greedy;
  NEED(!sampled || m->cfg.vocab_size <= sample_max_vocab(), "vocabulary of %lld exceeds the device sampler's %d",
       (long long)m->cfg.vocab_size, sample_max_vocab());
  DevScope ds(m->ctx->device);
  int rc = ensure_graphs(m, kv, true, sampled);
  if (rc) return rc;
  cudaStream_t st = m->ctx->own;
  m->h_io[0] = (int)token;
  m->h_io[1] = (int)pos;
  PRANA_CK(cudaMemcpyAsync(m->d_tokpos, m->h_io, 8, cudaMemcpyHostToDevice, st));
  if (sampled) {
    SampleState* h = reinterpret_cast<SampleState*>(m->h_io + 8);
    *h = SampleState{smp->state, smp->temp, 0};
    PRANA_CK(cudaMemcpyAsync(m->d_sample, h, sizeof(SampleState), cudaMemcpyHostToDevice, st));
  }
  PRANA_CK(cudaMemsetAsync(kv->ring_n, 0, sizeof(int), st));
  PRANA_CK(cudaStreamSynchronize(st));
  kv->loop_pos = pos;
  kv->loop_active = true;
  kv->loop_sampled = sampled;
  return PRANA_OK;
  API_END
}

int prana_decode_begin(prana_model* m, prana_kv* kv, uint32_t token, size_t pos) {
  return decode_begin(m, kv, token, pos, nullptr);
}

int prana_decode_begin_sampled(prana_model* m, prana_kv* kv, uint32_t token, size_t pos, const prana_sampler* s) {
  return decode_begin(m, kv, token, pos, s);
}

int prana_decode_run(prana_model* m, prana_kv* kv, size_t n_steps) {
  NEED(m && kv && kv->m == m && kv->loop_active, "decode loop not started");
  NEED(kv->loop_pos + n_steps <= kv->positions, "decode loop would pass kv capacity %zu", kv->positions);
  DevScope ds(m->ctx->device);
  cudaGraphExec_t g = kv->loop_sampled ? kv->g_loop_s : kv->g_loop;
  for (size_t i = 0; i < n_steps; i++) PRANA_CK(cudaGraphLaunch(g, m->ctx->own));
  kv->loop_pos += n_steps;
  return PRANA_OK;
}

int prana_decode_tokens(prana_model* m, prana_kv* kv, uint32_t* out, size_t max, size_t* n_out) {
  NEED(m && kv && kv->m == m && n_out, "null argument");
  DevScope ds(m->ctx->device);
  int n = 0;
  PRANA_CK(cudaStreamSynchronize(m->ctx->own));
  PRANA_CK(cudaMemcpy(&n, kv->ring_n, sizeof(int), cudaMemcpyDeviceToHost));
  size_t cnt = std::min((size_t)n, std::min(max, kv->positions));
  if (cnt && out) PRANA_CK(cudaMemcpy(out, kv->ring, cnt * 4, cudaMemcpyDeviceToHost));
  *n_out = cnt;
  return check_err(m);
}

static int generate(prana_model* m, const uint32_t* prompt, size_t p, size_t steps, int64_t stop_id, prana_sampler* smp,
                    uint32_t* out, size_t* n_out) {
  API_BEGIN
  NEED(m && prompt && n_out && (out || !steps), "null argument");
  NEED(p > 0, "prompt encoded to zero tokens");
  *n_out = 0;
  const size_t max_pos = std::min((size_t)m->cfg.seq_len, p + steps);
  prana_kv* kv = nullptr;
  int rc = prana_kv_create(m, max_pos, &kv);
  if (rc) return rc;
  std::unique_ptr<prana_kv, void (*)(prana_kv*)> guard(kv, destroy_kv);
  size_t start = 0;
  uint32_t token = prompt[0];
  if (p > 1 && p <= max_pos) {
    if ((rc = prana_prefill(m, kv, prompt, p - 1))) return rc;
    start = p - 1;
    token = prompt[p - 1];
  }
  size_t produced = 0;
  // teacher-forced positions (only when the prompt overflows the context)
  size_t pos = start;
  for (; pos + 1 < p && pos < max_pos; pos++) {
    if ((rc = prana_forward(m, kv, token, pos, nullptr, nullptr))) return rc;
    token = prompt[pos + 1];
  }
  if (pos + 1 < max_pos) {
    // every remaining position samples: run them on the device back to back
    const size_t n = max_pos - 1 - pos;
    if ((rc = decode_begin(m, kv, token, pos, smp))) return rc;
    if ((rc = prana_decode_run(m, kv, n))) return rc;
    std::vector<uint32_t> ids(n);
    size_t got = 0;
    if ((rc = prana_decode_tokens(m, kv, ids.data(), n, &got))) return rc;
    size_t draws = got;  // Sampler::sample calls the reference's loop makes
    for (size_t i = 0; i < got && produced < steps; i++) {
      if (stop_id >= 0 && ids[i] == (uint64_t)stop_id) {
        draws = i + 1;
        break;
      }
      out[produced++] = ids[i];
    }
    // the caller's sampler continues where the reference's would: one draw per
    // sampled position up to and including a stop token
    if (smp && !smp->greedy)
      for (size_t i = 0; i < draws; i++) smp->next_u64();
  }
  *n_out = produced;
  return PRANA_OK;
  API_END
}

int prana_generate(prana_model* m, const uint32_t* prompt, size_t p, size_t steps, int64_t stop_id, uint32_t* out,
                   size_t* n_out) {
  return generate(m, prompt, p, steps, stop_id, nullptr, out, n_out);
}

int prana_generate_sampled(prana_model* m, const uint32_t* prompt, size_t p, size_t steps, int64_t stop_id,
                           prana_sampler* s, uint32_t* out, size_t* n_out) {
  NEED(s, "null sampler");
  return generate(m, prompt, p, steps, stop_id, s, out, n_out);
}

int prana_generate_speculative(prana_model* target, prana_model* draft, const uint32_t* prompt, size_t p,
                               size_t steps, size_t k, int64_t stop_id, uint32_t* out, size_t* n_out,
                               size_t* stats) {
  API_BEGIN
  NEED(target && draft && prompt && n_out && (out || !steps), "null argument");
  NEED(k >= 1, "draft length must be >= 1");
  NEED(p > 0, "prompt encoded to zero tokens");
  NEED(target->cfg.vocab_size == draft->cfg.vocab_size, "draft and target must share a vocabulary");
  *n_out = 0;
  const size_t max_pos = std::min((size_t)target->cfg.seq_len, p + steps);
  prana_kv *tkv = nullptr, *dkv = nullptr;
  int rc = prana_kv_create(target, max_pos, &tkv);
  if (rc) return rc;
  std::unique_ptr<prana_kv, void (*)(prana_kv*)> g1(tkv, destroy_kv);
  if ((rc = prana_kv_create(draft, max_pos, &dkv))) return rc;
  std::unique_ptr<prana_kv, void (*)(prana_kv*)> g2(dkv, destroy_kv);
  NEED(dkv->positions >= max_pos, "draft context shorter than target's");
  if (p > 1) {
    if ((rc = prana_prefill(target, tkv, prompt, p - 1)) || (rc = prana_prefill(draft, dkv, prompt, p - 1))) return rc;
  }
  size_t pos = p - 1, generated = 0, proposed = 0, accepted = 0;
  uint32_t last = prompt[p - 1];
  std::vector<uint32_t> drafts(k), inputs(k + 1), tnext(k + 1);
  bool stop = false;
  while (!stop && pos + 1 < max_pos) {
    const size_t budget = std::min(max_pos - 1 - pos, k);
    uint32_t d = last;
    for (size_t j = 0; j < budget; j++) {
      if ((rc = prana_forward(draft, dkv, d, pos + j, nullptr, &d))) return rc;
      drafts[j] = d;
    }
    proposed += budget;
    inputs[0] = last;
    for (size_t j = 0; j < budget; j++) inputs[j + 1] = drafts[j];
    if ((rc = prana_forward_batch(target, tkv, inputs.data(), budget + 1, pos, nullptr, tnext.data()))) return rc;
    for (size_t i = 0; i <= budget; i++) {
      const uint32_t tn = tnext[i];
      if (i < budget && tn == drafts[i]) accepted++;
      if (stop_id >= 0 && tn == (uint64_t)stop_id) {
        stop = true;
        break;
      }
      out[generated++] = tn;
      pos++;
      last = tn;
      if (generated >= steps || pos + 1 >= max_pos) {
        stop = true;
        break;
      }
      if (i == budget || tn != drafts[i]) break;
    }
  }
  if (stats) {
    stats[0] = proposed;
    stats[1] = accepted;
  }
  *n_out = generated;
  return PRANA_OK;
  API_END
}

}  // extern "C"
