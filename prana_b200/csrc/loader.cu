// loader.cu -- streaming GGUF -> HBM weight upload (gguf.rs:157-334,
// kquant.rs:166-183 keep the blocks; here they are split into the planes the
// GEMV and the tensor-core GEMM read, on the device).
//
// A tensor's rows are gathered from the mapped file (in any row order: the
// Q|K|V concatenation, the NeoX pair order and the gate/up interleave are row
// maps) into one of two pinned chunks by a few host threads, copied to the
// device asynchronously, and split into planes by a repack kernel while the
// next chunk is gathered.  Q4_K super-blocks and f32 rows need no repack and
// are copied to their destination directly.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "host.h"

namespace prana {

namespace {

constexpr int kGatherThreads = 8;

size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

// The planes of a [rows, cols] matrix of `type` (see DevWeight): byte offsets
// and the total; 0 when the type does not hold cols.
size_t plane_layout(int type, size_t rows, size_t cols, size_t off[4]) {
  const size_t n = rows * cols;
  off[0] = off[1] = off[2] = off[3] = 0;
  switch (type) {
    case T_Q8_0:
      if (cols % 32) return 0;
      off[1] = al256(n);
      return off[1] + al256(n / 32 * 2);
    case T_Q4_0:
      if (cols % 32) return 0;
      off[1] = al256(n / 2);
      return off[1] + al256(n / 32 * 2);
    case T_Q4_K:
      if (cols % 256) return 0;
      return al256(n / 256 * 144);
    case T_Q6_K:
      if (cols % 256) return 0;
      off[1] = al256(n / 2);
      off[2] = off[1] + al256(n / 4);
      off[3] = off[2] + al256(n / 16);
      return off[3] + al256(n / 256 * 2);
    case T_F32:
    case T_F16:
      return al256(n * 4);
  }
  return 0;
}

// ---- repack kernels: `nb` GGUF blocks (chunk-linear) starting at block b0 of the matrix
__global__ void repack_q8_0(const uint8_t* src, size_t nb, size_t b0, uint8_t* qs, uint16_t* d) {
  const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const uint8_t* s = src + b * 34;
  d[b0 + b] = (uint16_t)(s[0] | (s[1] << 8));
  uint8_t* q = qs + (b0 + b) * 32;
#pragma unroll
  for (int i = 0; i < 32; i += 2) *reinterpret_cast<uint16_t*>(q + i) = (uint16_t)(s[2 + i] | (s[3 + i] << 8));
}
__global__ void repack_q4_0(const uint8_t* src, size_t nb, size_t b0, uint8_t* qs, uint16_t* d) {
  const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const uint8_t* s = src + b * 18;
  d[b0 + b] = (uint16_t)(s[0] | (s[1] << 8));
  uint8_t* q = qs + (b0 + b) * 16;
#pragma unroll
  for (int i = 0; i < 16; i += 2) *reinterpret_cast<uint16_t*>(q + i) = (uint16_t)(s[2 + i] | (s[3 + i] << 8));
}
__global__ void repack_q6_k(const uint8_t* src, size_t nb, size_t b0, uint8_t* ql, uint8_t* qh, uint8_t* sc,
                            uint16_t* d) {
  const size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const uint8_t* s = src + b * 210;  // 210 = 2 x 105: 2-byte pieces stay aligned
  const size_t g = b0 + b;
#pragma unroll 8
  for (int i = 0; i < 128; i += 2) *reinterpret_cast<uint16_t*>(ql + g * 128 + i) = *reinterpret_cast<const uint16_t*>(s + i);
#pragma unroll 8
  for (int i = 0; i < 64; i += 2)
    *reinterpret_cast<uint16_t*>(qh + g * 64 + i) = *reinterpret_cast<const uint16_t*>(s + 128 + i);
#pragma unroll
  for (int i = 0; i < 16; i += 2)
    *reinterpret_cast<uint16_t*>(sc + g * 16 + i) = *reinterpret_cast<const uint16_t*>(s + 192 + i);
  d[g] = *reinterpret_cast<const uint16_t*>(s + 208);
}
// f16 -> f32 (gguf.rs:208-267 widens F16 tensors)
__global__ void widen_f16(const uint16_t* src, size_t n, size_t e0, float* dst) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[e0 + i] = __half2float(__ushort_as_half(src[i]));
}

}  // namespace

size_t gguf_bytes_per_row(int type, size_t cols) {
  switch (type) {
    case T_Q8_0: return cols / 32 * 34;
    case T_Q4_0: return cols / 32 * 18;
    case T_Q4_K: return cols / 256 * 144;
    case T_Q6_K: return cols / 256 * 210;
    case T_F32: return cols * 4;
    case T_F16: return cols * 2;
  }
  return 0;
}

static void make_devweight(int type, size_t rows, size_t cols, uint8_t* base, const size_t off[4], DevWeight* dw) {
  *dw = DevWeight{};
  dw->type = type == T_F16 ? T_F32 : type;
  dw->rows = (int)rows;
  dw->cols = (int)cols;
  switch (dw->type) {
    case T_Q8_0:
    case T_Q4_0:
      dw->qs = base;
      dw->d = reinterpret_cast<const __half*>(base + off[1]);
      break;
    case T_Q4_K:
      dw->qs = base;
      break;
    case T_Q6_K:
      dw->qs = base;
      dw->qh = base + off[1];
      dw->sc = reinterpret_cast<const int8_t*>(base + off[2]);
      dw->d = reinterpret_cast<const __half*>(base + off[3]);
      break;
    default:
      dw->f32 = reinterpret_cast<const float*>(base);
  }
}

WeightStreamer::WeightStreamer(prana_ctx* c, size_t chunk_bytes) : ctx(c), chunk((chunk_bytes + 255) & ~(size_t)255) {}

WeightStreamer::~WeightStreamer() {
  if (ctx) {
    DevScope ds(ctx->device);
    if (pinned[0] || pinned[1]) cudaStreamSynchronize(ctx->own);
    for (int i = 0; i < 2; i++) {
      if (pinned[i]) cudaFreeHost(pinned[i]);
      if (stage[i]) dev_free(ctx, stage[i]);
      if (done[i]) cudaEventDestroy(done[i]);
    }
  }
}

int WeightStreamer::ready() {
  if (done[1]) return PRANA_OK;
  for (int i = 0; i < 2; i++) {
    if (cudaMallocHost(reinterpret_cast<void**>(&pinned[i]), chunk) != cudaSuccess) {
      cudaGetLastError();
      pinned[i] = nullptr;
      return fail(PRANA_E_OOM, "pinned staging of %zu bytes failed", chunk);
    }
    void* s = nullptr;
    if (int rc = dev_alloc(ctx, chunk, &s)) return rc;
    stage[i] = static_cast<uint8_t*>(s);
    PRANA_CK(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
    PRANA_CK(cudaEventRecord(done[i], ctx->own));
  }
  return PRANA_OK;
}

int WeightStreamer::upload(int type, size_t rows, size_t cols, const std::function<const uint8_t*(size_t)>& row_src,
                           prana_weight* w) {
  if (!rows || !cols) return fail(PRANA_E_INVALID, "empty weight [%zu, %zu]", rows, cols);
  if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX) return fail(PRANA_E_INVALID, "weight too large");
  size_t off[4];
  const size_t total = plane_layout(type, rows, cols, off);
  if (!total) {
    if (gguf_bytes_per_row(type, 256)) return fail(PRANA_E_INVALID, "ggml type %d cannot hold rows of %zu values", type, cols);
    return fail(PRANA_E_UNSUPPORTED, "ggml type %d is not supported", type);
  }
  const size_t rb = gguf_bytes_per_row(type, cols);
  if (rb > chunk) return fail(PRANA_E_UNSUPPORTED, "rows of %zu bytes exceed the staging chunk", rb);
  DevScope ds(ctx->device);
  if (int rc = ready()) return rc;
  void* mem = nullptr;
  if (int rc = dev_alloc(ctx, total, &mem)) return rc;
  uint8_t* base = static_cast<uint8_t*>(mem);
  cudaStream_t st = ctx->own;
  const size_t rows_per_chunk = chunk / rb;
  for (size_t r0 = 0; r0 < rows; r0 += rows_per_chunk) {
    const size_t nr = std::min(rows_per_chunk, rows - r0), bytes = nr * rb;
    // the chunk's buffers are free once their last copy and repack are done
    if (cudaEventSynchronize(done[cur]) != cudaSuccess) {
      dev_free(ctx, mem);
      return fail(PRANA_E_CUDA, "weight staging wait failed");
    }
    uint8_t* pin = pinned[cur];
    auto gather = [&](size_t a, size_t b) {
      for (size_t r = a; r < b; r++) memcpy(pin + (r - r0) * rb, row_src(r), rb);
    };
    if (bytes >= (size_t(4) << 20)) {  // a few threads share the gather of a large chunk
      std::vector<std::thread> th;
      const size_t per = (nr + kGatherThreads - 1) / kGatherThreads;
      for (int t = 0; t < kGatherThreads; t++) {
        const size_t a = r0 + t * per, b = std::min(r0 + nr, a + per);
        if (a < b) th.emplace_back(gather, a, b);
      }
      for (auto& t : th) t.join();
    } else {
      gather(r0, r0 + nr);
    }
    const size_t b0 = r0 * cols;  // first value of the chunk
    cudaError_t e = cudaSuccess;
    switch (type) {
      case T_Q4_K:  // super-blocks verbatim
        e = cudaMemcpyAsync(base + r0 * rb, pin, bytes, cudaMemcpyHostToDevice, st);
        break;
      case T_F32:
        e = cudaMemcpyAsync(base + b0 * 4, pin, bytes, cudaMemcpyHostToDevice, st);
        break;
      default: {
        e = cudaMemcpyAsync(stage[cur], pin, bytes, cudaMemcpyHostToDevice, st);
        const size_t nb = type == T_Q6_K ? nr * cols / 256 : nr * cols / 32, grid = (nb + 255) / 256;
        if (e == cudaSuccess) {
          if (type == T_Q8_0)
            repack_q8_0<<<grid, 256, 0, st>>>(stage[cur], nb, b0 / 32, base, reinterpret_cast<uint16_t*>(base + off[1]));
          else if (type == T_Q4_0)
            repack_q4_0<<<grid, 256, 0, st>>>(stage[cur], nb, b0 / 32, base, reinterpret_cast<uint16_t*>(base + off[1]));
          else if (type == T_Q6_K)
            repack_q6_k<<<grid, 256, 0, st>>>(stage[cur], nb, b0 / 256, base, base + off[1], base + off[2],
                                               reinterpret_cast<uint16_t*>(base + off[3]));
          else  // T_F16
            widen_f16<<<(nr * cols + 255) / 256, 256, 0, st>>>(reinterpret_cast<const uint16_t*>(stage[cur]), nr * cols,
                                                               b0, reinterpret_cast<float*>(base));
          e = cudaGetLastError();
        }
      }
    }
    if (e == cudaSuccess) e = cudaEventRecord(done[cur], st);
    if (e != cudaSuccess) {
      cudaStreamSynchronize(st);
      dev_free(ctx, mem);
      return fail(PRANA_E_CUDA, "weight upload failed: %s", cudaGetErrorString(e));
    }
    cur ^= 1;
  }
  make_devweight(type, rows, cols, base, off, &w->dw);
  w->ctx = ctx;
  w->mem = mem;
  w->bytes = total;
  bytes_streamed += rows * rb;
  return PRANA_OK;
}

int WeightStreamer::finish() {
  if (!ctx) return PRANA_OK;
  DevScope ds(ctx->device);
  PRANA_CK(cudaStreamSynchronize(ctx->own));
  return PRANA_OK;
}

}  // namespace prana
