// host.h -- host-side objects behind the opaque C-ABI handles.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/prana_cuda.h"
#include "internal.h"

namespace prana {

int fail(int code, const char* fmt, ...);
#define PRANA_CK(expr)                                                                                \
  do {                                                                                                \
    cudaError_t e_ = (expr);                                                                          \
    if (e_ != cudaSuccess) return ::prana::fail(PRANA_E_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// (cos, sin) tables of the two RoPE forms, computed on the host with libm
// exactly as the CPU loops compute them (attention.rs:96-99, 114-117).
struct RopeTable {
  float* cos = nullptr;
  float* sin = nullptr;
  int positions = 0;
};

// Device scratch that grows on demand; `counters` are zero between launches
// (every kernel that takes a ticket resets its counter).
struct Scratch {
  void* base = nullptr;
  size_t bytes = 0;
};

}  // namespace prana

struct prana_ctx {
  int device = 0;
  prana_pool* pool = nullptr;  // when set, the context's device memory comes from it
  int sm_count = 148;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  prana::Scratch scratch;
  unsigned* counters = nullptr;  // 4096 zeroed ticket counters (one per kv head of an attention launch)
  unsigned* err = nullptr;       // device error flag of kernel-level calls (a word of its own after the counters)
  std::map<std::tuple<int, uint32_t, int>, prana::RopeTable> rope;
  std::vector<void*> retired;  // outgrown RoPE tables: captured graphs may still point at them
};

struct prana_weight {
  prana_ctx* ctx = nullptr;
  prana::DevWeight dw{};
  void* mem = nullptr;
  size_t bytes = 0;
};

namespace prana {
// Grow the context scratch to at least `bytes` (synchronizes when it grows).
int ctx_scratch(prana_ctx* ctx, size_t bytes, void** out);
// Table for (head_dim, theta, neox) covering at least `positions` rows.
int ctx_rope(prana_ctx* ctx, int head_dim, float theta, int neox, int positions, const RopeTable** out);
// Address of row r's GGUF bytes (a [rows, cols] matrix taken from a file in any row order).
using RowSrc = std::function<const uint8_t*(size_t)>;

// Streams GGUF tensors to the device: rows are gathered into one of two pinned
// chunks, copied asynchronously on the context's own stream, and split into
// planes there by a repack kernel while the next chunk is gathered.  The
// destination is ready once finish() returns.
class WeightStreamer {
 public:
  WeightStreamer(prana_ctx* ctx, size_t chunk_bytes);
  ~WeightStreamer();
  WeightStreamer(const WeightStreamer&) = delete;
  WeightStreamer& operator=(const WeightStreamer&) = delete;
  int upload(int type, size_t rows, size_t cols, const RowSrc& row_src, prana_weight* w);
  int finish();
  size_t bytes_streamed = 0;

 private:
  int ready();
  prana_ctx* ctx;
  size_t chunk;
  uint8_t* pinned[2] = {nullptr, nullptr};
  uint8_t* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  int cur = 0;
};
// Bytes of one GGUF row of `type` holding `cols` values (0 for other types).
size_t gguf_bytes_per_row(int type, size_t cols);
// Repack GGUF bytes of a [rows, cols] tensor into device layout.
int upload_weight(prana_ctx* ctx, int type, size_t rows, size_t cols, const void* host, prana_weight* w);
// quantize_q8 (matmul.rs:61-84) on the host, then upload as T_Q8S
void quantize_q8_host(size_t rows, size_t cols, const float* w, int8_t* q, float* scales);
int upload_q8s(prana_ctx* ctx, size_t rows, size_t cols, const float* host, prana_weight* w);
void free_weight(prana_weight* w);
// Device memory of a context: its pool's when attached, else cudaMalloc.
int dev_alloc(prana_ctx* ctx, size_t bytes, void** out);
void dev_free(prana_ctx* ctx, void* p);
// Read and clear the error word of prana_attention_decode_noalloc on `device`.
int noalloc_take_error(int device, unsigned* out);
struct DevScope {
  int prev = -1;
  explicit DevScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace prana
