// pool.cu -- the device arena and buffer pool (prana-tensor's BufferPool,
// crates/prana-tensor/src/pool.rs:13-103, with its storage in HBM).
//
// One reservation (a single cudaMalloc, or host memory for tests) backs every
// buffer.  Requests up to kBucketMax are rounded to the reference's buckets (a
// power of two of at least 1 KiB, pool.rs:27-39) and recycled per bucket;
// larger ones (weights, KV caches) are carved at their own 256-byte-aligned
// size and recycled on an exact size match.  Released buffers wait in their
// bucket's list; clear() hands them back to the arena, whose free ranges are
// kept in address order and coalesced, so a cleared pool can carve any size
// again.  No allocator call happens after creation.
#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "host.h"

namespace {

constexpr size_t kMinBucket = 1024;              // pool.rs:22
constexpr size_t kAlignment = 64;                // pool.rs:21
constexpr size_t kBucketMax = size_t(64) << 20;  // larger requests are carved exactly
constexpr size_t kCarveAlign = 256;              // every buffer starts on 256 bytes (TMA, vector loads)

size_t bucket_of(size_t size) {
  if (size <= kMinBucket) return kMinBucket;
  const size_t aligned = (size + kAlignment - 1) & ~(kAlignment - 1);
  if (aligned > kBucketMax) return (aligned + kCarveAlign - 1) & ~(kCarveAlign - 1);
  size_t b = kMinBucket;
  while (b < aligned) b *= 2;
  return b;
}

}  // namespace

struct prana_pool {
  int device = -1;          // -1: host memory (bookkeeping tests)
  prana_ctx* ctx = nullptr;  // zeroing runs on its stream (device pools)
  uint8_t* base = nullptr;
  size_t cap = 0;
  std::map<size_t, size_t> ranges;                     // free ranges of the arena: offset -> size
  std::map<size_t, std::vector<size_t>> cached;        // released buffers by bucket: offsets
  std::unordered_map<size_t, size_t> live;             // offset -> bucket of every buffer out of the arena
  size_t active = 0, pooled = 0, peak = 0, carved = 0, carved_peak = 0;
  std::mutex mu;

  // first fit in address order; false when no range holds `bytes`
  bool carve(size_t bytes, size_t* off) {
    for (auto it = ranges.begin(); it != ranges.end(); ++it) {
      if (it->second < bytes) continue;
      *off = it->first;
      const size_t rest = it->second - bytes, at = it->first + bytes;
      ranges.erase(it);
      if (rest) ranges[at] = rest;
      carved += bytes;
      if (carved > carved_peak) carved_peak = carved;
      return true;
    }
    return false;
  }
  // return a range to the arena, merging with its neighbours
  void give_back(size_t off, size_t bytes) {
    carved -= bytes;
    auto next = ranges.lower_bound(off);
    if (next != ranges.end() && off + bytes == next->first) {
      bytes += next->second;
      next = ranges.erase(next);
    }
    if (next != ranges.begin()) {
      auto prev = std::prev(next);
      if (prev->first + prev->second == off) {
        prev->second += bytes;
        return;
      }
    }
    ranges[off] = bytes;
  }
};

using namespace prana;

extern "C" {

int prana_pool_create(prana_ctx* ctx, size_t capacity, prana_pool** out) {
  if (!out) return fail(PRANA_E_INVALID, "null argument");
  *out = nullptr;
  if (!capacity) return fail(PRANA_E_INVALID, "pool capacity must be positive");
  capacity = (capacity + kCarveAlign - 1) & ~(kCarveAlign - 1);
  prana_pool* p = new (std::nothrow) prana_pool();
  if (!p) return fail(PRANA_E_OOM, "host allocation failed");
  if (ctx) {
    DevScope ds(ctx->device);
    void* mem = nullptr;
    if (cudaMalloc(&mem, capacity) != cudaSuccess) {
      cudaGetLastError();
      delete p;
      return fail(PRANA_E_OOM, "device reservation of %zu bytes failed", capacity);
    }
    p->device = ctx->device;
    p->ctx = ctx;
    p->base = static_cast<uint8_t*>(mem);
  } else {
    p->base = static_cast<uint8_t*>(::operator new(capacity, std::nothrow));
    if (!p->base) {
      delete p;
      return fail(PRANA_E_OOM, "host reservation of %zu bytes failed", capacity);
    }
  }
  p->cap = capacity;
  p->ranges[0] = capacity;
  *out = p;
  return PRANA_OK;
}

int prana_pool_destroy(prana_pool* p) {
  if (!p) return PRANA_OK;
  if (p->device >= 0) {
    DevScope ds(p->device);
    cudaDeviceSynchronize();
    cudaFree(p->base);
  } else {
    ::operator delete(p->base);
  }
  delete p;
  return PRANA_OK;
}

}  // extern "C"

namespace {

// A buffer of at least `bytes` out of the pool (not cleared).
int pool_take(prana_pool* p, size_t bytes, uint8_t** out, size_t* got) {
  const size_t b = bucket_of(bytes);
  size_t off = 0;
  {
    std::lock_guard<std::mutex> lock(p->mu);
    auto it = p->cached.find(b);
    if (it != p->cached.end() && !it->second.empty()) {
      off = it->second.back();
      it->second.pop_back();
      p->pooled -= b;
    } else if (!p->carve(b, &off)) {
      return fail(PRANA_E_OOM, "pool of %zu bytes cannot hold another %zu-byte buffer (%zu carved)", p->cap, b,
                  p->carved);
    }
    p->live[off] = b;
    p->active += b;
    if (p->active > p->peak) p->peak = p->active;
  }
  *out = p->base + off;
  *got = b;
  return PRANA_OK;
}

}  // namespace

extern "C" {

int prana_pool_acquire(prana_pool* p, size_t bytes, void** ptr, size_t* got) {
  if (!p || !ptr) return fail(PRANA_E_INVALID, "null argument");
  *ptr = nullptr;
  if (got) *got = 0;
  if (!bytes) return PRANA_OK;  // pool.rs:44-46: a zero-byte request is an empty buffer
  uint8_t* q = nullptr;
  size_t b = 0;
  if (int rc = pool_take(p, bytes, &q, &b)) return rc;
  if (p->device >= 0) {  // zeroed like the reference's buffers, in the context's stream order
    DevScope ds(p->device);
    PRANA_CK(cudaMemsetAsync(q, 0, b, p->ctx->own));
  } else {
    memset(q, 0, b);
  }
  *ptr = q;
  if (got) *got = b;
  return PRANA_OK;
}

int prana_pool_release(prana_pool* p, void* ptr) {
  if (!p) return fail(PRANA_E_INVALID, "null pool");
  if (!ptr) return PRANA_OK;
  const uint8_t* q = static_cast<const uint8_t*>(ptr);
  if (q < p->base || q >= p->base + p->cap) return fail(PRANA_E_INVALID, "buffer does not belong to this pool");
  const size_t off = (size_t)(q - p->base);
  std::lock_guard<std::mutex> lock(p->mu);
  auto it = p->live.find(off);
  if (it == p->live.end()) return fail(PRANA_E_INVALID, "buffer is not checked out of this pool");
  const size_t b = it->second;
  p->live.erase(it);
  p->active -= b;
  p->pooled += b;
  p->cached[b].push_back(off);
  return PRANA_OK;
}

int prana_pool_clear(prana_pool* p) {
  if (!p) return fail(PRANA_E_INVALID, "null pool");
  std::lock_guard<std::mutex> lock(p->mu);
  for (auto& kv : p->cached)
    for (size_t off : kv.second) p->give_back(off, kv.first);
  p->cached.clear();
  p->pooled = 0;
  return PRANA_OK;
}

int prana_ctx_use_pool(prana_ctx* ctx, prana_pool* p) {
  if (!ctx) return fail(PRANA_E_INVALID, "ctx is null");
  if (p && p->device != ctx->device)
    return fail(PRANA_E_INVALID, "pool holds %s memory, the context runs on device %d",
                p->device < 0 ? "host" : "another device's", ctx->device);
  if (p == ctx->pool) return PRANA_OK;
  // the context's own buffers (kernel scratch, RoPE tables) go back to where
  // they came from before the switch, so none outlives the pool that holds it
  DevScope ds(ctx->device);
  PRANA_CK(cudaStreamSynchronize(ctx->own));
  PRANA_CK(cudaStreamSynchronize(ctx->stream));
  dev_free(ctx, ctx->scratch.base);
  ctx->scratch.base = nullptr;
  ctx->scratch.bytes = 0;
  for (auto& kv : ctx->rope) {
    dev_free(ctx, kv.second.cos);
    dev_free(ctx, kv.second.sin);
  }
  ctx->rope.clear();
  for (void* q : ctx->retired) dev_free(ctx, q);
  ctx->retired.clear();
  ctx->pool = p;
  return PRANA_OK;
}

int prana_pool_stats(prana_pool* p, size_t* active, size_t* pooled, size_t* peak, size_t* carved) {
  if (!p) return fail(PRANA_E_INVALID, "null pool");
  std::lock_guard<std::mutex> lock(p->mu);
  if (active) *active = p->active;
  if (pooled) *pooled = p->pooled;
  if (peak) *peak = p->peak;
  if (carved) *carved = p->carved;
  return PRANA_OK;
}

}  // extern "C"

namespace prana {

// Device memory of a context: from its pool when one is attached (no
// allocator call), else cudaMalloc.  Freed buffers go back where they came from.
int dev_alloc(prana_ctx* ctx, size_t bytes, void** out) {
  *out = nullptr;
  if (ctx && ctx->pool) {  // not cleared: every caller writes or clears what it takes
    uint8_t* q = nullptr;
    size_t got = 0;
    if (int rc = pool_take(ctx->pool, bytes ? bytes : 1, &q, &got)) return rc;
    *out = q;
    return PRANA_OK;
  }
  if (cudaMalloc(out, bytes ? bytes : 1) != cudaSuccess) {
    cudaGetLastError();
    *out = nullptr;
    return fail(PRANA_E_OOM, "device allocation of %zu bytes failed", bytes);
  }
  return PRANA_OK;
}

void dev_free(prana_ctx* ctx, void* p) {
  if (!p) return;
  if (ctx && ctx->pool) {
    const uint8_t* q = static_cast<const uint8_t*>(p);
    if (q >= ctx->pool->base && q < ctx->pool->base + ctx->pool->cap) {
      prana_pool_release(ctx->pool, p);
      return;
    }
  }
  cudaFree(p);
}

}  // namespace prana
