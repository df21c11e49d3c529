// noalloc.cu -- decode attention whose scratch is static device memory.
//
// prana_attention_decode takes the split partials from the context's scratch,
// which grows with cudaMalloc (and cudaFree, which synchronizes the device)
// the first time a larger shape arrives.  Some callers cannot allocate on the
// call path: a host that reserved all device memory up front for its own
// pool, or a latency-critical loop that must never block on the allocator.
// prana_attention_decode_noalloc runs the same kernels on a file-scope
// device array of fixed size instead, and never allocates.
#include <mutex>

#include "host.h"
#include "internal.h"

// 4 MiB of split partials: (max, sum) pairs and the unnormalized outputs of
// every (kv head, split, virtual head).  An 8B-shape decode (8 kv heads,
// 32 splits, 4 query heads per kv head, head_dim 128) needs 0.53 MiB.
constexpr size_t kScratchFloats = size_t(1) << 20;
constexpr int kMaxKvHeads = 1024;  // one ticket counter per kv head

// The counters must be zero whenever no call is running.  Static storage is
// zero when the module loads and each launch leaves every counter at zero
// again (the CTA that merges a kv head resets its counter), so they need no
// clearing between calls.  The partials need no initial value.
static __device__ __align__(256) float g_scratch[kScratchFloats];
static __device__ __align__(256) unsigned g_counters[kMaxKvHeads];
// Raised by a launch whose bounded mbarrier wait gave up (the output of that
// call is then incomplete); read and cleared by prana_ctx_synchronize.
static __device__ __align__(256) unsigned g_error;

namespace {

struct Slot {
  bool ready = false;
  float* scratch = nullptr;
  unsigned* counters = nullptr;
  unsigned* error = nullptr;
};
constexpr int kMaxDevices = 64;
Slot g_slots[kMaxDevices];
std::mutex g_mu;

// Device addresses of the static arrays on the current device, looked up once
// per device (the first call on a device does this set-up).
int setup(int device, Slot** out) {
  if (device < 0 || device >= kMaxDevices) return prana::fail(PRANA_E_INVALID, "device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_mu);
  Slot& s = g_slots[device];
  if (!s.ready) {
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.scratch), g_scratch);
    if (e != cudaSuccess)
      return prana::fail(PRANA_E_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.counters), g_counters);
    if (e != cudaSuccess)
      return prana::fail(PRANA_E_CUDA, "cudaGetSymbolAddress(counters) failed: %s", cudaGetErrorString(e));
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.error), g_error);
    if (e != cudaSuccess)
      return prana::fail(PRANA_E_CUDA, "cudaGetSymbolAddress(error) failed: %s", cudaGetErrorString(e));
    s.ready = true;
  }
  *out = &s;
  return PRANA_OK;
}

}  // namespace

namespace prana {

// The no-allocation entry point's error word on `device`: 0 when no call there
// has reported a timeout since the last look (or the device never ran one);
// a nonzero word is cleared.  The caller has synchronized the stream the
// calls ran on.
int noalloc_take_error(int device, unsigned* out) {
  *out = 0;
  if (device < 0 || device >= kMaxDevices) return PRANA_OK;
  unsigned* word = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_slots[device].ready) word = g_slots[device].error;
  }
  if (!word) return PRANA_OK;
  PRANA_CK(cudaMemcpy(out, word, sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (*out) PRANA_CK(cudaMemset(word, 0, sizeof(unsigned)));
  return PRANA_OK;
}

}  // namespace prana

using namespace prana;

extern "C" int prana_attention_decode_noalloc(prana_ctx* c, const float* q, const uint16_t* kc, const uint16_t* vc,
                                              size_t pos, size_t nh, size_t nkv, size_t hd, float* out) {
  if (!(c && q && kc && vc && out)) return fail(PRANA_E_INVALID, "null argument");
  if (!(nkv > 0 && nh % nkv == 0)) return fail(PRANA_E_INVALID, "n_heads must be a multiple of n_kv_heads");
  if (hd > 256 || hd * (nh / nkv) > 4096) return fail(PRANA_E_INVALID, "head_dim %zu x group exceeds 4096", hd);
  if (nkv > (size_t)kMaxKvHeads)
    return fail(PRANA_E_INVALID, "attention_decode_noalloc: %zu kv heads, the static scratch has counters for %d", nkv,
                kMaxKvHeads);
  try {
    DevScope ds(c->device);
    Slot* slot = nullptr;
    if (int rc = setup(c->device, &slot)) return rc;
    const int splits = attn_splits((int)(pos + 1), (int)nkv, (int)hd, c->sm_count);
    const size_t group = nh / nkv;
    const size_t ml = (nkv * splits * group * 2 + 3) / 4 * 4;  // keeps the outputs 16-byte aligned
    const size_t need = ml + nkv * splits * group * hd;
    if (need > kScratchFloats)
      return fail(PRANA_E_INVALID,
                  "attention_decode_noalloc: this shape needs %zu floats of split scratch, the static scratch holds %zu "
                  "(use prana_attention_decode)",
                  need, kScratchFloats);
    AttnArgs a{};
    a.q = q;
    a.kc = reinterpret_cast<const __half*>(kc);
    a.vc = reinterpret_cast<const __half*>(vc);
    a.m = 1;
    a.pos0 = (int)pos;
    a.n_heads = (int)nh;
    a.n_kv = (int)nkv;
    a.hd = (int)hd;
    a.n_splits = splits;
    a.part_ml = slot->scratch;
    a.part_o = slot->scratch + ml;
    a.counters = slot->counters;
    a.out = out;
    a.err = slot->error;
    attn_make_maps(a, (int)(pos + 1));
    const cudaError_t e = launch_attn_decode(a, c->stream, false);
    if (e == cudaErrorInvalidValue) return fail(PRANA_E_UNSUPPORTED, "attention: head_dim %zu not built", hd);
    PRANA_CK(e);
    return PRANA_OK;
  } catch (...) {
    return fail(PRANA_E_INVALID, "unexpected host exception");
  }
}
