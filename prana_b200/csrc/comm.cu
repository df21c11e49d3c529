// comm.cu -- NCCL entry points for tensor parallelism (see comm.h).
#include <dlfcn.h>

#include <mutex>
#include <vector>

#include "comm.h"

namespace prana {

const Nccl* nccl(const char** why) {
  static Nccl api;
  static const char* err = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy already in the process
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      err = "libnccl.so.2 not found";
      return;
    }
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!api.get_unique_id || !api.comm_init_rank || !api.comm_destroy || !api.all_reduce || !api.all_gather ||
        !api.error_string)
      err = "libnccl.so.2 lacks an entry point";
  });
  if (err) {
    if (why) *why = err;
    return nullptr;
  }
  return &api;
}


// ---------------------------------------------------------------- one-shot all-reduce

namespace {

// Every element travels as one 8-byte word: the value's bits in the low half,
// the call's epoch in the high half.  An aligned 8-byte store is single-copy
// atomic, so a reader that sees the epoch also sees the value: no fence and no
// separate flag, one NVLink crossing per call.
__device__ __forceinline__ void st_word(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

constexpr int kExThreads = 512;
constexpr int kExMaxCtas = 64;

// GATHER == false: x[i] = sum over ranks (all-reduce, in place).
// GATHER == true:  dst[r * n + i] = rank r's x[i] (all-gather).
// W ranks; each thread moves E elements per round, all of whose words are in
// flight together (the waits overlap instead of following one another).
// Each CTA keeps its own epoch (p.epoch[blockIdx.x]): every rank launches the
// same grids in the same order, so CTA b's counter agrees on every rank.
template <bool GATHER, int W, int E>
__global__ void __launch_bounds__(kExThreads) tp_exchange_kernel(const TpPeers p, float* x, int n, float* dst,
                                                                 unsigned* err) {
  // the next kernel may start streaming its weights while this one waits
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x is final
  __shared__ int timed_out;
  const int tid = threadIdx.x;
  if (tid == 0) timed_out = 0;
  unsigned* epoch = p.epoch + blockIdx.x;
  const unsigned e = *epoch + 1;  // this call's epoch
  const size_t area = (size_t)(e & 1) * W * p.cap;  // alternate halves on consecutive calls
  const uint64_t tag = (uint64_t)e << 32;
  const int per_cta = (int)((n + gridDim.x - 1) / gridDim.x);
  const int lo = blockIdx.x * per_cta, hi = min(n, lo + per_cta);
  uint32_t budget = p.budget;
  bool late = false;
  // push: this rank's values into its slot on every rank
  for (int b = lo; b < hi; b += kExThreads * E) {
    float v[E];
#pragma unroll
    for (int j = 0; j < E; j++) {
      const int i = b + j * kExThreads + tid;
      v[j] = i < hi ? x[i] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < W; r++) {
      uint64_t* slot = p.buf[r] + area + (size_t)p.rank * p.cap;
#pragma unroll
      for (int j = 0; j < E; j++) {
        const int i = b + j * kExThreads + tid;
        if (i < hi) st_word(slot + i, tag | __float_as_uint(v[j]));
      }
    }
  }
  // receive: every rank's word carries this epoch once it has landed (bounded wait)
  const uint64_t* own = p.buf[p.rank] + area;
  for (int b = lo; b < hi; b += kExThreads * E) {
    uint64_t w[E][W];
#pragma unroll
    for (int j = 0; j < E; j++)
#pragma unroll
      for (int r = 0; r < W; r++) {
        const int i = b + j * kExThreads + tid;
        w[j][r] = i < hi ? ld_word(own + (size_t)r * p.cap + i) : tag;
      }
    for (;;) {
      bool ready = true;
#pragma unroll
      for (int j = 0; j < E; j++)
#pragma unroll
        for (int r = 0; r < W; r++) ready &= (uint32_t)(w[j][r] >> 32) == e;
      if (ready || !budget) {
        late |= !ready;
        break;
      }
      budget--;
      __nanosleep(20);
#pragma unroll
      for (int j = 0; j < E; j++)
#pragma unroll
        for (int r = 0; r < W; r++) {
          const int i = b + j * kExThreads + tid;
          if ((uint32_t)(w[j][r] >> 32) != e) w[j][r] = ld_word(own + (size_t)r * p.cap + i);
        }
    }
#pragma unroll
    for (int j = 0; j < E; j++) {
      const int i = b + j * kExThreads + tid;
      if (i >= hi) continue;
      if (GATHER) {
#pragma unroll
        for (int r = 0; r < W; r++) dst[(size_t)r * n + i] = __uint_as_float((uint32_t)w[j][r]);
      } else {
        float s = __uint_as_float((uint32_t)w[j][0]);
#pragma unroll
        for (int r = 1; r < W; r++) s += __uint_as_float((uint32_t)w[j][r]);  // rank order on every rank
        x[i] = s;
      }
    }
  }
  if (late) timed_out = 1;
  __syncthreads();
  if (tid == 0) {
    if (timed_out && err) atomicExch(err, 1u);
    *epoch = e;
  }
}

template <bool GATHER, int W>
cudaError_t exchange_w(const TpPeers& p, float* x, int n, float* dst, unsigned* err, cudaLaunchConfig_t& cfg) {
  constexpr int E = 16 / W;
  // as many CTAs as keep each thread at one round or more, up to kExMaxCtas
  int grid = (n + kExThreads * E - 1) / (kExThreads * E);
  if (grid > kExMaxCtas) grid = kExMaxCtas;
  cfg.gridDim = dim3(grid);
  return cudaLaunchKernelEx(&cfg, tp_exchange_kernel<GATHER, W, E>, p, x, n, dst, err);
}

cudaError_t launch_exchange(const TpPeers& p, bool gather, float* x, int n, float* dst, unsigned* err,
                            cudaStream_t st, bool pdl) {
  if (n <= 0 || (size_t)n > p.cap) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kExThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  switch (p.world) {
    case 2: return gather ? exchange_w<true, 2>(p, x, n, dst, err, cfg) : exchange_w<false, 2>(p, x, n, dst, err, cfg);
    case 4: return gather ? exchange_w<true, 4>(p, x, n, dst, err, cfg) : exchange_w<false, 4>(p, x, n, dst, err, cfg);
    case 8: return gather ? exchange_w<true, 8>(p, x, n, dst, err, cfg) : exchange_w<false, 8>(p, x, n, dst, err, cfg);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_tp_allreduce(const TpPeers& p, float* x, int n, unsigned* err, cudaStream_t st, bool pdl) {
  return launch_exchange(p, false, x, n, nullptr, err, st, pdl);
}

cudaError_t launch_tp_allgather(const TpPeers& p, const float* src, int n, float* dst, unsigned* err,
                                cudaStream_t st, bool pdl) {
  return launch_exchange(p, true, const_cast<float*>(src), n, dst, err, st, pdl);
}

bool tp_peers_setup(ncclComm_t comm, int world, int rank, size_t cap, cudaStream_t st, TpPeers* out,
                    void** own_mem) {
  const Nccl* api = nccl(nullptr);
  if (!api || !(world == 2 || world == 4 || world == 8)) return false;
  TpPeers p;
  p.world = world;
  p.rank = rank;
  p.cap = cap;
  // [2][world][cap] words, then one epoch counter per exchange CTA
  const size_t buf_bytes = 2 * (size_t)world * cap * sizeof(uint64_t);
  const size_t bytes = buf_bytes + kExMaxCtas * sizeof(unsigned);
  void* mem = nullptr;
  if (cudaMalloc(&mem, bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  cudaMemset(mem, 0, bytes);
  cudaIpcMemHandle_t mine;
  bool ok = cudaIpcGetMemHandle(&mine, mem) == cudaSuccess;
  void* dev_handles = nullptr;
  std::vector<cudaIpcMemHandle_t> all(world);
  if (ok) ok = cudaMalloc(&dev_handles, world * sizeof(cudaIpcMemHandle_t)) == cudaSuccess;
  if (ok) {
    ok = cudaMemcpy(static_cast<char*>(dev_handles) + rank * sizeof(mine), &mine, sizeof(mine),
                    cudaMemcpyHostToDevice) == cudaSuccess;
    ok = ok && api->all_gather(static_cast<char*>(dev_handles) + rank * sizeof(mine), dev_handles, sizeof(mine),
                               ncclChar, comm, st) == ncclSuccess;
    ok = ok && cudaStreamSynchronize(st) == cudaSuccess;
    ok = ok && cudaMemcpy(all.data(), dev_handles, world * sizeof(mine), cudaMemcpyDeviceToHost) == cudaSuccess;
  }
  if (dev_handles) cudaFree(dev_handles);
  for (int r = 0; ok && r < world; r++) {
    void* base = mem;
    if (r != rank &&
        cudaIpcOpenMemHandle(&base, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      ok = false;
    if (ok) p.buf[r] = static_cast<uint64_t*>(base);
  }
  p.epoch = reinterpret_cast<unsigned*>(static_cast<char*>(mem) + buf_bytes);
  if (!ok) {
    cudaGetLastError();
    tp_peers_release(&p, mem);
    return false;
  }
  *out = p;
  *own_mem = mem;
  return true;
}

void tp_peers_release(TpPeers* p, void* own_mem) {
  for (int r = 0; r < p->world && r < kTpMaxWorld; r++)
    if (r != p->rank && p->buf[r]) cudaIpcCloseMemHandle(p->buf[r]);
  if (own_mem) cudaFree(own_mem);
  *p = TpPeers();
}

}  // namespace prana
