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

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// GATHER == false: x[i] = sum over ranks (all-reduce, in place).
// GATHER == true:  dst[r * n + i] = rank r's x[i] (all-gather).
template <bool GATHER>
__global__ void __launch_bounds__(1024) tp_exchange_kernel(const TpPeers p, float* x, int n, float* dst,
                                                           unsigned* err) {
  __shared__ int ok_all;
  const int tid = threadIdx.x;
  const unsigned e = *p.epoch + 1;  // this call's epoch (every rank counts in lockstep)
  const int par = (int)(e & 1);
  // push: this rank's values into its slot on every rank
  for (int r = 0; r < p.world; r++) {
    float* dst = p.buf[r] + ((size_t)par * p.world + p.rank) * p.cap;
    for (int i = tid; i < n; i += blockDim.x) dst[i] = x[i];
  }
  __syncthreads();
  // announce: the stores above happen before the flags (release at system scope)
  if (tid < p.world) {
    __threadfence_system();
    st_release_sys(p.flag[tid] + par * p.world + p.rank, e);
  }
  if (tid == 0) ok_all = 1;
  __syncthreads();
  // wait for every rank's values in this rank's area (bounded)
  if (tid < p.world) {
    const unsigned* f = p.flag[p.rank] + par * p.world + tid;
    bool ok = false;
    for (uint32_t i = 0; i < (1u << 24); i++) {
      if (ld_acquire_sys(f) == e) {
        ok = true;
        break;
      }
      __nanosleep(32);
    }
    if (!ok) {
      ok_all = 0;
      if (err) atomicExch(err, 1u);
    }
  }
  __syncthreads();
  // reduce in rank order (or lay the slots out side by side)
  const float* own = p.buf[p.rank] + (size_t)par * p.world * p.cap;
  if (GATHER) {
    if (ok_all)
      for (int r = 0; r < p.world; r++)
        for (int i = tid; i < n; i += blockDim.x) dst[(size_t)r * n + i] = own[(size_t)r * p.cap + i];
  } else if (ok_all)
    for (int i = tid; i < n; i += blockDim.x) {
      float s = own[i];
      for (int r = 1; r < p.world; r++) s += own[(size_t)r * p.cap + i];
      x[i] = s;
    }
  __syncthreads();
  if (tid == 0) *p.epoch = e;
}

}  // namespace

cudaError_t launch_tp_allreduce(const TpPeers& p, float* x, int n, unsigned* err, cudaStream_t st) {
  if (n <= 0 || (size_t)n > p.cap || p.world < 2) return cudaErrorInvalidValue;
  tp_exchange_kernel<false><<<1, 1024, 0, st>>>(p, x, n, nullptr, err);
  return cudaGetLastError();
}

cudaError_t launch_tp_allgather(const TpPeers& p, const float* src, int n, float* dst, unsigned* err,
                                cudaStream_t st) {
  if (n <= 0 || (size_t)n > p.cap || p.world < 2) return cudaErrorInvalidValue;
  tp_exchange_kernel<true><<<1, 1024, 0, st>>>(p, const_cast<float*>(src), n, dst, err);
  return cudaGetLastError();
}

bool tp_peers_setup(ncclComm_t comm, int world, int rank, size_t cap, cudaStream_t st, TpPeers* out,
                    void** own_mem) {
  const Nccl* api = nccl(nullptr);
  if (!api || world < 2 || world > kTpMaxWorld) return false;
  TpPeers p;
  p.world = world;
  p.rank = rank;
  p.cap = cap;
  // [2][world][cap] floats, then [2][world] flags, then the epoch counter
  const size_t buf_bytes = 2 * (size_t)world * cap * sizeof(float);
  const size_t bytes = buf_bytes + 2 * world * sizeof(unsigned) + 256;
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
    if (ok) {
      p.buf[r] = static_cast<float*>(base);
      p.flag[r] = reinterpret_cast<unsigned*>(static_cast<char*>(base) + buf_bytes);
    }
  }
  p.epoch = reinterpret_cast<unsigned*>(static_cast<char*>(mem) + buf_bytes + 2 * world * sizeof(unsigned));
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
