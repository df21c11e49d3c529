// comm.h -- the NCCL calls of the tensor-parallel decode step, resolved at run
// time.  The process may already hold a libnccl.so.2 (PyTorch ships one); the
// library binds to that copy when it is loaded, else opens one itself, so two
// NCCL builds never meet in one process.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

#include <cstdint>

namespace prana {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

// The resolved entry points, or nullptr (with *why set) when NCCL is unavailable.
const Nccl* nccl(const char** why);

// One-shot all-reduce over NVLink peer memory.  Every rank owns a receive
// area of 2 (alternating calls) x world slots of `cap` 8-byte words, mapped
// into every other rank's address space.  A call stores each of this rank's
// values, tagged with the call's epoch, into its slot on every rank, waits
// (bounded) until every slot of its own area carries the epoch, and sums the
// slots in rank order, so every rank computes identical bits.
constexpr int kTpMaxWorld = 8;
struct TpPeers {
  int world = 1, rank = 0;
  size_t cap = 0;                      // words per slot
  uint64_t* buf[kTpMaxWorld] = {};     // each rank's receive area (this process's mapping)
  unsigned* epoch = nullptr;           // this rank's call counters, one per exchange CTA (device)
  uint32_t budget = 1u << 22;          // polls (20 ns apart at least) before a wait gives up
};
// Map every rank's receive area (exchanged with an NCCL all-gather of IPC
// handles); false when peer access is unavailable or world is not 2, 4 or 8.
bool tp_peers_setup(ncclComm_t comm, int world, int rank, size_t cap, cudaStream_t st, TpPeers* out,
                    void** own_mem);
void tp_peers_release(TpPeers* p, void* own_mem);
// x[0..n) = sum over ranks of every rank's x[0..n); err is raised when a wait
// gives up.  pdl: launched as a programmatic dependent of the kernel before it.
cudaError_t launch_tp_allreduce(const TpPeers& p, float* x, int n, unsigned* err, cudaStream_t st, bool pdl);
// dst[r * n .. r * n + n) = rank r's src[0..n); the two calls share the epoch sequence.
cudaError_t launch_tp_allgather(const TpPeers& p, const float* src, int n, float* dst, unsigned* err,
                                cudaStream_t st, bool pdl);

}  // namespace prana
