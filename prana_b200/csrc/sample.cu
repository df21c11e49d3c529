// sample.cu -- Sampler::sample (sampler.rs:22-37) on the device, so that a
// temperature-sampled decode keeps its logits in HBM: softmax(logits / temp)
// (norms.rs:44-56), one xorshift64* draw r (sampler.rs:59-70), and the first
// index whose cumulative probability reaches r.
//
// One cluster of 8 CTAs x 1024 threads; each CTA keeps 1/8 of the row in
// shared memory, so the logits are read once.  The maximum, the sum and the
// per-CTA probability totals cross the cluster through distributed shared
// memory.  Cumulative sums are taken in f64 over fixed-order trees (the
// result is deterministic run to run); the reference subtracts the f32
// probabilities from r one by one, so the two agree except where r lies
// within that sequential sum's rounding of a bucket boundary.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "internal.h"

namespace cg = cooperative_groups;

namespace prana {

namespace {

constexpr int kCtas = 8;
constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxSlice = 49152;  // floats of one CTA's share (192 KiB)

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_incl_scan(double v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  return v;
}

__global__ void __cluster_dims__(kCtas, 1, 1) __launch_bounds__(kThreads, 1)
    sample_kernel(const float* __restrict__ logits, int n, int slice, SampleState* state, uint32_t* tok_out,
                  int* tok_next) {
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ float e[];  // this CTA's share: scaled logits, then exp
  __shared__ float red_f[kWarps];
  __shared__ double red_d[kWarps];
  __shared__ float x_max;    // published: this CTA's maximum
  __shared__ double x_sum;   // published: this CTA's sum of exp
  __shared__ double x_tot;   // published: this CTA's probability total
  __shared__ unsigned x_tok; // rank 0: first index reaching r
  const int rank = (int)cluster.block_rank();
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int lo = rank * slice, len = max(0, min(n, lo + slice) - lo);
  // every CTA reads the state before the first cluster barrier; rank 0 writes
  // it back after the last one
  const unsigned long long s0 = state->rng;
  const float temp = state->temp;

  // logits / temp (an IEEE divide, as the reference's l / temp) and its maximum
  // (f32::max folds NaN away, as fmaxf does)
  float mx = -INFINITY;
  for (int i = t; i < len; i += kThreads) {
    const float v = logits[lo + i] / temp;
    e[i] = v;
    mx = fmaxf(mx, v);
  }
  mx = warp_max(mx);
  if (lane == 0) red_f[warp] = mx;
  if (t == 0) x_tok = 0xffffffffu;
  __syncthreads();
  if (warp == 0) {
    const float v = warp_max(red_f[lane]);
    if (lane == 0) x_max = v;
  }
  cluster.sync();
  float M = -INFINITY;
  for (int r = 0; r < kCtas; r++) M = fmaxf(M, *cluster.map_shared_rank(&x_max, r));

  // exp(v - max) and the sum
  double sum = 0.0;
  for (int i = t; i < len; i += kThreads) {
    const float v = expf(e[i] - M);
    e[i] = v;
    sum += (double)v;
  }
  sum = warp_sum(sum);
  if (lane == 0) red_d[warp] = sum;
  __syncthreads();
  if (warp == 0) {
    const double v = warp_sum(red_d[lane]);
    if (lane == 0) x_sum = v;
  }
  cluster.sync();
  double S = 0.0;
  for (int r = 0; r < kCtas; r++) S += *cluster.map_shared_rank(&x_sum, r);
  // the probabilities are the reference's: p = e * (1 / sum) in f32
  const float sum_f = (float)S;
  const float inv = sum_f > 0.0f ? 1.0f / sum_f : 0.0f;

  // XorShift::next_f32
  unsigned long long x = s0;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  const float r = (float)((x * 0x2545F4914F6CDD1DULL) >> 40) / 16777216.0f;

  // each thread's contiguous run of p (odd length: conflict-free banks), its
  // total, and the block's exclusive prefix of those totals
  const int chunk = ((len + kThreads - 1) / kThreads) | 1;
  const int c0 = min(len, t * chunk), c1 = min(len, c0 + chunk);
  double cs = 0.0;
  for (int i = c0; i < c1; i++) cs += (double)(e[i] * inv);
  const double incl = warp_incl_scan(cs, lane);
  if (lane == 31) red_d[warp] = incl;  // red_d was last read before the barrier above
  __syncthreads();
  if (warp == 0) red_d[lane] = warp_incl_scan(red_d[lane], lane);
  __syncthreads();
  const double excl = (warp ? red_d[warp - 1] : 0.0) + incl - cs;
  if (t == 0) x_tot = red_d[kWarps - 1];
  cluster.sync();
  double acc = excl;
  for (int q = 0; q < rank; q++) acc += *cluster.map_shared_rank(&x_tot, q);
  if (sum_f > 0.0f) {
    const double rd = (double)r;
    for (int i = c0; i < c1; i++) {
      acc += (double)(e[i] * inv);
      if (acc >= rd) {
        atomicMin(cluster.map_shared_rank(&x_tok, 0), (unsigned)(lo + i));
        break;
      }
    }
  }
  cluster.sync();
  if (rank == 0 && t == 0) {
    unsigned tok;
    if (sum_f > 0.0f) {
      tok = x_tok != 0xffffffffu ? x_tok : (unsigned)(n - 1);  // round-off: the last bucket
    } else {
      // a NaN or infinite logit: every p is 0 or NaN, so r -= p stays r (or
      // turns NaN) and only r == 0 with a number at index 0 stops early
      tok = (r <= 0.0f && !isnan(e[0])) ? 0u : (unsigned)(n - 1);
    }
    state->rng = x;
    tok_out[0] = tok;
    if (tok_next) *tok_next = (int)tok;
  }
}

}  // namespace

int sample_max_vocab() { return kCtas * kMaxSlice; }

cudaError_t launch_sample(const float* logits, int n, SampleState* state, uint32_t* tok_out, int* tok_next,
                          cudaStream_t st) {
  if (n < 1 || n > kCtas * kMaxSlice || !logits || !state || !tok_out) return cudaErrorInvalidValue;
  const int slice = (n + kCtas - 1) / kCtas;
  const size_t smem = (size_t)slice * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  sample_kernel<<<kCtas, kThreads, smem, st>>>(logits, n, slice, state, tok_out, tok_next);
  return cudaGetLastError();
}

}  // namespace prana
