// finish.cuh -- block-level "prepare the next projection's input" step:
// optional rmsnorm (norms.rs:9-23) then per-32 activation quantization
// (matmul.rs:105-127) of m rows, written to global memory.  Each 32-group is
// quantized by one thread with exactly the CPU path's operations.
#pragma once
#include "common.cuh"

namespace prana {

__device__ __forceinline__ void bar_sync_n(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Threads 0..nthreads-1 of the block call this together; `bar` is a named
// barrier those threads (and only they) use.  red: >= 8 * (nthreads/32) floats,
// inv_s: >= 8 floats of shared memory.
static __device__ __noinline__ void block_quantize_rows(const float* x, const float* norm_w, float eps, int m_rows, int n,
                                                 int8_t* q, float* s, int32_t* sum, float* red, float* inv_s,
                                                 int nthreads, int bar) {
  const int tid = threadIdx.x, wi = tid >> 5, lane = tid & 31, nw = nthreads >> 5, G = n / 32;
  if (norm_w) {
    for (int m = 0; m < m_rows; m++) {
      const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)m * n);
      float p = 0.0f;
      for (int i = tid; i < n / 4; i += nthreads) {
        const float4 v = __ldcg(x4 + i);
        p = fmaf(v.x, v.x, p);
        p = fmaf(v.y, v.y, p);
        p = fmaf(v.z, v.z, p);
        p = fmaf(v.w, v.w, p);
      }
      p = warp_sum(p);
      if (lane == 0) red[m * nw + wi] = p;
    }
    bar_sync_n(bar, nthreads);
    if (tid < m_rows) {
      float ss = 0.0f;
      for (int w = 0; w < nw; w++) ss += red[tid * nw + w];
      inv_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    }
    bar_sync_n(bar, nthreads);
  }
  for (int task = tid; task < m_rows * G; task += nthreads) {
    const int m = task / G, grp = task - m * G;
    const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)m * n + grp * 32);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 t = __ldcg(x4 + i);
      v[4 * i] = t.x;
      v[4 * i + 1] = t.y;
      v[4 * i + 2] = t.z;
      v[4 * i + 3] = t.w;
    }
    if (norm_w) {
      const float inv = inv_s[m];
      const float4* w4 = reinterpret_cast<const float4*>(norm_w + grp * 32);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float4 t = __ldg(w4 + i);
        v[4 * i] = __fmul_rn(__fmul_rn(v[4 * i], inv), t.x);
        v[4 * i + 1] = __fmul_rn(__fmul_rn(v[4 * i + 1], inv), t.y);
        v[4 * i + 2] = __fmul_rn(__fmul_rn(v[4 * i + 2], inv), t.z);
        v[4 * i + 3] = __fmul_rn(__fmul_rn(v[4 * i + 3], inv), t.w);
      }
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(v[i]));
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    int total = 0;
    uint32_t packed[8];
#pragma unroll
    for (int w = 0; w < 8; w++) {
      uint32_t word = 0;
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int qi = round_clamp127(__fmul_rn(v[w * 4 + b], inv));
        total += qi;
        word |= (uint32_t)(qi & 0xff) << (8 * b);
      }
      packed[w] = word;
    }
    uint4* dst = reinterpret_cast<uint4*>(q + (size_t)m * n + grp * 32);
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    s[(size_t)m * G + grp] = scale;
    sum[(size_t)m * G + grp] = total;
  }
}

}  // namespace prana
