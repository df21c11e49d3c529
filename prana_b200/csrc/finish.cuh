// finish.cuh -- block-level "prepare the next projection's input" step:
// optional rmsnorm (norms.rs:9-23) then per-32 activation quantization
// (matmul.rs:105-127) of one row already staged in shared memory.
//
// Eight consecutive threads own one 32-group (a float4 each), so a warp
// quantizes four groups per step with 3-step shuffle reductions; every value
// goes through exactly the CPU path's operations (amax, scale = amax / 127,
// q = round(x * (1 / scale)), clamp).
#pragma once
#include "common.cuh"

namespace prana {

// All threads of the block call this together.  xs: the f32 row [n] and ws:
// the rmsnorm weight [n] (null: plain quantization), both in shared memory;
// red: >= blockDim.x / 32 floats and inv_s: 1 float of shared scratch.
static __device__ __noinline__ void block_quantize_smem(const float* xs, const float* ws, float eps, int n, int8_t* q,
                                                        float* s, int32_t* sum, float* red, float* inv_s) {
  const int tid = threadIdx.x, nthreads = blockDim.x, wi = tid >> 5, lane = tid & 31, nw = nthreads >> 5;
  const int n4 = n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const float4* w4 = reinterpret_cast<const float4*>(ws);
  float inv = 1.0f;
  if (ws) {
    float p = 0.0f;
    for (int i = tid; i < n4; i += nthreads) {
      const float4 v = x4[i];
      p = fmaf(v.x, v.x, p);
      p = fmaf(v.y, v.y, p);
      p = fmaf(v.z, v.z, p);
      p = fmaf(v.w, v.w, p);
    }
    p = warp_sum(p);
    if (lane == 0) red[wi] = p;
    __syncthreads();
    if (tid == 0) {
      float ss = 0.0f;
      for (int w = 0; w < nw; w++) ss += red[w];
      inv_s[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    }
    __syncthreads();
    inv = inv_s[0];
  }
  // float4 i belongs to group i / 8; the loop bound is warp-uniform so every
  // shuffle sees the full warp
  for (int base = 0; base < n4; base += nthreads) {
    const int i = base + tid;
    const bool act = i < n4;
    float4 v = act ? x4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (act && ws) {
      const float4 wv = w4[i];
      v.x = __fmul_rn(__fmul_rn(v.x, inv), wv.x);
      v.y = __fmul_rn(__fmul_rn(v.y, inv), wv.y);
      v.z = __fmul_rn(__fmul_rn(v.z, inv), wv.z);
      v.w = __fmul_rn(__fmul_rn(v.w, inv), wv.w);
    }
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float iv = __fdiv_rn(1.0f, scale);
    const int q0 = round_clamp127(__fmul_rn(v.x, iv)), q1 = round_clamp127(__fmul_rn(v.y, iv));
    const int q2 = round_clamp127(__fmul_rn(v.z, iv)), q3 = round_clamp127(__fmul_rn(v.w, iv));
    int t = q0 + q1 + q2 + q3;
    t += __shfl_xor_sync(0xffffffffu, t, 1);
    t += __shfl_xor_sync(0xffffffffu, t, 2);
    t += __shfl_xor_sync(0xffffffffu, t, 4);
    if (act) {
      reinterpret_cast<uint32_t*>(q)[i] = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) |
                                          ((uint32_t)(q2 & 0xff) << 16) | ((uint32_t)(q3 & 0xff) << 24);
      if ((i & 7) == 0) {
        s[i / 8] = scale;
        sum[i / 8] = t;
      }
    }
  }
}

}  // namespace prana
