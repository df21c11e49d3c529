// finish.cuh -- block-level "prepare the next projection's input" step:
// optional rmsnorm (norms.rs:9-23) then per-32 activation quantization
// (matmul.rs:105-127) of one row already staged in shared memory.
//
// One thread owns one 32-group: its 32 values are independent, so the
// per-element work (normalize, scale, round, clamp, pack) runs with full
// instruction-level parallelism and no shuffles; only amax and the group's two
// IEEE divides are serial.  Thread t reads the 16-byte pieces of its group
// starting at piece t mod 8, so a warp's shared-memory reads hit every bank
// once per wavefront.  Every value goes through exactly the CPU path's
// operations (amax, scale = amax / 127, q = round(x * (1 / scale)), clamp).
#pragma once
#include "common.cuh"

namespace prana {

// All threads of the block call this together.  xs: the f32 row [n] and ws:
// the rmsnorm weight [n] (null: plain quantization), both in shared memory;
// red: >= blockDim.x / 32 floats and inv_s: 1 float of shared scratch.
static __device__ __noinline__ void block_quantize_smem(const float* xs, const float* ws, float eps, int n, int8_t* q,
                                                        float* s, int32_t* sum, float* red, float* inv_s) {
  const int tid = threadIdx.x, nthreads = blockDim.x, wi = tid >> 5, lane = tid & 31, nw = nthreads >> 5;
  const int G = n / 32;
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const float4* w4 = reinterpret_cast<const float4*>(ws);
  float inv = 1.0f;
  if (ws) {
    float p = 0.0f;
    for (int grp = tid; grp < G; grp += nthreads) {
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const float4 v = x4[grp * 8 + ((k + tid) & 7)];
        p = fmaf(v.x, v.x, p);
        p = fmaf(v.y, v.y, p);
        p = fmaf(v.z, v.z, p);
        p = fmaf(v.w, v.w, p);
      }
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
  for (int grp = tid; grp < G; grp += nthreads) {
    float4 v[8];
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int idx = grp * 8 + ((k + tid) & 7);
      v[k] = x4[idx];
      if (ws) {
        const float4 wv = w4[idx];
        v[k].x = __fmul_rn(__fmul_rn(v[k].x, inv), wv.x);
        v[k].y = __fmul_rn(__fmul_rn(v[k].y, inv), wv.y);
        v[k].z = __fmul_rn(__fmul_rn(v[k].z, inv), wv.z);
        v[k].w = __fmul_rn(__fmul_rn(v[k].w, inv), wv.w);
      }
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
    }
    const float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float iv = __fdiv_rn(1.0f, scale);
    uint32_t* qw = reinterpret_cast<uint32_t*>(q) + grp * 8;
    int total = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int q0 = round_clamp127(__fmul_rn(v[k].x, iv)), q1 = round_clamp127(__fmul_rn(v[k].y, iv));
      const int q2 = round_clamp127(__fmul_rn(v[k].z, iv)), q3 = round_clamp127(__fmul_rn(v[k].w, iv));
      total += q0 + q1 + q2 + q3;
      qw[(k + tid) & 7] = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
                          ((uint32_t)(q3 & 0xff) << 24);
    }
    s[grp] = scale;
    sum[grp] = total;
  }
}

}  // namespace prana
