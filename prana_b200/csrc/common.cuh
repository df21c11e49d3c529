// common.cuh -- device-side building blocks shared by every prana_b200 kernel:
// the repacked weight views, streaming 128-bit loads, warp reductions,
// programmatic-dependent-launch hooks and the exact f16/quantization helpers
// the decode path needs to stay bit-compatible with Prana's CPU kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace prana {

// ggml type ids (crates/prana-model/src/gguf.rs:33-38), and one of this
// library: T_Q8S, the reference's in-memory QuantMatrix (int8 plane and one f32
// scale per 32 values, matmul.rs:21-30) that quantize_q8 (matmul.rs:61-84)
// produces -- its scales are arbitrary f32, not f16 like GGUF Q8_0's
enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_Q8S = 108 };

constexpr int WARP = 32;

// A quantized weight matrix [rows, cols] as laid out in HBM after upload.
//   Q8_0: qs = int8 plane [rows][cols],      d = f16 [rows][cols/32]
//   Q4_0: qs = nibble plane [rows][cols/2]   (16 B per block, GGUF byte order), d = f16 [rows][cols/32]
//   Q4_K: qs = GGUF super-blocks verbatim    [rows][cols/256][144] (144 = 9 x 16 B, so every
//         super-block is 16-byte aligned and needs no repacking)
//   Q6_K: qs = ql plane [rows][cols/2], qh = [rows][cols/4], sc = int8 [rows][cols/16], d = f16 [rows][cols/256]
//   Q8S : qs = int8 plane [rows][cols],      ds = f32 [rows][cols/32]
//   F32 : f32 = [rows][cols]
struct DevWeight {
  int type;
  int rows, cols;
  const uint8_t* qs;
  const uint8_t* qh;
  const int8_t* sc;
  const __half* d;
  const float* f32;
  const float* ds;
};

// ---- loads ----
// Weights are read exactly once per step: keep them out of L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned short ld_stream_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float h2f(unsigned short bits) { return __half2float(__ushort_as_half(bits)); }

// ---- programmatic dependent launch ----
// Kernels launched with the PDL attribute may start while their predecessor
// drains; they must wait here before touching anything it wrote.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bring a weight range toward L2 ahead of use (no register or smem cost).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- warp reductions ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- exact scalar semantics of the reference ----
// Rust `(x * inv).round().clamp(-127.0, 127.0) as i32`: roundf is round-half-away;
// clamp keeps a NaN (fminf/fmaxf would drop it) and `as` turns it into 0.
__device__ __forceinline__ int round_clamp127(float v) {
  const float r = roundf(v);
  if (r != r) return 0;
  return (int)fminf(fmaxf(r, -127.0f), 127.0f);
}

// Quantize one 32-group held one value per lane (crates/prana-kernels/src/matmul.rs:109-126):
// amax over |x| (NaN-ignoring), scale = amax/127 (1 if amax == 0), q = round(x * (1/scale)).
// Division and reciprocal are IEEE (built without fast-math), so the int8
// output is bit-identical to the CPU path for identical f32 input.
__device__ __forceinline__ void quant_group_lane(float x, int8_t* q_out, float* scale_out, int32_t* sum_out) {
  const int lane = threadIdx.x & 31;
  float amax = warp_max(fabsf(x));
  float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
  float inv = __fdiv_rn(1.0f, scale);
  int q = round_clamp127(__fmul_rn(x, inv));
  int s = warp_sum_i(q);
  q_out[lane] = (int8_t)q;
  if (lane == 0) {
    *scale_out = scale;
    *sum_out = s;
  }
}

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace prana
