// kernels.cu -- decode-path kernels other than attention:
//   * quantize_acts                         (matmul.rs:105-127)
//   * gemv: Q8_0 / Q4_0 / Q4_K / Q6_K / F32 x M<=8 activation rows, with
//       prologue  = pre-quantized | quantize f32 | rmsnorm + quantize
//       epilogue  = store (+bias) | residual add | logits + argmax
//   * qkv:    rmsnorm -> Q|K|V GEMV -> bias -> RoPE -> f16 KV-cache write
//   * swiglu: rmsnorm -> gate|up GEMV -> silu(g)*u -> per-32 quantize for ffn_down
//   * glue:   rmsnorm, RoPE, silu, silu*mul, softmax, f16 KV write, embedding, argmax
// Everything that has to match the CPU path bit for bit uses explicit
// round-to-nearest intrinsics (no FMA contraction), IEEE divide and sqrt.
#include <cfloat>
#include <climits>

#include "gemv.cuh"
#include "internal.h"
#include "mbar.cuh"

namespace prana {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;

// ------------------------------------------------------------------ prologues
// Stage M activation rows into shared memory as (q, scale, sum).

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[wi] = v;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < nw; i++) t += red[i];
  return t;
}

// rmsnorm scale (norms.rs:15-17): inv = 1 / sqrt(Σx²/dim + eps)
__device__ __forceinline__ float rms_inv(const float* x, int dim, float eps, float* red) {
  float p = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) p = fmaf(x[i], x[i], p);
  const float ss = block_sum(p, red);
  const float mean_sq = __fdiv_rn(ss, (float)dim);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean_sq, eps)));
}

// Dense f32 weights (F32/F16 tensors densified at upload, matmul.rs:150-156).
template <int M, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_f32_kernel(const GemvArgs g) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = g.w.cols, N = g.w.rows;
  float* sx = reinterpret_cast<float*>(smem);
  pdl_wait();
  for (int i = threadIdx.x; i < g.m * K; i += blockDim.x) sx[i] = __ldcg(g.x + i);
  __syncthreads();
  pdl_trigger();
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * GEMV_WARPS + wi;
  if (row >= N) return;
  float acc[M];
#pragma unroll
  for (int m = 0; m < M; m++) acc[m] = 0.0f;
  const float* wr = g.w.f32 + (size_t)row * K;
  for (int k = lane * 4; k < K; k += 128) {
    if (k + 4 <= K) {
      const float4 wv = __ldcs(reinterpret_cast<const float4*>(wr + k));
#pragma unroll
      for (int m = 0; m < M; m++)
        if (m < g.m) {
          const float* xm = sx + m * K + k;
          acc[m] = fmaf(wv.x, xm[0], acc[m]);
          acc[m] = fmaf(wv.y, xm[1], acc[m]);
          acc[m] = fmaf(wv.z, xm[2], acc[m]);
          acc[m] = fmaf(wv.w, xm[3], acc[m]);
        }
    } else {
      for (int kk = k; kk < K; kk++)
        for (int m = 0; m < M && m < g.m; m++) acc[m] = fmaf(wr[kk], sx[m * K + kk], acc[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < M; m++) acc[m] = warp_sum(acc[m]);
  if (lane == 0)
    for (int m = 0; m < g.m && m < M; m++) {
      float* o = g.out + (size_t)m * N + row;
      if (EPI == EPI_RESID) *o = __fadd_rn(*o, acc[m]);
      else *o = g.bias ? __fadd_rn(acc[m], g.bias[row]) : acc[m];
    }
}

// ------------------------------------------------------------------ small kernels

__global__ void quantize_acts_kernel(const float* x, int rows, int k, int8_t* q, float* s, int32_t* sum) {
  const int G = k / 32;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= rows * G) return;
  const int r = gw / G, grp = gw % G;
  const float v = x[(size_t)r * k + grp * 32 + (threadIdx.x & 31)];
  quant_group_lane(v, q + (size_t)r * k + grp * 32, s + (size_t)r * G + grp, sum + (size_t)r * G + grp);
}

__global__ void rmsnorm_kernel(const float* x, const float* w, int dim, float eps, float* out) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * dim;
  const float inv = rms_inv(xr, dim, eps, red);
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    out[(size_t)blockIdx.x * dim + i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// RoPE from a (cos, sin) table [positions][hd/2] computed on the host with the
// same libm calls as the CPU path (attention.rs:90-121).
__global__ void rope_kernel(float* x, int rows, int n, int pos0, int hd, int neox, const float* cos_t,
                            const float* sin_t) {
  const int half = hd / 2, pairs = n / 2;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * pairs) return;
  const int r = i / pairs, p = i % pairs;
  int ia, ib, j;
  if (neox) {
    const int head = p / half;
    j = p % half;
    ia = head * hd + j;
    ib = ia + half;
  } else {
    ia = 2 * p;
    ib = ia + 1;
    j = p % half;
  }
  float* xr = x + (size_t)r * n;
  const int pos = pos0 + r;
  const float c = cos_t[(size_t)pos * half + j], s = sin_t[(size_t)pos * half + j];
  const float a = xr[ia], b = xr[ib];
  xr[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  xr[ib] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
}

__global__ void silu_kernel(float* x, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float v = x[i];
    x[i] = __fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))));
  }
}

__global__ void silu_mul_kernel(float* g, const float* u, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float v = g[i];
    g[i] = __fmul_rn(__fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)))), u[i]);
  }
}

// softmax over each row (norms.rs:44-56): max-subtract, exp, 1/sum
__global__ void softmax_kernel(const float* x, int n, float* out) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * n;
  float* o = out + (size_t)blockIdx.x * n;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, xr[i]);
  mx = warp_max(mx);
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[wi] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int i = 0; i < nw; i++) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float e = expf(__fsub_rn(xr[i], mx));
    o[i] = e;
    s = __fadd_rn(s, e);
  }
  s = block_sum(s, red);
  const float inv = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = __fmul_rn(o[i], inv);
}

__global__ void kv_write_kernel(__half* cache, size_t start, const float* src, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) cache[start + i] = __float2half_rn(src[i]);
}

// Token-embedding rows, dequantized exactly like the CPU tables
// (checkpoint.rs:169-174; kquant.rs:39-112 for packed formats).
__global__ void embed_kernel(const DevWeight w, const uint32_t* toks_dev, const int* tok_single, int m_rows, float* x) {
  const int dim = w.cols;
  const int m = blockIdx.y;
  if (m >= m_rows) return;
  const uint32_t tok = tok_single ? (uint32_t)*tok_single : toks_dev[m];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
    x[(size_t)m * dim + i] = embed_value(w, tok, i);
}

// argmax over each row: first index of the maximum (infer.rs:560-568)
__global__ void argmax_kernel(const float* x, int n, uint32_t* out) {
  __shared__ float bvs[32];
  __shared__ int bis[32];
  const float* xr = x + (size_t)blockIdx.x * n;
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xr[i];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bvs[wi] = bv;
    bis[wi] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bv = bvs[0];
    bi = bis[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (bvs[w] > bv || (bvs[w] == bv && bis[w] < bi)) {
        bv = bvs[w];
        bi = bis[w];
      }
    out[blockIdx.x] = bi == INT_MAX ? 0u : (uint32_t)bi;
  }
}

template <int T>
__global__ void block_dots_kernel(const DevWeight w, int row, const int8_t* aq, const int32_t* asum, int32_t* out) {
  const Acts a{aq, nullptr, asum, w.cols, w.cols / 32};
  const int nu = units_per_row(T, w.cols);
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < nu; u += gridDim.x * blockDim.x)
    unit_block_dots<T>(w, row, u, a, out);
}

// Step bookkeeping for the device-resident decode loop: the sampled token
// becomes the next input, the position advances, and the token is appended to
// the output ring.
__global__ void advance_kernel(int* tok, int* pos, uint32_t* ring, int ring_cap, int* ring_n) {
  pdl_wait();
  const int n = *ring_n;
  if (ring && n < ring_cap) ring[n] = (uint32_t)*tok;
  *ring_n = n + 1;
  *pos = *pos + 1;
}

// ------------------------------------------------------------------ launchers

static cudaError_t launch(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelExC(&cfg, fn, args);
}

template <typename K>
static cudaError_t set_smem(K kern, size_t smem) {
  if (smem > 48 * 1024) return cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return cudaSuccess;
}

// Dense f32 weights only; every quantized weight streams through decode.cu.
cudaError_t launch_gemv(const GemvArgs& g, int pro, int epi, cudaStream_t st, bool pdl) {
  if (g.m < 1 || g.m > 8 || g.w.type != T_F32 || pro != PRO_F32 || epi == EPI_ARGMAX) return cudaErrorInvalidValue;
  const size_t smem = (size_t)g.m * g.w.cols * 4;
  const int grid = ceil_div(g.w.rows, GEMV_WARPS);
  GemvArgs a = g;
  void* args[] = {&a};
#define F32GO(MM)                                                                                          \
  do {                                                                                                     \
    auto k = epi == EPI_RESID ? gemv_f32_kernel<MM, EPI_RESID> : gemv_f32_kernel<MM, EPI_STORE>;           \
    cudaError_t e = set_smem(k, smem);                                                                     \
    if (e != cudaSuccess) return e;                                                                        \
    return launch((const void*)k, dim3(grid), dim3(GEMV_THREADS), smem, st, args, pdl);                    \
  } while (0)
  if (g.m == 1) F32GO(1);
  if (g.m <= 2) F32GO(2);
  if (g.m <= 4) F32GO(4);
  F32GO(8);
#undef F32GO
}

cudaError_t launch_quantize_acts(const float* x, int rows, int k, int8_t* q, float* s, int32_t* sum, cudaStream_t st) {
  const int warps = rows * (k / 32);
  quantize_acts_kernel<<<ceil_div(warps * 32, 256), 256, 0, st>>>(x, rows, k, q, s, sum);
  return cudaGetLastError();
}
cudaError_t launch_rmsnorm(const float* x, const float* w, int rows, int dim, float eps, float* out, cudaStream_t st) {
  rmsnorm_kernel<<<rows, 256, 0, st>>>(x, w, dim, eps, out);
  return cudaGetLastError();
}
cudaError_t launch_rope(float* x, int rows, int n, int pos0, int hd, int neox, const float* c, const float* s,
                        cudaStream_t st) {
  const int tot = rows * (n / 2);
  rope_kernel<<<ceil_div(tot, 256), 256, 0, st>>>(x, rows, n, pos0, hd, neox, c, s);
  return cudaGetLastError();
}
cudaError_t launch_silu(float* x, size_t n, cudaStream_t st) {
  silu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, n);
  return cudaGetLastError();
}
cudaError_t launch_silu_mul(float* g, const float* u, size_t n, cudaStream_t st) {
  silu_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, n);
  return cudaGetLastError();
}
cudaError_t launch_softmax(const float* x, int rows, int n, float* out, cudaStream_t st) {
  softmax_kernel<<<rows, 256, 0, st>>>(x, n, out);
  return cudaGetLastError();
}
cudaError_t launch_kv_write(__half* cache, size_t start, const float* src, size_t n, cudaStream_t st) {
  kv_write_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(cache, start, src, n);
  return cudaGetLastError();
}
cudaError_t launch_embed(const DevWeight& w, const uint32_t* toks, const int* tok_single, int m, float* x,
                         cudaStream_t st, bool pdl) {
  DevWeight ww = w;
  void* args[] = {&ww, (void*)&toks, (void*)&tok_single, &m, &x};
  const int bx = ceil_div(w.cols, 256) < 8 ? ceil_div(w.cols, 256) : 8;
  return launch((const void*)embed_kernel, dim3(bx, m), dim3(256), 0, st, args, pdl);
}
cudaError_t launch_argmax(const float* x, int rows, int n, uint32_t* out, cudaStream_t st) {
  argmax_kernel<<<rows, 1024, 0, st>>>(x, n, out);
  return cudaGetLastError();
}
cudaError_t launch_block_dots(const DevWeight& w, int row, const int8_t* aq, const int32_t* asum, int32_t* out,
                              cudaStream_t st) {
  const int nu = units_per_row(w.type, w.cols);
  const int grid = ceil_div(nu, 128);
  switch (w.type) {
    case T_Q8_0: block_dots_kernel<T_Q8_0><<<grid, 128, 0, st>>>(w, row, aq, asum, out); break;
    case T_Q8S: block_dots_kernel<T_Q8S><<<grid, 128, 0, st>>>(w, row, aq, asum, out); break;
    case T_Q4_0: block_dots_kernel<T_Q4_0><<<grid, 128, 0, st>>>(w, row, aq, asum, out); break;
    case T_Q4_K: block_dots_kernel<T_Q4_K><<<grid, 128, 0, st>>>(w, row, aq, asum, out); break;
    case T_Q6_K: block_dots_kernel<T_Q6_K><<<grid, 128, 0, st>>>(w, row, aq, asum, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}
cudaError_t launch_advance(int* tok, int* pos, uint32_t* ring, int ring_cap, int* ring_n, cudaStream_t st, bool pdl) {
  void* args[] = {&tok, &pos, &ring, &ring_cap, &ring_n};
  return launch((const void*)advance_kernel, dim3(1), dim3(1), 0, st, args, pdl);
}


// ---------------------------------------------------------------- tensor-parallel argmax
// Each rank's LM-head shard reported (max, global index) per row; the first
// maximum over the ranks (larger value, or equal value at the smaller index)
// is the token, as Model::argmax picks the first maximum (infer.rs:560-568).
__global__ void tp_argmax_kernel(const float* all, int world, int m, uint32_t* tok_out, int* tok_next) {
  const int i = threadIdx.x;
  if (i >= m) return;
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  for (int r = 0; r < world; r++) {
    const float v = all[r * 16 + i];
    const uint32_t idx = __float_as_uint(all[r * 16 + 8 + i]);
    if (v > bv || (v == bv && idx < bi)) {
      bv = v;
      bi = idx;
    }
  }
  if (bi == 0xffffffffu) bi = 0;
  tok_out[i] = bi;
  if (i == 0 && tok_next) *tok_next = (int)bi;
}

cudaError_t launch_tp_argmax(const float* all, int world, int m, uint32_t* tok_out, int* tok_next, cudaStream_t st) {
  tp_argmax_kernel<<<1, 32, 0, st>>>(all, world, m, tok_out, tok_next);
  return cudaGetLastError();
}

// A bounded mbarrier wait on a barrier nothing arrives at: the wait gives up
// after `polls` tries and raises the error flag, as every kernel's waits do
// when a copy never completes.
__global__ void wait_never_kernel(unsigned polls, unsigned* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const bool ok = mbar_wait(&bar, 0, polls);
  if (threadIdx.x == 0 && !ok && err) atomicExch(err, ERR_TIMEOUT);
}

cudaError_t launch_wait_never(unsigned polls, unsigned* err, cudaStream_t st) {
  wait_never_kernel<<<1, 32, 0, st>>>(polls, err);
  return cudaGetLastError();
}

}  // namespace prana
