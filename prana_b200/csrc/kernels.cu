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

template <int PRO>
__device__ void stage_acts(const GemvArgs& g, int K, int8_t* sq, float* ss, int32_t* ssum) {
  const int G = K / 32, wi = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if constexpr (PRO == PRO_Q) {
    const int nb = g.m * K / 16;
    for (int i = threadIdx.x; i < nb; i += blockDim.x)
      reinterpret_cast<uint4*>(sq)[i] = __ldcg(reinterpret_cast<const uint4*>(g.aq) + i);
    for (int i = threadIdx.x; i < g.m * G; i += blockDim.x) {
      ss[i] = __ldcg(g.as + i);
      ssum[i] = __ldcg(g.asum + i);
    }
  } else {
    __shared__ float red[32];
    for (int m = 0; m < g.m; m++) {
      const float* x = g.x + (size_t)m * K;
      float inv = 1.0f;
      if constexpr (PRO == PRO_NORM) inv = rms_inv(x, K, g.eps, red);
      for (int grp = wi; grp < G; grp += nw) {
        float v = __ldcg(x + grp * 32 + lane);
        if constexpr (PRO == PRO_NORM) v = __fmul_rn(__fmul_rn(v, inv), g.norm_w[grp * 32 + lane]);
        quant_group_lane(v, sq + m * K + grp * 32, ss + m * G + grp, ssum + m * G + grp);
      }
    }
  }
  __syncthreads();
  if (g.trace_q && blockIdx.x == 0) {
    for (int i = threadIdx.x; i < g.m * K; i += blockDim.x) g.trace_q[i] = sq[i];
    for (int i = threadIdx.x; i < g.m * G; i += blockDim.x) g.trace_s[i] = ss[i];
  }
}

__host__ __device__ inline size_t act_smem_bytes(int M, int K) { return (size_t)M * K + (size_t)M * (K / 32) * 8; }

// ------------------------------------------------------------------ generic GEMV

template <int T, int NR, int M, int UNR, int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_kernel(const GemvArgs g) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = g.w.cols, G = K / 32, N = g.w.rows;
  int8_t* sq = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(smem + (size_t)M * K);
  int32_t* ssum = reinterpret_cast<int32_t*>(ss + M * G);
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int rows[NR];
#pragma unroll
  for (int r = 0; r < NR; r++) {
    const int row = (blockIdx.x * GEMV_WARPS + wi) * NR + r;
    rows[r] = row < N ? row : -1;
  }
  pdl_wait();
  stage_acts<PRO>(g, K, sq, ss, ssum);
  pdl_trigger();
  const Acts a{sq, ss, ssum, K, G};
  float acc[NR][M];
  warp_dot<T, NR, M, UNR>(g.w, rows, a, g.m, acc);

  if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < NR; r++)
        if (rows[r] >= 0)
#pragma unroll
          for (int m = 0; m < M; m++)
            if (m < g.m) {
              float v = acc[r][m];
              float* o = g.out + (size_t)m * N + rows[r];
              if constexpr (EPI == EPI_STORE) {
                if (g.bias) v = __fadd_rn(v, g.bias[rows[r]]);
                *o = v;
              } else {
                *o = __fadd_rn(*o, v);
              }
            }
    }
  } else {  // EPI_ARGMAX: logits (optional) + first-max argmax per activation row
    __shared__ float wbest[GEMV_WARPS][M];
    __shared__ int widx[GEMV_WARPS][M];
    __shared__ unsigned ticket;
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < M; m++) {
        float bv = -INFINITY;
        int bi = INT_MAX;
#pragma unroll
        for (int r = 0; r < NR; r++)
          if (rows[r] >= 0 && m < g.m) {
            const float v = acc[r][m];
            if (g.out) g.out[(size_t)m * N + rows[r]] = v;
            if (v > bv || (v == bv && rows[r] < bi)) {
              bv = v;
              bi = rows[r];
            }
          }
        wbest[wi][m] = bv;
        widx[wi][m] = bi;
      }
    }
    __syncthreads();
    if (threadIdx.x < M && threadIdx.x < g.m) {
      const int m = threadIdx.x;
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int w = 0; w < GEMV_WARPS; w++) {
        const float v = wbest[w][m];
        const int i = widx[w][m];
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
      g.part_val[(size_t)m * gridDim.x + blockIdx.x] = bv;
      g.part_idx[(size_t)m * gridDim.x + blockIdx.x] = bi;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomicAdd(g.counter, 1u);
    __syncthreads();
    if (ticket == gridDim.x - 1) {
      __threadfence();
      for (int m = wi; m < g.m; m += GEMV_WARPS) {
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int b = lane; b < (int)gridDim.x; b += 32) {
          const float v = __ldcg(g.part_val + (size_t)m * gridDim.x + b);
          const int i = __ldcg(g.part_idx + (size_t)m * gridDim.x + b);
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
        if (lane == 0) {
          const uint32_t tok = bi == INT_MAX ? 0u : (uint32_t)bi;
          g.token_out[m] = tok;
          if (m == 0 && g.token_next) *g.token_next = (int)tok;
        }
      }
      if (threadIdx.x == 0) *g.counter = 0u;
    }
  }
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

// ------------------------------------------------------------------ fused Q|K|V

// Each warp computes one RoPE pair of rows of one of the three projections.
template <int T, int M, int PRO>
__global__ void __launch_bounds__(GEMV_THREADS) qkv_kernel(const QkvArgs g) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = g.w[0].cols, G = K / 32;
  int8_t* sq = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(smem + (size_t)M * K);
  int32_t* ssum = reinterpret_cast<int32_t*>(ss + M * G);
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = blockIdx.x * GEMV_WARPS + wi;
  int s = 0;
  while (s + 1 < g.nseg && p >= g.pair_start[s + 1]) s++;
  const bool active = p < g.pair_start[g.nseg];
  const int lp = p - g.pair_start[s];
  const int kind = g.kind[s];
  const int half = g.hd / 2;
  int ra, rb, j;
  if (kind != 2 && g.neox) {
    const int head = lp / half;
    j = lp % half;
    ra = head * g.hd + j;
    rb = ra + half;
  } else {
    ra = 2 * lp;
    rb = ra + 1;
    j = lp % half;
  }
  int rows[2] = {active ? ra : -1, active ? rb : -1};
  pdl_wait();
  stage_acts<PRO>(g.a, K, sq, ss, ssum);
  pdl_trigger();
  const Acts a{sq, ss, ssum, K, G};
  float acc[2][M];
  DevWeight w = g.w[0];
  if (s == 1) w = g.w[1];
  if (s == 2) w = g.w[2];
  warp_dot<T, 2, M, 4>(w, rows, a, g.a.m, acc);
  if (!active || lane >= M || lane >= g.a.m) return;
  // lane m finishes activation row m
  float va = acc[0][0], vb = acc[1][0];
#pragma unroll
  for (int m = 1; m < M; m++)
    if (lane == m) {
      va = acc[0][m];
      vb = acc[1][m];
    }
  const int m = lane;
  const float* bias = g.bias[s];
  if (bias) {
    va = __fadd_rn(va, bias[ra]);
    vb = __fadd_rn(vb, bias[rb]);
  }
  const int pos = (g.pos_dev ? *g.pos_dev : g.pos0) + m;
  if (kind != 2) {
    const float c = g.cos_t[(size_t)pos * half + j], sn = g.sin_t[(size_t)pos * half + j];
    const float a0 = va, b0 = vb;
    va = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(b0, sn));
    vb = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(b0, c));
  }
  if (kind == 0) {
    g.q_out[(size_t)m * g.q_dim + ra] = va;
    g.q_out[(size_t)m * g.q_dim + rb] = vb;
  } else {
    __half* cache = kind == 1 ? g.kc : g.vc;
    if (pos < g.cap) {
      cache[(size_t)pos * g.kv_dim + ra] = __float2half_rn(va);
      cache[(size_t)pos * g.kv_dim + rb] = __float2half_rn(vb);
    }
    float* win = kind == 1 ? g.k_f32 : g.v_f32;
    if (win) {
      win[(size_t)m * g.kv_dim + ra] = va;
      win[(size_t)m * g.kv_dim + rb] = vb;
    }
  }
}

// ------------------------------------------------------------------ fused gate|up -> SwiGLU -> quantize

template <int T, int M, int PRO>
__global__ void __launch_bounds__(GEMV_THREADS) swiglu_kernel(const SwigluArgs g) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = g.w1.cols, G = K / 32, H = g.w1.rows;
  int8_t* sq = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(smem + (size_t)M * K);
  int32_t* ssum = reinterpret_cast<int32_t*>(ss + M * G);
  __shared__ float hbuf[M][32];
  const int wi = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j0 = blockIdx.x * 32;
  int rows[4];
#pragma unroll
  for (int r = 0; r < 4; r++) rows[r] = j0 + wi * 4 + r < H ? j0 + wi * 4 + r : -1;
  pdl_wait();
  stage_acts<PRO>(g.a, K, sq, ss, ssum);
  pdl_trigger();
  const Acts a{sq, ss, ssum, K, G};
  float gt[4][M], up[4][M];
  warp_dot<T, 4, M, 2>(g.w1, rows, a, g.a.m, gt);
  warp_dot<T, 4, M, 2>(g.w3, rows, a, g.a.m, up);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < 4; r++)
#pragma unroll
      for (int m = 0; m < M; m++) {
        // silu(g)·u exactly as norms.rs:27-31 then infer.rs:197-199
        const float gv = gt[r][m];
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
        hbuf[m][wi * 4 + r] = __fmul_rn(__fmul_rn(gv, sg), up[r][m]);
      }
  }
  __syncthreads();
  const int HG = H / 32;
  for (int m = wi; m < g.a.m && m < M; m += GEMV_WARPS) {
    const float h = hbuf[m][lane];
    if (g.h_f32) g.h_f32[(size_t)m * H + j0 + lane] = h;
    quant_group_lane(h, g.hq + (size_t)m * H + j0, g.hs + (size_t)m * HG + blockIdx.x,
                     g.hsum + (size_t)m * HG + blockIdx.x);
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
  if (blockIdx.x == 0 && threadIdx.x == 0) pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
    float v;
    const size_t r = tok;
    switch (w.type) {
      case T_Q8_0:
        v = __fmul_rn((float)(int8_t)w.qs[r * dim + i], h2f(__half_as_ushort(w.d[r * (dim / 32) + i / 32])));
        break;
      case T_Q4_0: {
        const int b = i / 32, e = i % 32;
        const uint8_t byte = w.qs[r * (dim / 2) + b * 16 + (e & 15)];
        const int q = e < 16 ? (byte & 0xF) : (byte >> 4);
        v = __fmul_rn(h2f(__half_as_ushort(w.d[r * (dim / 32) + b])), __fsub_rn((float)q, 8.0f));
        break;
      }
      case T_Q4_K: {
        const uint8_t* sb = w.qs + r * (dim / 256) * 144 + (size_t)(i / 256) * 144;
        const int e = i % 256, pair = e / 64, hi = (e % 64) / 32, l = e % 32;
        int sc, mn;
        q4k_scale_min(pair * 2 + hi, sb + 4, sc, mn);
        const float d = h2f((unsigned short)(sb[0] | (sb[1] << 8))), dmin = h2f((unsigned short)(sb[2] | (sb[3] << 8)));
        const uint8_t byte = sb[16 + pair * 32 + l];
        const int q = hi ? (byte >> 4) : (byte & 0xF);
        v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
        break;
      }
      case T_Q6_K: {
        const int b = i / 256, e = i % 256, h = e / 128, g = (e % 128) / 32, l = e % 32;
        const uint8_t* ql = w.qs + r * (dim / 2) + (size_t)b * 128 + h * 64;
        const uint8_t* qh = w.qh + r * (dim / 4) + (size_t)b * 64 + h * 32;
        const int8_t* sc = w.sc + r * (dim / 16) + (size_t)b * 16;
        const int lo = (g & 1) ? ql[l + 32] : ql[l];
        const int nib = (g >> 1) ? (lo >> 4) : (lo & 0xF);
        const int q = (int)(int8_t)(nib | (((qh[l] >> (2 * g)) & 3) << 4)) - 32;
        const float d = h2f(__half_as_ushort(w.d[r * (dim / 256) + b]));
        v = __fmul_rn(__fmul_rn(d, (float)sc[h * 8 + l / 16 + 2 * g]), (float)q);
        break;
      }
      default:
        v = w.f32[r * dim + i];
    }
    x[(size_t)m * dim + i] = v;
  }
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

template <int T, int NR, int M, int UNR, int PRO, int EPI>
static cudaError_t gemv_go(const GemvArgs& g, cudaStream_t st, bool pdl) {
  const int rows_per_cta = GEMV_WARPS * NR;
  const int grid = ceil_div(g.w.rows, rows_per_cta);
  const size_t smem = act_smem_bytes(M, g.w.cols);
  auto kern = gemv_kernel<T, NR, M, UNR, PRO, EPI>;
  cudaError_t e = set_smem(kern, smem);
  if (e != cudaSuccess) return e;
  GemvArgs a = g;
  if (EPI == EPI_ARGMAX && a.n_parts < grid) return cudaErrorInvalidValue;
  void* args[] = {&a};
  return launch((const void*)kern, dim3(grid), dim3(GEMV_THREADS), smem, st, args, pdl);
}

template <int T, int PRO, int EPI>
static cudaError_t gemv_m(const GemvArgs& g, cudaStream_t st, bool pdl) {
  constexpr int NR = (T == T_Q8_0) ? 1 : 2;
  constexpr int UNR = (T == T_Q8_0) ? 4 : ((T == T_Q4_0) ? 4 : 2);
  if (g.m <= 1) return gemv_go<T, NR, 1, UNR, PRO, EPI>(g, st, pdl);
  if (g.m <= 2) return gemv_go<T, NR, 2, UNR, PRO, EPI>(g, st, pdl);
  if (g.m <= 4) return gemv_go<T, 1, 4, 2, PRO, EPI>(g, st, pdl);
  return gemv_go<T, 1, 8, 1, PRO, EPI>(g, st, pdl);
}

template <int PRO, int EPI>
static cudaError_t gemv_t(const GemvArgs& g, cudaStream_t st, bool pdl) {
  switch (g.w.type) {
    case T_Q8_0: return gemv_m<T_Q8_0, PRO, EPI>(g, st, pdl);
    case T_Q4_0: return gemv_m<T_Q4_0, PRO, EPI>(g, st, pdl);
    case T_Q4_K: return gemv_m<T_Q4_K, PRO, EPI>(g, st, pdl);
    case T_Q6_K: return gemv_m<T_Q6_K, PRO, EPI>(g, st, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemv(const GemvArgs& g, int pro, int epi, cudaStream_t st, bool pdl) {
  if (g.m < 1 || g.m > 8) return cudaErrorInvalidValue;
  if (g.w.type == T_F32) {
    if (pro != PRO_F32 || epi == EPI_ARGMAX) return cudaErrorInvalidValue;
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
#define GO(P, E) \
  if (pro == P && epi == E) return gemv_t<P, E>(g, st, pdl);
  GO(PRO_Q, EPI_STORE)
  GO(PRO_Q, EPI_RESID)
  GO(PRO_F32, EPI_STORE)
  GO(PRO_F32, EPI_RESID)
  GO(PRO_NORM, EPI_STORE)
  GO(PRO_NORM, EPI_ARGMAX)
  GO(PRO_F32, EPI_ARGMAX)
#undef GO
  return cudaErrorInvalidValue;
}

template <int T, int PRO>
static cudaError_t qkv_t(const QkvArgs& g, cudaStream_t st, bool pdl) {
  const int grid = ceil_div(g.pair_start[g.nseg], GEMV_WARPS);
  QkvArgs a = g;
  void* args[] = {&a};
#define QGO(MM)                                                                                     \
  do {                                                                                              \
    const size_t smem = act_smem_bytes(MM, g.w[0].cols);                                            \
    auto k = qkv_kernel<T, MM, PRO>;                                                                \
    cudaError_t e = set_smem(k, smem);                                                              \
    if (e != cudaSuccess) return e;                                                                 \
    return launch((const void*)k, dim3(grid), dim3(GEMV_THREADS), smem, st, args, pdl);             \
  } while (0)
  if (g.a.m <= 1) QGO(1);
  if (g.a.m <= 2) QGO(2);
  if (g.a.m <= 4) QGO(4);
  QGO(8);
#undef QGO
}

cudaError_t launch_qkv(const QkvArgs& g, int pro, cudaStream_t st, bool pdl) {
  if (g.a.m < 1 || g.a.m > 8 || g.nseg < 1 || g.nseg > 3) return cudaErrorInvalidValue;
  for (int i = 1; i < g.nseg; i++)
    if (g.w[i].type != g.w[0].type || g.w[i].cols != g.w[0].cols) return cudaErrorInvalidValue;
  const int t = g.w[0].type;
#define TGO(TT)                                              \
  if (t == TT) {                                             \
    if (pro == PRO_NORM) return qkv_t<TT, PRO_NORM>(g, st, pdl); \
    if (pro == PRO_F32) return qkv_t<TT, PRO_F32>(g, st, pdl);   \
    return qkv_t<TT, PRO_Q>(g, st, pdl);                     \
  }
  TGO(T_Q8_0) TGO(T_Q4_0) TGO(T_Q4_K) TGO(T_Q6_K)
#undef TGO
  return cudaErrorInvalidValue;
}

template <int T, int PRO>
static cudaError_t swiglu_t(const SwigluArgs& g, cudaStream_t st, bool pdl) {
  const int grid = g.w1.rows / 32;
  SwigluArgs a = g;
  void* args[] = {&a};
#define SGO(MM)                                                                                     \
  do {                                                                                              \
    const size_t smem = act_smem_bytes(MM, g.w1.cols);                                              \
    auto k = swiglu_kernel<T, MM, PRO>;                                                             \
    cudaError_t e = set_smem(k, smem);                                                              \
    if (e != cudaSuccess) return e;                                                                 \
    return launch((const void*)k, dim3(grid), dim3(GEMV_THREADS), smem, st, args, pdl);             \
  } while (0)
  if (g.a.m <= 1) SGO(1);
  if (g.a.m <= 2) SGO(2);
  if (g.a.m <= 4) SGO(4);
  SGO(8);
#undef SGO
}

cudaError_t launch_swiglu(const SwigluArgs& g, int pro, cudaStream_t st, bool pdl) {
  if (g.a.m < 1 || g.a.m > 8 || g.w1.type != g.w3.type || g.w1.rows != g.w3.rows || g.w1.cols != g.w3.cols ||
      g.w1.rows % 32)
    return cudaErrorInvalidValue;
#define TGO(TT)                                                     \
  if (g.w1.type == TT) {                                            \
    if (pro == PRO_NORM) return swiglu_t<TT, PRO_NORM>(g, st, pdl); \
    if (pro == PRO_F32) return swiglu_t<TT, PRO_F32>(g, st, pdl);   \
    return swiglu_t<TT, PRO_Q>(g, st, pdl);                         \
  }
  TGO(T_Q8_0) TGO(T_Q4_0) TGO(T_Q4_K) TGO(T_Q6_K)
#undef TGO
  return cudaErrorInvalidValue;
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

}  // namespace prana
