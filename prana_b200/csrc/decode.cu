// decode.cu -- the quantized GEMV that carries the decode step.
//
// Each warp owns RPW = 2 consecutive weight rows and streams them from HBM with
// 128-bit loads straight into registers (no shared-memory staging: at batch 1
// every weight byte is used once).  Rows longer than one chunk of loads are
// split across KS warps of the same CTA whose partial sums meet in shared
// memory.  The first chunk of weights is loaded before the kernel waits on its
// predecessor (programmatic dependent launch): weights never depend on it, so
// their DRAM latency overlaps the previous kernel's tail.  Lanes also
// bulk-prefetch the warp's next rows into L2 while it computes.
//
// Activation rows are staged in shared memory by the prologue:
//   PRO_Q     copy already-quantized int8 rows
//   PRO_F32   per-32 quantization of f32 rows            (matmul.rs:105-127)
//   PRO_NORM  rmsnorm, then per-32 quantization          (norms.rs:9-23)
// The per-block integer dots are exactly the reference's (gemv.cuh); each
// finished row goes through an epilogue:
//   EPI_STORE   out = W.x (+ bias)                      (Linear::apply)
//   EPI_RESID   out += W.x                              (x += wo.attn, x += w2.h)
//   EPI_ARGMAX  logits + first-max argmax               (Model::logits + argmax)
//   EPI_QKV     bias + RoPE + q / f16 K,V cache writes  (infer.rs:164-178)
//   EPI_SWIGLU  h = silu(gate) * up                     (infer.rs:192-199)
#include <climits>
#include <map>
#include <mutex>

#include "finish.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "mbar.cuh"

namespace prana {

constexpr int DG_WARPS = 8;
constexpr int DG_THREADS = DG_WARPS * 32;
constexpr int DG_RPW = 2;  // rows per warp; even, so RoPE and gate/up pairs never straddle warps

// Units a lane loads per chunk: enough 128-bit loads in flight per lane
// without spilling (a Q4_0 unit is 18 bytes, Q8_0 34, Q4_K 48, Q6_K 58).  At
// batch 1 two chunks per lane are in flight (the next one's while the current
// one computes), so the 48- and 58-byte units go one per chunk.
template <int T> constexpr int chunk_units() { return T == T_Q4_0 ? 4 : (T == T_Q4_K || T == T_Q6_K) ? 1 : 2; }
int gemv_chunk_units(int type) { return type == T_Q4_0 ? 4 : (type == T_Q4_K || type == T_Q6_K) ? 1 : 2; }

// Byte offset of the f32 staging row in a CTA's shared memory: after the int8
// rows, scales, sums and partial sums, rounded up to 16 bytes.
__host__ __device__ __forceinline__ size_t gemv_staging_offset(int M, int K) {
  const size_t b = (size_t)M * K + (size_t)M * (K / 32) * 8 + (size_t)DG_WARPS * DG_RPW * M * 4;
  return (b + 15) & ~(size_t)15;
}

// ---------------------------------------------------------------- epilogue of one finished row group

// Stored rows `row` (gate j) and row + 1 (up j) of activation row m:
// h[m][j] = silu(g) * u exactly as norms.rs:27-31 and infer.rs:197-199.
__device__ __forceinline__ void swiglu_pair(float* h, int N, int m, int row, float gv, float uv) {
  const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
  h[(size_t)m * (N / 2) + row / 2] = __fmul_rn(__fmul_rn(gv, sg), uv);
}

// Stored rows `row` and row + 1 (a RoPE pair of one projection; rows of a
// NeoX pair were made adjacent at upload) of activation row m: bias, RoPE at
// the row's position, then q out / f16 K and V cache rows / the f32 in-window
// K and V (infer.rs:164-178).
__device__ __forceinline__ void qkv_pair(const QkvMap& qm, int m, int row, float va, float vb) {
  int s = 0;
  while (s + 1 < qm.nseg && row >= qm.seg_start[s + 1]) s++;
  const int kind = qm.kind[s];
  const int p = (row - qm.seg_start[s]) / 2;  // pair index inside the projection
  const int half = qm.hd / 2;
  int ra, rb;
  if (kind != 2 && qm.neox) {
    ra = (p / half) * qm.hd + p % half;
    rb = ra + half;
  } else {
    ra = 2 * p;
    rb = ra + 1;
  }
  const int j = p % half;
  if (qm.bias[s]) {
    va = __fadd_rn(va, qm.bias[s][ra]);
    vb = __fadd_rn(vb, qm.bias[s][rb]);
  }
  const SeqRow* sr = qm.rows ? qm.rows + m : nullptr;
  const int pos = sr ? sr->pos : (qm.pos_dev ? *qm.pos_dev : qm.pos0) + m;
  if (kind != 2) {
    const float c = qm.cos_t[(size_t)pos * half + j], sn = qm.sin_t[(size_t)pos * half + j];
    const float a0 = va, b0 = vb;
    va = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(b0, sn));
    vb = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(b0, c));
  }
  if (kind == 0) {
    qm.q_out[(size_t)m * qm.q_dim + ra] = va;
    qm.q_out[(size_t)m * qm.q_dim + rb] = vb;
  } else {
    __half* cache = sr ? (kind == 1 ? sr->k : sr->v) + (size_t)qm.layer * sr->lstride : (kind == 1 ? qm.kc : qm.vc);
    if (pos < (sr ? sr->cap : qm.cap)) {
      cache[(size_t)pos * qm.kv_dim + ra] = __float2half_rn(va);
      cache[(size_t)pos * qm.kv_dim + rb] = __float2half_rn(vb);
    }
    float* win = kind == 1 ? qm.k_f32 : qm.v_f32;
    if (win) {
      win[(size_t)m * qm.kv_dim + ra] = va;
      win[(size_t)m * qm.kv_dim + rb] = vb;
    }
  }
}

// The batch path's epilogues over rows the tensor-core GEMM stored ([n][N]
// f32): the same per-pair arithmetic as the streaming GEMV's.
__global__ void qkv_finish_kernel(const float* y, int n, int N, const QkvMap qm) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // pair index over [n][N/2]
  if (i >= (size_t)n * (N / 2)) return;
  const int m = (int)(i / (N / 2)), row = 2 * (int)(i % (N / 2));
  qkv_pair(qm, m, row, y[(size_t)m * N + row], y[(size_t)m * N + row + 1]);
}

__global__ void swiglu_finish_kernel(const float* y, int n, int N, float* h) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)n * (N / 2)) return;
  const int m = (int)(i / (N / 2)), row = 2 * (int)(i % (N / 2));
  swiglu_pair(h, N, m, row, y[(size_t)m * N + row], y[(size_t)m * N + row + 1]);
}

cudaError_t launch_qkv_finish(const float* y, int n, int N, const QkvMap& qm, cudaStream_t st) {
  const size_t pairs = (size_t)n * (N / 2);
  qkv_finish_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, st>>>(y, n, N, qm);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_finish(const float* y, int n, int N, float* h, cudaStream_t st) {
  const size_t pairs = (size_t)n * (N / 2);
  swiglu_finish_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, st>>>(y, n, N, h);
  return cudaGetLastError();
}

// One CTA per row: (rmsnorm, then) per-32 quantization of an f32 row, with
// the streaming GEMV prologue's own routine (same int8 rows either path).
__global__ void __launch_bounds__(256) norm_quant_kernel(const float* x, const float* w, float eps, int K, int8_t* q,
                                                          float* s, int32_t* sum) {
  extern __shared__ __align__(16) float nq_smem[];
  __shared__ float red[8];
  __shared__ float inv_s[8];
  float* xs = nq_smem;
  float* ws = nq_smem + K;
  const size_t r = blockIdx.x;
  for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
    reinterpret_cast<float4*>(xs)[i] = __ldcg(reinterpret_cast<const float4*>(x + r * K) + i);
    if (w) reinterpret_cast<float4*>(ws)[i] = __ldg(reinterpret_cast<const float4*>(w) + i);
  }
  __syncthreads();
  block_quantize_smem(xs, w ? ws : nullptr, eps, K, q + r * K, s + r * (K / 32), sum + r * (K / 32), red, inv_s);
}

cudaError_t launch_norm_quant(const float* x, const float* w, float eps, int rows, int K, int8_t* q, float* s,
                              int32_t* sum, cudaStream_t st) {
  if (K % 32 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return cudaErrorInvalidValue;
  const size_t smem = (size_t)K * 4 * (w ? 2 : 1);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute((const void*)norm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) return e;
  }
  norm_quant_kernel<<<rows, 256, smem, st>>>(x, w, eps, K, q, s, sum);
  return cudaGetLastError();
}

// Lane m (< g.m) holds v[r] = row (r0 + r) . activation row m.
template <int EPI>
__device__ __forceinline__ void finish_rows(const StreamArgs& g, int r0, int m, const float (&v)[DG_RPW], float& run_v,
                                            int& run_i) {
  const int N = g.N;
  if constexpr (EPI == EPI_STORE || EPI == EPI_RESID || EPI == EPI_ARGMAX) {
#pragma unroll
    for (int r = 0; r < DG_RPW; r++) {
      const int row = r0 + r;
      if (row >= N) break;
      if constexpr (EPI == EPI_STORE) {
        float o = v[r];
        if (g.bias) o = __fadd_rn(o, g.bias[row]);
        g.out[(size_t)m * N + row] = o;
      } else if constexpr (EPI == EPI_RESID) {
        float* o = g.out + (size_t)m * N + row;
        *o = __fadd_rn(*o, v[r]);
      } else {
        if (g.out) g.out[(size_t)m * N + row] = v[r];
        if (v[r] > run_v || (v[r] == run_v && row < run_i)) {
          run_v = v[r];
          run_i = row;
        }
      }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
    for (int r = 0; r < DG_RPW; r += 2) {
      const int row = r0 + r;
      if (row >= N) break;
      swiglu_pair(g.out, N, m, row, v[r], v[r + 1]);
    }
  } else {  // EPI_QKV
#pragma unroll
    for (int r = 0; r < DG_RPW; r += 2) {
      const int row = r0 + r;
      if (row >= N) break;
      qkv_pair(g.qkv, m, row, v[r], v[r + 1]);
    }
  }
}

// Bulk-prefetch toward L2 the unit range [u0, u1) of rows [r0, r0 + RPW) of
// every plane; lane i < RPW * 4 issues at most one range.
template <int T>
__device__ __forceinline__ void prefetch_group(const DevWeight& w, int r0, int u0, int u1, int lane) {
  const int r = lane % DG_RPW, p = lane / DG_RPW;
  const int row = r0 + r;
  if (row >= w.rows || u0 >= u1) return;
  const size_t K = (size_t)w.cols;
  const size_t n = (size_t)(u1 - u0);
  if constexpr (T == T_Q8_0) {
    if (p == 0) prefetch_span(w.qs, row * K + (size_t)u0 * 32, n * 32);
    if (p == 1) prefetch_span(w.d, row * (K / 16) + (size_t)u0 * 2, n * 2);
  } else if constexpr (T == T_Q8S) {
    if (p == 0) prefetch_span(w.qs, row * K + (size_t)u0 * 32, n * 32);
    if (p == 1) prefetch_span(w.ds, row * (K / 8) + (size_t)u0 * 4, n * 4);
  } else if constexpr (T == T_Q4_0) {
    if (p == 0) prefetch_span(w.qs, row * (K / 2) + (size_t)u0 * 16, n * 16);
    if (p == 1) prefetch_span(w.d, row * (K / 16) + (size_t)u0 * 2, n * 2);
  } else if constexpr (T == T_Q4_K) {  // units are 64-weight pairs, 4 per 144-byte super-block
    const size_t b0 = u0 / 4, b1 = (u1 + 3) / 4;
    if (p == 0) prefetch_span(w.qs, row * (K / 256) * 144 + b0 * 144, (b1 - b0) * 144);
  } else {  // Q6_K: 4 units per 256-weight super-block
    const size_t b0 = u0 / 4, b1 = (u1 + 3) / 4;
    if (p == 0) prefetch_span(w.qs, row * (K / 2) + b0 * 128, (b1 - b0) * 128);
    if (p == 1) prefetch_span(w.qh, row * (K / 4) + b0 * 64, (b1 - b0) * 64);
    if (p == 2) prefetch_span(w.sc, row * (K / 16) + b0 * 16, (b1 - b0) * 16);
    if (p == 3) prefetch_span(w.d, row * (K / 128) + b0 * 2, (b1 - b0) * 2);
  }
}

// ---------------------------------------------------------------- the kernel

template <int T, int M, int EPI, int PRO>
__global__ void __launch_bounds__(DG_THREADS, 2) stream_gemv(const StreamArgs g) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int CH = chunk_units<T>();
  const DevWeight& w = g.w;
  const int K = g.K, G = K / 32, N = g.N;
  const int U = units_per_row(T, K);
  const int ks = g.ks, gpc = DG_WARPS / ks;  // warps per row group, row groups per CTA
  const int P = ceil_div(U, ks);             // units per K part
  const int n_groups = ceil_div(N, DG_RPW);
  const int n_tiles = ceil_div(n_groups, gpc);
  // shared layout: [int8 rows][scales][sums][partials][f32 row staging][norm weight][barriers]
  int8_t* sq = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(sq + (size_t)M * K);
  int32_t* ssum = reinterpret_cast<int32_t*>(ss + M * G);
  float* part = reinterpret_cast<float*>(ssum + M * G);  // [warp][RPW][M]
  // bulk-copy destinations start on 16 bytes (M * K + 8 * M * G bytes need not be a multiple of 16)
  float* xs = reinterpret_cast<float*>(smem + gemv_staging_offset(M, K));  // PRO_F32 / PRO_NORM: one f32 row
  float* ws = xs + (PRO == PRO_Q ? 0 : K);                                  // PRO_NORM: the rmsnorm weight
  uint64_t* bars = reinterpret_cast<uint64_t*>(ws + (PRO == PRO_NORM ? K : 0));  // [0]: rows, [1]: weight
  __shared__ float red[8 * DG_WARPS];
  __shared__ float inv_s[8];
  __shared__ int flag;
  __shared__ float wbest[DG_WARPS][8];
  __shared__ int widx[DG_WARPS][8];

  const int tid = threadIdx.x, wi = tid >> 5, lane = tid & 31;
  const int gs = wi / ks, kp = wi - gs * ks;
  const int u_lo = kp * P, u_hi = min(U, u_lo + P);
  if (PRO != PRO_Q && tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
    if (PRO == PRO_NORM) {  // the norm weight is constant: fetch it before the wait
      mbar_arrive_expect_tx(&bars[1], (uint32_t)K * 4);
      bulk_g2s(ws, g.norm_w, (uint32_t)K * 4, &bars[1]);
    }
  }

  Unit<T> buf[DG_RPW][CH];
  auto load_into = [&](Unit<T>(&b)[DG_RPW][CH], int r0, int c0) {
#pragma unroll
    for (int r = 0; r < DG_RPW; r++) {
      const int row = min(r0 + r, N - 1);
#pragma unroll
      for (int j = 0; j < CH; j++) {
        const int u = c0 + lane + 32 * j;
        if (u < u_hi) b[r][j] = load_unit<T>(w, row, u);
      }
    }
  };
  auto load = [&](int r0, int c0) { load_into(buf, r0, c0); };

  // Row groups: with whole rows per warp (ks == 1) the groups are dealt to the
  // warps of all CTAs in turn (group (k * 8 + warp) * grid + cta), so every SM
  // streams the same share of rows; with K split, CTA tiles of gpc groups.
  const int gstride = DG_WARPS * (int)gridDim.x;
  const int g_first = ks == 1 ? wi * (int)gridDim.x + (int)blockIdx.x : (int)blockIdx.x * gpc + gs;
  // weights first: they do not depend on the previous kernel
  int t = blockIdx.x;
  if ((ks == 1 || t < n_tiles) && g_first < n_groups) {
    const int r0 = g_first * DG_RPW;
    if (lane < DG_RPW * 4 && u_hi - u_lo > 32 * CH) prefetch_group<T>(w, r0, u_lo + 32 * CH, u_hi, lane);
    load(r0, u_lo);
  }
  // Batch-1 residual epilogue: the residual rows of the warp's first group are
  // read before the wait too.  The residual stream is never written by the
  // kernel this one waits on (attention before wo, gate|up before ffn_down):
  // its last writer finished before that kernel passed its own wait, which it
  // does before letting this kernel launch.
  float pre[DG_RPW] = {};
  constexpr bool kPre = EPI == EPI_RESID && M == 1;
  if (kPre && ks == 1 && lane == 0 && g_first < n_groups) {
#pragma unroll
    for (int r = 0; r < DG_RPW; r++)
      if (g_first * DG_RPW + r < N) pre[r] = __ldcg(g.out + g_first * DG_RPW + r);
  }
  __syncthreads();  // barrier initialization is visible to every waiting thread
  pdl_wait();
  if constexpr (PRO == PRO_Q) {
    const int nb = g.m * K / 16;
    for (int i = tid; i < nb; i += DG_THREADS)
      reinterpret_cast<uint4*>(sq)[i] = __ldcg(reinterpret_cast<const uint4*>(g.aq) + i);
    for (int i = tid; i < g.m * G; i += DG_THREADS) {
      ss[i] = __ldcg(g.as + i);
      ssum[i] = __ldcg(g.asum + i);
    }
  } else {
    // each f32 row arrives in shared memory with one bulk copy, then is
    // (normalized and) quantized from there
    bool ok = PRO != PRO_NORM || mbar_wait(&bars[1], 0);
    for (int m = 0; m < g.m; m++) {
      if (tid == 0) {
        mbar_arrive_expect_tx(&bars[0], (uint32_t)K * 4);
        bulk_g2s(xs, g.x + (size_t)m * K, (uint32_t)K * 4, &bars[0]);
      }
      ok = mbar_wait(&bars[0], m & 1) && ok;
      if (__syncthreads_or(!ok)) {
        if (tid == 0 && g.err) atomicExch(g.err, ERR_TIMEOUT);
        return;
      }
      block_quantize_smem(xs, PRO == PRO_NORM ? ws : nullptr, g.eps, K, sq + (size_t)m * K, ss + m * G, ssum + m * G,
                          red, inv_s);
      __syncthreads();  // the next row's copy overwrites the staging row
    }
  }
  __syncthreads();
  if (g.trace_q && blockIdx.x == 0) {
    for (int i = tid; i < g.m * K; i += DG_THREADS) g.trace_q[i] = sq[i];
    for (int i = tid; i < g.m * G; i += DG_THREADS) g.trace_s[i] = ss[i];
  }
  pdl_trigger();

  const Acts a{sq, ss, ssum, K, G};
  float run_v = -INFINITY;
  int run_i = INT_MAX;
  bool first = true;
  // Batch 1 with whole rows per warp: a flat sequence of (row group, chunk)
  // items with the next item's weights in flight while the current one computes.
  constexpr bool kPipe = M == 1;
  if (kPipe && ks == 1) {
    Unit<T> nb[DG_RPW][CH];
    int c0 = u_lo, gcur = g_first;
    bool have = gcur < n_groups;
    float accv[DG_RPW];
#pragma unroll
    for (int r = 0; r < DG_RPW; r++) accv[r] = 0.0f;
    auto step = [&](Unit<T>(&cur)[DG_RPW][CH], Unit<T>(&nxt)[DG_RPW][CH]) {
      int ng = gcur, nc = c0 + 32 * CH;
      if (nc >= u_hi) {
        nc = u_lo;
        ng = gcur + gstride;
      }
      const bool nhave = ng < n_groups;
      if (nhave) {
        load_into(nxt, ng * DG_RPW, nc);
        // the group after that toward L2 when a new group starts
        const int pg = ng + gstride;
        if (nc == u_lo && lane < DG_RPW * 4 && pg < n_groups) prefetch_group<T>(w, pg * DG_RPW, u_lo, u_hi, lane);
      }
#pragma unroll
      for (int j = 0; j < CH; j++) {
        const int u = c0 + lane + 32 * j;
        if (u < u_hi) {
          const ActU<T> au = load_act<T>(a, u);
#pragma unroll
          for (int r = 0; r < DG_RPW; r++) accum_r(cur[r][j], au, u, accv[r]);
        }
      }
      if (c0 + 32 * CH >= u_hi) {  // last chunk of the group: finish its rows
        float v[DG_RPW];
#pragma unroll
        for (int r = 0; r < DG_RPW; r++) {
          v[r] = warp_sum(accv[r]);
          accv[r] = 0.0f;
        }
        if (lane == 0) {
          if (kPre && gcur == g_first) {
#pragma unroll
            for (int r = 0; r < DG_RPW; r++)
              if (gcur * DG_RPW + r < N) g.out[gcur * DG_RPW + r] = __fadd_rn(pre[r], v[r]);
          } else {
            finish_rows<EPI>(g, gcur * DG_RPW, 0, v, run_v, run_i);
          }
        }
      }
      gcur = ng;
      c0 = nc;
      have = nhave;
    };
    while (have) {
      step(buf, nb);
      if (!have) break;
      step(nb, buf);
    }
  }
  for (int it = 0; !(kPipe && ks == 1); it++) {
    // ks == 1: this warp's it-th group (warps leave independently); ks > 1: the
    // CTA's it-th tile, every warp stays for the tile's barriers
    int grp, nxt;
    if (ks == 1) {
      grp = g_first + it * gstride;
      if (grp >= n_groups) break;
      nxt = grp + gstride;
    } else {
      t = blockIdx.x + it * gridDim.x;
      if (t >= n_tiles) break;
      grp = t * gpc + gs;
      nxt = t + (int)gridDim.x < n_tiles ? (t + gridDim.x) * gpc + gs : n_groups;
    }
    const bool live = grp < n_groups;
    const int r0 = grp * DG_RPW;
    // the next group's rows toward L2 while this one computes
    if (lane < DG_RPW * 4 && nxt < n_groups) prefetch_group<T>(w, nxt * DG_RPW, u_lo, u_hi, lane);
    float acc[DG_RPW][M];
#pragma unroll
    for (int r = 0; r < DG_RPW; r++)
#pragma unroll
      for (int m = 0; m < M; m++) acc[r][m] = 0.0f;
    if (live) {
      for (int c0 = u_lo; c0 < u_hi; c0 += 32 * CH) {
        if (!first) load(r0, c0);
        first = false;
        if constexpr (M == 1) {  // activations once per chunk, reused by every row
#pragma unroll
          for (int j = 0; j < CH; j++) {
            const int u = c0 + lane + 32 * j;
            if (u < u_hi) {
              const ActU<T> au = load_act<T>(a, u);
#pragma unroll
              for (int r = 0; r < DG_RPW; r++) accum_r(buf[r][j], au, u, acc[r][0]);
            }
          }
        } else {
#pragma unroll
          for (int r = 0; r < DG_RPW; r++)
#pragma unroll
            for (int j = 0; j < CH; j++) {
              const int u = c0 + lane + 32 * j;
              if (u < u_hi) accum_unit<M>(buf[r][j], u, a, g.m, acc[r]);
            }
        }
      }
    }
    first = false;
#pragma unroll
    for (int r = 0; r < DG_RPW; r++)
#pragma unroll
      for (int m = 0; m < M; m++) acc[r][m] = warp_sum(acc[r][m]);
    // lane m keeps activation row m's sums
    float v[DG_RPW];
#pragma unroll
    for (int r = 0; r < DG_RPW; r++) {
      v[r] = acc[r][0];
#pragma unroll
      for (int m = 1; m < M; m++)
        if (lane == m) v[r] = acc[r][m];
    }
    if (ks > 1) {  // K parts of a row group meet in shared memory; the part-0 warp finishes
      if (lane < M) {
#pragma unroll
        for (int r = 0; r < DG_RPW; r++) part[(wi * DG_RPW + r) * M + lane] = v[r];
      }
      __syncthreads();
      if (kp == 0 && lane < g.m) {
#pragma unroll
        for (int r = 0; r < DG_RPW; r++) {
          float s = 0.0f;
          for (int k = 0; k < ks; k++) s += part[((wi + k) * DG_RPW + r) * M + lane];
          v[r] = s;
        }
        if (live) finish_rows<EPI>(g, r0, lane, v, run_v, run_i);
      }
      __syncthreads();
    } else if (live && lane < g.m) {
      finish_rows<EPI>(g, r0, lane, v, run_v, run_i);
    }
  }

  // -------------------------------------------------- the next weights toward L2
  // A warp done with its rows spends the kernel's tail starting the next
  // matrix's first rows, so DRAM stays busy while the last rows finish and
  // the next kernel's first loads find L2.
  if (g.pf_rows > 0 && lane == 0) {
    const int nw = (int)gridDim.x * DG_WARPS, gw = (int)blockIdx.x * DG_WARPS + wi;
    const int rp = (g.pf_rows + nw - 1) / nw, r0 = gw * rp;
    if (r0 < g.pf_rows) prefetch_rows(g.pf_w, r0, min(rp, g.pf_rows - r0));
  }

  // -------------------------------------------------- cross-CTA argmax (Model::argmax: first maximum)
  if constexpr (EPI == EPI_ARGMAX) {
    if (lane < 8) {
      wbest[wi][lane] = run_v;
      widx[wi][lane] = run_i;
    }
    __syncthreads();
    if (tid < g.m) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int q = 0; q < DG_WARPS; q++)
        if (wbest[q][tid] > bv || (wbest[q][tid] == bv && widx[q][tid] < bi)) {
          bv = wbest[q][tid];
          bi = widx[q][tid];
        }
      g.part_val[(size_t)tid * gridDim.x + blockIdx.x] = bv;
      g.part_idx[(size_t)tid * gridDim.x + blockIdx.x] = bi;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) flag = atomicAdd(g.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!flag) return;
    __threadfence();
    for (int m = wi; m < g.m; m += DG_WARPS) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int b = lane; b < (int)gridDim.x; b += 32) {
        const float v_ = __ldcg(g.part_val + (size_t)m * gridDim.x + b);
        const int i_ = __ldcg(g.part_idx + (size_t)m * gridDim.x + b);
        if (v_ > bv || (v_ == bv && i_ < bi)) {
          bv = v_;
          bi = i_;
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
        const uint32_t tok = bi == INT_MAX ? 0u : (uint32_t)(bi + g.idx_offset);
        g.token_out[m] = tok;
        if (g.best_val) g.best_val[m] = bv;
        if (m == 0 && g.token_next) *g.token_next = (int)tok;
      }
    }
    if (tid == 0) *g.counter = 0u;
  }
}

// ---------------------------------------------------------------- launch

static int sw_sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev] && cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n[dev] = 148;
  return n[dev];
}

// Warps per row group.  A warp streams its rows chunk after chunk (the rest of
// its rows already on the way to L2), so K is split across warps only when the
// matrix has too few rows to give every SM a CTA.
int gemv_split_k(int type, int K, int N, int sm_count) {
  const int need = ceil_div(units_per_row(type, K), 32 * gemv_chunk_units(type));
  int ks = 1;
  while (ks < need && ks < DG_WARPS && ceil_div(ceil_div(N, DG_RPW), DG_WARPS / ks) < sm_count) ks *= 2;
  return ks;
}

size_t gemv_smem_bytes(int M, int K, int pro) {
  const size_t staging = pro == PRO_Q ? 0 : (size_t)K * 4 * (pro == PRO_NORM ? 2 : 1);
  return gemv_staging_offset(M, K) + staging + 16;
}

// Resident CTAs per SM of one kernel instance at a given shared-memory size
// (cached: the decode step asks on every launch).
static int resident_ctas(const void* k, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, size_t>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({k, smem});
  if (it != cache.end()) return it->second;
  int b = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k, DG_THREADS, smem) != cudaSuccess || b < 1) {
    cudaGetLastError();
    b = 1;
  }
  cache[{k, smem}] = b;
  return b;
}

template <int T, int M, int EPI, int PRO>
static cudaError_t stream_go(const StreamArgs& g, cudaStream_t st, bool pdl) {
  const size_t smem = gemv_smem_bytes(M, g.K, PRO);
  auto k = stream_gemv<T, M, EPI, PRO>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  StreamArgs a = g;
  a.ks = gemv_split_k(T, g.K, g.N, sw_sm_count());
  const int n_groups = ceil_div(g.N, DG_RPW);
  const int n_tiles = ceil_div(n_groups, DG_WARPS / a.ks);
  int grid = sw_sm_count() * resident_ctas((const void*)k, smem);
  // K split: one CTA per tile at most; whole rows: every resident CTA takes a share
  if (grid > (a.ks == 1 ? n_groups : n_tiles)) grid = a.ks == 1 ? n_groups : n_tiles;
  if (EPI == EPI_ARGMAX && (g.n_parts < grid || g.counter == nullptr)) return cudaErrorInvalidValue;
  void* args[] = {&a};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(DG_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelExC(&cfg, (const void*)k, args);
}

template <int T, int EPI, int PRO>
static cudaError_t stream_m(const StreamArgs& g, cudaStream_t st, bool pdl) {
  if (g.m <= 1) return stream_go<T, 1, EPI, PRO>(g, st, pdl);
  if (g.m <= 2) return stream_go<T, 2, EPI, PRO>(g, st, pdl);
  if (g.m <= 4) return stream_go<T, 4, EPI, PRO>(g, st, pdl);
  return stream_go<T, 8, EPI, PRO>(g, st, pdl);
}

template <int EPI, int PRO>
static cudaError_t stream_t(const StreamArgs& g, cudaStream_t st, bool pdl) {
  switch (g.w.type) {
    case T_Q8_0: return stream_m<T_Q8_0, EPI, PRO>(g, st, pdl);
    case T_Q8S: return stream_m<T_Q8S, EPI, PRO>(g, st, pdl);
    case T_Q4_0: return stream_m<T_Q4_0, EPI, PRO>(g, st, pdl);
    case T_Q4_K: return stream_m<T_Q4_K, EPI, PRO>(g, st, pdl);
    case T_Q6_K: return stream_m<T_Q6_K, EPI, PRO>(g, st, pdl);
  }
  return cudaErrorInvalidValue;
}

// The (epilogue, prologue) pairs the decode path uses:
//   Q|K|V, gate|up, LM head:  rmsnorm + quantize the residual stream in the prologue
//   wo, ffn_down:             quantize the attention output / silu(g)*u, residual epilogue
//   kernel-level matmuls:     pre-quantized rows, plain store (or rmsnorm'd for unfused gate/up)
//   tensor-parallel wo / ffn_down on ranks > 0: f32 rows, plain store of the partial product
cudaError_t launch_stream(const StreamArgs& g, int epi, int pro, cudaStream_t st, bool pdl) {
  if (g.m < 1 || g.m > 8 || g.K != g.w.cols || g.N != g.w.rows || g.K % 32) return cudaErrorInvalidValue;
  // bulk copies of f32 rows need 16-byte aligned sources
  if (pro != PRO_Q && ((reinterpret_cast<uintptr_t>(g.x) | reinterpret_cast<uintptr_t>(g.norm_w)) & 15))
    return cudaErrorInvalidValue;
  if ((epi == EPI_QKV || epi == EPI_SWIGLU) && g.N % 2) return cudaErrorInvalidValue;
  if (epi == EPI_QKV && pro == PRO_NORM) return stream_t<EPI_QKV, PRO_NORM>(g, st, pdl);
  if (epi == EPI_SWIGLU && pro == PRO_NORM) return stream_t<EPI_SWIGLU, PRO_NORM>(g, st, pdl);
  if (epi == EPI_ARGMAX && pro == PRO_NORM) return stream_t<EPI_ARGMAX, PRO_NORM>(g, st, pdl);
  if (epi == EPI_RESID && pro == PRO_F32) return stream_t<EPI_RESID, PRO_F32>(g, st, pdl);
  if (epi == EPI_STORE && pro == PRO_Q) return stream_t<EPI_STORE, PRO_Q>(g, st, pdl);
  if (epi == EPI_STORE && pro == PRO_NORM) return stream_t<EPI_STORE, PRO_NORM>(g, st, pdl);
  if (epi == EPI_STORE && pro == PRO_F32) return stream_t<EPI_STORE, PRO_F32>(g, st, pdl);  // tensor-parallel partials
  return cudaErrorInvalidValue;
}

}  // namespace prana
