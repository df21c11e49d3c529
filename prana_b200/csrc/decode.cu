// decode.cu -- the streaming quantized GEMV that carries the decode step.
//
// Persistent CTAs, one producer thread + 8 consumer warps.  The producer
// streams contiguous row tiles of the packed weight planes global -> shared
// through a ring of `stages` bulk copies (cp.async.bulk + mbarrier), issuing
// the first stages before waiting on the predecessor kernel (weights do not
// depend on it), so the weight stream starts while the previous kernel drains.
// Consumer warps stage the int8 activations once per CTA, then compute
// per-block dp4a dots from shared memory (exactly the reference's per-block
// integers, see gemv.cuh) and run the epilogue for each finished row:
//   EPI_STORE   out = W.x (+ bias)                      (Linear::apply)
//   EPI_RESID   out += W.x                              (x += wo.attn, x += w2.h)
//   EPI_ARGMAX  logits + first-max argmax               (Model::logits + argmax)
//   EPI_QKV     bias + RoPE + q / f16 K,V cache writes  (infer.rs:164-178)
//   EPI_SWIGLU  h = silu(gate) * up                     (infer.rs:192-199)
// and the last CTA to finish runs a "finisher" that prepares the next kernel's
// input once for everyone: rmsnorm + per-32 quantization of the residual
// stream (FIN_NORM_Q) or plain quantization (FIN_Q).
#include <climits>

#include "finish.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "tma.cuh"

namespace prana {

constexpr int SW_CONSUMERS = 8;                     // consumer warps
constexpr int SW_THREADS = (SW_CONSUMERS + 1) * 32;  // + one producer warp
constexpr int SW_CT = SW_CONSUMERS * 32;

// ---------------------------------------------------------------- units from shared memory

struct StageView {
  const uint8_t* p[4];  // plane bases inside the stage
  int rb[4];            // bytes per row of each plane
};

template <int T> __device__ __forceinline__ Unit<T> load_unit_s(const StageView& v, int lr, int u);

template <> __device__ __forceinline__ Unit<T_Q8_0> load_unit_s<T_Q8_0>(const StageView& v, int lr, int u) {
  Unit<T_Q8_0> x;
  const uint8_t* q = v.p[0] + lr * v.rb[0] + u * 32;
  x.a = *reinterpret_cast<const uint4*>(q);
  x.b = *reinterpret_cast<const uint4*>(q + 16);
  x.d = *reinterpret_cast<const unsigned short*>(v.p[1] + lr * v.rb[1] + u * 2);
  return x;
}
template <> __device__ __forceinline__ Unit<T_Q4_0> load_unit_s<T_Q4_0>(const StageView& v, int lr, int u) {
  Unit<T_Q4_0> x;
  x.q = *reinterpret_cast<const uint4*>(v.p[0] + lr * v.rb[0] + u * 16);
  x.d = *reinterpret_cast<const unsigned short*>(v.p[1] + lr * v.rb[1] + u * 2);
  return x;
}
template <> __device__ __forceinline__ Unit<T_Q4_K> load_unit_s<T_Q4_K>(const StageView& v, int lr, int u) {
  Unit<T_Q4_K> x;
  const uint8_t* sb = v.p[0] + lr * v.rb[0] + (u >> 2) * 144;
  x.a = *reinterpret_cast<const uint4*>(sb + 16 + (u & 3) * 32);
  x.b = *reinterpret_cast<const uint4*>(sb + 32 + (u & 3) * 32);
  x.meta = *reinterpret_cast<const uint4*>(sb);
  return x;
}
template <> __device__ __forceinline__ Unit<T_Q6_K> load_unit_s<T_Q6_K>(const StageView& v, int lr, int u) {
  Unit<T_Q6_K> x;
  const int b = u >> 2, h = (u >> 1) & 1, l0 = (u & 1) * 16;
  const uint8_t* ql = v.p[0] + lr * v.rb[0] + b * 128 + h * 64 + l0;
  x.lo = *reinterpret_cast<const uint4*>(ql);
  x.hi = *reinterpret_cast<const uint4*>(ql + 32);
  x.qh = *reinterpret_cast<const uint4*>(v.p[1] + lr * v.rb[1] + b * 64 + h * 32 + l0);
  x.sc = *reinterpret_cast<const uint2*>(v.p[2] + lr * v.rb[2] + b * 16 + h * 8);
  x.d = *reinterpret_cast<const unsigned short*>(v.p[3] + lr * v.rb[3] + b * 2);
  return x;
}

// ---------------------------------------------------------------- the kernel

// PRO selects how the consumers stage the activation rows while the producer's
// first weight tiles are already in flight: PRO_Q copies int8 rows, PRO_F32
// quantizes f32 rows, PRO_NORM applies rmsnorm then quantizes.
template <int T, int M, int EPI, int PRO>
__global__ void __launch_bounds__(SW_THREADS, 1) stream_gemv(const StreamArgs g) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = g.K, G = K / 32, N = g.N;
  const TilePlan& tp = g.plan;
  const int R = tp.R, wpr = tp.wpr, S = tp.stages;
  const int ntiles = ceil_div(N, R);
  const int n_my = (int)blockIdx.x < ntiles ? ceil_div(ntiles - (int)blockIdx.x, (int)gridDim.x) : 0;
  // shared layout: [stages x stage_bytes][acts][partials][barriers]
  uint8_t* stage0 = smem;
  int8_t* sq = reinterpret_cast<int8_t*>(smem + (size_t)S * tp.stage_bytes);
  float* ss = reinterpret_cast<float*>(sq + (size_t)M * K);
  int32_t* ssum = reinterpret_cast<int32_t*>(ss + M * G);
  float* part = reinterpret_cast<float*>(ssum + M * G);  // [R][wpr][M]
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(part + R * wpr * M) + 7) & ~(uintptr_t)7);
  uint64_t* empty = full + S;
  __shared__ float red[8 * SW_CONSUMERS];
  __shared__ float inv_s[8];
  __shared__ int flag;
  __shared__ float wbest[SW_CONSUMERS][8];
  __shared__ int widx[SW_CONSUMERS][8];

  const int tid = threadIdx.x, wi = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (wi == SW_CONSUMERS) {
    // ------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      for (int i = 0; i < n_my; i++) {
        const int st = i % S;
        if (i >= S && !mbar_wait(&empty[st], ((i / S) - 1) & 1)) {
          atomicExch(g.err, ERR_TIMEOUT);
          break;
        }
        const int t = blockIdx.x + i * gridDim.x;
        const int r0 = t * R, rows = min(R, N - r0);
        uint32_t bytes[4], total = 0;
        for (int p = 0; p < tp.nplanes; p++) {
          bytes[p] = (uint32_t)(((size_t)rows * tp.row_bytes[p] + 15) & ~(size_t)15);
          total += bytes[p];
        }
        mbar_arrive_expect_tx(&full[st], total);
        uint8_t* dst = stage0 + (size_t)st * tp.stage_bytes;
        for (int p = 0; p < tp.nplanes; p++)
          bulk_g2s(dst + tp.smem_off[p], tp.plane[p] + (size_t)r0 * tp.row_bytes[p], bytes[p], &full[st], pol);
      }
    }
    return;
  }

  // -------------------------------------------------- consumers
  pdl_wait();
  if constexpr (PRO == PRO_Q) {  // stage already-quantized activation rows
    const int nb = g.m * K / 16;
    for (int i = tid; i < nb; i += SW_CT) reinterpret_cast<uint4*>(sq)[i] = __ldcg(reinterpret_cast<const uint4*>(g.aq) + i);
    for (int i = tid; i < g.m * G; i += SW_CT) {
      ss[i] = __ldcg(g.as + i);
      ssum[i] = __ldcg(g.asum + i);
    }
  } else {  // (rmsnorm +) per-32 quantization, one group per thread
    block_quantize_rows(g.x, PRO == PRO_NORM ? g.norm_w : nullptr, g.eps, g.m, K, sq, ss, ssum, red, inv_s, SW_CT, 1);
  }
  consumer_sync(SW_CT);
  if (g.trace_q && blockIdx.x == 0) {
    for (int i = tid; i < g.m * K; i += SW_CT) g.trace_q[i] = sq[i];
    for (int i = tid; i < g.m * G; i += SW_CT) g.trace_s[i] = ss[i];
  }
  pdl_trigger();
  const Acts a{sq, ss, ssum, K, G};
  const int U = units_per_row(T, K);
  float run_v[M];
  int run_i[M];
#pragma unroll
  for (int m = 0; m < M; m++) {
    run_v[m] = -INFINITY;
    run_i[m] = INT_MAX;
  }
  bool ok = true;
  for (int i = 0; i < n_my; i++) {
    const int st = i % S;
    if (tid == 0) flag = mbar_wait(&full[st], (i / S) & 1) ? 1 : 0;
    consumer_sync(SW_CT);
    if (!flag) {
      if (tid == 0) atomicExch(g.err, ERR_TIMEOUT);
      ok = false;
      break;
    }
    const int t = blockIdx.x + i * gridDim.x;
    const int r0 = t * R, rows = min(R, N - r0);
    StageView v;
    const uint8_t* sb = stage0 + (size_t)st * tp.stage_bytes;
#pragma unroll
    for (int p = 0; p < 4; p++) {
      v.p[p] = sb + tp.smem_off[p];
      v.rb[p] = tp.row_bytes[p];
    }
    // work items: (row, K-segment); a warp takes items wi, wi + 8, ...
    const int items = rows * wpr;
    for (int it = wi; it < items; it += SW_CONSUMERS) {
      const int lr = it / wpr, ks = it - lr * wpr;
      const int u0 = ks * U / wpr, u1 = (ks + 1) * U / wpr;
      float acc[M];
#pragma unroll
      for (int m = 0; m < M; m++) acc[m] = 0.0f;
      int u = u0 + lane;
      for (; u + 32 < u1; u += 64) {
        const Unit<T> x0 = load_unit_s<T>(v, lr, u);
        const Unit<T> x1 = load_unit_s<T>(v, lr, u + 32);
        accum_unit<M>(x0, u, a, g.m, acc);
        accum_unit<M>(x1, u + 32, a, g.m, acc);
      }
      if (u < u1) accum_unit<M>(load_unit_s<T>(v, lr, u), u, a, g.m, acc);
#pragma unroll
      for (int m = 0; m < M; m++) acc[m] = warp_sum(acc[m]);
      if (lane < M) {
        float mine = acc[0];
#pragma unroll
        for (int m = 1; m < M; m++)
          if (lane == m) mine = acc[m];
        part[(lr * wpr + ks) * M + lane] = mine;
      }
    }
    consumer_sync(SW_CT);
    if (tid == 0) mbar_arrive(&empty[st]);  // the stage's bytes are no longer read
    // ---- epilogue: one thread per (output, activation row)
    const int pairs = (EPI == EPI_QKV || EPI == EPI_SWIGLU) ? 2 : 1;
    const int outs = rows / pairs;
    for (int o = tid; o < outs * g.m; o += SW_CT) {
      const int oi = o / g.m, m = o - oi * g.m;
      float val[2] = {0.0f, 0.0f};
      for (int pp = 0; pp < pairs; pp++)
        for (int ks = 0; ks < wpr; ks++) val[pp] += part[((oi * pairs + pp) * wpr + ks) * M + m];
      const int row = r0 + oi * pairs;  // stored row (first of the pair)
      if constexpr (EPI == EPI_STORE) {
        float r = val[0];
        if (g.bias) r = __fadd_rn(r, g.bias[row]);
        g.out[(size_t)m * N + row] = r;
      } else if constexpr (EPI == EPI_RESID) {
        float* o_ = g.out + (size_t)m * N + row;
        *o_ = __fadd_rn(*o_, val[0]);
      } else if constexpr (EPI == EPI_ARGMAX) {
        if (g.out) g.out[(size_t)m * N + row] = val[0];
        // per-thread running max over the rows it finalizes
        if (val[0] > run_v[m < M ? m : 0] || (val[0] == run_v[m < M ? m : 0] && row < run_i[m < M ? m : 0])) {
          run_v[m < M ? m : 0] = val[0];
          run_i[m < M ? m : 0] = row;
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        // stored rows 2j (gate) and 2j+1 (up): silu(g)*u exactly as norms.rs:27-31, infer.rs:197-199
        const float gv = val[0];
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
        g.out[(size_t)m * (N / 2) + row / 2] = __fmul_rn(__fmul_rn(gv, sg), val[1]);
      } else {  // EPI_QKV
        const QkvMap& qm = g.qkv;
        int s = 0;
        while (s + 1 < qm.nseg && row >= qm.seg_start[s + 1]) s++;
        const int kind = qm.kind[s];
        const int p = (row - qm.seg_start[s]) / 2;  // pair index inside the projection
        const int half = qm.hd / 2;
        int ra, rb, j;
        if (kind != 2 && qm.neox) {
          ra = (p / half) * qm.hd + p % half;
          rb = ra + half;
          j = p % half;
        } else {
          ra = 2 * p;
          rb = ra + 1;
          j = p % half;
        }
        float va = val[0], vb = val[1];
        if (qm.bias[s]) {
          va = __fadd_rn(va, qm.bias[s][ra]);
          vb = __fadd_rn(vb, qm.bias[s][rb]);
        }
        const int pos = (qm.pos_dev ? *qm.pos_dev : qm.pos0) + m;
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
          __half* cache = kind == 1 ? qm.kc : qm.vc;
          if (pos < qm.cap) {
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
    }
    consumer_sync(SW_CT);  // `part` is rewritten by the next tile
  }
  if (!ok) return;

  // -------------------------------------------------- cross-CTA completion
  if constexpr (EPI == EPI_ARGMAX) {
    // reduce the per-thread running maxima of this CTA, per activation row
    for (int m = 0; m < g.m && m < M; m++) {
      float bv = run_v[m];
      int bi = run_i[m];
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
        wbest[wi][m] = bv;
        widx[wi][m] = bi;
      }
    }
    consumer_sync(SW_CT);
    if (tid < g.m) {
      float bv = -INFINITY;
      int bi = INT_MAX;
      for (int w = 0; w < SW_CONSUMERS; w++)
        if (wbest[w][tid] > bv || (wbest[w][tid] == bv && widx[w][tid] < bi)) {
          bv = wbest[w][tid];
          bi = widx[w][tid];
        }
      g.part_val[(size_t)tid * gridDim.x + blockIdx.x] = bv;
      g.part_idx[(size_t)tid * gridDim.x + blockIdx.x] = bi;
    }
  }
  if (g.counter == nullptr) return;
  __threadfence();
  consumer_sync(SW_CT);
  if (tid == 0) flag = atomicAdd(g.counter, 1u) == gridDim.x - 1;
  consumer_sync(SW_CT);
  if (!flag) return;
  __threadfence();
  if constexpr (EPI == EPI_ARGMAX) {
    for (int m = wi; m < g.m; m += SW_CONSUMERS) {
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
        const uint32_t tok = bi == INT_MAX ? 0u : (uint32_t)bi;
        g.token_out[m] = tok;
        if (m == 0 && g.token_next) *g.token_next = (int)tok;
      }
    }
  }
  if (g.fin_x)
    block_quantize_rows(g.fin_x, g.fin_norm, g.fin_eps, g.m, g.fin_n, g.fin_q, g.fin_s, g.fin_sum, red, inv_s, SW_CT, 1);
  if (tid == 0) *g.counter = 0u;
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

int row_plane_bytes(int type, int K, int* rb) {
  switch (type) {
    case T_Q8_0: rb[0] = K; rb[1] = K / 16; return 2;
    case T_Q4_0: rb[0] = K / 2; rb[1] = K / 16; return 2;
    case T_Q4_K: rb[0] = K / 256 * 144; return 1;
    case T_Q6_K: rb[0] = K / 2; rb[1] = K / 4; rb[2] = K / 16; rb[3] = K / 128; return 4;
  }
  return 0;
}

static size_t acts_bytes(int M, int K) { return (size_t)M * K + (size_t)M * (K / 32) * 8; }

// Tile plan for a weight: rows per tile, warps per row, ring depth.
// Budget: SMEM_BUDGET bytes per CTA (one CTA per SM).
bool plan_tiles(const DevWeight& w, int M, int budget, int min_rows_multiple, TilePlan& tp) {
  int rb[4] = {0, 0, 0, 0};
  const int np = row_plane_bytes(w.type, w.cols, rb);
  if (!np) return false;
  int row = 0;
  bool aligned = true;
  for (int p = 0; p < np; p++) {
    row += rb[p];
    if (rb[p] % 16) aligned = false;
  }
  const size_t acts = acts_bytes(M, w.cols);
  const int cand[] = {64, 48, 32, 24, 16, 8, 4, 2, 1};
  // largest tile that still leaves >= 3 stages in flight, else >= 2
  for (int pass = 0; pass < 2; pass++)
  for (int R : cand) {
    if (R % min_rows_multiple) continue;
    if (R < 8 && !aligned) continue;
    const int wpr = R >= SW_CONSUMERS ? 1 : SW_CONSUMERS / R;
    size_t stage = 0;
    for (int p = 0; p < np; p++) stage += ((size_t)R * rb[p] + 15) & ~(size_t)15;
    stage = (stage + 127) & ~(size_t)127;
    const size_t fixed = acts + (size_t)R * wpr * M * 4 + 64 + 16 * 8;
    if ((size_t)budget <= fixed) continue;
    const int S = (int)std::min<size_t>(6, ((size_t)budget - fixed) / stage);
    if (S < (pass == 0 ? 3 : 2) || stage > 48 * 1024) continue;
    tp.R = R;
    tp.wpr = wpr;
    tp.stages = S;
    tp.stage_bytes = (int)stage;
    tp.nplanes = np;
    int off = 0;
    const uint8_t* base[4] = {w.qs, w.type == T_Q6_K ? w.qh : reinterpret_cast<const uint8_t*>(w.d),
                              reinterpret_cast<const uint8_t*>(w.sc), reinterpret_cast<const uint8_t*>(w.d)};
    for (int p = 0; p < 4; p++) {
      tp.row_bytes[p] = p < np ? rb[p] : 0;
      tp.plane[p] = p < np ? base[p] : nullptr;
      tp.smem_off[p] = off;
      if (p < np) off += (int)(((size_t)R * rb[p] + 15) & ~(size_t)15);
    }
    return true;
  }
  return false;
}

size_t stream_smem_bytes(const TilePlan& tp, int M, int K) {
  return (size_t)tp.stages * tp.stage_bytes + acts_bytes(M, K) + (size_t)tp.R * tp.wpr * M * 4 + 8 + 16 * tp.stages;
}

template <int T, int M, int EPI, int PRO>
static cudaError_t stream_go(const StreamArgs& g, cudaStream_t st, bool pdl, int ctas_per_sm) {
  const size_t smem = stream_smem_bytes(g.plan, M, g.K);
  auto k = stream_gemv<T, M, EPI, PRO>;
  cudaError_t e = cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int ntiles = ceil_div(g.N, g.plan.R);
  int grid = sw_sm_count() * ctas_per_sm;
  if (grid > ntiles) grid = ntiles;
  if (EPI == EPI_ARGMAX && g.n_parts < grid) return cudaErrorInvalidValue;
  StreamArgs a = g;
  void* args[] = {&a};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(SW_THREADS);
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
static cudaError_t stream_m(const StreamArgs& g, cudaStream_t st, bool pdl, int cps) {
  if (g.m <= 1) return stream_go<T, 1, EPI, PRO>(g, st, pdl, cps);
  if (g.m <= 2) return stream_go<T, 2, EPI, PRO>(g, st, pdl, cps);
  if (g.m <= 4) return stream_go<T, 4, EPI, PRO>(g, st, pdl, cps);
  return stream_go<T, 8, EPI, PRO>(g, st, pdl, cps);
}

template <int EPI, int PRO>
static cudaError_t stream_t(const StreamArgs& g, int type, cudaStream_t st, bool pdl, int cps) {
  switch (type) {
    case T_Q8_0: return stream_m<T_Q8_0, EPI, PRO>(g, st, pdl, cps);
    case T_Q4_0: return stream_m<T_Q4_0, EPI, PRO>(g, st, pdl, cps);
    case T_Q4_K: return stream_m<T_Q4_K, EPI, PRO>(g, st, pdl, cps);
    case T_Q6_K: return stream_m<T_Q6_K, EPI, PRO>(g, st, pdl, cps);
  }
  return cudaErrorInvalidValue;
}

// The (epilogue, prologue) pairs the decode path uses:
//   Q|K|V, gate|up, LM head:  rmsnorm + quantize the residual stream in the prologue
//   wo, ffn_down:             quantize the attention output / silu(g)*u, residual epilogue
//   kernel-level matmuls:     pre-quantized rows, plain store (or rmsnorm'd for unfused gate/up)
cudaError_t launch_stream(const StreamArgs& g, int type, int epi, int pro, cudaStream_t st, bool pdl) {
  if (g.m < 1 || g.m > 8) return cudaErrorInvalidValue;
  static int cps = -1;
  if (cps < 0) {
    const char* e = getenv("PRANA_STREAM_CTAS_PER_SM");
    cps = e ? atoi(e) : 1;
    if (cps < 1) cps = 1;
  }
  if (epi == EPI_QKV && pro == PRO_NORM) return stream_t<EPI_QKV, PRO_NORM>(g, type, st, pdl, cps);
  if (epi == EPI_SWIGLU && pro == PRO_NORM) return stream_t<EPI_SWIGLU, PRO_NORM>(g, type, st, pdl, cps);
  if (epi == EPI_ARGMAX && pro == PRO_NORM) return stream_t<EPI_ARGMAX, PRO_NORM>(g, type, st, pdl, cps);
  if (epi == EPI_RESID && pro == PRO_F32) return stream_t<EPI_RESID, PRO_F32>(g, type, st, pdl, cps);
  if (epi == EPI_STORE && pro == PRO_Q) return stream_t<EPI_STORE, PRO_Q>(g, type, st, pdl, cps);
  if (epi == EPI_STORE && pro == PRO_NORM) return stream_t<EPI_STORE, PRO_NORM>(g, type, st, pdl, cps);
  return cudaErrorInvalidValue;
}

// One CTA per token row: the embedding row (checkpoint.rs:169-174) into x, then
// the first layer's rmsnorm + quantization of that row for the Q|K|V stream.
__global__ void __launch_bounds__(256) embed_norm_kernel(const DevWeight w, const uint32_t* toks, const int* tok_single,
                                                         float* x, const float* norm_w, float eps, int8_t* q, float* s,
                                                         int32_t* sum) {
  __shared__ float red[8 * 8];
  __shared__ float inv_s[8];
  const int m = blockIdx.x, dim = w.cols;
  pdl_wait();
  const uint32_t tok = tok_single ? (uint32_t)*tok_single : toks[m];
  float* xr = x + (size_t)m * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) xr[i] = embed_value(w, tok, i);
  __syncthreads();
  pdl_trigger();
  block_quantize_rows(xr, norm_w, eps, 1, dim, q + (size_t)m * dim, s + (size_t)m * (dim / 32),
                      sum + (size_t)m * (dim / 32), red, inv_s, 256, 1);
}

cudaError_t launch_embed_norm(const DevWeight& emb, const uint32_t* toks, const int* tok_single, int m, float* x,
                              const float* norm_w, float eps, int8_t* q, float* s, int32_t* sum, cudaStream_t st,
                              bool pdl) {
  DevWeight w = emb;
  void* args[] = {&w, (void*)&toks, (void*)&tok_single, &x, (void*)&norm_w, &eps, &q, &s, &sum};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelExC(&cfg, (const void*)embed_norm_kernel, args);
}

}  // namespace prana
