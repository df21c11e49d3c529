// attention.cu -- grouped-query attention for the decode path.
//
// Decode / verify (attention.rs:129-195, 296-333): the f16 KV cache of one
// layer is split along positions into n_splits ranges; CTA (split, kv_head)
// streams its K/V tiles through shared memory with cp.async double buffering
// and runs an online softmax for every query head that shares the kv head and
// every query row (verify rows i see positions <= pos0 + i).  Partial
// (max, sum, o) triples go to scratch; the last CTA of a kv head to finish
// (ticket counter, no waiting) merges them and writes the output.
//
// Prefill (attention.rs:236-284): the same kernel body over the f32 in-window
// K/V of the prompt (the CPU path attends over f32 there, not the f16 cache),
// one CTA per (query-row chunk, kv head), no split.
#include <climits>

#include "finish.cuh"
#include "internal.h"

namespace prana {

constexpr int AT_THREADS = 256;
constexpr int AT_TT = 32;          // positions per tile
constexpr int AT_MAX_VHD = 4096;   // (query rows x group) x head_dim per CTA

int attn_max_rows_per_cta(int hd) { return AT_MAX_VHD / hd; }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int HD, bool F32KV>
struct AttnSmem {
  using KvT = typename std::conditional<F32KV, float, __half>::type;
  static constexpr int PAD = F32KV ? 4 : 8;  // 16 B of padding per row: conflict-free 128-bit reads
  static constexpr int ROW = HD + PAD;
  static size_t bytes(int vh) {
    return sizeof(float) * (size_t)vh * HD          // q
           + 2 * 2 * sizeof(KvT) * AT_TT * ROW      // K, V double-buffered
           + sizeof(float) * (size_t)vh * AT_TT     // scores / probabilities
           + sizeof(float) * 3 * (size_t)vh;        // running max, sum, rescale
  }
};

// Shared body.  Query "virtual heads" vh = row * group + g map to query row
// `row` (position pos_base + row0 + row) and head kvh * group + g.
template <int HD, bool F32KV>
__device__ void attn_body(const float* __restrict__ q, int q_stride, const void* kbase, const void* vbase,
                          int kv_stride, int kvh, int group, int row0, int n_rows, int pos_base, int t_begin,
                          int t_end, float* sm, float (&acc)[(AT_MAX_VHD / 2 + AT_THREADS - 1) / AT_THREADS][2],
                          float*& m_row, float*& l_row) {
  using S = AttnSmem<HD, F32KV>;
  using KvT = typename S::KvT;
  constexpr int ROW = S::ROW;
  constexpr int NP = (AT_MAX_VHD / 2 + AT_THREADS - 1) / AT_THREADS;
  const int VH = n_rows * group;
  const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
  float* q_s = sm;
  KvT* kv_s = reinterpret_cast<KvT*>(q_s + VH * HD);  // [2 stages][K|V][AT_TT][ROW]
  float* p_s = reinterpret_cast<float*>(kv_s + 2 * 2 * AT_TT * ROW);
  m_row = p_s + VH * AT_TT;
  l_row = m_row + VH;
  float* a_row = l_row + VH;
  const float scale = 1.0f / sqrtf((float)HD);

  for (int i = tid; i < VH * HD; i += AT_THREADS) {
    const int vh = i / HD, d = i % HD;
    const int row = vh / group, head = kvh * group + vh % group;
    q_s[i] = q[(size_t)(row0 + row) * q_stride + head * HD + d];
  }
  for (int i = tid; i < VH; i += AT_THREADS) {
    m_row[i] = -INFINITY;
    l_row[i] = 0.0f;
  }
#pragma unroll
  for (int i = 0; i < NP; i++) acc[i][0] = acc[i][1] = 0.0f;

  constexpr int CH = HD * (int)sizeof(KvT) / 16;  // 16-byte chunks per row
  auto load_tile = [&](int stage, int t0) {
    KvT* ks = kv_s + (size_t)stage * 2 * AT_TT * ROW;
    KvT* vs = ks + AT_TT * ROW;
    for (int c = tid; c < 2 * AT_TT * CH; c += AT_THREADS) {
      const int which = c / (AT_TT * CH), rem = c % (AT_TT * CH), tt = rem / CH, ch = rem % CH;
      const int t = t0 + tt;
      KvT* dst = (which ? vs : ks) + tt * ROW + ch * (16 / sizeof(KvT));
      if (t < t_end) {
        const KvT* src = reinterpret_cast<const KvT*>(which ? vbase : kbase) + (size_t)t * kv_stride + kvh * HD +
                         ch * (16 / sizeof(KvT));
        cp_async16(dst, src);
      } else {
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
  };

  const int n_tiles = t_end > t_begin ? (t_end - t_begin + AT_TT - 1) / AT_TT : 0;
  if (n_tiles > 0) load_tile(0, t_begin);
  __syncthreads();
  for (int it = 0; it < n_tiles; it++) {
    const int t0 = t_begin + it * AT_TT, stage = it & 1;
    if (it + 1 < n_tiles) {
      load_tile(stage ^ 1, t0 + AT_TT);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const KvT* ks = kv_s + (size_t)stage * 2 * AT_TT * ROW;
    const KvT* vs = ks + AT_TT * ROW;
    // scores: warp -> virtual head, lane -> position
    for (int vh = wi; vh < VH; vh += AT_THREADS / 32) {
      const int t = t0 + lane, row = vh / group;
      float s = -INFINITY;
      if (t < t_end && t <= pos_base + row0 + row) {
        const float* qv = q_s + vh * HD;
        const KvT* kr = ks + lane * ROW;
        float dot = 0.0f;
        if constexpr (F32KV) {
#pragma unroll 8
          for (int d = 0; d < HD; d += 4) {
            const float4 kk = *reinterpret_cast<const float4*>(kr + d);
            const float4 qq = *reinterpret_cast<const float4*>(qv + d);
            dot = fmaf(qq.x, kk.x, dot);
            dot = fmaf(qq.y, kk.y, dot);
            dot = fmaf(qq.z, kk.z, dot);
            dot = fmaf(qq.w, kk.w, dot);
          }
        } else {
#pragma unroll 4
          for (int d = 0; d < HD; d += 8) {
            const uint4 raw = *reinterpret_cast<const uint4*>(kr + d);
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
            const float4 q0 = *reinterpret_cast<const float4*>(qv + d);
            const float4 q1 = *reinterpret_cast<const float4*>(qv + d + 4);
            float2 f;
            f = __half22float2(h2[0]); dot = fmaf(q0.x, f.x, dot); dot = fmaf(q0.y, f.y, dot);
            f = __half22float2(h2[1]); dot = fmaf(q0.z, f.x, dot); dot = fmaf(q0.w, f.y, dot);
            f = __half22float2(h2[2]); dot = fmaf(q1.x, f.x, dot); dot = fmaf(q1.y, f.y, dot);
            f = __half22float2(h2[3]); dot = fmaf(q1.z, f.x, dot); dot = fmaf(q1.w, f.y, dot);
          }
        }
        s = __fmul_rn(dot, scale);
      }
      // online softmax update for this virtual head
      const float tmax = warp_max(s);
      const float m_old = m_row[vh];
      const float m_new = fmaxf(m_old, tmax);
      float p = 0.0f, alpha = 1.0f;
      if (m_new != -INFINITY) {
        p = s == -INFINITY ? 0.0f : expf(s - m_new);
        alpha = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
      }
      p_s[vh * AT_TT + lane] = p;
      const float psum = warp_sum(p);
      if (lane == 0) {
        m_row[vh] = m_new;
        l_row[vh] = fmaf(l_row[vh], alpha, psum);
        a_row[vh] = alpha;
      }
    }
    __syncthreads();
    // o = o * alpha + P V   (each thread owns pairs of adjacent dims)
#pragma unroll
    for (int i = 0; i < NP; i++) {
      const int pi = tid + i * AT_THREADS;
      if (pi * 2 >= VH * HD) break;
      const int vh = (pi * 2) / HD, d = (pi * 2) % HD;
      const float alpha = a_row[vh];
      float o0 = acc[i][0] * alpha, o1 = acc[i][1] * alpha;
      const float* pr = p_s + vh * AT_TT;
#pragma unroll 8
      for (int tt = 0; tt < AT_TT; tt++) {
        float2 v;
        if constexpr (F32KV) v = *reinterpret_cast<const float2*>(vs + tt * ROW + d);
        else v = __half22float2(*reinterpret_cast<const __half2*>(vs + tt * ROW + d));
        o0 = fmaf(pr[tt], v.x, o0);
        o1 = fmaf(pr[tt], v.y, o1);
      }
      acc[i][0] = o0;
      acc[i][1] = o1;
    }
    __syncthreads();
  }
}

template <int HD>
__device__ void attn_merge_splits(const AttnArgs& a, int kvh, int split, int row0, int VH, int group, int q_stride,
                                  float (&acc)[(AT_MAX_VHD / 2 + AT_THREADS - 1) / AT_THREADS][2], const float* m_row,
                                  const float* l_row, unsigned* ticket);

template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_decode_kernel(const AttnArgs a, int row0, int n_rows) {
  extern __shared__ __align__(16) float sm[];
  constexpr int NP = (AT_MAX_VHD / 2 + AT_THREADS - 1) / AT_THREADS;
  const int kvh = blockIdx.y, split = blockIdx.x;
  const int group = a.n_heads / a.n_kv, VH = n_rows * group;
  pdl_wait();
  const int pos0 = a.pos_dev ? *a.pos_dev : a.pos0;
  const int L = pos0 + row0 + n_rows;  // positions 0..L-1 are visible to some row
  int per = (L + a.n_splits - 1) / a.n_splits;
  per = (per + AT_TT - 1) / AT_TT * AT_TT;
  const int t_begin = split * per, t_end = min(L, t_begin + per);
  float acc[NP][2];
  float *m_row, *l_row;
  attn_body<HD, false>(a.q, a.n_heads * HD, a.kc, a.vc, a.n_kv * HD, kvh, group, row0, n_rows, pos0,
                       t_begin, t_end, sm, acc, m_row, l_row);
  pdl_trigger();
  const int tid = threadIdx.x;
  const int q_stride = a.n_heads * HD;
  __shared__ unsigned ticket;
  if (a.n_splits == 1) {
#pragma unroll
    for (int i = 0; i < NP; i++) {
      const int pi = tid + i * AT_THREADS;
      if (pi * 2 >= VH * HD) break;
      const int vh = (pi * 2) / HD, d = (pi * 2) % HD;
      const int row = vh / group, head = kvh * group + vh % group;
      const float inv = 1.0f / l_row[vh];
      float* o = a.out + (size_t)(row0 + row) * q_stride + head * HD + d;
      o[0] = acc[i][0] * inv;
      o[1] = acc[i][1] * inv;
    }
  } else {
    attn_merge_splits<HD>(a, kvh, split, row0, VH, group, q_stride, acc, m_row, l_row, &ticket);
    if (ticket != (unsigned)a.n_splits - 1) return;
  }
  // every kv head of these rows finished: quantize the rows for the wo projection
  if (a.out_q) {
    __shared__ float red[8 * (AT_THREADS / 32)];
    __shared__ float inv_s[8];
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket = atomicAdd(a.counters + a.n_kv, 1u);
    __syncthreads();
    if (ticket != (unsigned)a.n_kv - 1) return;
    __threadfence();
    block_quantize_rows(a.out + (size_t)row0 * q_stride, nullptr, 0.0f, n_rows, q_stride,
                        a.out_q + (size_t)row0 * q_stride, a.out_s + (size_t)row0 * (q_stride / 32),
                        a.out_sum + (size_t)row0 * (q_stride / 32), red, inv_s, AT_THREADS, 1);
    if (tid == 0) a.counters[a.n_kv] = 0u;
  }
}

// Publish this split's (max, sum, o) and, in the last split CTA of the kv head
// to finish, merge all splits into the output.  `ticket` tells the caller
// whether this CTA merged (== n_splits - 1).
template <int HD>
__device__ void attn_merge_splits(const AttnArgs& a, int kvh, int split, int row0, int VH, int group, int q_stride,
                                  float (&acc)[(AT_MAX_VHD / 2 + AT_THREADS - 1) / AT_THREADS][2], const float* m_row,
                                  const float* l_row, unsigned* ticket) {
  constexpr int NP = (AT_MAX_VHD / 2 + AT_THREADS - 1) / AT_THREADS;
  const int tid = threadIdx.x;
  const size_t base = ((size_t)kvh * a.n_splits + split) * VH;
  for (int vh = tid; vh < VH; vh += AT_THREADS) {
    a.part_ml[(base + vh) * 2] = m_row[vh];
    a.part_ml[(base + vh) * 2 + 1] = l_row[vh];
  }
#pragma unroll
  for (int i = 0; i < NP; i++) {
    const int pi = tid + i * AT_THREADS;
    if (pi * 2 >= VH * HD) break;
    const int vh = (pi * 2) / HD, d = (pi * 2) % HD;
    *reinterpret_cast<float2*>(a.part_o + (base + vh) * HD + d) = make_float2(acc[i][0], acc[i][1]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) *ticket = atomicAdd(a.counters + kvh, 1u);
  __syncthreads();
  if (*ticket != (unsigned)a.n_splits - 1) return;
  __threadfence();
  // last CTA of this kv head: merge all splits
#pragma unroll
  for (int i = 0; i < NP; i++) {
    const int pi = tid + i * AT_THREADS;
    if (pi * 2 >= VH * HD) break;
    const int vh = (pi * 2) / HD, d = (pi * 2) % HD;
    float mx = -INFINITY;
    for (int s = 0; s < a.n_splits; s++)
      mx = fmaxf(mx, __ldcg(a.part_ml + (((size_t)kvh * a.n_splits + s) * VH + vh) * 2));
    float lsum = 0.0f, o0 = 0.0f, o1 = 0.0f;
    for (int s = 0; s < a.n_splits; s++) {
      const size_t pb = ((size_t)kvh * a.n_splits + s) * VH + vh;
      const float ms = __ldcg(a.part_ml + pb * 2);
      if (ms == -INFINITY) continue;
      const float w = expf(ms - mx);
      lsum = fmaf(__ldcg(a.part_ml + pb * 2 + 1), w, lsum);
      const float2 po = __ldcg(reinterpret_cast<const float2*>(a.part_o + pb * HD + d));
      o0 = fmaf(po.x, w, o0);
      o1 = fmaf(po.y, w, o1);
    }
    const float inv = 1.0f / lsum;
    const int row = vh / group, head = kvh * group + vh % group;
    float* o = a.out + (size_t)(row0 + row) * q_stride + head * HD + d;
    o[0] = o0 * inv;
    o[1] = o1 * inv;
  }
  if (tid == 0) a.counters[kvh] = 0u;
}

template <int HD>
__global__ void __launch_bounds__(AT_THREADS) attn_prefill_kernel(const PrefillAttnArgs a, int rows_per_cta) {
  extern __shared__ __align__(16) float sm[];
  constexpr int NP = (AT_MAX_VHD / 2 + AT_THREADS - 1) / AT_THREADS;
  const int kvh = blockIdx.y, group = a.n_heads / a.n_kv;
  const int row0 = blockIdx.x * rows_per_cta;
  const int n_rows = min(rows_per_cta, a.n - row0);
  const int VH = n_rows * group;
  float acc[NP][2];
  float *m_row, *l_row;
  attn_body<HD, true>(a.q, a.n_heads * HD, a.k, a.v, a.n_kv * HD, kvh, group, row0, n_rows, 0, 0,
                      row0 + n_rows, sm, acc, m_row, l_row);
  const int q_stride = a.n_heads * HD;
#pragma unroll
  for (int i = 0; i < NP; i++) {
    const int pi = threadIdx.x + i * AT_THREADS;
    if (pi * 2 >= VH * HD) break;
    const int vh = (pi * 2) / HD, d = (pi * 2) % HD;
    const int row = vh / group, head = kvh * group + vh % group;
    const float inv = 1.0f / l_row[vh];
    float* o = a.out + (size_t)(row0 + row) * q_stride + head * HD + d;
    o[0] = acc[i][0] * inv;
    o[1] = acc[i][1] * inv;
  }
}

template <int HD>
static cudaError_t decode_go(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int group = a.n_heads / a.n_kv;
  const int max_rows = AT_MAX_VHD / (HD * group);
  if (max_rows < 1) return cudaErrorInvalidValue;
  for (int row0 = 0; row0 < a.m; row0 += max_rows) {
    const int n_rows = min(max_rows, a.m - row0);
    const size_t smem = AttnSmem<HD, false>::bytes(n_rows * group);
    auto k = attn_decode_kernel<HD>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    AttnArgs aa = a;
    void* args[] = {&aa, (void*)&row0, (void*)&n_rows};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_splits, a.n_kv);
    cfg.blockDim = dim3(AT_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl && row0 == 0) {
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)k, args);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.n_kv <= 0 || a.n_heads % a.n_kv || a.m < 1 || a.n_splits < 1) return cudaErrorInvalidValue;
  switch (a.hd) {
    case 32: return decode_go<32>(a, st, pdl);
    case 48: return decode_go<48>(a, st, pdl);
    case 64: return decode_go<64>(a, st, pdl);
    case 96: return decode_go<96>(a, st, pdl);
    case 128: return decode_go<128>(a, st, pdl);
    case 256: return decode_go<256>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

template <int HD>
static cudaError_t prefill_go(const PrefillAttnArgs& a, cudaStream_t st) {
  const int group = a.n_heads / a.n_kv;
  const int rows = AT_MAX_VHD / (HD * group);
  if (rows < 1) return cudaErrorInvalidValue;
  const size_t smem = AttnSmem<HD, true>::bytes(rows * group);
  auto k = attn_prefill_kernel<HD>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  k<<<dim3((a.n + rows - 1) / rows, a.n_kv), AT_THREADS, smem, st>>>(a, rows);
  return cudaGetLastError();
}

cudaError_t launch_attn_prefill(const PrefillAttnArgs& a, cudaStream_t st) {
  if (a.n_kv <= 0 || a.n_heads % a.n_kv || a.n < 1) return cudaErrorInvalidValue;
  switch (a.hd) {
    case 32: return prefill_go<32>(a, st);
    case 48: return prefill_go<48>(a, st);
    case 64: return prefill_go<64>(a, st);
    case 96: return prefill_go<96>(a, st);
    case 128: return prefill_go<128>(a, st);
    case 256: return prefill_go<256>(a, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace prana
