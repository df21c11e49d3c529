// attention.cu -- grouped-query attention for the decode path.
//
// Decode / verify (attention.rs:129-195, 296-333): flash-decoding over the f16
// KV cache of one layer.  The positions are split into n_splits ranges; CTA
// (split, kv_head) runs an online softmax for every query head that shares the
// kv head and every query row (verify rows i see positions <= pos0 + i).
// Partial (max, sum, o) triples go to scratch; the last CTA of a kv head to
// finish (ticket counter, no waiting) merges them and writes the output.
//
// Prefill (attention.rs:236-284): a tiled body over the f32 in-window K/V of
// the prompt (the CPU path attends over f32 there, not the f16 cache), one CTA
// per (query-row chunk, kv head), no split.
#include <climits>

#include <cooperative_groups.h>

#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <tuple>
#include <mutex>

#include "internal.h"
#include "mbar.cuh"
#include "tc.cuh"

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

// ---------------------------------------------------------------- decode / verify over the f16 cache
//
// Flash-decoding split: CTA (split, kv_head) owns a contiguous range of cache
// positions and moves it through shared memory AD_C positions at a time, every
// K and V row of a pass requested at once (cp.async, 16 bytes per request).
// Rows written by earlier decode steps (positions < pos0) do not depend on the
// Q|K|V kernel that precedes this one, so they are requested before the
// programmatic-launch wait; q and this step's rows are read after it.
//
// Work layout (256 threads): scores take one position and half of the head
// dims per thread for AD_VG query heads at once (8 independent FMA chains);
// P.V takes one pair of dims and a slice of the positions per thread, again
// for AD_VG heads, and the slices meet in shared memory.  The running output
// lives in shared memory and is rescaled once per pass (online softmax).
constexpr int AD_THREADS = 256;
constexpr int AD_C = 128;  // positions per pass
constexpr int AD_VG = 4;   // query heads per compute chunk

// Splits for a cache of `positions` rows: one pass per CTA at full length,
// at most ~4 CTAs per SM, and few enough that the (max, sum, weight) triples of
// every split fit in the merging CTA's idle K/V buffers.
int attn_splits(int positions, int n_kv, int hd, int sm_count) {
  const int by_len = (positions + AD_C - 1) / AD_C;
  const int by_sm = (4 * sm_count + n_kv - 1) / n_kv;
  const int by_smem = AD_C * (hd + 8) * hd / (3 * AT_MAX_VHD);
  return std::max(1, std::min(std::min(by_len, by_sm), by_smem));
}

template <int HD>
struct AdSmem {
  static constexpr int ROW = HD + 8;  // halves; 16 bytes of padding per row
  static constexpr int RED = 2048;    // floats: (threads / (HD/2)) slices x AD_VG x HD
  static size_t bytes(int vh) {
    return 2 * sizeof(__half) * (size_t)AD_C * ROW  // K, V
           + sizeof(float) * (size_t)vh * HD        // q
           + sizeof(float) * (size_t)vh * HD        // running output
           + sizeof(float) * (size_t)vh * AD_C      // scores / probabilities
           + sizeof(float) * RED                    // P.V slices
           + sizeof(float) * 3 * (size_t)vh;        // running max, sum, rescale
  }
};

// Ticket of a cross-CTA completion count: the CTA's writes (ordered before
// this by the caller's __syncthreads) are released at gpu scope, and the CTA
// that draws the last ticket acquires every other CTA's writes.
__device__ __forceinline__ unsigned ticket_acq_rel(unsigned* counter) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
  return old;
}

// End of a decode CTA: (m_run, l_run, o_s) hold this CTA's softmax state for
// its VH virtual heads (o_s unnormalized).  With one split the rows are final;
// otherwise they are published as a partial and the last CTA of the kv head
// to finish merges every split.  `smem_raw` is shared memory the caller no
// longer needs (>= 3 x VH x n_splits floats), `red` >= 4 KB.
template <int HD, int NTH = AD_THREADS>
__device__ __forceinline__ void attn_finish(const AttnArgs& a, int kvh, int split, int row0, int VH, int group,
                                            const float* o_s, const float* m_run, float* l_run, uint8_t* smem_raw,
                                            float* red) {
  const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
  const int q_stride = a.n_heads * HD;
  if (a.n_splits == 1) {
    for (int e = tid; e < VH * HD; e += NTH) {
      const int vh = e / HD, d = e - vh * HD;
      const int row = vh / group, head = kvh * group + vh % group;
      a.out[(size_t)(row0 + row) * q_stride + head * HD + d] = o_s[e] / l_run[vh];
    }
    return;
  }
  // ---- publish this split's (max, sum, o); the last split CTA of the kv head merges
  const size_t base = ((size_t)kvh * a.n_splits + split) * VH;
  for (int vh = tid; vh < VH; vh += NTH)
    reinterpret_cast<float2*>(a.part_ml)[base + vh] = make_float2(m_run[vh], l_run[vh]);
  for (int e = tid; e < VH * HD / 4; e += NTH)
    reinterpret_cast<float4*>(a.part_o + base * HD)[e] = reinterpret_cast<const float4*>(o_s)[e];
  __shared__ unsigned ticket;
  __syncthreads();
  if (tid == 0) ticket = ticket_acq_rel(a.counters + kvh);
  __syncthreads();
  if (ticket != (unsigned)a.n_splits - 1) return;
  // (max, sum) of every split in one round trip, then the split weights
  // exp(m_s - max) (attn_splits keeps 3 x VH x NS floats in range)
  const int NS = a.n_splits;
  float2* ml_s = reinterpret_cast<float2*>(smem_raw);  // [VH][NS]
  const size_t hb = (size_t)kvh * NS * VH;  // this kv head's first partial
  for (int i = tid; i < VH * NS; i += NTH) {
    const int vh = i / NS, s = i - vh * NS;
    ml_s[i] = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + hb + (size_t)s * VH + vh);
  }
  __syncthreads();
  float* w_s = reinterpret_cast<float*>(ml_s + VH * NS);  // [VH][NS]
  for (int vh = wi; vh < VH; vh += NTH / 32) {
    float mx = -INFINITY;
    for (int s = lane; s < NS; s += 32) mx = fmaxf(mx, ml_s[vh * NS + s].x);
    mx = warp_max(mx);
    float lsum = 0.0f;
    for (int s = lane; s < NS; s += 32) {
      const float2 ml = ml_s[vh * NS + s];
      const float w = ml.x == -INFINITY ? 0.0f : expf(ml.x - mx);
      w_s[vh * NS + s] = w;
      lsum = fmaf(ml.y, w, lsum);
    }
    lsum = warp_sum(lsum);
    if (lane == 0) l_run[vh] = lsum;
  }
  __syncthreads();
  // weighted sum of the partial outputs: item = 4 dims of one head; the
  // splits of an item are shared by `nsub` threads so all loads go out at once
  const int items = VH * HD / 4;
  const int nsub = items >= NTH ? 1 : NTH / items;
  const int sub = tid / items < nsub ? tid / items : nsub;  // == nsub: idle
  float4* red4 = reinterpret_cast<float4*>(red);  // [nsub][items] when nsub > 1
  for (int it = tid % items; sub < nsub && it < items; it += (nsub > 1 ? items : NTH)) {
    const int vh = (it * 4) / HD;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 8
    for (int s = sub; s < NS; s += nsub) {
      const float w = w_s[vh * NS + s];
      const float4 po = __ldcg(reinterpret_cast<const float4*>(a.part_o + (hb + (size_t)s * VH) * HD) + it);
      acc.x = fmaf(po.x, w, acc.x);
      acc.y = fmaf(po.y, w, acc.y);
      acc.z = fmaf(po.z, w, acc.z);
      acc.w = fmaf(po.w, w, acc.w);
    }
    if (nsub > 1) {
      red4[sub * items + it] = acc;
    } else {
      const int d = it * 4 - vh * HD, row = vh / group, head = kvh * group + vh % group;
      const float inv = 1.0f / l_run[vh];
      float* o = a.out + (size_t)(row0 + row) * q_stride + head * HD + d;
      *reinterpret_cast<float4*>(o) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
  }
  if (nsub > 1) {
    __syncthreads();
    for (int it = tid; it < items; it += NTH) {
      const int vh = (it * 4) / HD, d = it * 4 - vh * HD, row = vh / group, head = kvh * group + vh % group;
      float4 acc = red4[it];
      for (int s = 1; s < nsub; s++) {
        const float4 t = red4[s * items + it];
        acc.x += t.x;
        acc.y += t.y;
        acc.z += t.z;
        acc.w += t.w;
      }
      const float inv = 1.0f / l_run[vh];
      float* o = a.out + (size_t)(row0 + row) * q_stride + head * HD + d;
      *reinterpret_cast<float4*>(o) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
  }
  if (tid == 0) a.counters[kvh] = 0u;
}

template <int HD>
__global__ void __launch_bounds__(AD_THREADS) attn_decode_kernel(const AttnArgs a, int row0, int n_rows) {
  using S = AdSmem<HD>;
  constexpr int ROW = S::ROW, CPR = HD / 8, HP = HD / 2, NPART = AD_THREADS / HP;
  static_assert(NPART * AD_VG * HD <= S::RED, "P.V slice buffer");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __half* k_s = reinterpret_cast<__half*>(smem_raw);
  __half* v_s = k_s + AD_C * ROW;
  float* q_s = reinterpret_cast<float*>(v_s + AD_C * ROW);
  const int group = a.n_heads / a.n_kv, VH = n_rows * group;
  float* o_s = q_s + VH * HD;
  float* s_s = o_s + VH * HD;
  float* red = s_s + VH * AD_C;
  float* m_run = red + S::RED;
  float* l_run = m_run + VH;
  float* alpha = l_run + VH;
  const int kvh = blockIdx.y, split = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
  const int kv_stride = a.n_kv * HD, q_stride = a.n_heads * HD;
  const float scale = 1.0f / sqrtf((float)HD);

  // the position counter of a graph-driven step was advanced before the
  // previous step's kernels finished, so it is safe to read before the wait
  const int pos0 = a.pos_dev ? *a.pos_dev : a.pos0;
  const int L = pos0 + row0 + n_rows;  // positions 0..L-1 are visible to some row
  int per = (L + a.n_splits - 1) / a.n_splits;
  per = (per + 15) / 16 * 16;
  const int t_begin = min(L, split * per), t_end = min(L, t_begin + per);

  auto request = [&](int t0, int n, int lo, int hi) {  // rows t0 + [0, n) with lo <= t < hi
    for (int c = tid; c < 2 * AD_C * CPR; c += AD_THREADS) {
      const int which = c / (AD_C * CPR), r = (c / CPR) % AD_C, ch = c % CPR;
      const int t = t0 + r;
      if (r >= n || t < lo || t >= hi) continue;
      const __half* src = (which ? a.vc : a.kc) + (size_t)t * kv_stride + kvh * HD + ch * 8;
      cp_async16((which ? v_s : k_s) + r * ROW + ch * 8, src);
    }
  };

  const int n0 = min(AD_C, t_end - t_begin);
  if (n0 > 0) request(t_begin, n0, 0, pos0);
  cp_async_commit();
  pdl_wait();
  if (n0 > 0) request(t_begin, n0, pos0, INT_MAX);
  cp_async_commit();
  for (int i = tid; i < VH * HD; i += AD_THREADS) {
    const int vh = i / HD, d = i - vh * HD;
    const int row = vh / group, head = kvh * group + vh % group;
    q_s[i] = a.q[(size_t)(row0 + row) * q_stride + head * HD + d];
    o_s[i] = 0.0f;
  }
  for (int i = tid; i < VH; i += AD_THREADS) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.0f;
  }
  pdl_trigger();

  for (int t0 = t_begin; t0 < t_end; t0 += AD_C) {
    const int n = min(AD_C, t_end - t0);
    if (t0 != t_begin) {
      request(t0, n, 0, INT_MAX);
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();
    // ---- scores: thread -> (position p, half h of the dims), AD_VG heads at a time
    {
      const int p = tid >> 1, h = tid & 1;
      for (int v0 = 0; v0 < VH; v0 += AD_VG) {
        float d0[AD_VG], d1[AD_VG];
#pragma unroll
        for (int g = 0; g < AD_VG; g++) d0[g] = d1[g] = 0.0f;
        if (p < n) {
          const __half* kr = k_s + p * ROW + h * HP;
#pragma unroll 4
          for (int dd = 0; dd < HP; dd += 8) {
            const uint4 raw = *reinterpret_cast<const uint4*>(kr + dd);
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
            const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
            const float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
#pragma unroll
            for (int g = 0; g < AD_VG; g++) {
              if (v0 + g < VH) {
                const float* qv = q_s + (v0 + g) * HD + h * HP + dd;
                const float4 qa = *reinterpret_cast<const float4*>(qv);
                const float4 qb = *reinterpret_cast<const float4*>(qv + 4);
                d0[g] = fmaf(qa.x, f0.x, d0[g]);
                d1[g] = fmaf(qa.y, f0.y, d1[g]);
                d0[g] = fmaf(qa.z, f1.x, d0[g]);
                d1[g] = fmaf(qa.w, f1.y, d1[g]);
                d0[g] = fmaf(qb.x, f2.x, d0[g]);
                d1[g] = fmaf(qb.y, f2.y, d1[g]);
                d0[g] = fmaf(qb.z, f3.x, d0[g]);
                d1[g] = fmaf(qb.w, f3.y, d1[g]);
              }
            }
          }
        }
#pragma unroll
        for (int g = 0; g < AD_VG; g++) {
          float d = d0[g] + d1[g];
          d += __shfl_xor_sync(0xffffffffu, d, 1);
          const int vh = v0 + g;
          if (h == 0 && p < n && vh < VH)
            s_s[vh * AD_C + p] = (t0 + p <= pos0 + row0 + vh / group) ? __fmul_rn(d, scale) : -INFINITY;
        }
      }
    }
    __syncthreads();
    // ---- online softmax: one warp per head
    for (int vh = wi; vh < VH; vh += AD_THREADS / 32) {
      float mx = -INFINITY;
      for (int r = lane; r < n; r += 32) mx = fmaxf(mx, s_s[vh * AD_C + r]);
      mx = warp_max(mx);
      const float m_old = m_run[vh], m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
      for (int r = lane; r < n; r += 32) {
        const float s = s_s[vh * AD_C + r];
        const float pr = (s == -INFINITY) ? 0.0f : expf(s - m_new);
        s_s[vh * AD_C + r] = pr;
        sum += pr;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float al = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
        m_run[vh] = m_new;
        l_run[vh] = fmaf(l_run[vh], al, sum);
        alpha[vh] = al;
      }
    }
    __syncthreads();
    // ---- P.V: thread -> (dim pair dp, slice of the positions), AD_VG heads at a time
    {
      const int dp = tid % HP, part = tid / HP;  // part == NPART: idle (HD/2 does not divide the block)
      const int per_part = (n + NPART - 1) / NPART;
      const int r_lo = part < NPART ? min(n, part * per_part) : n, r_hi = min(n, r_lo + per_part);
      for (int v0 = 0; v0 < VH; v0 += AD_VG) {
        float o0[AD_VG], o1[AD_VG];
#pragma unroll
        for (int g = 0; g < AD_VG; g++) o0[g] = o1[g] = 0.0f;
#pragma unroll 4
        for (int r = r_lo; r < r_hi; r++) {
          const float2 v = __half22float2(*reinterpret_cast<const __half2*>(v_s + r * ROW + 2 * dp));
#pragma unroll
          for (int g = 0; g < AD_VG; g++) {
            if (v0 + g < VH) {
              const float pr = s_s[(v0 + g) * AD_C + r];
              o0[g] = fmaf(pr, v.x, o0[g]);
              o1[g] = fmaf(pr, v.y, o1[g]);
            }
          }
        }
        if (part < NPART) {
#pragma unroll
          for (int g = 0; g < AD_VG; g++)
            *reinterpret_cast<float2*>(red + (part * AD_VG + g) * HD + 2 * dp) = make_float2(o0[g], o1[g]);
        }
        __syncthreads();
        for (int e = tid; e < AD_VG * HD; e += AD_THREADS) {
          const int g = e / HD, d = e - g * HD, vh = v0 + g;
          if (vh >= VH) continue;
          float s = 0.0f;
#pragma unroll 4
          for (int pp = 0; pp < NPART; pp++) s += red[(pp * AD_VG + g) * HD + d];
          o_s[vh * HD + d] = fmaf(o_s[vh * HD + d], alpha[vh], s);
        }
        __syncthreads();
      }
    }
  }

  attn_finish<HD>(a, kvh, split, row0, VH, group, o_s, m_run, l_run, smem_raw, red);
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

// ---------------------------------------------------------------- tensor-core decode (head_dim 64 / 128)
//
// Same split / pass / merge structure as attn_decode_kernel, with Q.K^T and
// P.V on the tensor cores (mma.sync m16n8k16, f16 inputs, f32 accumulate).
// A CTA's pass holds AM_C = 128 positions; warp w owns positions 16w..16w+15
// of the pass and keeps its own online-softmax state (m, l, O) for up to 16
// virtual heads (the rows of the MMA tile).  f32 operands reach f16 as a
// hi + lo pair (x = hi + lo to ~2^-22 relative), two MMAs each, so scores and
// outputs carry f32-level accuracy: the K/V cache is f16 already and every
// f16 x f16 product is exact in the f32 accumulator.
constexpr int AM_C = 128;  // positions per pass (8 warps x 16)
constexpr int AM_ROWS = 16;  // virtual heads per CTA (MMA rows)

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// (x0, x1) -> f16 hi pair and f16 lo pair (lo = x - hi), low half = x0
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  const __half l0 = __float2half_rn(x0 - __half2float(h0)), l1 = __float2half_rn(x1 - __half2float(h1));
  hi = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
  lo = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
}

template <int HD>
struct AmSmem {
  static constexpr int ROW = HD + 8;  // halves; 16 bytes of padding per row (conflict-free ldmatrix)
  static constexpr size_t KV = 2 * sizeof(__half) * (size_t)AM_C * ROW;
  static constexpr size_t Q = 2 * sizeof(__half) * (size_t)AM_ROWS * ROW;  // hi, lo
  static constexpr size_t O = sizeof(float) * (size_t)AM_ROWS * HD;
  static constexpr size_t RED = 4096;
  static constexpr size_t bytes = KV + Q + O + RED + sizeof(float) * 2 * AM_ROWS;
  // the warps' (m, l, O) meet in the K/V buffers after the last pass
  static_assert(sizeof(float) * 8 * AM_ROWS * (HD + 2) <= KV, "warp merge buffer");
};

template <int HD>
__global__ void __launch_bounds__(256) attn_decode_mma(const AttnArgs a, int row0, int n_rows) {
  using S = AmSmem<HD>;
  constexpr int ROW = S::ROW, CPR = HD / 8, KS = HD / 16, NT = HD / 8;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __half* k_s = reinterpret_cast<__half*>(smem_raw);
  __half* v_s = k_s + AM_C * ROW;
  __half* qh_s = v_s + AM_C * ROW;
  __half* ql_s = qh_s + AM_ROWS * ROW;
  float* o_s = reinterpret_cast<float*>(ql_s + AM_ROWS * ROW);
  float* red = o_s + AM_ROWS * HD;
  float* m_run = red + S::RED / sizeof(float);
  float* l_run = m_run + AM_ROWS;
  const int group = a.n_heads / a.n_kv, VH = n_rows * group;  // VH <= 16
  const int kvh = blockIdx.y, split = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int kv_stride = a.n_kv * HD, q_stride = a.n_heads * HD;
  const float scale = 1.0f / sqrtf((float)HD);

  // the position counter of a graph-driven step was advanced before the
  // previous step's kernels finished, so it is safe to read before the wait
  const int pos0 = a.pos_dev ? *a.pos_dev : a.pos0;
  const int L = pos0 + row0 + n_rows;
  int per = (L + a.n_splits - 1) / a.n_splits;
  per = (per + 15) / 16 * 16;
  const int t_begin = min(L, split * per), t_end = min(L, t_begin + per);

  // thread -> 16-byte chunk `ch` of pass rows r_first, r_first + RSTEP, ... of K and V
  constexpr int RSTEP = 256 / CPR;
  const int ch = tid % CPR, r_first = tid / CPR;
  auto request = [&](int t0, int r_lo, int r_hi) {  // pass rows [r_lo, r_hi)
    int r = r_first;
    if (r < r_lo) r += (r_lo - r + RSTEP - 1) / RSTEP * RSTEP;
    const size_t src0 = (size_t)(t0 + r) * kv_stride + kvh * HD + ch * 8;
    const __half* ks = a.kc + src0;
    const __half* vs = a.vc + src0;
    for (; r < r_hi; r += RSTEP, ks += (size_t)RSTEP * kv_stride, vs += (size_t)RSTEP * kv_stride) {
      cp_async16(k_s + r * ROW + ch * 8, ks);
      cp_async16(v_s + r * ROW + ch * 8, vs);
    }
  };
  // V rows past the end of a short pass enter the P.V MMA with P = 0; zero
  // them so stale shared memory cannot inject NaN (0 x NaN)
  auto zero_tail = [&](int n) {
    const int n16 = min(AM_C, (n + 15) / 16 * 16);
    for (int c = tid; c < (n16 - n) * CPR; c += 256) {
      const int r = n + c / CPR, ch = c % CPR;
      *reinterpret_cast<uint4*>(v_s + r * ROW + ch * 8) = make_uint4(0, 0, 0, 0);
    }
  };

  __shared__ int q_off[AM_ROWS];  // where virtual head vh's q row starts (-1: padding row)
  if (tid < AM_ROWS) q_off[tid] = tid < VH ? (row0 + tid / group) * q_stride + (kvh * group + tid % group) * HD : -1;
  const int n0 = min(AM_C, t_end - t_begin);
  const int split_at = min(n0, max(0, pos0 - t_begin));  // rows before it were written by earlier steps
  if (split_at > 0) request(t_begin, 0, split_at);
  cp_async_commit();
  pdl_wait();
  if (n0 > split_at) request(t_begin, split_at, n0);
  if (n0 > 0) zero_tail(n0);
  cp_async_commit();
  __syncthreads();
  // q rows of the virtual heads as f16 hi/lo tiles; rows >= VH are zero
  for (int i = tid; i < AM_ROWS * HD; i += 256) {
    const int vh = i / HD, d = i - vh * HD;
    const int off = q_off[vh];
    const float x = off >= 0 ? a.q[off + d] : 0.0f;
    const __half h = __float2half_rn(x);
    qh_s[vh * ROW + d] = h;
    ql_s[vh * ROW + d] = __float2half_rn(x - __half2float(h));
  }
  pdl_trigger();

  // per-warp online softmax state: rows g and g + 8 of the MMA tile
  float m_w[2] = {-INFINITY, -INFINITY}, l_w[2] = {0.0f, 0.0f};
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  const int lr = lane & 7, lj = lane >> 3;  // ldmatrix: row within matrix, matrix index

  for (int t0 = t_begin; t0 < t_end; t0 += AM_C) {
    const int n = min(AM_C, t_end - t0);
    if (t0 != t_begin) {
      request(t0, 0, n);
      zero_tail(n);
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();
    const int p0 = wi * 16;  // this warp's first position in the pass
    if (p0 < n) {
      // ---- S[16 x 16] = Q . K^T over HD (hi and lo halves of Q)
      float sc[2][4];
#pragma unroll
      for (int i = 0; i < 2; i++) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
        uint32_t ah[4], al[4], kb[4];
        const int qoff = ((lj & 1) * 8 + lr) * ROW + ks * 16 + (lj >> 1) * 8;
        ldsm_x4(ah, qh_s + qoff);
        ldsm_x4(al, ql_s + qoff);
        ldsm_x4(kb, k_s + (p0 + (lj >> 1) * 8 + lr) * ROW + ks * 16 + (lj & 1) * 8);
        mma_f16(sc[0], ah, kb[0], kb[1]);
        mma_f16(sc[0], al, kb[0], kb[1]);
        mma_f16(sc[1], ah, kb[2], kb[3]);
        mma_f16(sc[1], al, kb[2], kb[3]);
      }
      // ---- mask, scale, online softmax per row (a row's 16 values live in one lane quad)
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int row = g + (c >> 1) * 8, p = p0 + nt * 8 + tig * 2 + (c & 1);
          const bool ok = row < VH && p < n && t0 + p <= pos0 + row0 + row / group;
          sc[nt][c] = ok ? __fmul_rn(sc[nt][c], scale) : -INFINITY;
          mx[c >> 1] = fmaxf(mx[c >> 1], sc[nt][c]);
        }
      float alpha[2], sum[2] = {0.0f, 0.0f};
#pragma unroll
      for (int h = 0; h < 2; h++) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float m_new = fmaxf(m_w[h], mx[h]);
        alpha[h] = (m_w[h] == -INFINITY) ? 0.0f : expf(m_w[h] - m_new);
        m_w[h] = m_new;
      }
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float s = sc[nt][c];
          const float pr = (s == -INFINITY) ? 0.0f : expf(s - m_w[c >> 1]);
          sc[nt][c] = pr;
          sum[c >> 1] += pr;
        }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
        sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
        l_w[h] = fmaf(l_w[h], alpha[h], sum[h]);
      }
#pragma unroll
      for (int i = 0; i < NT; i++) {
        o[i][0] *= alpha[0];
        o[i][1] *= alpha[0];
        o[i][2] *= alpha[1];
        o[i][3] *= alpha[1];
      }
      // ---- O += P . V: the two S tiles are exactly the A fragment of P (16 x 16)
      uint32_t ph[4], pl[4];
      split_pair(sc[0][0], sc[0][1], ph[0], pl[0]);
      split_pair(sc[0][2], sc[0][3], ph[1], pl[1]);
      split_pair(sc[1][0], sc[1][1], ph[2], pl[2]);
      split_pair(sc[1][2], sc[1][3], ph[3], pl[3]);
#pragma unroll
      for (int dt = 0; dt < NT; dt += 2) {
        uint32_t vb[4];
        ldsm_x4_t(vb, v_s + (p0 + (lj & 1) * 8 + lr) * ROW + dt * 8 + (lj >> 1) * 8);
        mma_f16(o[dt], ph, vb[0], vb[1]);
        mma_f16(o[dt], pl, vb[0], vb[1]);
        mma_f16(o[dt + 1], ph, vb[2], vb[3]);
        mma_f16(o[dt + 1], pl, vb[2], vb[3]);
      }
    }
    __syncthreads();  // the next pass overwrites K and V
  }

  // ---- the warps' states meet in the K/V buffers: wm/wl [8][16], wo [8][VH][HD]
  float* wm = reinterpret_cast<float*>(smem_raw);
  float* wl = wm + 8 * AM_ROWS;
  float* wo = wl + 8 * AM_ROWS;
  if (tig == 0) {
    wm[wi * AM_ROWS + g] = m_w[0];
    wl[wi * AM_ROWS + g] = l_w[0];
    wm[wi * AM_ROWS + g + 8] = m_w[1];
    wl[wi * AM_ROWS + g + 8] = l_w[1];
  }
#pragma unroll
  for (int i = 0; i < NT; i++) {
    const int d = i * 8 + tig * 2;
    if (g < VH) *reinterpret_cast<float2*>(wo + (wi * AM_ROWS + g) * HD + d) = make_float2(o[i][0], o[i][1]);
    if (g + 8 < VH) *reinterpret_cast<float2*>(wo + (wi * AM_ROWS + g + 8) * HD + d) = make_float2(o[i][2], o[i][3]);
  }
  __syncthreads();
  if (tid < VH) {
    float mx = -INFINITY;
    for (int w = 0; w < 8; w++) mx = fmaxf(mx, wm[w * AM_ROWS + tid]);
    float l = 0.0f;
    for (int w = 0; w < 8; w++) {
      const float mw = wm[w * AM_ROWS + tid];
      const float sw = mw == -INFINITY ? 0.0f : expf(mw - mx);
      wm[w * AM_ROWS + tid] = sw;  // the warp's weight from here on
      l = fmaf(wl[w * AM_ROWS + tid], sw, l);
    }
    m_run[tid] = mx;
    l_run[tid] = l;
  }
  __syncthreads();
  for (int e = tid; e < VH * HD; e += 256) {
    const int vh = e / HD;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) acc = fmaf(wo[(w * AM_ROWS + vh) * HD + (e - vh * HD)], wm[w * AM_ROWS + vh], acc);
    o_s[e] = acc;
  }
  __syncthreads();
  attn_finish<HD>(a, kvh, split, row0, VH, group, o_s, m_run, l_run, smem_raw, red);
}

// ---------------------------------------------------------------- cluster decode (head_dim 64 / 128)
//
// The C (<= 16) splits of a kv head form one thread-block cluster.  Each CTA
// streams its ~1/C of the positions through two shared-memory stages of AC_C
// rows.  A stage is filled by tensor-map (TMA) copies of 64-dim x 128-position
// boxes of K and V, 128-byte swizzled so the ldmatrix reads below hit every
// bank once; boxes that hold only rows of earlier steps are requested before
// the programmatic-launch wait.  Each pass runs the tensor-core QK^T / online
// softmax / P.V of attn_decode_mma; the 8 warps then merge, and the splits
// meet through distributed shared memory: after a cluster barrier, CTA r
// combines its share of the head's outputs from all C CTAs' (max, sum, o).
// No global scratch, atomics or fences; a second cluster barrier keeps every
// CTA's shared memory alive until the others have read it.
constexpr int AC_MAX = 16;  // largest cluster (splits per kv head)
constexpr int AC_C = 128;   // positions per pass (8 warps x 16)
constexpr int AC_BOX = 64;  // dims per TMA box: 64 halves = one 128-byte swizzle line

template <int HD>
struct AcSmem {
  static constexpr int NB = HD / AC_BOX;                             // boxes per row of K (or V)
  static constexpr size_t BOX = (size_t)AC_C * AC_BOX * 2;            // 16 KB
  static constexpr size_t STAGE = 2 * NB * BOX;                       // K and V
  static constexpr int QROW = HD + 8;                                 // padded q tile rows (halves)
  static constexpr size_t Q = 2 * sizeof(__half) * (size_t)AM_ROWS * QROW;
  static constexpr size_t O = sizeof(float) * (size_t)AM_ROWS * HD;
  static constexpr size_t ML = sizeof(float) * (4 * AM_ROWS + AM_ROWS * AC_MAX);
  static constexpr size_t bytes = 1024 + 2 * STAGE + Q + O + ML + 16;  // + alignment slack
  static_assert(sizeof(float) * 8 * AM_ROWS * (HD + 2) <= 2 * STAGE, "warp merge buffer (both stages)");
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// byte offset of the 16-byte chunk `chunk` (of 8 halves) of position row r in a
// 128-byte-swizzled box
__device__ __forceinline__ int swz(int r, int chunk) { return r * 128 + ((chunk ^ (r & 7)) << 4); }

template <int HD>
__global__ void __launch_bounds__(256, 2) attn_decode_cluster(const __grid_constant__ AttnArgs a, int row0, int n_rows) {
  using S = AcSmem<HD>;
  constexpr int NB = S::NB, QROW = S::QROW, KS = HD / 16, NT = HD / 8;
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  // stages start on 1024 bytes, as 128-byte swizzled TMA boxes require
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~(uintptr_t)1023);
  uint8_t* stage0 = base;
  __half* qh_s = reinterpret_cast<__half*>(base + 2 * S::STAGE);
  __half* ql_s = qh_s + AM_ROWS * QROW;
  float* o_s = reinterpret_cast<float*>(ql_s + AM_ROWS * QROW);
  float* m_run = o_s + AM_ROWS * HD;
  float* l_run = m_run + AM_ROWS;
  float* l_tot = l_run + AM_ROWS;
  float* w_s = l_tot + 2 * AM_ROWS;  // [AM_ROWS][AC_MAX]
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_s + AM_ROWS * AC_MAX);
  const int group = a.n_heads / a.n_kv, VH = n_rows * group;  // VH <= 16
  const int C = (int)cluster.num_blocks(), split = (int)cluster.block_rank();
  // K clusters per kv head: the positions are split over all K * C CTAs
  const int K = (int)gridDim.x / C, cq = (int)blockIdx.x / C, gsplit = (int)blockIdx.x;
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const int q_stride = a.n_heads * HD;
  const float scale = 1.0f / sqrtf((float)HD);
  // several sequences: this CTA's one (its cache views, position, scratch, q / out row)
  const AttnSeq* sq = a.seqs ? a.seqs + blockIdx.z : nullptr;
  const CUtensorMap* tm_k = sq ? &sq->tm_k : &a.tm_k;
  const CUtensorMap* tm_v = sq ? &sq->tm_v : &a.tm_v;
  const float* qz = a.q + (sq ? (size_t)blockIdx.z * q_stride : 0);
  float* outz = a.out + (sq ? (size_t)blockIdx.z * q_stride : 0);
  float* part_ml = sq ? sq->part_ml : a.part_ml;
  float* part_o = sq ? sq->part_o : a.part_o;
  unsigned* counters = sq ? sq->counters : a.counters;

  // the position counter of a graph-driven step was advanced before the
  // previous step's kernels finished, so it is safe to read before the wait
  const int pos0 = sq ? sq->pos0 : (a.pos_dev ? *a.pos_dev : a.pos0);
  const int L = pos0 + row0 + n_rows;
  int per = (L + K * C - 1) / (K * C);
  per = (per + 15) / 16 * 16;
  const int t_begin = min(L, gsplit * per), t_end = min(L, t_begin + per);
  const int n_pass = (t_end - t_begin + AC_C - 1) / AC_C;

  auto kbox = [&](int st, int b) { return stage0 + st * S::STAGE + b * S::BOX; };
  auto vbox = [&](int st, int b) { return stage0 + st * S::STAGE + (NB + b) * S::BOX; };
  // pass p -> stage p & 1: every box of K and V from position t_begin + p * AC_C
  auto issue = [&](int p) {
    const int st = p & 1, t0 = t_begin + p * AC_C;
    mbar_arrive_expect_tx(&bars[st], (uint32_t)(2 * NB * S::BOX));
#pragma unroll
    for (int b = 0; b < NB; b++) {
      tma_load_3d(kbox(st, b), tm_k, b * AC_BOX, kvh, t0, &bars[st]);
      tma_load_3d(vbox(st, b), tm_v, b * AC_BOX, kvh, t0, &bars[st]);
    }
  };
  // a pass holding only rows written by earlier steps may load before the wait
  auto early = [&](int p) { return t_begin + p * AC_C + AC_C <= pos0; };

  __shared__ int q_off[AM_ROWS];
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
    for (int p = 0; p < 2 && p < n_pass; p++)
      if (early(p)) issue(p);
  }
  if (tid < AM_ROWS) q_off[tid] = tid < VH ? (row0 + tid / group) * q_stride + (kvh * group + tid % group) * HD : -1;
  pdl_wait();
  if (tid == 0)
    for (int p = 0; p < 2 && p < n_pass; p++)
      if (!early(p)) issue(p);
  __syncthreads();
  for (int i = tid; i < AM_ROWS * HD; i += 256) {
    const int vh = i / HD, d = i - vh * HD;
    const int off = q_off[vh];
    const float x = off >= 0 ? qz[off + d] : 0.0f;
    const __half h = __float2half_rn(x);
    qh_s[vh * QROW + d] = h;
    ql_s[vh * QROW + d] = __float2half_rn(x - __half2float(h));
  }
  __syncthreads();
  pdl_trigger();

  float m_w[2] = {-INFINITY, -INFINITY}, l_w[2] = {0.0f, 0.0f};
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  const int lr = lane & 7, lj = lane >> 3;
  bool ok = true;
  for (int p = 0; p < n_pass; p++) {
    const int st = p & 1, t0 = t_begin + p * AC_C, n = min(AC_C, t_end - t0);
    ok = mbar_wait(&bars[st], (p >> 1) & 1) && ok;
    const int p0 = wi * 16;
    if (p0 < n) {
      float sc[2][4];
#pragma unroll
      for (int i = 0; i < 2; i++) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.0f;
      const int kr = p0 + (lj >> 1) * 8 + lr;  // K row this lane addresses
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
        uint32_t ah[4], al[4], kb[4];
        const int qoff = ((lj & 1) * 8 + lr) * QROW + ks * 16 + (lj >> 1) * 8;
        ldsm_x4(ah, qh_s + qoff);
        ldsm_x4(al, ql_s + qoff);
        const int c = ks * 2 + (lj & 1);  // 8-dim chunk along the head
        ldsm_x4(kb, kbox(st, c / 8) + swz(kr, c % 8));
        mma_f16(sc[0], ah, kb[0], kb[1]);
        mma_f16(sc[0], al, kb[0], kb[1]);
        mma_f16(sc[1], ah, kb[2], kb[3]);
        mma_f16(sc[1], al, kb[2], kb[3]);
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
          const int row = g + (cc >> 1) * 8, pp = p0 + nt * 8 + tig * 2 + (cc & 1);
          const bool vis = row < VH && pp < n && t0 + pp <= pos0 + row0 + row / group;
          sc[nt][cc] = vis ? __fmul_rn(sc[nt][cc], scale) : -INFINITY;
          mx[cc >> 1] = fmaxf(mx[cc >> 1], sc[nt][cc]);
        }
      float alpha[2], sum[2] = {0.0f, 0.0f};
#pragma unroll
      for (int h = 0; h < 2; h++) {
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        const float m_new = fmaxf(m_w[h], mx[h]);
        alpha[h] = (m_w[h] == -INFINITY) ? 0.0f : expf(m_w[h] - m_new);
        m_w[h] = m_new;
      }
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int cc = 0; cc < 4; cc++) {
          const float sv = sc[nt][cc];
          const float pr = (sv == -INFINITY) ? 0.0f : expf(sv - m_w[cc >> 1]);
          sc[nt][cc] = pr;
          sum[cc >> 1] += pr;
        }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 1);
        sum[h] += __shfl_xor_sync(0xffffffffu, sum[h], 2);
        l_w[h] = fmaf(l_w[h], alpha[h], sum[h]);
      }
#pragma unroll
      for (int i = 0; i < NT; i++) {
        o[i][0] *= alpha[0];
        o[i][1] *= alpha[0];
        o[i][2] *= alpha[1];
        o[i][3] *= alpha[1];
      }
      uint32_t ph[4], pl[4];
      split_pair(sc[0][0], sc[0][1], ph[0], pl[0]);
      split_pair(sc[0][2], sc[0][3], ph[1], pl[1]);
      split_pair(sc[1][0], sc[1][1], ph[2], pl[2]);
      split_pair(sc[1][2], sc[1][3], ph[3], pl[3]);
      const int vr = p0 + (lj & 1) * 8 + lr;  // V row this lane addresses
#pragma unroll
      for (int dt = 0; dt < NT; dt += 2) {
        uint32_t vb[4];
        const int c = dt + (lj >> 1);
        ldsm_x4_t(vb, vbox(st, c / 8) + swz(vr, c % 8));
        mma_f16(o[dt], ph, vb[0], vb[1]);
        mma_f16(o[dt], pl, vb[0], vb[1]);
        mma_f16(o[dt + 1], ph, vb[2], vb[3]);
        mma_f16(o[dt + 1], pl, vb[2], vb[3]);
      }
    }
    __syncthreads();  // the stage is free again
    if (tid == 0 && p + 2 < n_pass) issue(p + 2);
  }
  if (!ok && tid == 0 && a.err) atomicExch(a.err, 1u);

  // ---- this CTA's warps meet in the (now idle) stages: wm/wl [8][16], wo [8][VH][HD]
  float* wm = reinterpret_cast<float*>(stage0);
  float* wl = wm + 8 * AM_ROWS;
  float* wo = wl + 8 * AM_ROWS;
  if (tig == 0) {
    wm[wi * AM_ROWS + g] = m_w[0];
    wl[wi * AM_ROWS + g] = l_w[0];
    wm[wi * AM_ROWS + g + 8] = m_w[1];
    wl[wi * AM_ROWS + g + 8] = l_w[1];
  }
#pragma unroll
  for (int i = 0; i < NT; i++) {
    const int d = i * 8 + tig * 2;
    if (g < VH) *reinterpret_cast<float2*>(wo + (wi * AM_ROWS + g) * HD + d) = make_float2(o[i][0], o[i][1]);
    if (g + 8 < VH) *reinterpret_cast<float2*>(wo + (wi * AM_ROWS + g + 8) * HD + d) = make_float2(o[i][2], o[i][3]);
  }
  __syncthreads();
  if (tid < VH) {
    float mx = -INFINITY;
    for (int w = 0; w < 8; w++) mx = fmaxf(mx, wm[w * AM_ROWS + tid]);
    float l = 0.0f;
    for (int w = 0; w < 8; w++) {
      const float mw = wm[w * AM_ROWS + tid];
      const float sw = mw == -INFINITY ? 0.0f : expf(mw - mx);
      wm[w * AM_ROWS + tid] = sw;
      l = fmaf(wl[w * AM_ROWS + tid], sw, l);
    }
    m_run[tid] = mx;
    l_run[tid] = l;
  }
  __syncthreads();
  for (int e = tid; e < VH * HD; e += 256) {
    const int vh = e / HD;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) acc = fmaf(wo[(w * AM_ROWS + vh) * HD + (e - vh * HD)], wm[w * AM_ROWS + vh], acc);
    o_s[e] = acc;
  }

  // ---- the C splits meet through distributed shared memory
  cluster.sync();
  const int n_w = VH * AC_MAX;  // weight of split j for virtual head vh: 16 lanes per head
  if (tid < ((n_w + 31) & ~31)) {  // whole warps, so every shuffle sees all its lanes
    const int vh = tid / AC_MAX, j = tid % AC_MAX;
    const bool act = tid < n_w && j < C;
    float mj = -INFINITY, lj_ = 0.0f;
    if (act) {
      mj = *cluster.map_shared_rank(m_run + vh, j);
      lj_ = *cluster.map_shared_rank(l_run + vh, j);
    }
    float mx = mj;
#pragma unroll
    for (int o_ = AC_MAX / 2; o_ > 0; o_ >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o_));
    const float w = mj == -INFINITY ? 0.0f : expf(mj - mx);
    float lw = w * lj_;
#pragma unroll
    for (int o_ = AC_MAX / 2; o_ > 0; o_ >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o_);
    if (tid < n_w) {
      w_s[vh * AC_MAX + j] = w;
      if (j == 0) {
        l_tot[vh] = lw;
        l_tot[AM_ROWS + vh] = mx;  // the cluster's running max
      }
    }
  }
  __syncthreads();
  const int E = VH * HD, chunk = (E + C - 1) / C;
  const int e_end = min(E, (split + 1) * chunk);
  // one cluster: final rows; K clusters: this cluster's unnormalized partial
  // (attn_finish's partial layout, with the K clusters as the splits)
  const size_t pbase = ((size_t)kvh * K + cq) * VH;
  for (int e = split * chunk + tid; e < e_end; e += 256) {
    const int vh = e / HD, d = e - vh * HD;
    float acc = 0.0f;
    for (int j = 0; j < C; j++) acc = fmaf(*cluster.map_shared_rank(o_s + e, j), w_s[vh * AC_MAX + j], acc);
    if (K == 1) {
      const int row = vh / group, head = kvh * group + vh % group;
      outz[(size_t)(row0 + row) * q_stride + head * HD + d] = acc / l_tot[vh];
    } else {
      part_o[pbase * HD + e] = acc;
    }
  }
  if (K > 1 && split == 0 && tid < VH)
    reinterpret_cast<float2*>(part_ml)[pbase + tid] = make_float2(l_tot[AM_ROWS + tid], l_tot[tid]);
  cluster.sync();  // every CTA's shared memory stays alive until the others have read it
  if (K == 1) return;

  // ---- the last of the kv head's K * C CTAs merges the K cluster partials
  __shared__ unsigned ticket;
  __syncthreads();
  if (tid == 0) ticket = ticket_acq_rel(counters + kvh);
  __syncthreads();
  if (ticket != (unsigned)(K * C) - 1) return;
  const size_t hb = (size_t)kvh * K * VH;
  if (tid < VH) {
    float mx = -INFINITY;
    for (int q = 0; q < K; q++) mx = fmaxf(mx, __ldcg(reinterpret_cast<const float2*>(part_ml) + hb + q * VH + tid).x);
    float l = 0.0f;
    for (int q = 0; q < K; q++) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(part_ml) + hb + q * VH + tid);
      const float wq = ml.x == -INFINITY ? 0.0f : expf(ml.x - mx);
      w_s[tid * AC_MAX + q] = wq;
      l = fmaf(ml.y, wq, l);
    }
    l_tot[tid] = l;
  }
  __syncthreads();
  for (int e = tid; e < E; e += 256) {
    const int vh = e / HD;
    float acc = 0.0f;
    for (int q = 0; q < K; q++) acc = fmaf(__ldcg(part_o + (hb + (size_t)q * VH) * HD + e), w_s[vh * AC_MAX + q], acc);
    const int row = vh / group, head = kvh * group + vh % group, d = e - vh * HD;
    outz[(size_t)(row0 + row) * q_stride + head * HD + d] = acc / l_tot[vh];
  }
  if (tid == 0) counters[kvh] = 0u;
}

// ---------------------------------------------------------------- tcgen05 decode / verify
// The same attention on the 5th-generation tensor cores, one tile of 128
// positions at a time, warp-specialized:
//   warp 8 (one lane)   TMA: K and V boxes of each tile into a 2- or 3-stage
//                       ring, the tiles before pos0 ahead of the programmatic
//                       wait
//   warp 9 (one lane)   MMAs: S = K . [q_hi | q_lo]^T (M = 128 positions,
//                       N = 2 NQ: the hi and lo halves side by side) into one
//                       of two TMEM buffers as soon as a tile lands, and
//                       O^T = V^T . [P_hi | P_lo] (M = 128 dims, V read
//                       MN-major straight from its TMA box) once P is
//                       written; whichever of the two is ready goes first, so
//                       a late tile never holds back the P.V of an earlier one
//   warps 0-3, 4-7      two softmax groups on alternate tiles (group g takes
//                       tiles g, g + 2, ...: its own S, P and O buffers), one
//                       thread per position: scores = hi + lo columns,
//                       masked and scaled, exp against the group's running
//                       reference max that moves only when a score passes it
//                       by more than 8 (then the tile's exact max, and a
//                       rescale); P to shared memory as f16 hi / lo; one
//                       thread per dim folds O_hi + O_lo of the group's
//                       previous tile into its registers.  Per-thread sums of
//                       P meet once at the end, then the two groups' (max,
//                       sum, o) as two partials.
// q and P enter as f16 hi + lo pairs (each product carries ~22 bits of the
// f32 operand; K and V are f16 already); accumulation is f32.  The n_splits
// position ranges of a kv head meet as in attn_finish.
constexpr int TC_C = 128;
constexpr int TC_THREADS = 320;   // warps 0-7 softmax (two groups), 8 TMA, 9 MMA
constexpr int TC_TMA_WARP = 8, TC_MMA_WARP = 9;
constexpr int TC_COLS = 128;      // TMEM: S buffers [0, 64), O buffers [64, 128)
constexpr float TC_TAU = 8.0f;    // largest exponent before the reference max moves

template <int HD, int NS>
struct TcSmem {
  static constexpr int NB = HD / AC_BOX;                   // 64-dim boxes per K (or V) row
  static constexpr size_t BOX = (size_t)TC_C * AC_BOX * 2;  // 16 KB
  static constexpr size_t STAGE = 2 * NB * BOX;             // K boxes, then V boxes
  static constexpr size_t OP = 32 * 128 * 2;                // a 32-row x 128-value f16 operand tile
  static constexpr size_t OFF_Q = NS * STAGE;
  static constexpr size_t OFF_P = OFF_Q + OP;               // two P tiles
  static constexpr size_t OFF_RED = OFF_P + 2 * OP;         // [2 groups][4 warps][16] floats
  static constexpr size_t bytes = 1024 + OFF_RED + 8 * 16 * sizeof(float) + 64;
  static_assert(sizeof(float) * 16 * HD <= STAGE, "o staging");
};

// byte offset of element (row r < 32, column k < 128) of a K-major f16
// operand tile: 128-byte swizzle atoms of 64 columns x 32 rows, 4 KB apart
__device__ __forceinline__ int op_off(int r, int k) {
  return (k >> 6) * 4096 + (r >> 3) * 1024 + (r & 7) * 128 + ((((k & 63) >> 3) ^ (r & 7)) << 4) + (k & 7) * 2;
}
// f16 instruction descriptor: f32 accumulate, M = 128, N = n; A MN-major when `a_mn`
constexpr uint32_t f16_idesc(bool a_mn, int n) {
  return (1u << 4) | ((a_mn ? 1u : 0u) << 15) | ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t* r) {
  tc_ld16(taddr, r);
  tc_ld16(taddr + 16, r + 16);
}
// Bounded wait that also gives up once another role of the CTA has.
__device__ __forceinline__ bool twait(uint64_t* bar, uint32_t phase, volatile int* abort) {
  for (uint32_t i = 0; i < kMbarPolls; i++) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((i & 255) == 255 && *abort) return false;
  }
  *abort = 1;
  return false;
}
// named barriers of softmax group g (1 + g: its four warps) and of both
// groups (3); the OR of `pred` over a group
__device__ __forceinline__ void grp_sync(int g) { asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory"); }
__device__ __forceinline__ void both_sync() { asm volatile("bar.sync 3, 256;" ::: "memory"); }
__device__ __forceinline__ bool grp_any(int g, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, 128, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(1 + g)
      : "memory");
  return r != 0;
}

// The n_splits partials of one kv head (and sequence) of attn_decode_tc meet
// here, in the kernel launched right behind it: the (max, sum) pairs by plain
// loads while one bulk copy brings the o rows (contiguous per kv head) into
// shared memory when they fit, then attn_finish's arithmetic.  One thread
// per dim.
constexpr size_t TC_MERGE_SMEM = 160 * 1024;
template <int HD>
__global__ void __launch_bounds__(HD) attn_merge_tc(const __grid_constant__ AttnArgs a, int row0, int n_rows) {
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float l_s[16];
  const int kvh = blockIdx.x, z = blockIdx.y, tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
  const int group = a.n_heads / a.n_kv, VH = n_rows * group, NS = a.n_splits;
  const int q_stride = a.n_heads * HD;
  const AttnSeq* sq = a.seqs ? a.seqs + z : nullptr;
  const float* part_ml = sq ? sq->part_ml : a.part_ml;
  const float* part_o = sq ? sq->part_o : a.part_o;
  float* out = a.out + (sq ? (size_t)z * q_stride : 0);
  const size_t hb = (size_t)kvh * NS * VH;  // this kv head's first partial
  const size_t o_bytes = (size_t)NS * VH * HD * 4;
  float* w_s = reinterpret_cast<float*>(smem_dyn);  // [VH][NS]
  float* po = w_s + ((VH * NS + 3) & ~3);           // [NS][VH][HD] when it fits
  const bool bulk = (size_t)((VH * NS + 3) & ~3) * 4 + o_bytes <= TC_MERGE_SMEM;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();  // the attention grid has finished and its partials are visible
  pdl_trigger();
  if (bulk && tid == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    mbar_arrive_expect_tx(&bar, (uint32_t)o_bytes);
    bulk_g2s(po, part_o + hb * HD, (uint32_t)o_bytes, &bar);
  }
  // (max, sum) of every split -> weights exp(m_s - max) and the total
  for (int vh = wi; vh < VH; vh += HD / 32) {
    float mx = -INFINITY;
    for (int s = lane; s < NS; s += 32) mx = fmaxf(mx, __ldcg(reinterpret_cast<const float2*>(part_ml) + hb + (size_t)s * VH + vh).x);
    mx = warp_max(mx);
    float lsum = 0.0f;
    for (int s = lane; s < NS; s += 32) {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(part_ml) + hb + (size_t)s * VH + vh);
      const float w = v.x == -INFINITY ? 0.0f : expf(v.x - mx);
      w_s[vh * NS + s] = w;
      lsum = fmaf(v.y, w, lsum);
    }
    lsum = warp_sum(lsum);
    if (lane == 0) l_s[vh] = lsum;
  }
  if (bulk && !mbar_wait(&bar, 0) && a.err) atomicExch(a.err, ERR_TIMEOUT);
  __syncthreads();
  for (int vh = 0; vh < VH; vh++) {
    float acc = 0.0f;
    if (bulk) {
      for (int s = 0; s < NS; s++) acc = fmaf(po[((size_t)s * VH + vh) * HD + tid], w_s[vh * NS + s], acc);
    } else {
#pragma unroll 8
      for (int s = 0; s < NS; s++) acc = fmaf(__ldcg(part_o + (hb + (size_t)s * VH + vh) * HD + tid), w_s[vh * NS + s], acc);
    }
    const int row = vh / group, head = kvh * group + vh % group;
    out[(size_t)(row0 + row) * q_stride + head * HD + tid] = acc / l_s[vh];
  }
}

// NQ: virtual-head columns of each half (8 when VH <= 8, else 16); NS: K/V
// stages; VHC: a compile-time bound on VH, the heads the per-position loops run
template <int HD, int NQ, int NS, int VHC>
__global__ void __launch_bounds__(TC_THREADS, 1) attn_decode_tc(const __grid_constant__ AttnArgs a, int row0, int n_rows) {
  static_assert(VHC <= NQ, "virtual heads");
  using S = TcSmem<HD, NS>;
  constexpr int TC_NS = NS;
  constexpr int NB = S::NB, KSTEPS = HD / 16, PSTEPS = TC_C / 16;
  constexpr uint32_t IDESC_S = f16_idesc(false, 2 * NQ), IDESC_O = f16_idesc(true, 2 * NQ);
  extern __shared__ __align__(16) uint8_t smem_dyn[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~(uintptr_t)1023);
  uint8_t* q_t = base + S::OFF_Q;
  uint8_t* p_t = base + S::OFF_P;
  float* red = reinterpret_cast<float*>(base + S::OFF_RED);  // [2][4][16]
  // full[3] stage_free[3] s_full[2] s_free[2] p_full[2] o_full[2] o_free[2] q_ready mma_done
  __shared__ __align__(8) uint64_t bars[18];
  uint64_t* full = bars;
  uint64_t* stage_free = bars + 3;
  uint64_t* s_full = bars + 6;
  uint64_t* s_free = bars + 8;
  uint64_t* p_full = bars + 10;
  uint64_t* o_full = bars + 12;
  uint64_t* o_free = bars + 14;
  uint64_t* q_ready = bars + 16;
  uint64_t* mma_done = bars + 17;
  __shared__ uint32_t tmem_s;
  __shared__ int s_abort;
  volatile int* abort = &s_abort;

  const int group = a.n_heads / a.n_kv, VH = n_rows * group;  // VH <= VHC
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5;
  const int q_stride = a.n_heads * HD;
  const float scale = 1.0f / sqrtf((float)HD);
  const AttnSeq* sq = a.seqs ? a.seqs + blockIdx.z : nullptr;
  const CUtensorMap* tm_k = sq ? &sq->tm_k : &a.tm_k;
  const CUtensorMap* tm_v = sq ? &sq->tm_v : &a.tm_v;
  const float* qz = a.q + (sq ? (size_t)blockIdx.z * q_stride : 0);

  // the position counter of a graph-driven step was advanced before the
  // previous step's kernels finished, so it is safe to read before the wait
  const int pos0 = sq ? sq->pos0 : (a.pos_dev ? *a.pos_dev : a.pos0);
  const int L = pos0 + row0 + n_rows;
  int per = (L + a.n_splits - 1) / a.n_splits;
  per = (per + 15) / 16 * 16;
  const int t_begin = min(L, split * per), t_end = min(L, t_begin + per);
  const int n_tiles = (t_end - t_begin + TC_C - 1) / TC_C;

  auto kbox = [&](int st, int b) { return base + st * S::STAGE + b * S::BOX; };
  auto vbox = [&](int st, int b) { return base + st * S::STAGE + (NB + b) * S::BOX; };

  auto issue = [&](int i) {  // the K and V boxes of tile i
    const int st = i % TC_NS, t0 = t_begin + i * TC_C;
    mbar_arrive_expect_tx(&full[st], (uint32_t)(2 * NB * S::BOX));
#pragma unroll
    for (int b = 0; b < NB; b++) {
      tma_load_3d(kbox(st, b), tm_k, b * AC_BOX, kvh, t0, &full[st]);
      tma_load_3d(vbox(st, b), tm_v, b * AC_BOX, kvh, t0, &full[st]);
    }
  };
  int pre = 0;  // tiles issued ahead of the setup barrier
  if (wi == TC_TMA_WARP && lane == 0) {
    s_abort = 0;
    for (int i = 0; i < 3; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&stage_free[i], 1);
    }
    for (int i = 0; i < 2; i++) {  // buffer i belongs to softmax group i
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(q_ready, 128);
    mbar_init(mma_done, 1);
    fence_barrier_init();
    // tiles holding only rows written by earlier steps go first, before the
    // programmatic wait and the rest of the setup
    for (; pre < TC_NS && pre < n_tiles && t_begin + (pre + 1) * TC_C <= pos0; pre++) issue(pre);
  }
  if (wi == TC_MMA_WARP) {
    tc_alloc(&tmem_s, TC_COLS);
    tc_relinquish();
  }
  // P rows >= VHC (and their lo rows) stay zero; the others are rewritten every tile
  for (int i = tid; i < (int)(2 * S::OP / 16); i += TC_THREADS)
    reinterpret_cast<uint4*>(p_t)[i] = make_uint4(0u, 0u, 0u, 0u);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;
  pdl_trigger();
  bool ok = true;

  if (wi == TC_TMA_WARP) {
    // ------------------------------------------------ TMA
    if (lane == 0) {
      int i = pre;
      pdl_wait();
      int issued = i;
      for (; i < n_tiles; i++) {
        const int st = i % TC_NS;
        if (i >= TC_NS && !twait(&stage_free[st], ((i / TC_NS) - 1) & 1, abort)) break;
        issue(i);
        issued = i + 1;
      }
      // wind down: every copy issued has landed before the CTA may exit
      for (int j = issued > TC_NS ? issued - TC_NS : 0; j < issued; j++)
        ok = mbar_wait(&full[j % TC_NS], (j / TC_NS) & 1, *abort ? (1u << 16) : kMbarPolls) && ok;
    }
    __syncwarp();
  } else if (wi == TC_MMA_WARP) {
    // ------------------------------------------------ MMA
    // S(j) goes once its tile has landed and group j & 1 has read S(j - 2);
    // P.V(j) once P(j) is written and the group has folded O(j - 2) (the
    // group folds O(j - 2) before it writes P(j), so that P tile is free).
    // Non-blocking tests: neither stream waits behind the other.
    if (lane == 0) {
      const uint64_t qd = sw128_desc(smem_u32(q_t));
      bool go = twait(q_ready, 0, abort);
      int ns = 0, np = 0;
      uint32_t idle = 0;
      while (go && np < n_tiles) {
        bool moved = false;
        if (ns < n_tiles && mbar_test_wait(&full[ns % TC_NS], (ns / TC_NS) & 1) &&
            (ns < 2 || mbar_test_wait(&s_free[ns & 1], ((ns - 2) >> 1) & 1))) {
          const int st = ns % TC_NS, sb = ns & 1;
          tc_fence_after();
          const uint64_t k0 = sw128_desc(smem_u32(kbox(st, 0)));
#pragma unroll
          for (int ks = 0; ks < KSTEPS; ks++)
            tc_mma_f16(tmem + (uint32_t)(sb * 32), k0 + (uint64_t)((ks >> 2) * (S::BOX >> 4) + (ks & 3) * 2),
                       qd + (uint64_t)((ks >> 2) * 256 + (ks & 3) * 2), IDESC_S, ks > 0);
          tc_commit(&s_full[sb]);
          ns++;
          moved = true;
        }
        if (np < ns && mbar_test_wait(&p_full[np & 1], (np >> 1) & 1) &&
            (np < 2 || mbar_test_wait(&o_free[np & 1], ((np - 2) >> 1) & 1))) {
          const int st = np % TC_NS, pb = np & 1;
          tc_fence_after();
          const uint64_t v0 = sw128_desc_mn(smem_u32(vbox(st, 0)), (uint32_t)S::BOX, 1024u);
          const uint64_t p0 = sw128_desc(smem_u32(p_t + pb * S::OP));
#pragma unroll
          for (int ks = 0; ks < PSTEPS; ks++)
            tc_mma_f16(tmem + 64u + (uint32_t)(pb * 32), v0 + (uint64_t)(ks * 128),
                       p0 + (uint64_t)((ks >> 2) * 256 + (ks & 3) * 2), IDESC_O, ks > 0);
          tc_commit(&o_full[pb]);
          tc_commit(&stage_free[st]);
          np++;
          moved = true;
        }
        if (moved) {
          idle = 0;
        } else if (++idle >= kMbarPolls || ((idle & 255) == 255 && *abort)) {
          *abort = 1;
          break;
        }
      }
      // wind down: every MMA issued has completed before TMEM is freed
      tc_commit(mma_done);
      ok = mbar_wait(mma_done, 0, *abort ? (1u << 16) : kMbarPolls) && ok;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ softmax groups (warps 0-3, 4-7)
    const int g = wi >> 2, wq = wi & 3;  // group; warp in the group = its TMEM lane quarter
    const int r = tid & 127;              // TMEM lane: tile position r for S, dim r for O
    pdl_wait();
    if (g == 0) {
      // q rows of the virtual heads as f16 hi (rows 0..NQ) and lo (NQ..2 NQ); rows >= VH zero
      for (int c = r; c < NQ * (HD / 4); c += 128) {
        const int vh = c / (HD / 4), d = (c - vh * (HD / 4)) * 4;
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (vh < VH)
          x = *reinterpret_cast<const float4*>(qz + (size_t)(row0 + vh / group) * q_stride +
                                               (size_t)(kvh * group + vh % group) * HD + d);
        const float xs[4] = {x.x, x.y, x.z, x.w};
        __half hh[4], hl[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          hh[e] = __float2half_rn(xs[e]);
          hl[e] = __float2half_rn(xs[e] - __half2float(hh[e]));
        }
        *reinterpret_cast<uint2*>(q_t + op_off(vh, d)) = *reinterpret_cast<const uint2*>(hh);
        *reinterpret_cast<uint2*>(q_t + op_off(NQ + vh, d)) = *reinterpret_cast<const uint2*>(hl);
      }
      fence_async_smem();
      mbar_arrive(q_ready);
    }

    float m_run[VHC], l_thr[VHC], o_acc[VHC], alpha_prev[VHC];
#pragma unroll
    for (int h = 0; h < VHC; h++) {
      m_run[h] = -INFINITY;
      l_thr[h] = 0.0f;
      o_acc[h] = 0.0f;
      alpha_prev[h] = 1.0f;
    }
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t s_col = (uint32_t)(g * 32), o_col = 64u + (uint32_t)(g * 32);
    // hi columns [0, VHC) and lo columns [NQ, NQ + VHC) of this lane
    auto ld_cols = [&](uint32_t taddr, uint32_t* v) {
      if constexpr (VHC <= 4) {
        tc_ld4(taddr, v);
        tc_ld4(taddr + NQ, v + NQ);
      } else if constexpr (NQ == 8) {
        tc_ld16(taddr, v);
      } else {
        tc_ld32(taddr, v);
      }
      tc_wait_ld();
    };
    // O of the group's tile i into the registers, rescaled by that tile's alpha
    auto fold = [&](int i, const float* al) {
      ok = twait(&o_full[g], (i >> 1) & 1, abort) && ok;
      tc_fence_after();
      uint32_t ov[2 * NQ];
      ld_cols(tmem + lane_base + o_col, ov);
      tc_fence_before();
      mbar_arrive(&o_free[g]);
#pragma unroll
      for (int h = 0; h < VHC; h++)
        o_acc[h] = fmaf(o_acc[h], al[h], __uint_as_float(ov[h]) + __uint_as_float(ov[NQ + h]));
    };
    int last = -1;  // the group's last tile
    for (int i = g; i < n_tiles; i += 2) {
      const int st = i % TC_NS, t = t_begin + i * TC_C + r;
      // O of the group's previous tile while S(i) is on its way; once it is
      // in, P.V(i - 2) has completed and its P tile may be rewritten
      if (i >= 2) fold(i - 2, alpha_prev);
      ok = twait(&s_full[g], (i >> 1) & 1, abort) && ok;
      tc_fence_after();
      uint32_t sv[2 * NQ];
      ld_cols(tmem + lane_base + s_col, sv);
      tc_fence_before();
      mbar_arrive(&s_free[g]);
      float sc[VHC], alpha[VHC];
      bool over = false;
#pragma unroll
      for (int h = 0; h < VHC; h++) {
        const bool vis = h < VH && t < t_end && t <= pos0 + row0 + h / group;
        sc[h] = vis ? __fmul_rn(__uint_as_float(sv[h]) + __uint_as_float(sv[NQ + h]), scale) : -INFINITY;
        over |= sc[h] > m_run[h] + TC_TAU;
        alpha[h] = 1.0f;
      }
      if (grp_any(g, over || *abort != 0)) {
        if (grp_any(g, *abort != 0)) break;  // a uniform decision: the named barriers stay matched
        // the tile's exact max becomes the reference
        float* rg = red + g * 64;
#pragma unroll
        for (int h = 0; h < VHC; h++)
          if (h < VH) {
            const float mw = warp_max(sc[h]);
            if (lane == 0) rg[wq * 16 + h] = mw;
          }
        grp_sync(g);
#pragma unroll
        for (int h = 0; h < VHC; h++)
          if (h < VH) {
            const float mt = fmaxf(fmaxf(rg[h], rg[16 + h]), fmaxf(rg[32 + h], rg[48 + h]));
            const float m_new = fmaxf(m_run[h], mt);
            alpha[h] = m_run[h] == -INFINITY ? 0.0f : expf(m_run[h] - m_new);
            m_run[h] = m_new;
            l_thr[h] *= alpha[h];
          }
      }
      uint8_t* pt = p_t + g * S::OP;
#pragma unroll
      for (int h = 0; h < VHC; h++) {
        const float pv = sc[h] == -INFINITY ? 0.0f : expf(sc[h] - m_run[h]);
        l_thr[h] += pv;
        const __half ph = __float2half_rn(pv);
        *reinterpret_cast<__half*>(pt + op_off(h, r)) = ph;
        *reinterpret_cast<__half*>(pt + op_off(NQ + h, r)) = __float2half_rn(pv - __half2float(ph));
      }
      // V rows at positions not yet written may hold anything: zero them (P is 0 there)
      if (t >= L) {
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
          for (int c = 0; c < 8; c++)
            *reinterpret_cast<uint4*>(vbox(st, b) + r * 128 + c * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_async_smem();
      mbar_arrive(&p_full[g]);
#pragma unroll
      for (int h = 0; h < VHC; h++) alpha_prev[h] = alpha[h];
      last = i;
    }
    if (last >= 0 && !*abort) fold(last, alpha_prev);
    // the sums over the group's positions, once
#pragma unroll
    for (int h = 0; h < VHC; h++)
      if (h < VH) {
        const float sw = warp_sum(l_thr[h]);
        if (lane == 0) red[g * 64 + wq * 16 + h] = sw;
      }
    // both groups' last folds are done, so every MMA has completed: the
    // stages are idle.  Group g's o goes to stage 0 at g * NQ * HD, its
    // (max, sum) to stage 1 at 32 g.
    both_sync();
    float* o_g = reinterpret_cast<float*>(base) + g * NQ * HD;
    float* ml = reinterpret_cast<float*>(base + S::STAGE) + 32 * g;
#pragma unroll
    for (int h = 0; h < VHC; h++)
      if (h < VH) o_g[h * HD + r] = o_acc[h];
    if (r < VH) {
      float mv = m_run[0];
#pragma unroll
      for (int h = 1; h < VHC; h++)
        if (h == r) mv = m_run[h];
      const float* rg = red + g * 64;
      ml[r] = mv;
      ml[16 + r] = (rg[r] + rg[16 + r]) + (rg[32 + r] + rg[48 + r]);
    }
  }
  if (!ok) *abort = 1;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abort && tid == 0 && a.err) atomicExch(a.err, ERR_TIMEOUT);
  if (wi == TC_MMA_WARP) tc_dealloc(tmem, TC_COLS);
  {
    // the two groups' partials -> this split's (max, sum) in stage 1 [0, 32)
    // and o in stage 0 [0, VH * HD)
    float* o_s = reinterpret_cast<float*>(base);
    float* ml = reinterpret_cast<float*>(base + S::STAGE);
    __shared__ float wg[2][16];
    if (tid < VH) {
      const float m0 = ml[tid], m1 = ml[32 + tid], mx = fmaxf(m0, m1);
      const float w0 = m0 == -INFINITY ? 0.0f : expf(m0 - mx), w1 = m1 == -INFINITY ? 0.0f : expf(m1 - mx);
      wg[0][tid] = w0;
      wg[1][tid] = w1;
      ml[tid] = mx;
      ml[16 + tid] = fmaf(ml[16 + tid], w0, ml[48 + tid] * w1);
    }
    __syncthreads();
    for (int e = tid; e < VH * HD; e += TC_THREADS) {
      const int vh = e / HD;
      o_s[e] = fmaf(o_s[e], wg[0][vh], o_s[NQ * HD + e] * wg[1][vh]);
    }
    __syncthreads();
  }

  // ---- this split's (max, sum, o): the final rows with one split, else a
  // partial for attn_merge_tc (stage 0 holds o, stage 1 m / l)
  const float* o_s = reinterpret_cast<const float*>(base);
  const float* ml = reinterpret_cast<const float*>(base + S::STAGE);
  float* out = a.out + (sq ? (size_t)blockIdx.z * q_stride : 0);
  if (a.n_splits == 1) {
    for (int e = tid; e < VH * HD; e += TC_THREADS) {
      const int vh = e / HD, d = e - vh * HD;
      const int row = vh / group, head = kvh * group + vh % group;
      out[(size_t)(row0 + row) * q_stride + head * HD + d] = o_s[e] / ml[16 + vh];
    }
    return;
  }
  float* part_ml = sq ? sq->part_ml : a.part_ml;
  float* part_o = sq ? sq->part_o : a.part_o;
  const int NSP = a.n_splits;
  const size_t pbase = ((size_t)kvh * NSP + split) * VH;
  for (int vh = tid; vh < VH; vh += TC_THREADS)
    reinterpret_cast<float2*>(part_ml)[pbase + vh] = make_float2(ml[vh], ml[16 + vh]);
  for (int e = tid; e < VH * HD / 4; e += TC_THREADS)
    reinterpret_cast<float4*>(part_o + pbase * HD)[e] = reinterpret_cast<const float4*>(o_s)[e];
  if (!a.tail_merge) return;  // attn_merge_tc follows
  // ---- the last split CTA of the kv head merges: every split's o rows by one
  // bulk copy into the idle stages, the (max, sum) pairs by plain loads
  unsigned* counters = sq ? sq->counters : a.counters;
  __shared__ unsigned ticket;
  __syncthreads();
  if (tid == 0) ticket = ticket_acq_rel(counters + kvh);
  __syncthreads();
  if (ticket != (unsigned)NSP - 1) return;
  const size_t hb = (size_t)kvh * NSP * VH;
  const uint32_t o_bytes = (uint32_t)((size_t)NSP * VH * HD * 4);
  float* po = reinterpret_cast<float*>(base + S::STAGE);  // [NSP][VH][HD] (the host checked it fits)
  __shared__ float w_m[16 * 64];                           // [vh][split] weights (splits <= 64)
  __shared__ float l_m[16];
  if (tid == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the acquired partials, to the bulk copy
    mbar_arrive_expect_tx(&bars[0], o_bytes);
    bulk_g2s(po, part_o + hb * HD, o_bytes, &bars[0]);
  }
  for (int vh = wi; vh < VH; vh += TC_THREADS / 32) {
    float mx = -INFINITY;
    for (int j = lane; j < NSP; j += 32) mx = fmaxf(mx, __ldcg(reinterpret_cast<const float2*>(part_ml) + hb + (size_t)j * VH + vh).x);
    mx = warp_max(mx);
    float lsum = 0.0f;
    for (int j = lane; j < NSP; j += 32) {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(part_ml) + hb + (size_t)j * VH + vh);
      const float w = v.x == -INFINITY ? 0.0f : expf(v.x - mx);
      w_m[vh * 64 + j] = w;
      lsum = fmaf(v.y, w, lsum);
    }
    lsum = warp_sum(lsum);
    if (lane == 0) l_m[vh] = lsum;
  }
  // full[0] completed every use the tile loop made of it; this is its next phase
  const int uses0 = (n_tiles + NS - 1) / NS;
  if (!mbar_wait(&bars[0], uses0 & 1) && a.err) atomicExch(a.err, ERR_TIMEOUT);
  __syncthreads();
  for (int e = tid; e < VH * HD; e += TC_THREADS) {
    const int vh = e / HD, d = e - vh * HD;
    float acc = 0.0f;
    for (int j = 0; j < NSP; j++) acc = fmaf(po[((size_t)j * VH + vh) * HD + d], w_m[vh * 64 + j], acc);
    const int row = vh / group, head = kvh * group + vh % group;
    out[(size_t)(row0 + row) * q_stride + head * HD + d] = acc / l_m[vh];
  }
  if (tid == 0) counters[kvh] = 0u;
}

template <int HD, bool MMA>
static cudaError_t decode_go(const AttnArgs& a, cudaStream_t st, bool pdl) {
  const int group = a.n_heads / a.n_kv;
  const int max_rows = MMA ? AM_ROWS / group : AT_MAX_VHD / (HD * group);
  if (max_rows < 1) return cudaErrorInvalidValue;
  for (int row0 = 0; row0 < a.m; row0 += max_rows) {
    const int n_rows = min(max_rows, a.m - row0);
    size_t smem;
    const void* k;
    if constexpr (MMA) {
      smem = AmSmem<HD>::bytes;
      k = (const void*)attn_decode_mma<HD>;
    } else {
      smem = AdSmem<HD>::bytes(n_rows * group);
      k = (const void*)attn_decode_kernel<HD>;
    }
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    AttnArgs aa = a;
    void* args[] = {&aa, (void*)&row0, (void*)&n_rows};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_splits, a.n_kv);
    cfg.blockDim = dim3(AD_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (pdl && row0 == 0) {
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelExC(&cfg, k, args);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// ---- tensor maps of the f16 cache (driver entry point, looked up once)
using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  });
  return fn;
}

// {hd, n_kv, positions} view of one layer's K or V cache; a box is 64 dims x
// 1 head x 128 positions, 128-byte swizzled; rows past `positions` read as 0
static bool encode_cache_map(CUtensorMap* m, const __half* base, int positions, int n_kv, int hd) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || positions < 1 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)n_kv, (cuuint64_t)positions};
  const cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)n_kv * hd * 2};
  const cuuint32_t box[3] = {(cuuint32_t)AC_BOX, 1, (cuuint32_t)AC_C};
  const cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void attn_make_maps(AttnArgs& a, int positions) {
  a.has_tm = 0;
  if (a.hd != 64 && a.hd != 128) return;
  if (encode_cache_map(&a.tm_k, a.kc, positions, a.n_kv, a.hd) && encode_cache_map(&a.tm_v, a.vc, positions, a.n_kv, a.hd))
    a.has_tm = 1;
}

// Cluster shape for n_kv kv heads: C CTAs per cluster (the largest C <= 16
// for which all n_kv clusters are resident at once) and, when C reaches 16
// with room to spare (few kv heads: a tensor-parallel shard), K clusters per
// kv head whose partials meet through global memory; K is capped by the split
// scratch (max_k) and by AC_MAX.  Asked once per device, n_kv and max_k.
// C == 0: no cluster fits.
struct ClusterPlan {
  int c = 0, k = 1;
};
template <int HD>
static ClusterPlan cluster_plan(int n_kv, int max_k) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, ClusterPlan> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return {};
  if (max_k > AC_MAX) max_k = AC_MAX;
  if (max_k < 1) max_k = 1;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, n_kv, max_k});
  if (it != cache.end()) return it->second;
  auto k = attn_decode_cluster<HD>;
  ClusterPlan best;
  if (cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AcSmem<HD>::bytes) ==
          cudaSuccess &&
      cudaFuncSetAttribute((const void*)k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
    for (int c = AC_MAX; c >= 2 && !best.c; c--) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(c, n_kv);
      cfg.blockDim = dim3(256);
      cfg.dynamicSmemBytes = AcSmem<HD>::bytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = c;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, (const void*)k, &cfg) == cudaSuccess && n >= n_kv) {
        best.c = c;
        // several clusters per kv head only at full cluster size: below it the
        // global merge costs more than the extra CTAs gain
        if (c == AC_MAX) best.k = std::min(max_k, n / n_kv);
      }
    }
  }
  cudaGetLastError();
  cache[{dev, n_kv, max_k}] = best;
  return best;
}

template <int HD>
static cudaError_t cluster_go(const AttnArgs& a, ClusterPlan pl, cudaStream_t st, bool pdl, int n_seq = 1) {
  const int c = pl.c;
  const int group = a.n_heads / a.n_kv;
  const int max_rows = AM_ROWS / group;
  for (int row0 = 0; row0 < a.m; row0 += max_rows) {
    const int n_rows = min(max_rows, a.m - row0);
    void* args[] = {const_cast<AttnArgs*>(&a), (void*)&row0, (void*)&n_rows};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c * pl.k, a.n_kv, n_seq);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = AcSmem<HD>::bytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    int na = 1;
    if (pdl && row0 == 0) {
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    cudaError_t e = cudaLaunchKernelExC(&cfg, (const void*)attn_decode_cluster<HD>, args);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// SMs of the current device (asked once per device)
static int device_sms() {
  static std::mutex mu;
  static std::map<int, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
  cudaGetLastError();
  cache[dev] = n;
  return n;
}

// tcgen05 attention: one CTA per SM across (splits, kv heads, sequences);
// the split count is capped by the partial scratch the caller sized
template <int HD, int NQ, int VHC>
static const void* tc_kernel_v(bool two) {
  return two ? (const void*)attn_decode_tc<HD, NQ, 2, VHC> : (const void*)attn_decode_tc<HD, NQ, 3, VHC>;
}
// the kernel for launches of at most `vh` virtual heads
template <int HD>
static const void* tc_kernel(int vh, bool two) {
  if (vh <= 2) return tc_kernel_v<HD, 8, 2>(two);
  if (vh <= 4) return tc_kernel_v<HD, 8, 4>(two);
  if (vh <= 8) return tc_kernel_v<HD, 8, 8>(two);
  return tc_kernel_v<HD, 16, 16>(two);
}

// Launch shape of the tcgen05 decode kernel for `n_seq` sequences.
struct TcPlan {
  int splits = 1;
  bool two = false;  // two K/V stages (at most two tiles per CTA), else three
  int max_rows = 0, max_vh = 0;
};
template <int HD>
static bool tc_plan(const AttnArgs& a, int n_seq, TcPlan& p) {
  const int group = a.n_heads / a.n_kv;
  // up to 8 virtual heads per launch run the narrow form (N = 16), else N = 32
  const bool narrow = a.m * group <= 8;
  p.max_rows = (narrow ? 8 : 16) / group;
  if (p.max_rows < 1) return false;
  p.max_vh = std::min(a.m, p.max_rows) * group;
  const int cap = a.cap > 0 ? a.cap : a.pos0 + a.m;
  auto pick = [&](int splits) {  // at most two tiles per CTA: two stages, else three
    return (cap + splits - 1) / splits <= 2 * TC_C;
  };
  // one CTA per SM over (splits, kv heads, sequences); the splits of a kv
  // head meet in its last CTA or in a merge kernel behind.  (Clusters of a kv
  // head's splits merging through distributed shared memory measured slower:
  // fewer SMs, and the cluster waits for its slowest CTA at two barriers.)
  p.splits = std::max(1, std::min(a.n_splits, device_sms() / (a.n_kv * n_seq)));
  p.two = pick(p.splits);
  return true;
}

template <int HD>
static cudaError_t tc_go(const AttnArgs& a, cudaStream_t st, bool pdl, int n_seq) {
  const int group = a.n_heads / a.n_kv;
  TcPlan pl;
  if (!tc_plan<HD>(a, n_seq, pl)) return cudaErrorInvalidValue;
  const int max_rows = pl.max_rows, max_vh = pl.max_vh;
  const bool two = pl.two;
  AttnArgs aa = a;
  aa.n_splits = pl.splits;
  const void* kern = tc_kernel<HD>(max_vh, two);
  const size_t smem = two ? TcSmem<HD, 2>::bytes : TcSmem<HD, 3>::bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // split partials: merged by the kernel's last CTA when every split's o rows
  // fit its idle stages, else by attn_merge_tc behind it
  const size_t stage_bytes = TcSmem<HD, 2>::STAGE;
  aa.tail_merge = aa.n_splits > 1 && aa.n_splits <= 64 &&
                  (size_t)aa.n_splits * max_vh * HD * 4 <= (two ? 1 : 2) * stage_bytes;
  const bool merge = aa.n_splits > 1 && !aa.tail_merge;
  if (merge) {
    e = cudaFuncSetAttribute((const void*)attn_merge_tc<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)TC_MERGE_SMEM);
    if (e != cudaSuccess) return e;
  }
  for (int row0 = 0; row0 < a.m; row0 += max_rows) {
    int n_rows = min(max_rows, a.m - row0);
    void* args[] = {&aa, (void*)&row0, (void*)&n_rows};
    cudaLaunchAttribute attr[1];
    int na = 0;
    if (pdl && row0 == 0) {
      attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[na].val.programmaticStreamSerializationAllowed = 1;
      na++;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(aa.n_splits, a.n_kv, n_seq);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = na ? attr : nullptr;
    cfg.numAttrs = na;
    e = cudaLaunchKernelExC(&cfg, kern, args);
    if (e != cudaSuccess) return e;
    if (merge) {  // the merge, right behind (programmatic: it waits for the whole grid)
      const size_t vhn = (size_t)n_rows * group * aa.n_splits, w_bytes = ((vhn + 3) & ~(size_t)3) * 4;
      const size_t need = w_bytes + vhn * HD * 4;
      cudaLaunchAttribute pa[1];
      pa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      pa[0].val.programmaticStreamSerializationAllowed = 1;
      cudaLaunchConfig_t mc = {};
      mc.gridDim = dim3(a.n_kv, n_seq);
      mc.blockDim = dim3(HD);
      mc.dynamicSmemBytes = need <= TC_MERGE_SMEM ? need : w_bytes;
      mc.stream = st;
      if (pdl) {
        mc.attrs = pa;
        mc.numAttrs = 1;
      }
      e = cudaLaunchKernelExC(&mc, (const void*)attn_merge_tc<HD>, args);
      if (e != cudaSuccess) return e;
    }
  }
  return cudaSuccess;
}

cudaError_t launch_attn_decode(const AttnArgs& a, cudaStream_t st, bool pdl) {
  if (a.n_kv <= 0 || a.n_heads % a.n_kv || a.m < 1 || a.n_splits < 1) return cudaErrorInvalidValue;
  // tensor cores for the common head sizes while a kv head's query heads fit one MMA tile;
  // the cluster kernel (no global merge) when the cache has tensor maps and the clusters fit
  const bool mma = a.n_heads / a.n_kv <= AM_ROWS;
  switch (a.hd) {
    case 32: return decode_go<32, false>(a, st, pdl);
    case 48: return decode_go<48, false>(a, st, pdl);
    case 64: {
      if (!mma) return decode_go<64, false>(a, st, pdl);
      const ClusterPlan pl = a.has_tm ? cluster_plan<64>(a.n_kv, a.n_splits) : ClusterPlan{};
      return pl.c ? cluster_go<64>(a, pl, st, pdl) : decode_go<64, true>(a, st, pdl);
    }
    case 96: return decode_go<96, false>(a, st, pdl);
    case 128: {
      if (!mma) return decode_go<128, false>(a, st, pdl);
      if (a.has_tm) return tc_go<128>(a, st, pdl, 1);
      return decode_go<128, true>(a, st, pdl);
    }
    case 256: return decode_go<256, false>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_attn_decode_seqs(const AttnArgs& a, int n_seq, cudaStream_t st, bool pdl) {
  if (!a.seqs || a.m != 1 || n_seq < 1 || a.n_kv <= 0 || a.n_heads % a.n_kv || a.n_splits < 1)
    return cudaErrorInvalidValue;
  if (a.n_heads / a.n_kv > AM_ROWS || !a.has_tm || !(a.hd == 64 || a.hd == 128) || n_seq > 65535)
    return cudaErrorNotSupported;
  if (a.hd == 128) return tc_go<128>(a, st, pdl, n_seq);
  const ClusterPlan pl = cluster_plan<64>(a.n_kv, a.n_splits);
  if (!pl.c) return cudaErrorNotSupported;
  return cluster_go<64>(a, pl, st, pdl, n_seq);
}

// ---------------------------------------------------------------- tensor-core prefill attention
//
// Causal attention of the prompt rows over their own f32 K/V (attention.rs:
// 236-284) with Q.K^T and P.V on the tensor cores: mma.sync m16n8k8 TF32, each
// f32 operand split into a TF32 head and its remainder (x = hi + lo), three
// MMAs per product (lo.hi + hi.lo + hi.hi), so scores and outputs keep about
// 2^-21 relative accuracy.  A CTA owns PT_M consecutive virtual heads
// (query row x head of the group) of one kv head, 16 per warp, and walks the
// key positions up to its last row in tiles of KT (cp.async, two stages) with
// a running maximum and sum per row; the division by the sum comes last.
constexpr int PT_WARPS = 4;
constexpr int PT_M = 16 * PT_WARPS;  // virtual heads per CTA

template <int HD>
struct PtCfg {
  static constexpr int KT = HD <= 64 ? 64 : 32;  // key positions per tile
  // row pitches (floats) that make every fragment load of a warp hit 32
  // distinct banks: K, Q and P rows at 4g + t, V rows at 8t + g
  static constexpr int ROWK = HD + 4, ROWV = HD + 8, ROWQ = HD + 4, ROWP = KT + 4;
  static constexpr int STAGE = KT * (ROWK + ROWV);  // floats
  static constexpr size_t SMEM = sizeof(float) * ((size_t)2 * STAGE + (size_t)PT_M * ROWQ + (size_t)PT_M * ROWP);
};

__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  const uint32_t h = __float_as_uint(x) & 0xffffe000u;
  hi = h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(x - __uint_as_float(h)));
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// d += a.b with split operands: the two small cross terms first
__device__ __forceinline__ void mma_tf32x3(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                           const uint32_t (&bh)[2], const uint32_t (&bl)[2]) {
  mma_tf32(d, al, bh);
  mma_tf32(d, ah, bl);
  mma_tf32(d, ah, bh);
}

template <int HD>
__global__ void __launch_bounds__(PT_WARPS * 32) attn_prefill_tc(const PrefillAttnArgs a) {
  using C = PtCfg<HD>;
  constexpr int KT = C::KT, NTS = KT / 8, NTO = HD / 8, KS = HD / 8, CPR = HD / 4;
  extern __shared__ __align__(16) float pt_sm[];
  float* kv_s = pt_sm;                     // [2][K: KT x ROWK, V: KT x ROWV]
  float* q_s = kv_s + 2 * C::STAGE;        // [PT_M][ROWQ]
  float* p_s = q_s + PT_M * C::ROWQ;       // [PT_M][ROWP]
  const int group = a.n_heads / a.n_kv, kvh = blockIdx.y;
  const int VH = a.n * group;
  const int vh0 = ((int)gridDim.x - 1 - (int)blockIdx.x) * PT_M;  // the longest rows start first
  const int tid = threadIdx.x, lane = tid & 31, wi = tid >> 5, g = lane >> 2, t4 = lane & 3;
  const int q_stride = a.n_heads * HD, kv_stride = a.n_kv * HD;
  const int n_tiles = (min(VH, vh0 + PT_M) - 1) / group / KT + 1;

  auto load_tile = [&](int stage, int t0) {
    float* ks = kv_s + stage * C::STAGE;
    float* vs = ks + KT * C::ROWK;
    for (int c = tid; c < 2 * KT * CPR; c += PT_WARPS * 32) {
      const int which = c / (KT * CPR), rem = c - which * (KT * CPR), r = rem / CPR, ch = rem - r * CPR;
      const int t = t0 + r;
      float* dst = (which ? vs + r * C::ROWV : ks + r * C::ROWK) + ch * 4;
      if (t < a.n)
        cp_async16(dst, (which ? a.v : a.k) + (size_t)t * kv_stride + kvh * HD + ch * 4);
      else  // past the prompt: zeros, masked below (finite, so 0 x V stays 0)
        *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_commit();
  };
  load_tile(0, 0);
  for (int i = tid; i < PT_M * CPR; i += PT_WARPS * 32) {
    const int r = i / CPR, c = i - r * CPR, vh = vh0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (vh < VH) {
      const int row = vh / group, head = kvh * group + vh % group;
      v = *reinterpret_cast<const float4*>(a.q + (size_t)row * q_stride + head * HD + c * 4);
    }
    *reinterpret_cast<float4*>(q_s + r * C::ROWQ + c * 4) = v;
  }

  // this thread's two fragment rows: virtual heads vw + g and vw + g + 8
  const int vw = vh0 + 16 * wi;
  const int va = min(vw + g, VH - 1), vb = min(vw + g + 8, VH - 1);  // rows past the end compute, never store
  const int qa = va / group, qb = vb / group;                         // their query positions
  const int wmax = min(vw + 15, VH - 1) / group;                      // the warp's last query position
  const float scale = 1.0f / sqrtf((float)HD);
  float o[NTO][4];
#pragma unroll
  for (int n = 0; n < NTO; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  const float* qw = q_s + 16 * wi * C::ROWQ;
  float* pw = p_s + 16 * wi * C::ROWP;

  for (int it = 0; it < n_tiles; it++) {
    const int t0 = it * KT;
    if (it + 1 < n_tiles) {
      load_tile((it + 1) & 1, t0 + KT);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* ks = kv_s + (it & 1) * C::STAGE;
    const float* vs = ks + KT * C::ROWK;
    if (t0 <= wmax) {
      // ---- S = Q K^T (rows: virtual heads, columns: key positions t0 ..)
      float s[NTS][4];
#pragma unroll
      for (int n = 0; n < NTS; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll 2
      for (int kk = 0; kk < KS; kk++) {
        uint32_t ah[4], al[4];
        tf32_split(qw[g * C::ROWQ + kk * 8 + t4], ah[0], al[0]);
        tf32_split(qw[(g + 8) * C::ROWQ + kk * 8 + t4], ah[1], al[1]);
        tf32_split(qw[g * C::ROWQ + kk * 8 + t4 + 4], ah[2], al[2]);
        tf32_split(qw[(g + 8) * C::ROWQ + kk * 8 + t4 + 4], ah[3], al[3]);
#pragma unroll
        for (int n = 0; n < NTS; n++) {
          uint32_t bh[2], bl[2];
          tf32_split(ks[(n * 8 + g) * C::ROWK + kk * 8 + t4], bh[0], bl[0]);
          tf32_split(ks[(n * 8 + g) * C::ROWK + kk * 8 + t4 + 4], bh[1], bl[1]);
          mma_tf32x3(s[n], ah, al, bh, bl);
        }
      }
      // ---- scale, causal mask, running maximum (a row's four lanes agree)
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int n = 0; n < NTS; n++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
          const int tc = t0 + n * 8 + 2 * t4 + j;
          s[n][j] = tc <= qa ? __fmul_rn(s[n][j], scale) : -INFINITY;
          s[n][2 + j] = tc <= qb ? __fmul_rn(s[n][2 + j], scale) : -INFINITY;
          mx_a = fmaxf(mx_a, s[n][j]);
          mx_b = fmaxf(mx_b, s[n][2 + j]);
        }
#pragma unroll
      for (int x = 1; x <= 2; x <<= 1) {
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, x));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, x));
      }
      // key 0 is in every row's first tile, so the running maxima are finite from then on
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float al_a = m_a == -INFINITY ? 0.f : expf(m_a - mn_a);
      const float al_b = m_b == -INFINITY ? 0.f : expf(m_b - mn_b);
      m_a = mn_a;
      m_b = mn_b;
      float ls_a = 0.f, ls_b = 0.f;
#pragma unroll
      for (int n = 0; n < NTS; n++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
          const float pa = s[n][j] == -INFINITY ? 0.f : expf(s[n][j] - mn_a);
          const float pb = s[n][2 + j] == -INFINITY ? 0.f : expf(s[n][2 + j] - mn_b);
          ls_a += pa;
          ls_b += pb;
          pw[g * C::ROWP + n * 8 + 2 * t4 + j] = pa;
          pw[(g + 8) * C::ROWP + n * 8 + 2 * t4 + j] = pb;
        }
      l_a = fmaf(l_a, al_a, ls_a);
      l_b = fmaf(l_b, al_b, ls_b);
#pragma unroll
      for (int n = 0; n < NTO; n++) {
        o[n][0] *= al_a;
        o[n][1] *= al_a;
        o[n][2] *= al_b;
        o[n][3] *= al_b;
      }
      __syncwarp();
      // ---- O += P V
#pragma unroll 2
      for (int kk = 0; kk < KT / 8; kk++) {
        uint32_t ah[4], al[4];
        tf32_split(pw[g * C::ROWP + kk * 8 + t4], ah[0], al[0]);
        tf32_split(pw[(g + 8) * C::ROWP + kk * 8 + t4], ah[1], al[1]);
        tf32_split(pw[g * C::ROWP + kk * 8 + t4 + 4], ah[2], al[2]);
        tf32_split(pw[(g + 8) * C::ROWP + kk * 8 + t4 + 4], ah[3], al[3]);
#pragma unroll
        for (int n = 0; n < NTO; n++) {
          uint32_t bh[2], bl[2];
          tf32_split(vs[(kk * 8 + t4) * C::ROWV + n * 8 + g], bh[0], bl[0]);
          tf32_split(vs[(kk * 8 + t4 + 4) * C::ROWV + n * 8 + g], bh[1], bl[1]);
          mma_tf32x3(o[n], ah, al, bh, bl);
        }
      }
      __syncwarp();  // P is rewritten by the next tile
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
  }

  // ---- out = O / sum
#pragma unroll
  for (int x = 1; x <= 2; x <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, x);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, x);
  }
  const float inv_a = 1.0f / l_a, inv_b = 1.0f / l_b;
  const int ra = vw + g, rb = vw + g + 8;
  float* out_a = ra < VH ? a.out + (size_t)(ra / group) * q_stride + (kvh * group + ra % group) * HD : nullptr;
  float* out_b = rb < VH ? a.out + (size_t)(rb / group) * q_stride + (kvh * group + rb % group) * HD : nullptr;
#pragma unroll
  for (int n = 0; n < NTO; n++) {
    const int d = n * 8 + 2 * t4;
    if (out_a) *reinterpret_cast<float2*>(out_a + d) = make_float2(o[n][0] * inv_a, o[n][1] * inv_a);
    if (out_b) *reinterpret_cast<float2*>(out_b + d) = make_float2(o[n][2] * inv_b, o[n][3] * inv_b);
  }
}

template <int HD>
static cudaError_t prefill_tc_go(const PrefillAttnArgs& a, cudaStream_t st) {
  using C = PtCfg<HD>;
  auto k = attn_prefill_tc<HD>;
  const cudaError_t e = cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
  if (e != cudaSuccess) return e;
  const long long vh = (long long)a.n * (a.n_heads / a.n_kv);
  k<<<dim3((unsigned)((vh + PT_M - 1) / PT_M), a.n_kv), PT_WARPS * 32, C::SMEM, st>>>(a);
  return cudaGetLastError();
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
  // f32 K/V rows are read with 16-byte copies
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
       reinterpret_cast<uintptr_t>(a.out)) & 15)
    return cudaErrorInvalidValue;
  switch (a.hd) {  // tensor cores up to head dim 128; the CUDA-core kernel beyond
    case 32: return prefill_tc_go<32>(a, st);
    case 48: return prefill_tc_go<48>(a, st);
    case 64: return prefill_tc_go<64>(a, st);
    case 96: return prefill_tc_go<96>(a, st);
    case 128: return prefill_tc_go<128>(a, st);
    case 256: return prefill_go<256>(a, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace prana
