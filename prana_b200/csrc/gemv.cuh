// gemv.cuh -- the quantized GEMV core: one warp streams whole weight rows with
// 128-bit loads, dequantizes in registers and accumulates int8 x int8 block
// dots with dp4a against activations staged in shared memory.
//
// Work unit per lane (a "unit"):
//   Q8_0: one 32-weight block (32 B int8 + f16 d)
//   Q4_0: one 32-weight block (16 B nibbles + f16 d)
//   Q4_K: one 64-weight pair of a super-block (32 B nibbles + the super-block's 16 B header)
//   Q6_K: one 64-weight quarter of a super-block (16 B low nibbles x2 + 16 B high bits + scales)
// Lanes take consecutive units, so a warp reads a contiguous stretch of the row.
//
// The per-block integer dots are exactly the reference's:
//   Q8_0 Σ qa·qw (matmul.rs:395-406), Q4_0 Σ qa·q − 8·Σqa (kquant.rs:240-252),
//   Q4_K Σ qa·nibble per 32-group (kquant.rs:257-282), Q6_K Σ qa·(q6−32) per
//   16-element sub-block (kquant.rs:287-318); only the f32 sum order differs.
#pragma once
#include "common.cuh"

namespace prana {

// Activations of up to M rows staged in shared memory.
struct Acts {
  const int8_t* q;    // [M][K]
  const float* s;     // [M][G]
  const int32_t* sum; // [M][G]
  int K, G;
};

__host__ __device__ inline int units_per_row(int type, int cols) {
  return (type == T_Q4_K || type == T_Q6_K) ? cols / 64 : cols / 32;
}

// Bulk-prefetch the bytes of rows [r0, r0 + R) of every plane toward L2.
// Ranges are widened to 16-byte boundaries; planes are 256-byte padded, so the
// widened range stays inside the allocation.
__device__ __forceinline__ void prefetch_span(const void* base, size_t off, size_t bytes) {
  const uintptr_t a = (reinterpret_cast<uintptr_t>(base) + off) & ~(uintptr_t)15;
  const uintptr_t e = (reinterpret_cast<uintptr_t>(base) + off + bytes + 15) & ~(uintptr_t)15;
  if (e > a) prefetch_l2_bulk(reinterpret_cast<const void*>(a), (uint32_t)(e - a));
}
__device__ __forceinline__ void prefetch_rows(const DevWeight& w, int r0, int R) {
  if (r0 >= w.rows) return;
  if (r0 + R > w.rows) R = w.rows - r0;
  const size_t K = (size_t)w.cols;
  switch (w.type) {
    case T_Q8_0:
      prefetch_span(w.qs, r0 * K, R * K);
      prefetch_span(w.d, r0 * K / 16, R * K / 16);
      break;
    case T_Q8S:
      prefetch_span(w.qs, r0 * K, R * K);
      prefetch_span(w.ds, r0 * K / 8, R * K / 8);
      break;
    case T_Q4_0:
      prefetch_span(w.qs, r0 * K / 2, R * K / 2);
      prefetch_span(w.d, r0 * K / 16, R * K / 16);
      break;
    case T_Q4_K:
      prefetch_span(w.qs, r0 * (K / 256) * 144, R * (K / 256) * 144);
      break;
    case T_Q6_K:
      prefetch_span(w.qs, r0 * K / 2, R * K / 2);
      prefetch_span(w.qh, r0 * K / 4, R * K / 4);
      prefetch_span(w.sc, r0 * K / 16, R * K / 16);
      prefetch_span(w.d, r0 * K / 128, R * K / 128);
      break;
  }
}

template <int T> struct Unit;
template <> struct Unit<T_Q8_0> { uint4 a, b; unsigned short d; };
template <> struct Unit<T_Q8S> { uint4 a, b; float d; };
template <> struct Unit<T_Q4_0> { uint4 q; unsigned short d; };
template <> struct Unit<T_Q4_K> { uint4 a, b, meta; };
template <> struct Unit<T_Q6_K> { uint4 lo, hi, qh; uint2 sc; unsigned short d; };

template <int T> __device__ __forceinline__ Unit<T> load_unit(const DevWeight& w, int row, int u);

template <> __device__ __forceinline__ Unit<T_Q8_0> load_unit<T_Q8_0>(const DevWeight& w, int row, int u) {
  Unit<T_Q8_0> x;
  const uint8_t* p = w.qs + (size_t)row * w.cols + (size_t)u * 32;
  x.a = ld_stream16(p);
  x.b = ld_stream16(p + 16);
  x.d = ld_stream_u16(w.d + (size_t)row * (w.cols / 32) + u);
  return x;
}
template <> __device__ __forceinline__ Unit<T_Q8S> load_unit<T_Q8S>(const DevWeight& w, int row, int u) {
  Unit<T_Q8S> x;
  const uint8_t* p = w.qs + (size_t)row * w.cols + (size_t)u * 32;
  x.a = ld_stream16(p);
  x.b = ld_stream16(p + 16);
  x.d = __ldg(w.ds + (size_t)row * (w.cols / 32) + u);
  return x;
}
template <> __device__ __forceinline__ Unit<T_Q4_0> load_unit<T_Q4_0>(const DevWeight& w, int row, int u) {
  Unit<T_Q4_0> x;
  x.q = ld_stream16(w.qs + (size_t)row * (w.cols / 2) + (size_t)u * 16);
  x.d = ld_stream_u16(w.d + (size_t)row * (w.cols / 32) + u);
  return x;
}
template <> __device__ __forceinline__ Unit<T_Q4_K> load_unit<T_Q4_K>(const DevWeight& w, int row, int u) {
  Unit<T_Q4_K> x;
  const uint8_t* sb = w.qs + (size_t)row * (w.cols / 256) * 144 + (size_t)(u >> 2) * 144;
  x.a = ld_stream16(sb + 16 + (u & 3) * 32);
  x.b = ld_stream16(sb + 32 + (u & 3) * 32);
  x.meta = ld_stream16(sb);
  return x;
}
template <> __device__ __forceinline__ Unit<T_Q6_K> load_unit<T_Q6_K>(const DevWeight& w, int row, int u) {
  Unit<T_Q6_K> x;
  const int b = u >> 2, h = (u >> 1) & 1, l0 = (u & 1) * 16;
  const uint8_t* ql = w.qs + (size_t)row * (w.cols / 2) + (size_t)b * 128 + h * 64 + l0;
  x.lo = ld_stream16(ql);
  x.hi = ld_stream16(ql + 32);
  x.qh = ld_stream16(w.qh + (size_t)row * (w.cols / 4) + (size_t)b * 64 + h * 32 + l0);
  x.sc = ld_stream8(w.sc + (size_t)row * (w.cols / 16) + (size_t)b * 16 + h * 8);
  x.d = ld_stream_u16(w.d + (size_t)row * (w.cols / 256) + b);
  return x;
}

__device__ __forceinline__ int dp4(unsigned a, int b, int c) { return __dp4a((int)a, b, c); }

// ---- per-unit integer dots (exact) ----
template <class U>
__device__ __forceinline__ int idot_q8(const U& x, const int8_t* a) {
  const int4 a0 = *reinterpret_cast<const int4*>(a), a1 = *reinterpret_cast<const int4*>(a + 16);
  int s = dp4(x.a.x, a0.x, 0);
  s = dp4(x.a.y, a0.y, s); s = dp4(x.a.z, a0.z, s); s = dp4(x.a.w, a0.w, s);
  s = dp4(x.b.x, a1.x, s); s = dp4(x.b.y, a1.y, s); s = dp4(x.b.z, a1.z, s); s = dp4(x.b.w, a1.w, s);
  return s;
}
// Σ qa·q with raw nibbles (0..15); caller subtracts 8·Σqa.
__device__ __forceinline__ int idot_q4_0(const Unit<T_Q4_0>& x, const int8_t* a) {
  const int4 a0 = *reinterpret_cast<const int4*>(a), a1 = *reinterpret_cast<const int4*>(a + 16);
  const unsigned m = 0x0F0F0F0Fu;
  int s = dp4(x.q.x & m, a0.x, 0);
  s = dp4(x.q.y & m, a0.y, s); s = dp4(x.q.z & m, a0.z, s); s = dp4(x.q.w & m, a0.w, s);
  s = dp4((x.q.x >> 4) & m, a1.x, s); s = dp4((x.q.y >> 4) & m, a1.y, s);
  s = dp4((x.q.z >> 4) & m, a1.z, s); s = dp4((x.q.w >> 4) & m, a1.w, s);
  return s;
}
// Q4_K pair: s1 = Σ a_lo·(q & 0xF), s2 = Σ a_hi·(q >> 4) over the pair's 32 bytes.
__device__ __forceinline__ void idot_q4_k(const Unit<T_Q4_K>& x, const int8_t* a, int& s1, int& s2) {
  const unsigned m = 0x0F0F0F0Fu;
  const int4 l0 = *reinterpret_cast<const int4*>(a), l1 = *reinterpret_cast<const int4*>(a + 16);
  const int4 h0 = *reinterpret_cast<const int4*>(a + 32), h1 = *reinterpret_cast<const int4*>(a + 48);
  int s = dp4(x.a.x & m, l0.x, 0);
  s = dp4(x.a.y & m, l0.y, s); s = dp4(x.a.z & m, l0.z, s); s = dp4(x.a.w & m, l0.w, s);
  s = dp4(x.b.x & m, l1.x, s); s = dp4(x.b.y & m, l1.y, s); s = dp4(x.b.z & m, l1.z, s); s = dp4(x.b.w & m, l1.w, s);
  int t = dp4((x.a.x >> 4) & m, h0.x, 0);
  t = dp4((x.a.y >> 4) & m, h0.y, t); t = dp4((x.a.z >> 4) & m, h0.z, t); t = dp4((x.a.w >> 4) & m, h0.w, t);
  t = dp4((x.b.x >> 4) & m, h1.x, t); t = dp4((x.b.y >> 4) & m, h1.y, t);
  t = dp4((x.b.z >> 4) & m, h1.z, t); t = dp4((x.b.w >> 4) & m, h1.w, t);
  s1 = s;
  s2 = t;
}
// Q4_K (scale, min) pair j from the 12 packed bytes (kquant.rs:52-61).
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* s, int& sc, int& mn) {
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}
// Q4_K (scale, min) of sub-blocks 2p and 2p + 1 (kquant.rs:52-61) taken from
// the header's packed words y = bytes 0-3, z = 4-7, w = 8-11 with shifts, so
// the twelve bytes never go through a local array (p differs per lane).
__device__ __forceinline__ void q4k_pair_scales(int p, const uint4& meta, int& sc1, int& m1, int& sc2, int& m2) {
  const int sh = 8 * ((2 * p) & 3);
  const unsigned y = meta.y >> sh, z = meta.z >> sh, w = meta.w >> sh;
  const bool hi = p >= 2;
  sc1 = hi ? (int)((w & 0xFu) | (((y >> 6) & 3u) << 4)) : (int)(y & 63u);
  m1 = hi ? (int)(((w >> 4) & 0xFu) | (((z >> 6) & 3u) << 4)) : (int)(z & 63u);
  sc2 = hi ? (int)(((w >> 8) & 0xFu) | (((y >> 14) & 3u) << 4)) : (int)((y >> 8) & 63u);
  m2 = hi ? (int)(((w >> 12) & 0xFu) | (((z >> 14) & 3u) << 4)) : (int)((z >> 8) & 63u);
}
// Q6_K quarter: per-group (g = 0..3) sums over 16 elements of (q6 − 32)·qa.
__device__ __forceinline__ void q6_words(unsigned lo, unsigned hi, unsigned qh, unsigned q[4]) {
  const unsigned m4 = 0x0F0F0F0Fu, m2 = 0x03030303u;
  q[0] = __vsub4((lo & m4) | ((qh & m2) << 4), 0x20202020u);
  q[1] = __vsub4((hi & m4) | (((qh >> 2) & m2) << 4), 0x20202020u);
  q[2] = __vsub4(((lo >> 4) & m4) | (((qh >> 4) & m2) << 4), 0x20202020u);
  q[3] = __vsub4(((hi >> 4) & m4) | (((qh >> 6) & m2) << 4), 0x20202020u);
}
__device__ __forceinline__ void idot_q6_k(const Unit<T_Q6_K>& x, const int8_t* a /* block base + h*128 + l0 */,
                                          int s[4]) {
  const unsigned lo[4] = {x.lo.x, x.lo.y, x.lo.z, x.lo.w}, hi[4] = {x.hi.x, x.hi.y, x.hi.z, x.hi.w},
                 qh[4] = {x.qh.x, x.qh.y, x.qh.z, x.qh.w};
  int4 av[4];
#pragma unroll
  for (int g = 0; g < 4; g++) av[g] = *reinterpret_cast<const int4*>(a + g * 32);
  s[0] = s[1] = s[2] = s[3] = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    unsigned q[4];
    q6_words(lo[k], hi[k], qh[k], q);
#pragma unroll
    for (int g = 0; g < 4; g++) {
      const int aw = k == 0 ? av[g].x : (k == 1 ? av[g].y : (k == 2 ? av[g].z : av[g].w));
      s[g] = dp4(q[g], aw, s[g]);
    }
  }
}

// ---- per-unit float accumulation for M activation rows ----
template <int T, int M>
__device__ __forceinline__ void accum_unit(const Unit<T>& x, int u, const Acts& a, int m_rt, float (&acc)[M]);

template <int M>
__device__ __forceinline__ void accum_unit(const Unit<T_Q8_0>& x, int u, const Acts& a, int m_rt, float (&acc)[M]) {
  const float d = h2f(x.d);
#pragma unroll
  for (int m = 0; m < M; m++)
    if (m < m_rt) {
      const int s = idot_q8(x, a.q + m * a.K + u * 32);
      acc[m] = fmaf(__fmul_rn(d, a.s[m * a.G + u]), (float)s, acc[m]);
    }
}
template <int M>
__device__ __forceinline__ void accum_unit(const Unit<T_Q8S>& x, int u, const Acts& a, int m_rt, float (&acc)[M]) {
#pragma unroll
  for (int m = 0; m < M; m++)
    if (m < m_rt) {
      const int s = idot_q8(x, a.q + m * a.K + u * 32);
      acc[m] = fmaf(__fmul_rn(x.d, a.s[m * a.G + u]), (float)s, acc[m]);
    }
}
template <int M>
__device__ __forceinline__ void accum_unit(const Unit<T_Q4_0>& x, int u, const Acts& a, int m_rt, float (&acc)[M]) {
  const float d = h2f(x.d);
#pragma unroll
  for (int m = 0; m < M; m++)
    if (m < m_rt) {
      const int s = idot_q4_0(x, a.q + m * a.K + u * 32) - 8 * a.sum[m * a.G + u];
      acc[m] = fmaf(__fmul_rn(d, a.s[m * a.G + u]), (float)s, acc[m]);
    }
}
template <int M>
__device__ __forceinline__ void accum_unit(const Unit<T_Q4_K>& x, int u, const Acts& a, int m_rt, float (&acc)[M]) {
  const float d = h2f((unsigned short)(x.meta.x & 0xffffu)), dmin = h2f((unsigned short)(x.meta.x >> 16));
  const int p = u & 3;
  int sc1, m1, sc2, m2;
  q4k_pair_scales(p, x.meta, sc1, m1, sc2, m2);
  const float dsc1 = __fmul_rn(d, (float)sc1), dm1 = __fmul_rn(dmin, (float)m1);
  const float dsc2 = __fmul_rn(d, (float)sc2), dm2 = __fmul_rn(dmin, (float)m2);
  const int g_lo = (u >> 2) * 8 + 2 * p;
#pragma unroll
  for (int m = 0; m < M; m++)
    if (m < m_rt) {
      int s1, s2;
      idot_q4_k(x, a.q + m * a.K + g_lo * 32, s1, s2);
      const float t1 = __fsub_rn(__fmul_rn(dsc1, (float)s1), __fmul_rn(dm1, (float)a.sum[m * a.G + g_lo]));
      const float t2 = __fsub_rn(__fmul_rn(dsc2, (float)s2), __fmul_rn(dm2, (float)a.sum[m * a.G + g_lo + 1]));
      acc[m] = fmaf(a.s[m * a.G + g_lo], t1, acc[m]);
      acc[m] = fmaf(a.s[m * a.G + g_lo + 1], t2, acc[m]);
    }
}
template <int M>
__device__ __forceinline__ void accum_unit(const Unit<T_Q6_K>& x, int u, const Acts& a, int m_rt, float (&acc)[M]) {
  const float d = h2f(x.d);
  const int b = u >> 2, h = (u >> 1) & 1, half16 = u & 1;
  float scf[4];  // sub-block scales of this quarter: int8 at byte 2g + half16 of x.sc
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const unsigned word = g < 2 ? x.sc.x : x.sc.y;
    scf[g] = (float)(int)(int8_t)((word >> (8 * ((g * 2 + half16) & 3))) & 0xffu);
  }
#pragma unroll
  for (int m = 0; m < M; m++)
    if (m < m_rt) {
      int s[4];
      idot_q6_k(x, a.q + m * a.K + b * 256 + h * 128 + half16 * 16, s);
#pragma unroll
      for (int g = 0; g < 4; g++) {
        const float sa = a.s[m * a.G + b * 8 + h * 4 + g];
        acc[m] = fmaf(__fmul_rn(__fmul_rn(d, sa), scf[g]), (float)s[g], acc[m]);
      }
    }
}

// ---- one activation row held in registers (the batch-1 decode path) ----
// A lane loads the activation data of its unit once per chunk and reuses it
// for every weight row the warp streams; the arithmetic is accum_unit's with
// a single activation row, operation for operation.
template <int T> struct ActU;
template <> struct ActU<T_Q8_0> { int4 a0, a1; float s; };
template <> struct ActU<T_Q8S> { int4 a0, a1; float s; };
template <> struct ActU<T_Q4_0> { int4 a0, a1; float s; int sum8; };
template <> struct ActU<T_Q4_K> { int4 l0, l1, h0, h1; float s1, s2; int sum1, sum2; };
template <> struct ActU<T_Q6_K> { int4 a[4]; float s[4]; };

template <int T> __device__ __forceinline__ ActU<T> load_act(const Acts& a, int u);
template <> __device__ __forceinline__ ActU<T_Q8_0> load_act<T_Q8_0>(const Acts& a, int u) {
  ActU<T_Q8_0> r;
  r.a0 = *reinterpret_cast<const int4*>(a.q + u * 32);
  r.a1 = *reinterpret_cast<const int4*>(a.q + u * 32 + 16);
  r.s = a.s[u];
  return r;
}
template <> __device__ __forceinline__ ActU<T_Q8S> load_act<T_Q8S>(const Acts& a, int u) {
  ActU<T_Q8S> r;
  r.a0 = *reinterpret_cast<const int4*>(a.q + u * 32);
  r.a1 = *reinterpret_cast<const int4*>(a.q + u * 32 + 16);
  r.s = a.s[u];
  return r;
}
template <> __device__ __forceinline__ ActU<T_Q4_0> load_act<T_Q4_0>(const Acts& a, int u) {
  ActU<T_Q4_0> r;
  r.a0 = *reinterpret_cast<const int4*>(a.q + u * 32);
  r.a1 = *reinterpret_cast<const int4*>(a.q + u * 32 + 16);
  r.s = a.s[u];
  r.sum8 = 8 * a.sum[u];
  return r;
}
template <> __device__ __forceinline__ ActU<T_Q4_K> load_act<T_Q4_K>(const Acts& a, int u) {
  ActU<T_Q4_K> r;
  const int g_lo = (u >> 2) * 8 + 2 * (u & 3);
  const int8_t* q = a.q + g_lo * 32;
  r.l0 = *reinterpret_cast<const int4*>(q);
  r.l1 = *reinterpret_cast<const int4*>(q + 16);
  r.h0 = *reinterpret_cast<const int4*>(q + 32);
  r.h1 = *reinterpret_cast<const int4*>(q + 48);
  r.s1 = a.s[g_lo];
  r.s2 = a.s[g_lo + 1];
  r.sum1 = a.sum[g_lo];
  r.sum2 = a.sum[g_lo + 1];
  return r;
}
template <> __device__ __forceinline__ ActU<T_Q6_K> load_act<T_Q6_K>(const Acts& a, int u) {
  ActU<T_Q6_K> r;
  const int b = u >> 2, h = (u >> 1) & 1, half16 = u & 1;
  const int8_t* q = a.q + b * 256 + h * 128 + half16 * 16;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    r.a[g] = *reinterpret_cast<const int4*>(q + g * 32);
    r.s[g] = a.s[b * 8 + h * 4 + g];
  }
  return r;
}

__device__ __forceinline__ void accum_r(const Unit<T_Q8_0>& x, const ActU<T_Q8_0>& a, int, float& acc) {
  int s = dp4(x.a.x, a.a0.x, 0);
  s = dp4(x.a.y, a.a0.y, s); s = dp4(x.a.z, a.a0.z, s); s = dp4(x.a.w, a.a0.w, s);
  s = dp4(x.b.x, a.a1.x, s); s = dp4(x.b.y, a.a1.y, s); s = dp4(x.b.z, a.a1.z, s); s = dp4(x.b.w, a.a1.w, s);
  acc = fmaf(__fmul_rn(h2f(x.d), a.s), (float)s, acc);
}
__device__ __forceinline__ void accum_r(const Unit<T_Q8S>& x, const ActU<T_Q8S>& a, int, float& acc) {
  int s = dp4(x.a.x, a.a0.x, 0);
  s = dp4(x.a.y, a.a0.y, s); s = dp4(x.a.z, a.a0.z, s); s = dp4(x.a.w, a.a0.w, s);
  s = dp4(x.b.x, a.a1.x, s); s = dp4(x.b.y, a.a1.y, s); s = dp4(x.b.z, a.a1.z, s); s = dp4(x.b.w, a.a1.w, s);
  acc = fmaf(__fmul_rn(x.d, a.s), (float)s, acc);
}
__device__ __forceinline__ void accum_r(const Unit<T_Q4_0>& x, const ActU<T_Q4_0>& a, int, float& acc) {
  const unsigned m = 0x0F0F0F0Fu;
  int s = dp4(x.q.x & m, a.a0.x, 0);
  s = dp4(x.q.y & m, a.a0.y, s); s = dp4(x.q.z & m, a.a0.z, s); s = dp4(x.q.w & m, a.a0.w, s);
  s = dp4((x.q.x >> 4) & m, a.a1.x, s); s = dp4((x.q.y >> 4) & m, a.a1.y, s);
  s = dp4((x.q.z >> 4) & m, a.a1.z, s); s = dp4((x.q.w >> 4) & m, a.a1.w, s);
  acc = fmaf(__fmul_rn(h2f(x.d), a.s), (float)(s - a.sum8), acc);
}
__device__ __forceinline__ void accum_r(const Unit<T_Q4_K>& x, const ActU<T_Q4_K>& a, int u, float& acc) {
  const float d = h2f((unsigned short)(x.meta.x & 0xffffu)), dmin = h2f((unsigned short)(x.meta.x >> 16));
  const int p = u & 3;
  int sc1, m1, sc2, m2;
  q4k_pair_scales(p, x.meta, sc1, m1, sc2, m2);
  const float dsc1 = __fmul_rn(d, (float)sc1), dm1 = __fmul_rn(dmin, (float)m1);
  const float dsc2 = __fmul_rn(d, (float)sc2), dm2 = __fmul_rn(dmin, (float)m2);
  const unsigned m = 0x0F0F0F0Fu;
  int s1 = dp4(x.a.x & m, a.l0.x, 0);
  s1 = dp4(x.a.y & m, a.l0.y, s1); s1 = dp4(x.a.z & m, a.l0.z, s1); s1 = dp4(x.a.w & m, a.l0.w, s1);
  s1 = dp4(x.b.x & m, a.l1.x, s1); s1 = dp4(x.b.y & m, a.l1.y, s1); s1 = dp4(x.b.z & m, a.l1.z, s1);
  s1 = dp4(x.b.w & m, a.l1.w, s1);
  int s2 = dp4((x.a.x >> 4) & m, a.h0.x, 0);
  s2 = dp4((x.a.y >> 4) & m, a.h0.y, s2); s2 = dp4((x.a.z >> 4) & m, a.h0.z, s2); s2 = dp4((x.a.w >> 4) & m, a.h0.w, s2);
  s2 = dp4((x.b.x >> 4) & m, a.h1.x, s2); s2 = dp4((x.b.y >> 4) & m, a.h1.y, s2);
  s2 = dp4((x.b.z >> 4) & m, a.h1.z, s2); s2 = dp4((x.b.w >> 4) & m, a.h1.w, s2);
  const float t1 = __fsub_rn(__fmul_rn(dsc1, (float)s1), __fmul_rn(dm1, (float)a.sum1));
  const float t2 = __fsub_rn(__fmul_rn(dsc2, (float)s2), __fmul_rn(dm2, (float)a.sum2));
  acc = fmaf(a.s1, t1, acc);
  acc = fmaf(a.s2, t2, acc);
}
__device__ __forceinline__ void accum_r(const Unit<T_Q6_K>& x, const ActU<T_Q6_K>& a, int u, float& acc) {
  const float d = h2f(x.d);
  const int half16 = u & 1;
  const unsigned lo[4] = {x.lo.x, x.lo.y, x.lo.z, x.lo.w}, hi[4] = {x.hi.x, x.hi.y, x.hi.z, x.hi.w},
                 qh[4] = {x.qh.x, x.qh.y, x.qh.z, x.qh.w};
  int s[4] = {0, 0, 0, 0};
#pragma unroll
  for (int k = 0; k < 4; k++) {
    unsigned q[4];
    q6_words(lo[k], hi[k], qh[k], q);
#pragma unroll
    for (int g = 0; g < 4; g++) {
      const int aw = k == 0 ? a.a[g].x : (k == 1 ? a.a[g].y : (k == 2 ? a.a[g].z : a.a[g].w));
      s[g] = dp4(q[g], aw, s[g]);
    }
  }
  // sub-block scales of this quarter: int8 at byte 2g + half16 of x.sc
#pragma unroll
  for (int g = 0; g < 4; g++) {
    const unsigned word = g < 2 ? x.sc.x : x.sc.y;
    const int sc = (int)(int8_t)((word >> (8 * ((g * 2 + half16) & 3))) & 0xffu);
    acc = fmaf(__fmul_rn(__fmul_rn(d, a.s[g]), (float)sc), (float)s[g], acc);
  }
}

// Warp computes NR rows (rows[r] < 0 = idle) x up to M activation rows.
// UNR units per lane are loaded before any is consumed, so NR*UNR 128-bit
// loads per lane are in flight.
template <int T, int NR, int M, int UNR>
__device__ __forceinline__ void warp_dot(const DevWeight& w, const int (&rows)[NR], const Acts& a, int m_rt,
                                         float (&acc)[NR][M]) {
  const int lane = threadIdx.x & 31;
  const int nu = units_per_row(T, w.cols);
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int m = 0; m < M; m++) acc[r][m] = 0.0f;
  for (int u0 = 0; u0 < nu; u0 += 32 * UNR) {
    Unit<T> buf[NR][UNR];
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
      for (int j = 0; j < UNR; j++) {
        const int u = u0 + j * 32 + lane;
        if (u < nu && rows[r] >= 0) buf[r][j] = load_unit<T>(w, rows[r], u);
      }
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
      for (int j = 0; j < UNR; j++) {
        const int u = u0 + j * 32 + lane;
        if (u < nu && rows[r] >= 0) accum_unit<M>(buf[r][j], u, a, m_rt, acc[r]);
      }
  }
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int m = 0; m < M; m++) acc[r][m] = warp_sum(acc[r][m]);
}

// Element i of token row `tok` of an embedding table, dequantized exactly like
// the CPU tables (checkpoint.rs:169-174; kquant.rs:39-112 for packed formats;
// Q8_0 tables are f32 `q * d` in gguf.rs:238-247).
__device__ __forceinline__ float embed_value(const DevWeight& w, uint32_t tok, int i) {
  const int dim = w.cols;
  const size_t r = tok;
  switch (w.type) {
    case T_Q8_0:
      return __fmul_rn((float)(int8_t)w.qs[r * dim + i], h2f(__half_as_ushort(w.d[r * (dim / 32) + i / 32])));
    case T_Q4_0: {
      const int b = i / 32, e = i % 32;
      const uint8_t byte = w.qs[r * (dim / 2) + b * 16 + (e & 15)];
      const int q = e < 16 ? (byte & 0xF) : (byte >> 4);
      return __fmul_rn(h2f(__half_as_ushort(w.d[r * (dim / 32) + b])), __fsub_rn((float)q, 8.0f));
    }
    case T_Q4_K: {
      const uint8_t* sb = w.qs + r * (dim / 256) * 144 + (size_t)(i / 256) * 144;
      const int e = i % 256, pair = e / 64, hi = (e % 64) / 32, l = e % 32;
      int sc, mn;
      q4k_scale_min(pair * 2 + hi, sb + 4, sc, mn);
      const float d = h2f((unsigned short)(sb[0] | (sb[1] << 8))), dmin = h2f((unsigned short)(sb[2] | (sb[3] << 8)));
      const uint8_t byte = sb[16 + pair * 32 + l];
      const int q = hi ? (byte >> 4) : (byte & 0xF);
      return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)mn));
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
      return __fmul_rn(__fmul_rn(d, (float)sc[h * 8 + l / 16 + 2 * g]), (float)q);
    }
    default:
      return w.f32[r * dim + i];
  }
}

// Per-block integer dots of one row (debug/parity entry): one value per
// 32-group (Q8_0, Q4_0, Q4_K) or per 16-element sub-block (Q6_K).
template <int T>
__device__ __forceinline__ void unit_block_dots(const DevWeight& w, int row, int u, const Acts& a, int32_t* out) {
  Unit<T> x = load_unit<T>(w, row, u);
  if constexpr (T == T_Q8_0 || T == T_Q8S) {
    out[u] = idot_q8(x, a.q + u * 32);
  } else if constexpr (T == T_Q4_0) {
    out[u] = idot_q4_0(x, a.q + u * 32) - 8 * a.sum[u];
  } else if constexpr (T == T_Q4_K) {
    int s1, s2;
    const int g_lo = (u >> 2) * 8 + 2 * (u & 3);
    idot_q4_k(x, a.q + g_lo * 32, s1, s2);
    out[g_lo] = s1;
    out[g_lo + 1] = s2;
  } else {
    const int b = u >> 2, h = (u >> 1) & 1, half16 = u & 1;
    int s[4];
    idot_q6_k(x, a.q + b * 256 + h * 128 + half16 * 16, s);
    for (int g = 0; g < 4; g++) out[b * 16 + h * 8 + g * 2 + half16] = s[g];
  }
}

}  // namespace prana
