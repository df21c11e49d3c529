// qgemm.cu -- block-scaled int8 GEMM on the 5th-generation tensor cores for
// the dense cases of the decode path: prefill, the (k+1)-row speculative
// verify pass and batches of independent sequences
// (matmul_q8_prefill, matmul.rs:185-232; matmul_kquant_prefill,
// kquant.rs:368-370).
//
//   out[t][r] = sum over blocks b of  scale(r, t, b) * dot_b(W[r], a[t])
//
// dot_b is the integer dot of one 32-value block (16 for Q6_K's sub-blocks)
// of weight row r with activation row t: exactly the reference's per-block
// int32 (matmul.rs:395-406, kquant.rs:240-318).  Each block is its own
// tcgen05.mma.kind::i8 (K = 32) into a fresh TMEM accumulator, so the tensor
// core produces exactly those integers; the epilogue applies the per-block
// scales in f32, operation for operation as the CPU path does (only the
// order of the f32 sum over blocks differs).
//
// CTA tile: 128 weight rows (the MMA's M) x NT tokens (its N); K in stages
// of BK values.  Warp roles (14 warps):
//   warps 0-3   producers: one weight row per thread; unpack the stage's
//               packed blocks (staged by TMA) into int8 in the 128-byte
//               swizzled K-major layout the MMA reads (Q8_0 needs none:
//               TMA writes that layout itself)
//   warps 4-11  epilogue: warp w owns TMEM lanes 32*(w%4).. (32 weight
//               rows); the two warps of a lane quarter split the tokens.
//               Per block: tcgen05.ld the int32 dots, release the slot,
//               scale and accumulate in registers
//   warp 12     TMEM allocation; lane 0 issues the MMAs
//   warp 13     lane 0 issues the TMA copies of each stage: activations,
//               their per-block scales (and group sums), packed weights
//
// Q6_K's 16-value sub-blocks carry their own scales, so its 32-blocks are
// two MMAs over the same activations: one with the upper 16 weights of every
// block zeroed, one with the lower 16 zeroed.
//
// A stage is refilled once its MMAs completed (tcgen05.commit) and the
// epilogue finished with its staged scales.  Every mbarrier wait is bounded
// and also gives up when another role has given up; the CTA then waits
// (bounded) for its own copies and MMAs, frees its TMEM and raises the error
// flag.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <map>
#include <mutex>

#include "gemv.cuh"
#include "host.h"
#include "internal.h"
#include "mbar.cuh"
#include "tc.cuh"

namespace prana {

namespace {

constexpr int QG_BM = 128;         // weight rows per CTA (MMA M)
constexpr int QG_PRODUCERS = 128;  // warps 0-3
constexpr int QG_SMEM_MAX = 224 * 1024;

template <int T> struct QgFmt;
// BK: K values per stage; RAW: packed bytes per weight row per stage, staged
// by TMA (0: TMA writes the int8 tile itself); A_TILES: int8 tiles per stage
// (2 for Q6_K: lower and upper sub-block halves).  Q6_K's raw row is its ql
// bytes (128) then its qh bytes (64), staged as two regions.
template <> struct QgFmt<T_Q8_0> { static constexpr int BK = 256, RAW = 0, A_TILES = 1; };
template <> struct QgFmt<T_Q8S> { static constexpr int BK = 256, RAW = 0, A_TILES = 1; };
template <> struct QgFmt<T_Q4_0> { static constexpr int BK = 256, RAW = 128, A_TILES = 1; };
template <> struct QgFmt<T_Q4_K> { static constexpr int BK = 256, RAW = 144, A_TILES = 1; };
template <> struct QgFmt<T_Q6_K> { static constexpr int BK = 256, RAW = 192, A_TILES = 2; };

template <int T, int NT>
struct QgLayout {
  using F = QgFmt<T>;
  static constexpr int BK = F::BK;
  static constexpr int BLK = BK / 32;                       // 32-value blocks per stage
  static constexpr int KATOMS = BK / 128;                   // 128-byte swizzle atoms along K
  static constexpr int A_ATOM = QG_BM * 128;                // bytes of one atom of one tile
  static constexpr int A_BYTES = A_ATOM * KATOMS * F::A_TILES;
  static constexpr int B_BYTES = NT * BK;
  static constexpr int RAW_BYTES = QG_BM * F::RAW;
  static constexpr int SA_BYTES = BLK * NT * 4;             // activation scales [BLK][NT]
  static constexpr int SUM_BYTES = T == T_Q4_K ? BLK * NT * 4 : 0;  // activation group sums
  static constexpr int OFF_B = A_BYTES;
  static constexpr int OFF_RAW = OFF_B + B_BYTES;
  static constexpr int OFF_SA = OFF_RAW + RAW_BYTES;
  static constexpr int OFF_SUM = OFF_SA + SA_BYTES;
  static constexpr int STAGE = (OFF_SUM + SUM_BYTES + 1023) / 1024 * 1024;
  static constexpr int NS_FIT = (QG_SMEM_MAX - 2048) / STAGE;
  static constexpr int NS = NS_FIT > 6 ? 6 : NS_FIT;        // pipeline stages
  static_assert(NS >= 2, "stage too large");
  static constexpr int MPB = F::A_TILES;                    // MMAs per 32-value block
  static constexpr int SLOTS_MAX = 512 / NT;
  static constexpr int SLOTS = SLOTS_MAX > 16 ? 16 : SLOTS_MAX;  // TMEM accumulator slots (one MMA each)
  // MMAs are committed, waited on and released in groups of GS slots (a
  // group never spans two stages); NG groups in flight
  static constexpr int GS = SLOTS / 2 < 8 ? SLOTS / 2 : 8;
  static constexpr int NG = SLOTS / GS;
  static_assert((BLK * F::A_TILES) % GS == 0, "groups tile a stage");
  static constexpr int TMEM_COLS = SLOTS * NT < 32 ? 32 : SLOTS * NT;
  static constexpr size_t SMEM = (size_t)NS * STAGE + 1024 /* alignment */ + 1024 /* barriers */;
  static constexpr uint32_t TX = (uint32_t)(B_BYTES + (F::RAW ? RAW_BYTES : A_BYTES) + SA_BYTES + SUM_BYTES);
  // warps: 0-3 producers, then the epilogue (four per TMEM lane quarter at 16
  // tokens, where a thread's share is small; two otherwise), MMA, TMA
  static constexpr int EPI = NT == 16 ? 16 : 8;
  static constexpr int MMA_WARP = 4 + EPI;
  static constexpr int TMA_WARP = MMA_WARP + 1;
  static constexpr int THREADS = (TMA_WARP + 1) * 32;
};

// Instruction descriptor: s8 x s8 -> s32, K-major A and B, M = 128, N = nt.
constexpr uint32_t i8_idesc(int nt) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(nt >> 3) << 17) | ((uint32_t)(QG_BM >> 4) << 24);
}

// byte offset of 16-byte chunk c (0..7) of row r inside a 128-row x 128-byte swizzle atom
__device__ __forceinline__ int sw_off(int r, int c) { return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4); }

// Bounded wait that also gives up when another role of the CTA has.
__device__ __forceinline__ bool qwait(uint64_t* bar, uint32_t phase, volatile int* abort) {
  for (uint32_t i = 0; i < kMbarPolls; i++) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((i & 255) == 255 && *abort) return false;
  }
  return false;
}

// Unpack weight row r of one stage from its staged packed bytes into the
// int8 tile(s), swizzled.  Bytes past the matrix were filled with zeros by
// TMA; the values they become are never scaled into a result (their blocks
// lie past K, their rows past N).
template <int T>
__device__ __forceinline__ void unpack_row(const uint8_t* raw, const uint8_t* raw2, uint8_t* a, int r) {
  constexpr int ATOM = QG_BM * 128;
  if constexpr (T == T_Q4_0) {
    // 8 blocks of 16 bytes: byte j holds value j (low nibble) and j + 16 (high), q - 8.
    // Rows are 128 bytes apart: each row starts at another block (bank) so a
    // warp's reads spread over the banks.
#pragma unroll
    for (int b_ = 0; b_ < 8; b_++) {
      const int b = (b_ + r) & 7;
      const uint4 x = *reinterpret_cast<const uint4*>(raw + b * 16);
      const unsigned m = 0x0F0F0F0Fu, e = 0x08080808u;
      const uint4 lo = make_uint4(__vsub4(x.x & m, e), __vsub4(x.y & m, e), __vsub4(x.z & m, e), __vsub4(x.w & m, e));
      const uint4 hi = make_uint4(__vsub4((x.x >> 4) & m, e), __vsub4((x.y >> 4) & m, e), __vsub4((x.z >> 4) & m, e),
                                  __vsub4((x.w >> 4) & m, e));
      uint8_t* at = a + (b >> 2) * ATOM;
      *reinterpret_cast<uint4*>(at + sw_off(r, (2 * b) & 7)) = lo;
      *reinterpret_cast<uint4*>(at + sw_off(r, (2 * b + 1) & 7)) = hi;
    }
  } else if constexpr (T == T_Q4_K) {
    // 16-byte header, then pair p (32 bytes): low nibbles = group 2p, high = group 2p + 1
#pragma unroll
    for (int c = 0; c < 16; c++) {  // 16-value chunk c: pair c/4, high half (c/2)%2, bytes (c%2)*16..
      const int p = c >> 2, hi = (c >> 1) & 1, l0 = (c & 1) * 16;
      const uint4 x = *reinterpret_cast<const uint4*>(raw + 16 + p * 32 + l0);
      const unsigned m = 0x0F0F0F0Fu;
      const uint4 v = hi ? make_uint4((x.x >> 4) & m, (x.y >> 4) & m, (x.z >> 4) & m, (x.w >> 4) & m)
                         : make_uint4(x.x & m, x.y & m, x.z & m, x.w & m);
      *reinterpret_cast<uint4*>(a + (c >> 3) * ATOM + sw_off(r, c & 7)) = v;
    }
  } else if constexpr (T == T_Q6_K) {
    // one super-block: ql 128 bytes (raw), qh 64 bytes (raw2).  Half h, value e = 32 g + l
    // (g = 0..3): low 4 bits from ql[64 h + l + 32 (g & 1)] (high nibble when
    // g >= 2), high 2 bits from qh[32 h + l] >> 2g; minus 32.  16-value chunk c
    // (one sub-block) goes to the lower tile when c is even, to the upper when
    // odd; the other tile holds zeros there.
    uint8_t* lo_t = a;
    uint8_t* hi_t = a + 2 * ATOM;
#pragma unroll
    for (int c_ = 0; c_ < 16; c_++) {
      const int c = (c_ + r) & 15;  // rows start at different chunks: spread banks
      const int h = c >> 3, g = (c >> 1) & 3, l0 = (c & 1) * 16;
      const uint4 x = *reinterpret_cast<const uint4*>(raw + h * 64 + (g & 1) * 32 + l0);
      const uint4 q = *reinterpret_cast<const uint4*>(raw2 + h * 32 + l0);
      const int sh = (g >> 1) * 4, hs = 2 * g;
      const unsigned m4 = 0x0F0F0F0Fu, m2 = 0x03030303u, k = 0x20202020u;
      const uint4 v = make_uint4(__vsub4(((x.x >> sh) & m4) | (((q.x >> hs) & m2) << 4), k),
                                 __vsub4(((x.y >> sh) & m4) | (((q.y >> hs) & m2) << 4), k),
                                 __vsub4(((x.z >> sh) & m4) | (((q.z >> hs) & m2) << 4), k),
                                 __vsub4(((x.w >> sh) & m4) | (((q.w >> hs) & m2) << 4), k));
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      const int at = h * ATOM + sw_off(r, c & 7);
      *reinterpret_cast<uint4*>(lo_t + at) = (c & 1) ? z : v;
      *reinterpret_cast<uint4*>(hi_t + at) = (c & 1) ? v : z;
    }
  }
}

template <int T, int NT>
__global__ void __launch_bounds__(QgLayout<T, NT>::THREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
                 const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_sa,
                 const __grid_constant__ CUtensorMap tm_sum, const QgemmArgs g) {
  using L = QgLayout<T, NT>;
  using F = QgFmt<T>;
  constexpr int NS = L::NS, BK = L::BK, SLOTS = L::SLOTS, MPB = L::MPB, BLK = L::BLK, GS = L::GS, NG = L::NG;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + NS * L::STAGE);
  uint64_t* full = bars;                   // [NS] every TMA byte of the stage landed
  uint64_t* conv = bars + NS;              // [NS] producers wrote the int8 tile
  uint64_t* freed = bars + 2 * NS;         // [NS] MMAs completed and epilogue done with the stage
  uint64_t* acc_full = bars + 3 * NS;      // [NG] a group's MMAs landed in its slots
  uint64_t* acc_empty = acc_full + NG;     // [NG] every epilogue warp read the group's slots
  uint64_t* mma_done = acc_empty + NG;     // every MMA issued has completed (before TMEM is freed)
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ int s_abort;
  volatile int* abort = &s_abort;

  auto stage = [&](int st) { return base + st * L::STAGE; };

  const int tid = threadIdx.x, wi = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * QG_BM, tok0 = blockIdx.y * NT;
  const int K = g.K, N = g.N;
  const int n_blk = K / 32;
  // split-K: this CTA takes stages [s_lo, s_lo + n_stage) of the row
  const int all_stages = (K + BK - 1) / BK;
  const int s_lo = (int)(((long long)all_stages * blockIdx.z) / gridDim.z);
  const int n_stage = (int)(((long long)all_stages * (blockIdx.z + 1)) / gridDim.z) - s_lo;
  // CTAs walk their stages from different starting points, so that at any
  // moment the grid's copies read different offsets of the weight rows rather
  // than one column band of every row (which concentrates on few DRAM
  // channels); each CTA's order is fixed, so results are reproducible
  const int rot = n_stage > 0 ? (int)(blockIdx.x % (unsigned)n_stage) : 0;
  auto gstage = [&](int s) { return s_lo + (s + rot) % n_stage; };

  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < NS; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&conv[i], QG_PRODUCERS);
      mbar_init(&freed[i], 1 + L::EPI);
    }
    for (int i = 0; i < NG; i++) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], L::EPI);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (wi == L::MMA_WARP) {
    tc_alloc(tmem_base_s, L::TMEM_COLS);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_s;

  if (wi == L::TMA_WARP) {
    // ------------------------------------------------ TMA issue
    if (lane == 0) {
      int issued = 0;
      for (int s = 0; s < n_stage; s++) {
        const int st = s % NS;
        if (s >= NS && !qwait(&freed[st], ((s / NS) - 1) & 1, abort)) break;
        if (*abort) break;
        uint8_t* sm = stage(st);
        mbar_arrive_expect_tx(&full[st], L::TX);
        const int sg = gstage(s), k0 = sg * BK;
#pragma unroll
        for (int a = 0; a < L::KATOMS; a++) tma_load_2d(sm + L::OFF_B + a * NT * 128, &tm_x, k0 + a * 128, tok0, &full[st]);
        if constexpr (F::RAW == 0) {
#pragma unroll
          for (int a = 0; a < L::KATOMS; a++) tma_load_2d(sm + a * L::A_ATOM, &tm_w, k0 + a * 128, row0, &full[st]);
        } else if constexpr (T == T_Q6_K) {
          tma_load_2d(sm + L::OFF_RAW, &tm_w, sg * 128, row0, &full[st]);                 // ql
          tma_load_2d(sm + L::OFF_RAW + QG_BM * 128, &tm_w2, sg * 64, row0, &full[st]);  // qh
        } else {
          tma_load_2d(sm + L::OFF_RAW, &tm_w, sg * F::RAW, row0, &full[st]);
        }
        tma_load_2d(sm + L::OFF_SA, &tm_sa, tok0, sg * BLK, &full[st]);
        if constexpr (L::SUM_BYTES > 0) tma_load_2d(sm + L::OFF_SUM, &tm_sum, tok0, sg * BLK, &full[st]);
        issued = s + 1;
      }
      // wind down: the copies still possibly in flight are those of the last NS stages issued
      const bool ab = *abort != 0;
      for (int s = issued > NS ? issued - NS : 0; s < issued; s++)
        mbar_wait(&full[s % NS], (s / NS) & 1, ab ? (1u << 16) : kMbarPolls);
    }
    __syncwarp();
  } else if (wi == L::MMA_WARP) {
    // ------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = i8_idesc(NT);
      int grp = 0, last_stage = -1;
      bool ok = true;
      for (int s = 0; s < n_stage && ok; s++) {
        const int st = s % NS, ph = (s / NS) & 1;
        ok = qwait(&full[st], ph, abort);
        if (ok && F::RAW > 0) ok = qwait(&conv[st], ph, abort);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_base = smem_u32(stage(st)), b_base = a_base + L::OFF_B;
        const int nb = min(BLK, n_blk - gstage(s) * BLK);
        const int total = nb * MPB;  // MMAs of this stage: (block j, half h) in order
        for (int i0 = 0; i0 < total && ok; i0 += GS, grp++) {
          const int gslot = grp % NG;
          if (grp >= NG && !qwait(&acc_empty[gslot], ((grp / NG) - 1) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int cnt = min(GS, total - i0);
          for (int i = 0; i < cnt; i++) {
            const int j = (i0 + i) / MPB, h = (i0 + i) % MPB;
            const uint32_t koff = (uint32_t)((j & 3) * 32);
            const uint32_t a_at = a_base + (uint32_t)((j >> 2) * L::A_ATOM) + koff +
                                  (uint32_t)(h * L::KATOMS * L::A_ATOM);
            const uint32_t b_at = b_base + (uint32_t)((j >> 2) * NT * 128) + koff;
            tc_mma_i8(tmem + (uint32_t)((gslot * GS + i) * NT), sw128_desc(a_at), sw128_desc(b_at), idesc);
          }
          tc_commit(&acc_full[gslot]);
        }
        tc_commit(&freed[st]);
        last_stage = s;
      }
      if (!ok) *abort = 1;
      // wind down: every MMA issued has completed before TMEM is freed
      (void)last_stage;
      tc_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
    __syncwarp();
  } else if (wi < 4) {
    // ------------------------------------------------ producers: unpack one weight row each
    if constexpr (F::RAW > 0) {
      const int r = tid;
      for (int s = 0; s < n_stage; s++) {
        const int st = s % NS;
        if (!qwait(&full[st], (s / NS) & 1, abort)) {
          *abort = 1;
          break;
        }
        uint8_t* sm = stage(st);
        if constexpr (T == T_Q6_K)
          unpack_row<T>(sm + L::OFF_RAW + r * 128, sm + L::OFF_RAW + QG_BM * 128 + r * 64, sm, r);
        else
          unpack_row<T>(sm + L::OFF_RAW + r * F::RAW, nullptr, sm, r);
        fence_async_smem();
        mbar_arrive(&conv[st]);
      }
    }
  } else {
    // ------------------------------------------------ epilogue
    const int q4 = wi & 3, part = (wi - 4) >> 2;  // lane quarter, token slice
    const int rl = q4 * 32 + lane;                 // row within the tile
    const int r = row0 + rl;
    const int rr = min(r, N - 1);                  // rows past N read row N-1's scales (never stored)
    constexpr int NC = NT / (L::EPI / 4);    // tokens per thread
    const int c0 = part * NC;
    float acc[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) acc[c] = 0.0f;
    // weight scales of a stage, loaded one stage ahead: Q8_0 / Q4_0 the f16 d
    // of each block; Q6_K the super-block's d and its 16 int8 sub-block scales
    // (Q4_K's live in the staged super-block header)
    // f16 scales: two per word at up to 32 tokens, one per register at 64
    // (where the epilogue's accumulators leave fewer registers)
    uint32_t dn[BLK / 2], dc[BLK / 2];
    unsigned short dn1[BLK], dc1[BLK];
    float dnf[BLK], dcf[BLK];  // Q8S: f32 scales
    uint4 scn = make_uint4(0u, 0u, 0u, 0u), scc = scn;
    auto load_scales = [&](int s) {  // s: global stage (< 0: none)
      if (s < 0) return;
      if constexpr (T == T_Q8_0 || T == T_Q4_0) {
        const unsigned short* d = reinterpret_cast<const unsigned short*>(g.w.d) + (size_t)rr * n_blk + s * BLK;
        const int nb = min(BLK, n_blk - s * BLK);
        // the stage's 8 scales: one 16-byte load (16-token tiles, whose
        // epilogue has the registers to spare)
        if (NT <= 32 && nb == BLK && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(d));
          dn[0] = v.x;
          dn[1] = v.y;
          dn[2] = v.z;
          dn[3] = v.w;
        } else if constexpr (NT <= 32) {
#pragma unroll
          for (int j = 0; j < BLK / 2; j++) dn[j] = 0u;
#pragma unroll
          for (int j = 0; j < BLK; j++)
            if (j < nb) dn[j >> 1] |= (uint32_t)__ldg(d + j) << (16 * (j & 1));
        } else {
#pragma unroll
          for (int j = 0; j < BLK; j++)
            if (j < nb) dn1[j] = __ldg(d + j);
        }
      } else if constexpr (T == T_Q8S) {
        const float* d = g.w.ds + (size_t)rr * n_blk + s * BLK;
        const int nb = min(BLK, n_blk - s * BLK);
        if (NT <= 32 && nb == BLK && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
          const float4 v0 = __ldg(reinterpret_cast<const float4*>(d)), v1 = __ldg(reinterpret_cast<const float4*>(d) + 1);
          dnf[0] = v0.x; dnf[1] = v0.y; dnf[2] = v0.z; dnf[3] = v0.w;
          dnf[4] = v1.x; dnf[5] = v1.y; dnf[6] = v1.z; dnf[7] = v1.w;
        } else {
#pragma unroll
          for (int j = 0; j < BLK; j++)
            if (j < nb) dnf[j] = __ldg(d + j);
        }
      } else if constexpr (T == T_Q6_K) {
        dn[0] = __ldg(reinterpret_cast<const unsigned short*>(g.w.d) + (size_t)rr * (K / 256) + s);
        scn = __ldg(reinterpret_cast<const uint4*>(g.w.sc + (size_t)rr * (K / 16)) + s);
      }
    };
    load_scales(n_stage > 0 ? gstage(0) : -1);
    int grp = 0;
    bool ok = true;
    constexpr int NB = (32 / NC) < 1 ? 1 : ((32 / NC) < GS ? (32 / NC) : GS);  // slots per load batch (<= 32 registers)
    // A stage that is one slot group read in one load batch (16-token tiles,
    // one MMA per block): the group and batch offsets below are always 0, and
    // saying so lets every block index, and with it the choice of the block's
    // weight scale, resolve at compile time.
    constexpr bool kOneGroup = GS == BLK * MPB && NB == GS;
    for (int s = 0; s < n_stage && ok; s++) {
      const int st = s % NS, sg = gstage(s);
      const uint8_t* sm = stage(st);
#pragma unroll
      for (int j = 0; j < BLK / 2; j++) dc[j] = dn[j];
#pragma unroll
      for (int j = 0; j < BLK; j++) dc1[j] = dn1[j];
#pragma unroll
      for (int j = 0; j < BLK; j++) dcf[j] = dnf[j];
      scc = scn;
      load_scales(s + 1 < n_stage ? gstage(s + 1) : -1);
      if (!qwait(&full[st], (s / NS) & 1, abort)) {
        ok = false;
        break;
      }
      const float* sa_s = reinterpret_cast<const float*>(sm + L::OFF_SA);
      const int nb = min(BLK, n_blk - sg * BLK);
      const int total = nb * MPB;
      for (int i0 = 0; i0 < total && ok; i0 += GS, grp++) {
        const int gslot = grp % NG;
        if (!qwait(&acc_full[gslot], (grp / NG) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int cnt = min(GS, total - i0);
        for (int b0_ = 0; b0_ < cnt; b0_ += NB) {
          const int b0 = kOneGroup ? 0 : b0_, ib = kOneGroup ? 0 : i0 + b0_;
          uint32_t v[NB][NC];
#pragma unroll
          for (int k = 0; k < NB; k++)
            if (b0 + k < cnt) {
              if constexpr (NC == 4) {
                tc_ld4(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)((gslot * GS + b0 + k) * NT + c0), &v[k][0]);
              } else {
#pragma unroll
                for (int c = 0; c < NC; c += 8)
                  tc_ld8(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)((gslot * GS + b0 + k) * NT + c0 + c), &v[k][c]);
              }
            }
          tc_wait_ld();
#pragma unroll
          for (int k = 0; k < NB; k++) {
            if (b0 + k >= cnt) break;
            const int i = ib + k, j = i / MPB, h = i % MPB;
            const int b = sg * BLK + j;  // global block
            if (g.dots) {
              if (r < N)
#pragma unroll
                for (int c = 0; c < NC; c++) {
                  const int t = tok0 + c0 + c;
                  if (t < g.M)
                    g.dots[((size_t)t * N + r) * (size_t)(n_blk * MPB) + (size_t)b * MPB + h] = (int32_t)v[k][c];
                }
              continue;
            }
            const float* sa = sa_s + j * NT + c0;
            if constexpr (T == T_Q8_0 || T == T_Q4_0 || T == T_Q8S) {
              // (d * sa) * dot (matmul.rs:395-406, kquant.rs:240-252)
              float ws0;
              if constexpr (T == T_Q8S) {
                ws0 = dcf[0];
#pragma unroll
                for (int q = 1; q < BLK; q++)
                  if (q == j) ws0 = dcf[q];  // a register select, not an indexed local array
              } else {
                if constexpr (NT <= 32) {
                  uint32_t wsel = dc[0];
#pragma unroll
                  for (int q = 1; q < BLK / 2; q++)
                    if (q == (j >> 1)) wsel = dc[q];  // register selects, not an indexed local array
                  ws0 = h2f((unsigned short)(wsel >> (16 * (j & 1))));
                } else {
                  unsigned short dj = dc1[0];
#pragma unroll
                  for (int q = 1; q < BLK; q++)
                    if (q == j) dj = dc1[q];
                  ws0 = h2f(dj);
                }
              }
#pragma unroll
              for (int c = 0; c < NC; c++) acc[c] = fmaf(__fmul_rn(ws0, sa[c]), (float)(int32_t)v[k][c], acc[c]);
            } else if constexpr (T == T_Q4_K) {
              // sa * (d sc * dot - dmin m * sum) (kquant.rs:257-282)
              const uint8_t* hdr = sm + L::OFF_RAW + rl * F::RAW;
              int sc, mn;
              q4k_scale_min(j, hdr + 4, sc, mn);
              const float d = h2f((unsigned short)(hdr[0] | (hdr[1] << 8)));
              const float dmin = h2f((unsigned short)(hdr[2] | (hdr[3] << 8)));
              const float dsc = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)mn);
              const int32_t* sm_s = reinterpret_cast<const int32_t*>(sm + L::OFF_SUM) + j * NT + c0;
#pragma unroll
              for (int c = 0; c < NC; c++) {
                const float t = __fsub_rn(__fmul_rn(dsc, (float)(int32_t)v[k][c]), __fmul_rn(dm, (float)sm_s[c]));
                acc[c] = fmaf(sa[c], t, acc[c]);
              }
            } else {
              // (d * sa) * sc * dot per 16-value sub-block (kquant.rs:287-318)
              const float d = h2f((unsigned short)dc[0]);
              const int si = 2 * j + h;  // sub-block scale byte si of the 16
              const unsigned word = si < 8 ? (si < 4 ? scc.x : scc.y) : (si < 12 ? scc.z : scc.w);
              const float scf = (float)(int8_t)((word >> (8 * (si & 3))) & 0xffu);
#pragma unroll
              for (int c = 0; c < NC; c++)
                acc[c] = fmaf(__fmul_rn(__fmul_rn(d, sa[c]), scf), (float)(int32_t)v[k][c], acc[c]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[gslot]);
      }
      // this warp is done with the stage's staged scales
      __syncwarp();
      if (lane == 0) mbar_arrive(&freed[st]);
    }
    if (!ok) *abort = 1;
    if (ok && r < N && !g.dots) {
      if (gridDim.z > 1) {  // split-K: this split's partial, summed in split order by qgemm_reduce_kernel
        float* pz = g.part + (size_t)blockIdx.z * g.M * N;
#pragma unroll
        for (int c = 0; c < NC; c++) {
          const int t = tok0 + c0 + c;
          if (t < g.M) pz[(size_t)t * N + r] = acc[c];
        }
      } else {
#pragma unroll
        for (int c = 0; c < NC; c++) {
          const int t = tok0 + c0 + c;
          if (t < g.M) {
            float* o = g.out + (size_t)t * N + r;
            float v = acc[c];
            if (g.bias) v = __fadd_rn(v, g.bias[r]);
            *o = g.resid ? __fadd_rn(*o, v) : v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && s_abort && g.err) atomicExch(g.err, ERR_TIMEOUT);
  if (wi == L::MMA_WARP) {
    tc_fence_after();
    tc_dealloc(tmem, L::TMEM_COLS);
  }
}

// Activation rows, quantized, into the GEMM's layout: the scales (and group
// sums) of block b for tokens t at [b][t] with rows padded to m_pad (zeros).
__global__ void qgemm_prep_kernel(const float* s, const int32_t* sum, int m, int G, int m_pad, float* s_t,
                                  int32_t* sum_t) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= G * m_pad) return;
  const int b = i / m_pad, t = i - b * m_pad;
  s_t[i] = t < m ? s[(size_t)t * G + b] : 0.0f;
  if (sum_t) sum_t[i] = t < m ? sum[(size_t)t * G + b] : 0;
}

// Split-K partials [splits][M][N] summed in split order (the same bits every
// run), then the epilogue: + bias, stored or added to out.
__global__ void qgemm_reduce_kernel(const float* part, int splits, int M, int N, const float* bias, int resid,
                                    float* out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t mn = (size_t)M * N;
  if (i >= mn) return;
  float v = part[i];
  for (int z = 1; z < splits; z++) v = __fadd_rn(v, part[(size_t)z * mn + i]);
  if (bias) v = __fadd_rn(v, bias[i % N]);
  out[i] = resid ? __fadd_rn(out[i], v) : v;
}

// ---- host: tensor maps, launch

using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeTiledFn qg_encode() {
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

// 2-D view: `rows` rows of `cols` elements (row pitch `pitch` bytes), box
// {bx, by}; out-of-range elements read as zero.
bool map2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t cols, uint64_t rows,
           uint64_t pitch, uint32_t bx, uint32_t by, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = qg_encode();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (pitch & 15) || ((uint64_t)bx * esize) % 16) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {bx, by};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int T, int NT>
cudaError_t qgemm_go(const QgemmArgs& g, const int8_t* q, const float* sa_t, const int32_t* sum_t, cudaStream_t st) {
  using L = QgLayout<T, NT>;
  const DevWeight& w = g.w;
  CUtensorMap tm_w{}, tm_w2{}, tm_x{}, tm_sa{}, tm_sum{};
  const uint64_t K = (uint64_t)g.K, N = (uint64_t)g.N, G = K / 32;
  bool ok = map2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, K, (uint64_t)g.M, K, 128, NT, CU_TENSOR_MAP_SWIZZLE_128B) &&
            map2d(&tm_sa, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, sa_t, (uint64_t)g.m_pad, G, (uint64_t)g.m_pad * 4, NT,
                  L::BLK, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (T == T_Q4_K)
    ok = ok && map2d(&tm_sum, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, sum_t, (uint64_t)g.m_pad, G, (uint64_t)g.m_pad * 4, NT,
                     L::BLK, CU_TENSOR_MAP_SWIZZLE_NONE);
  if constexpr (T == T_Q8_0 || T == T_Q8S) {
    ok = ok && map2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.qs, K, N, K, 128, QG_BM, CU_TENSOR_MAP_SWIZZLE_128B);
  } else if constexpr (T == T_Q4_0) {
    ok = ok && map2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.qs, K / 2, N, K / 2, 128, QG_BM,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
  } else if constexpr (T == T_Q4_K) {
    ok = ok && map2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.qs, K / 256 * 144, N, K / 256 * 144, 144, QG_BM,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    ok = ok && map2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.qs, K / 2, N, K / 2, 128, QG_BM,
                     CU_TENSOR_MAP_SWIZZLE_NONE) &&
         map2d(&tm_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.qh, K / 4, N, K / 4, 64, QG_BM, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!ok) return cudaErrorNotSupported;
  auto kern = qgemm_kernel<T, NT>;
  static bool attr_set[64] = {};  // per device and instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)L::SMEM);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const dim3 grid((unsigned)((N + QG_BM - 1) / QG_BM), (unsigned)(g.m_pad / NT), (unsigned)g.splits);
  kern<<<grid, L::THREADS, L::SMEM, st>>>(tm_w, tm_w2, tm_x, tm_sa, tm_sum, g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || g.splits == 1 || g.dots) return e;
  const size_t mn = (size_t)g.M * g.N;
  qgemm_reduce_kernel<<<(unsigned)((mn + 255) / 256), 256, 0, st>>>(g.part, g.splits, g.M, g.N, g.bias, g.resid, g.out);
  return cudaGetLastError();
}

template <int T>
cudaError_t qgemm_t(const QgemmArgs& g, const int8_t* q, const float* sa_t, const int32_t* sum_t, cudaStream_t st) {
  switch (qgemm_tokens_per_tile(g.M)) {
    case 16: return qgemm_go<T, 16>(g, q, sa_t, sum_t, st);
    case 32: return qgemm_go<T, 32>(g, q, sa_t, sum_t, st);
    default: return qgemm_go<T, 64>(g, q, sa_t, sum_t, st);
  }
}

}  // namespace

int qgemm_tokens_per_tile(int m) { return m <= 16 ? 16 : m <= 32 ? 32 : 64; }

namespace {
constexpr int QG_SMS = 148;
constexpr int QG_MAX_SPLITS = 16;
constexpr int QG_MAX_CTAS = 4 * QG_SMS;  // split grids stay within this (partial scratch)
// K splits for an [n x k] weight times m rows: the count whose waves of one
// CTA per SM, each CTA paying about three stages of pipeline fill, finish
// first; each split keeps at least 2 stages
int qgemm_splits(int m, int n, int k) {
  const int nt = qgemm_tokens_per_tile(m);
  const int tiles = ((n + QG_BM - 1) / QG_BM) * ((m + nt - 1) / nt);
  const int stages = (k + 255) / 256;
  int best = 1;
  long long best_cost = LLONG_MAX;
  for (int sp = 1; sp <= QG_MAX_SPLITS && sp <= std::max(1, stages / 2) && (sp == 1 || tiles * sp <= QG_MAX_CTAS); sp++) {
    const long long waves = (tiles * (long long)sp + QG_SMS - 1) / QG_SMS;
    const long long cost = waves * ((stages + sp - 1) / sp + 3);
    if (cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}
}  // namespace

size_t qgemm_scratch_bytes(int m, int k) {
  const int nt = qgemm_tokens_per_tile(m);
  const size_t m_pad = (size_t)(m + nt - 1) / nt * nt;
  // scale tables, then split partials: splits x m x n <= QG_MAX_CTAS x 128 x nt floats
  const size_t tables = (2 * m_pad * (size_t)(k / 32) * 4 + 255) & ~(size_t)255;
  return tables + (size_t)QG_MAX_CTAS * QG_BM * nt * 4 + 256;
}

cudaError_t launch_qgemm(QgemmArgs g, const int8_t* q, const float* s, const int32_t* sums, void* scratch,
                         cudaStream_t st) {
  if (g.M < 1 || g.K % 32 || g.K != g.w.cols || g.N != g.w.rows || g.N < 1) return cudaErrorInvalidValue;
  if ((g.w.type == T_Q4_K || g.w.type == T_Q6_K) && g.K % 256) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(q) & 15) return cudaErrorInvalidValue;
  const int nt = qgemm_tokens_per_tile(g.M);
  g.m_pad = (g.M + nt - 1) / nt * nt;
  const int G = g.K / 32;
  float* sa_t = static_cast<float*>(scratch);
  int32_t* sum_t = reinterpret_cast<int32_t*>(sa_t + (size_t)g.m_pad * G);
  g.splits = g.dots ? 1 : qgemm_splits(g.M, g.N, g.K);
  g.part = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) +
                                    ((2 * (size_t)g.m_pad * G * 4 + 255) & ~(size_t)255));
  const int n = G * g.m_pad;
  qgemm_prep_kernel<<<(n + 255) / 256, 256, 0, st>>>(s, g.w.type == T_Q4_K ? sums : nullptr, g.M, G, g.m_pad, sa_t,
                                                      g.w.type == T_Q4_K ? sum_t : nullptr);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  switch (g.w.type) {
    case T_Q8_0: return qgemm_t<T_Q8_0>(g, q, sa_t, sum_t, st);
    case T_Q8S: return qgemm_t<T_Q8S>(g, q, sa_t, sum_t, st);
    case T_Q4_0: return qgemm_t<T_Q4_0>(g, q, sa_t, sum_t, st);
    case T_Q4_K: return qgemm_t<T_Q4_K>(g, q, sa_t, sum_t, st);
    case T_Q6_K: return qgemm_t<T_Q6_K>(g, q, sa_t, sum_t, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace prana

// ---------------------------------------------------------------- C ABI

using namespace prana;

static int qgemm_entry(prana_ctx* c, const int8_t* q, const float* s, const int32_t* sums, size_t n_tokens,
                       const prana_weight* w, float* out, int32_t* dots) {
  if (!(c && q && s && sums && w && (out || dots))) return fail(PRANA_E_INVALID, "null argument");
  if (w->dw.type == T_F32) return fail(PRANA_E_INVALID, "the tensor-core GEMM takes a quantized weight");
  if (!n_tokens) return PRANA_OK;
  if (n_tokens > (1u << 20)) return fail(PRANA_E_INVALID, "too many rows");
  if (reinterpret_cast<uintptr_t>(q) & 15) return fail(PRANA_E_INVALID, "activation rows must be 16-byte aligned");
  DevScope ds(c->device);
  void* sp = nullptr;
  if (int rc = ctx_scratch(c, qgemm_scratch_bytes((int)n_tokens, w->dw.cols), &sp)) return rc;
  QgemmArgs g{};
  g.w = w->dw;
  g.N = w->dw.rows;
  g.K = w->dw.cols;
  g.M = (int)n_tokens;
  g.out = out;
  g.dots = dots;
  g.err = c->err;
  const cudaError_t e = launch_qgemm(g, q, s, sums, sp, c->stream);
  if (e == cudaErrorNotSupported) return fail(PRANA_E_UNSUPPORTED, "tensor map for this shape could not be made");
  PRANA_CK(e);
  return PRANA_OK;
}

extern "C" int prana_qgemm(prana_ctx* c, const int8_t* q, const float* s, const int32_t* sums, size_t n_tokens,
                           const prana_weight* w, float* out) {
  return qgemm_entry(c, q, s, sums, n_tokens, w, out, nullptr);
}

extern "C" int prana_qgemm_block_dots(prana_ctx* c, const int8_t* q, const float* s, const int32_t* sums,
                                      size_t n_tokens, const prana_weight* w, int32_t* dots) {
  return qgemm_entry(c, q, s, sums, n_tokens, w, nullptr, dots);
}
