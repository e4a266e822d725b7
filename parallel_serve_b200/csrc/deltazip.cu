// Route-A DeltaZip linear on sm_100a: base fp16 GEMM plus an int4, 2:4-sparse,
// group-quantised delta, in one kernel that reads the compressed delta.
//
// Route A of the reference serves an RL policy as base weights plus a
// compressed delta through an external Marlin-24 kernel with an
// epilogue-accumulate op (docs/deltazip_progress_2026-04-17.md:154-162; no
// source in the reference). Here, for tokens in routed order:
//
//   y[:c0]      = x[:c0]  @ W_base                 (base-model tokens)
//   y[c0:c0+c1] = x[c0:]  @ (W_base + deq(D))      (policy tokens)
//
// deq(D)[k, n] = q[k, n] * scale[k / 128, n], with two kept entries in every
// group of 4 consecutive k (2:4 along K) and q in [-7, 7].
//
// Design: one CTA per SM, stream-K over (128-column tile, 64-k block). Per
// stage, TMA brings the W_base tile (MN-major, 128-byte swizzle), the x tile
// of both token groups (K-major) and, by one bulk copy, the packed delta of
// the tile (3328 B: 128 columns x [16 B values, 8 B indices, 2 B scale]).
// A converter warpgroup expands the delta into a K-major fp16 tile in shared
// memory (two-buffer ring); the MMA thread issues the base MMAs over all
// tokens and the delta MMAs over the policy tokens into the same TMEM
// accumulator. W_base bytes are read once for both models, so a step moves
// base + ~0.19 x base bytes instead of 2 x base.
#include <cuda_runtime.h>

#include "ps_common.cuh"
#include "ps_host.h"

namespace ps {
namespace dz {

constexpr int kBM = 128;                    // weight columns per tile
constexpr int kBK = 64;                     // k per stage
constexpr int kGroup = 128;                 // quantisation group along K
constexpr int kMaxTok = 128;                // base + policy tokens per tile (padded)
constexpr int kThreads = 448;               // 14 warps: TMA, MMA, 4 epilogue, 8 converter
constexpr int kABytes = kBM * kBK * 2;      // 16 KB W_base tile
constexpr int kAHalf = 64 * kBK * 2;        // 8 KB per 64-column box
constexpr int kPackBytes = kBM * 16 + kBM * 8 + kBM * 2;  // 3328 B per (tile, 64 k)
constexpr int kDqBytes = kBM * kBK * 2;     // 16 KB expanded delta
constexpr int kDqBufs = 2;
constexpr int kXBoxRows = 16;
constexpr int kXBoxBytes = kXBoxRows * 128;
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;
constexpr int kStageBytes = 16 * kBM * 2;    // epilogue output stage: 16 columns x 128 rows
constexpr int kSmemFixed = 1024 + 512 + 128 + 128 + kStageBytes + kDqBufs * kDqBytes;

struct Args {
  void* y;
  const int32_t* counts;
  const uint8_t* packed;
  float* partial;
  int32_t* counter;
  int32_t* status;
  int M, K, N, split_point, tokpad, stages, bf16;
};

struct Sched {
  int c0, c1, n0, n1, nt, KB, I, C;
};

PS_DEV bool make_sched(const Args& a, Sched& s) {
  int c0 = a.counts ? a.counts[0] : a.split_point;
  int c1 = a.counts ? a.counts[1] : a.M - a.split_point;
  const int n0 = (c0 + 15) & ~15, n1 = (c1 + 15) & ~15;
  bool ok = c0 >= 0 && c1 >= 0 && c0 + c1 <= a.M && n0 + n1 <= a.tokpad;
  if (!ok) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_status(a.status, PS_ERR_BAD_INDEX);
    c0 = c1 = 0;
  }
  s.c0 = c0;
  s.c1 = c1;
  s.n0 = ok ? n0 : 0;
  s.n1 = ok ? n1 : 0;
  s.nt = (a.N + kBM - 1) / kBM;
  s.KB = (a.K + kBK - 1) / kBK;
  s.I = (c0 + c1 > 0) ? s.nt * s.KB : 0;
  s.C = (s.I + gridDim.x - 1) / gridDim.x;
  return ok;
}

// Expand one packed column (32 kept int4 values, their 2-bit positions, the
// group scale) into 64 fp16/bf16 values and store them as row `row` of a
// K-major, 128-byte-swizzled 128 x 64 tile.
template <typename T>
PS_DEV void expand_row(const uint8_t* pk, int row, uint8_t* dq) {
  const uint4 vals = *reinterpret_cast<const uint4*>(pk + row * 16);
  const uint2 meta = *reinterpret_cast<const uint2*>(pk + kBM * 16 + row * 8);
  const float scale = __half2float(*reinterpret_cast<const __half*>(pk + kBM * 24 + row * 2));
  const uint32_t vw[4] = {vals.x, vals.y, vals.z, vals.w};
  const uint32_t mw[2] = {meta.x, meta.y};
  uint8_t* rowp = dq + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = k in [8c, 8c + 8) = groups 2c, 2c+1
    float f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = 0.f;
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const int g = 2 * c + gg;  // group 0..15, kept values j = 2g, 2g + 1
#pragma unroll
      for (int sl = 0; sl < 2; ++sl) {
        const int j = 2 * g + sl;
        const int q = (int)((vw[j >> 3] >> ((j & 7) * 4)) & 0xF);
        const int qs = q >= 8 ? q - 16 : q;
        const int p = (int)((mw[j >> 4] >> ((j & 15) * 2)) & 0x3);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (p == e) f[gg * 4 + e] = (float)qs * scale;
      }
    }
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      T lo = from_f32<T>(f[2 * i]), hi = from_f32<T>(f[2 * i + 1]);
      o[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) |
             ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
    }
    *reinterpret_cast<uint4*>(rowp + ((c ^ (row & 7)) << 4)) = out;
  }
}

// fp16 fast path: thread (row, half) expands kept values 16*half .. 16*half+15
// (groups 8*half .. 8*half+7, k = 32*half .. 32*half+31) into 4 swizzled
// 16-byte chunks. Two int4 values become an fp16 pair through the exponent
// bias trick (0x6400 | (q+8) is 1024 + q + 8 exactly; subtract 1032), one
// HMUL2 applies the scale (q * scale is exact in fp32, so rounding the fp16
// product once equals rounding the fp32 product), and two byte permutes put
// the pair into its 2:4 slots; `lut` maps the group's 4-bit position code to
// the two permute selectors.
PS_DEV void expand_half_f16(const uint8_t* pk, int row, int half, uint8_t* dq,
                            const uint2* lut) {
  const uint2 vals = *reinterpret_cast<const uint2*>(pk + row * 16 + half * 8);
  const uint32_t meta = *reinterpret_cast<const uint32_t*>(pk + kBM * 16 + row * 8 + half * 4);
  const __half sc = *reinterpret_cast<const __half*>(pk + kBM * 24 + row * 2);
  const __half2 s2 = __halves2half2(sc, sc);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  uint8_t* rowp = dq + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {       // chunk c = 4*half + cc holds groups 2c, 2c+1
    uint32_t w[4];
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const int g = 2 * cc + gg;           // local group 0..7
      const uint32_t word = g < 4 ? vals.x : vals.y;
      const uint32_t byte = (word >> ((g & 3) * 8)) & 0xFFu;
      const uint32_t t = ((byte & 0x0Fu) | ((byte & 0xF0u) << 12)) ^ 0x00080008u;
      const uint32_t hb = t | 0x64006400u;
      const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&hb), bias);
      const __half2 dv = __hmul2(qv, s2);
      const uint32_t d = *reinterpret_cast<const uint32_t*>(&dv);
      const uint2 sel = lut[(meta >> (4 * g)) & 0xFu];
      w[2 * gg] = __byte_perm(d, 0u, sel.x);
      w[2 * gg + 1] = __byte_perm(d, 0u, sel.y);
    }
    const int c = 4 * half + cc;
    *reinterpret_cast<uint4*>(rowp + ((c ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Sparse path (fp16): thread (row, half) writes the 16 kept values of groups
// 8*half .. 8*half+7 of its row — dequantised, in k order, two per group —
// as 2 chunks of a K-major compressed tile (32 kept values = 64 bytes per
// row, 64-byte swizzle: 16-byte chunk c of row r sits at c ^ ((r & 7) >> 1)).
PS_DEV void compress_half_f16(const uint8_t* pk, int row, int half, uint8_t* dq) {
  const uint2 vals = *reinterpret_cast<const uint2*>(pk + row * 16 + half * 8);
  const __half sc = *reinterpret_cast<const __half*>(pk + kBM * 24 + row * 2);
  const __half2 s2 = __halves2half2(sc, sc);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  uint8_t* rowp = dq + (row >> 3) * 512 + (row & 7) * 64;
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    uint32_t w[4];
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {
      const int g = 4 * cc + gg;  // local group 0..7
      const uint32_t word = g < 4 ? vals.x : vals.y;
      const uint32_t byte = (word >> ((g & 3) * 8)) & 0xFFu;
      const uint32_t t = ((byte & 0x0Fu) | ((byte & 0xF0u) << 12)) ^ 0x00080008u;
      const uint32_t hb = t | 0x64006400u;
      const __half2 dv = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&hb), bias), s2);
      w[gg] = *reinterpret_cast<const uint32_t*>(&dv);
    }
    const int c = 2 * half + cc;
    *reinterpret_cast<uint4*>(rowp + ((c ^ ((row & 7) >> 1)) << 4)) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Sparse-MMA metadata word of TMEM lane L for the MMA covering k = 32*kk ..
// 32*kk+31 of the stage. For kind::f16 the lane holds rows m0 + 16*m2 (bits
// 0-15) and m0 + 8 + 16*m2 (bits 16-31), m0 = L & 7, m2 = L >> 4, for the
// k-half (L >> 3) & 1; one bit per logical element, i.e. one 4-bit code
// (two 2-bit positions) per group of 4 — the packed format's nibbles.
PS_DEV uint32_t meta_word(const uint8_t* pk, int L, int kk) {
  const int m0 = L & 7, k1 = (L >> 3) & 1, m2 = L >> 4;
  const int ra = m0 + 16 * m2, rb = ra + 8;
  const uint32_t* ma = reinterpret_cast<const uint32_t*>(pk + kBM * 16 + ra * 8);
  const uint32_t* mb = reinterpret_cast<const uint32_t*>(pk + kBM * 16 + rb * 8);
  return ((ma[kk] >> (16 * k1)) & 0xFFFFu) | (((mb[kk] >> (16 * k1)) & 0xFFFFu) << 16);
}

// Byte-permute selectors for a group whose kept values sit at positions
// p0 = code & 3, p1 = code >> 2 (p0 < p1): output halves 0..3 take bytes
// 0-1 (first value), 2-3 (second value) or 4-5 (zero).
PS_DEV uint2 lut_entry(int code) {
  const int p0 = code & 3, p1 = code >> 2;
  uint32_t sel[2] = {0u, 0u};
  for (int slot = 0; slot < 4; ++slot) {
    const uint32_t hs = (p0 < p1 && slot == p0) ? 0x10u : (p0 < p1 && slot == p1) ? 0x32u : 0x54u;
    sel[slot >> 1] |= hs << ((slot & 1) * 8);
  }
  return make_uint2(sel[0], sel[1]);
}

// Output row of token column col (base tokens occupy columns [0, n0), policy
// tokens [n0, n0 + n1)); -1 for padding columns.
PS_DEV int out_row(const Sched& s, int col) {
  if (col < s.n0) return col < s.c0 ? col : -1;
  return col - s.n0 < s.c1 ? s.c0 + (col - s.n0) : -1;
}

// 16 token columns of tile t -> y. The 128 epilogue threads (one tile row
// each) write their values into a shared-memory stage [16][128]; after a
// barrier the stage goes out as 16-byte stores, one token's 8 consecutive
// features each (scalar 2-byte stores left the last tile's epilogue
// latency-bound).
template <typename T>
PS_DEV void store_cols(const Args& a, const Sched& s, int t, int row, int col0, const float* v,
                       T* stg) {
#pragma unroll
  for (int j = 0; j < 16; ++j) stg[j * kBM + row] = from_f32<T>(v[j]);
  named_bar_sync(2, 128);
  const int et = threadIdx.x - 64;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = et + k * 128;
    const int r = out_row(s, col0 + (i >> 4));
    const int n0 = t * kBM + (i & 15) * 8;
    if (r >= 0 && n0 < a.N)
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.y) + (size_t)r * a.N + n0) =
          reinterpret_cast<const uint4*>(stg)[i];
  }
  named_bar_sync(2, 128);
}

// Sum of the fp32 partials of tile t (contributors bf..bl, summed in that
// order: deterministic) for token columns [c0, c0 + 32) of this thread's tile
// row; ncol (16 or 32) columns are valid. Loads of two contributors x 32
// columns are issued before any add, so the last-arriving CTA pays one L2
// round trip per two contributors.
PS_DEV void reduce_partials(const float* partial, int tokpad, const Sched& s, int t, int bf,
                            int bl, int c0, int ncol, int row, float* v) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = 0.f;
  for (int b0 = bf; b0 <= bl; b0 += 2) {
    float tv[2][32];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int bb = b0 + u;
      if (bb <= bl) {
        const int wb = (t == (bb * s.C) / s.KB) ? 0 : 1;
        const float* pr = partial + (size_t)(bb * 2 + wb) * tokpad * kBM + (size_t)c0 * kBM + row;
#pragma unroll
        for (int j = 0; j < 32; ++j) tv[u][j] = (j < ncol) ? __ldcg(pr + (size_t)j * kBM) : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (b0 + u <= bl) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += tv[u][j];
      }
    }
  }
}

// Sparse: the delta product runs on tcgen05.mma.sp over the compressed
// values with metadata in TMEM (fp16); dense: the delta is expanded to a dense
// tile and multiplied with tcgen05.mma (bf16, and the cross-check).
constexpr int kMetaCol = 256;  // first TMEM column of the sparse metadata

PS_DEV uint32_t meta_col(int qb, int kk) { return kMetaCol + (qb * 2 + kk) * 4; }

template <typename T, bool kSparse>
__global__ void __launch_bounds__(kThreads, 1)
    deltazip_kernel(const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_x, const Args a) {
  constexpr uint32_t kTmemCols = kSparse ? 512 : 2 * kMaxTok;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const int xstage = a.tokpad * 128;
  uint8_t* sDq = smem;                                  // kDqBufs x 16 KB
  uint8_t* sA = sDq + kDqBufs * kDqBytes;               // S x 16 KB
  uint8_t* sX = sA + S * kABytes;                       // S x tokpad x 128
  uint8_t* sP = sX + S * xstage;                        // S x 3328
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(sP + S * kPackBytes) + 15) & ~uintptr_t(15));
  uint64_t* full = bars;
  uint64_t* empty = full + S;
  uint64_t* dq_full = empty + S;
  uint64_t* dq_empty = dq_full + kDqBufs;
  uint64_t* acc_full = dq_empty + kDqBufs;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint2* lut = reinterpret_cast<uint2*>(
      (reinterpret_cast<uintptr_t>(tmem_slot) + 64) & ~uintptr_t(15));
  T* stg = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(lut + 16) + 127) & ~uintptr_t(127));

  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    for (int i = 0; i < kDqBufs; ++i) {
      mbar_init(dq_full + i, 8);
      mbar_init(dq_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 4);
    }
    mbar_init(drain, 1);
    flags[0] = 0;
    flags[1] = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 16) lut[threadIdx.x] = lut_entry(threadIdx.x);
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Before the dependency wait: warm L2 with this CTA's first base tiles and
  // packed deltas (static data). The (tile, k-block) ranges do not depend on
  // the token counts unless there are no tokens at all.
  if (warp == 0 && lane == 0) {
    const int nt = (a.N + kBM - 1) / kBM, KB = (a.K + kBK - 1) / kBK;
    const int C = (nt * KB + gridDim.x - 1) / gridDim.x;
    const int g0 = b * C, g1 = min(g0 + C, nt * KB);
    for (int g = g0, n = 0; g < g1 && n < S; ++g, ++n) {
      const int t = g / KB, kb = g % KB;
      tma_prefetch_l2_2d(&tmap_w, t * kBM, kb * kBK);
      tma_prefetch_l2_2d(&tmap_w, t * kBM + 64, kb * kBK);
      bulk_prefetch_l2(a.packed + ((size_t)t * KB + kb) * kPackBytes, kPackBytes);
    }
  }
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();

  Sched s;
  make_sched(a, s);
  const int start = b * s.C;
  const int end = min(start + s.C, s.I);
  const bool has_delta = s.n1 > 0;

  if (start >= end) {
    // no work for this CTA
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint32_t tx = kABytes + kPackBytes + (uint32_t)((s.n0 + s.n1) / 16) * kXBoxBytes;
      int it = 0;
      for (int g = start; g < end && !flags[0]; ++g, ++it) {
        const int t = g / s.KB, kb = g % s.KB;
        const int st = it % S;
        if (!mbar_wait(empty + st, ((it / S) & 1) ^ 1, a.status)) {
          flags[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(full + st, tx);
        uint8_t* dA = sA + st * kABytes;
        tma_load_2d(dA, &tmap_w, full + st, t * kBM, kb * kBK, pol_w);
        tma_load_2d(dA + kAHalf, &tmap_w, full + st, t * kBM + 64, kb * kBK, pol_w);
        bulk_load(sP + st * kPackBytes, a.packed + ((size_t)t * s.KB + kb) * kPackBytes,
                  kPackBytes, full + st, pol_w);
        uint8_t* dX = sX + st * xstage;
        for (int bx = 0; bx < s.n0 / 16; ++bx)
          tma_load_2d(dX + bx * kXBoxBytes, &tmap_x, full + st, kb * kBK, bx * 16, pol_x);
        for (int bx = 0; bx < s.n1 / 16; ++bx)
          tma_load_2d(dX + s.n0 * 128 + bx * kXBoxBytes, &tmap_x, full + st, kb * kBK,
                      s.c0 + bx * 16, pol_x);
      }
      if (flags[0]) {
        for (int st = 0; st < S && st < it; ++st) {
          const int last = st + S * ((it - 1 - st) / S);
          mbar_wait(full + st, (last / S) & 1, a.status);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issue
    if (lane == 0) {
      const uint32_t id_all = idesc_f16(a.bf16, 1, 0, kBM, s.n0 + s.n1);
      const uint32_t id_dq = idesc_f16(a.bf16, 0, 0, kBM, has_delta ? s.n1 : 16);
      const uint32_t id_sp = id_dq | (1u << 2);  // sparse flag
      int it = 0, acc_it = 0;
      for (int g = start; g < end && !flags[0];) {
        const int t = g / s.KB, kb0 = g % s.KB;
        const int kb1 = min(s.KB, kb0 + (end - g));
        (void)t;
        const int ab = acc_it & 1;
        if (!mbar_wait(acc_empty + ab, ((acc_it >> 1) & 1) ^ 1, a.status)) {
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + ab * kMaxTok;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int st = it % S;
          if (!mbar_wait(full + st, (it / S) & 1, a.status)) {
            flags[0] = 1;
            break;
          }
          const int qb = it % kDqBufs;
          if (has_delta && !mbar_wait(dq_full + qb, (it / kDqBufs) & 1, a.status)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t aaddr = smem_u32(sA + st * kABytes);
          const uint32_t xaddr = smem_u32(sX + st * xstage);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(aaddr + kk * 2048, kAHalf, 1024);
            const uint64_t bd = smem_desc_sw128(xaddr + kk * 32, 16, 1024);
            umma_f16(d, ad, bd, id_all, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          if (has_delta) {
            const uint32_t qaddr = smem_u32(sDq + qb * kDqBytes);
            if (kSparse) {
              // K = 32 logical (16 kept) per MMA; A rows are 64 B, 64-byte swizzle
#pragma unroll
              for (int kk = 0; kk < kBK / 32; ++kk) {
                const uint64_t ad = smem_desc(qaddr + kk * 32, 16, 512, 4);
                const uint64_t bd = smem_desc_sw128(xaddr + s.n0 * 128 + kk * 64, 16, 1024);
                umma_sp_f16(d + s.n0, ad, bd, tmem + meta_col(qb, kk), id_sp, 1u);
              }
            } else {
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk) {
                const uint64_t ad = smem_desc_sw128(qaddr + kk * 32, 16, 1024);
                const uint64_t bd = smem_desc_sw128(xaddr + s.n0 * 128 + kk * 32, 16, 1024);
                umma_f16(d + s.n0, ad, bd, id_dq, 1u);
              }
            }
            umma_commit(dq_empty + qb);
          }
          umma_commit(empty + st);
        }
        umma_commit(acc_full + ab);
        ++acc_it;
        g += kb1 - kb0;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, a.status);
    }
  } else if (warp >= 6) {
    // ------------------------------------------------- delta expansion
    if (has_delta) {
      const int ct = (warp - 6) * 32 + lane;  // 0..255: two threads per tile row
      const int row = ct >> 1, half = ct & 1;
      int it = 0;
      for (int g = start; g < end; ++g, ++it) {
        const int st = it % S;
        const int qb = it % kDqBufs;
        const bool ok = !flags[0] && mbar_wait(full + st, (it / S) & 1, a.status) &&
                        mbar_wait(dq_empty + qb, ((it / kDqBufs) & 1) ^ 1, a.status);
        if (__any_sync(0xffffffffu, !ok)) {
          flags[0] = 1;
          break;
        }
        if (kSparse) {
          compress_half_f16(sP + st * kPackBytes, row, half, sDq + qb * kDqBytes);
          if (warp < 10) {  // warps 6..9 cover the four TMEM lane quadrants once
            const int qd = warp & 3;
            const int L = qd * 32 + lane;
            const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);
            tmem_st1(lane_addr + meta_col(qb, 0), meta_word(sP + st * kPackBytes, L, 0));
            tmem_st1(lane_addr + meta_col(qb, 1), meta_word(sP + st * kPackBytes, L, 1));
            tmem_wait_st();
          }
        } else if (sizeof(T) == 2 && !a.bf16) {
          expand_half_f16(sP + st * kPackBytes, row, half, sDq + qb * kDqBytes, lut);
        } else if (half == 0) {
          expand_row<T>(sP + st * kPackBytes, row, sDq + qb * kDqBytes);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_full + qb);
      }
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int et = threadIdx.x - 64;
    const int nchunk = (s.n0 + s.n1) >> 4;
    int acc_it = 0;
    for (int g = start; g < end;) {
      const int t = g / s.KB, kb0 = g % s.KB;
      const int kb1 = min(s.KB, kb0 + (end - g));
      const int ab = acc_it & 1;
      const bool ok = !flags[0] && mbar_wait(acc_full + ab, (acc_it >> 1) & 1, a.status);
      if (named_bar_or(1, 128, !ok)) {
        flags[0] = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + ab * kMaxTok + ((uint32_t)(q * 32) << 16);
      if (kb0 == 0 && kb1 == s.KB) {
        for (int c = 0; c < nchunk; ++c) {
          float v[16];
          tmem_ld16(taddr + c * 16, v);
          store_cols<T>(a, s, t, row, c * 16, v, stg);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + ab);
      } else {
        const int which = (t == (b * s.C) / s.KB) ? 0 : 1;
        const uint64_t keep = l2_policy_evict_last();
        float* pw = a.partial + (size_t)(b * 2 + which) * a.tokpad * kBM;
        for (int c = 0; c < nchunk; ++c) {
          float v[16];
          tmem_ld16(taddr + c * 16, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) st_global_keep(pw + (size_t)(c * 16 + j) * kBM + row, v[j], keep);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + ab);
        named_bar_sync(1, 128);
        if (et == 0) {
          const int len = kb1 - kb0;
          fence_acq_rel_gpu();
          const int old = atom_add_acq_rel_gpu(a.counter + t, len);
          const int last = (old + len == s.KB) ? 1 : 0;
          if (last) a.counter[t] = 0;
          flags[1] = last;
        }
        named_bar_sync(1, 128);
        if (flags[1]) {
          const int bf = (t * s.KB) / s.C;
          const int bl = ((t + 1) * s.KB - 1) / s.C;
          for (int c = 0; c < nchunk; c += 2) {
            float v[32];
            const int ncol = (c + 1 < nchunk) ? 32 : 16;
            reduce_partials(a.partial, a.tokpad, s, t, bf, bl, c * 16, ncol, row, v);
            store_cols<T>(a, s, t, row, c * 16, v, stg);
            if (ncol == 32) store_cols<T>(a, s, t, row, c * 16 + 16, v + 16, stg);
          }
        }
      }
      ++acc_it;
      g += kb1 - kb0;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

struct Plan {
  int tokpad, stages, smem, grid, max_tiles;
  size_t counter_bytes, partial_bytes;
};

static Plan plan_for(int M, int N, int device) {
  Plan p;
  // Base and policy tokens are padded to 16 separately.
  p.tokpad = min(kMaxTok, max(32, round_up(M, 16) + 16));
  const int stage = kABytes + p.tokpad * 128 + kPackBytes;
  p.stages = min(kMaxStages, (kSmemLimit - kSmemFixed) / stage);
  p.smem = p.stages * stage + kSmemFixed;
  p.grid = sm_count(device);
  p.max_tiles = cdiv(N, kBM);
  p.counter_bytes = kCounterRegionBytes;
  p.partial_bytes = (size_t)p.grid * 2 * p.tokpad * kBM * sizeof(float);
  return p;
}

}  // namespace dz
}  // namespace ps

using namespace ps;

extern "C" size_t ps_deltazip_packed_bytes(int K, int N) {
  if (K <= 0 || N <= 0 || K % dz::kGroup) return 0;
  return (size_t)cdiv(N, dz::kBM) * (K / dz::kBK) * dz::kPackBytes;
}

extern "C" size_t ps_deltazip_workspace_bytes(int M, int N, int device) {
  if (M < 0 || N <= 0) return 0;
  const dz::Plan p = dz::plan_for(M, N, device);
  return p.counter_bytes + p.partial_bytes;
}

extern "C" int ps_deltazip_linear(const void* x, const void* W_base, const void* packed_delta,
                                  void* y, int M, int K, int N, int split_point,
                                  const int32_t* counts, int dtype, void* workspace,
                                  size_t workspace_bytes, int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && K > 0 && N > 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  PS_CHECK_ARG(K % dz::kGroup == 0 && N % 8 == 0);
  if (!counts) PS_CHECK_ARG(split_point >= 0 && split_point <= M);
  if (M == 0) return PS_OK;
  if (M > dz::kMaxTok - 16 && !(counts == nullptr && (split_point == 0 || split_point == M) &&
                                M <= dz::kMaxTok))
    return PS_ERR_UNSUPPORTED;
  PS_CHECK_ARG(x && W_base && packed_delta && y);
  PS_CHECK_ARG(aligned16(x) && aligned16(W_base) && aligned16(packed_delta) && aligned16(y));
  const int device = current_device();
  if (!is_sm100(device)) return PS_ERR_UNSUPPORTED;
  const dz::Plan p = dz::plan_for(M, N, device);
  if (p.max_tiles > kMaxCounters) return PS_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < p.counter_bytes + p.partial_bytes) return PS_ERR_WORKSPACE;
  PS_CHECK_ARG(aligned16(workspace));

  CUtensorMap tw, tx;
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)N * 2};
    const uint32_t box[2] = {64, (uint32_t)dz::kBK};
    if (!make_tmap_16bit(&tw, W_base, 2, dims, strides, box, dtype == PS_DTYPE_BF16, 256))
      return PS_ERR_CUDA;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, (uint32_t)dz::kXBoxRows};
    if (!make_tmap_16bit(&tx, x, 2, dims, strides, box, dtype == PS_DTYPE_BF16))
      return PS_ERR_CUDA;
  }
  dz::Args a;
  a.y = y;
  a.counts = counts;
  a.packed = reinterpret_cast<const uint8_t*>(packed_delta);
  a.counter = reinterpret_cast<int32_t*>(workspace);
  a.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + p.counter_bytes);
  a.status = status;
  a.M = M;
  a.K = K;
  a.N = N;
  a.split_point = split_point;
  a.tokpad = p.tokpad;
  a.stages = p.stages;
  a.bf16 = dtype == PS_DTYPE_BF16;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PS_DTYPE_BF16) {
    PS_CUDA_RET(allow_dynamic_smem(dz::deltazip_kernel<__nv_bfloat16, false>, dz::kSmemLimit));
    PS_CUDA_RET(launch(dz::deltazip_kernel<__nv_bfloat16, false>, dim3(p.grid),
                       dim3(dz::kThreads), p.smem, st, tw, tx, a));
  } else {
    PS_CUDA_RET(allow_dynamic_smem(dz::deltazip_kernel<__half, true>, dz::kSmemLimit));
    PS_CUDA_RET(launch(dz::deltazip_kernel<__half, true>, dim3(p.grid), dim3(dz::kThreads),
                       p.smem, st, tw, tx, a));
  }
  return PS_OK;
}
