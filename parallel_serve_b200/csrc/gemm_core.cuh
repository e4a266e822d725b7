// Building blocks of the routed two-model GEMM on sm_100a shared by the
// per-projection kernel (routed_gemm.cu) and the persistent projection-chain
// kernel (chain.cu): tile shape, launch arguments, the stream-K schedule
// (host-and-device code), the per-tile token staging, the fused epilogues and
// the split-tile reduction.
#pragma once
#include <cuda_runtime.h>

#include "ps_common.cuh"
#include "ps_host.h"

#include <cstring>

namespace ps {
namespace gemm {

constexpr int kBM = 128;                     // weight columns per tile (MMA M)
constexpr int kBK = 128;                     // K per pipeline stage
constexpr int kMaxTok = 128;                 // tokens per tile (MMA N upper bound)
constexpr int kThreads = 192;                // 6 warps
constexpr int kABytes = kBM * kBK * 2;       // 32 KB weight tile per stage
constexpr int kAHalf = 64 * kBK * 2;         // one 64-column TMA box (16 KB)
// Packed weights (ps_pack_weights): every (model, weight tile, 128-k block) is
// one contiguous 32 KB block holding exactly the shared-memory image a stage
// needs, so the producer moves it with one bulk copy and HBM sees long
// sequential runs instead of 128 row pieces of 128-256 bytes. Tile index n and
// the block order follow tile_of (SwiGLU tiles pair gate and up columns).
constexpr int kPackedTileBytes = kABytes;
// TMEM columns: two accumulator buffers [0, 256), the tile's residual staged
// as fp32 [256, 384) (one column per token), unused [384, 512).
constexpr int kTmemCols = 4 * kMaxTok;
constexpr int kTmemResidual = 2 * kMaxTok;
constexpr int kTmemSpare = 3 * kMaxTok;  // [384, 512): partials of a split tile's other contributors
constexpr int kMaxStages = 8;
constexpr int kPrefetchStages = 12;  // weight tiles per CTA warmed in L2 before the wait
constexpr int kSmemLimit = 232448;           // 227 KB opt-in per CTA
// align slack, barriers, epilogue exchange, per-token values of the tile
constexpr int kSmemFixed = 1024 + 256 + 128 * 16 * 4 + 3 * kMaxTok * 4;

struct Args {
  void* y;
  const void* residual;
  const int32_t* counts;
  const int32_t* scatter;
  float* partial;
  int32_t* counter;
  int32_t* status;
  int M, K, N;
  int split_point;
  int n_out;  // row length of y (N, or N/2 for SwiGLU)
  int gated;
  int ff;     // SwiGLU: N/2
  int tokpad;
  int stages;
  int bf16;
  int mode;  // PS_EPI_STORE / PS_EPI_SWIGLU / PS_EPI_QKV_ROPE
  // folded RMSNorm of the input rows:
  //   acc *= rsqrt(sum_p in_sumsq[row * in_parts + p] * inv_dim + eps)
  const float* in_sumsq;
  int in_parts;
  float norm_inv_dim, eps;
  // sum of squares of the stored (rounded) outputs per (row, 128-feature tile):
  //   out_sumsq[row * out_parts + out0 / 128]
  float* out_sumsq;
  int out_parts;
  // PS_EPI_QKV_ROPE: q -> y, k / v -> the token's model pools at pos[row]
  void* kp0;
  void* vp0;
  void* kp1;
  void* vp1;
  const int32_t* pos;
  const float* rcos;
  const float* rsin;
  int n_heads, L_cap, slots0, slots1, apply_rope;
  const int32_t* bt;  // paged pools: block table [table_rows, max_pages]
  int max_pages, page_size, table_rows;
  const int32_t* kv_rows;  // slot (contiguous) or block-table row (paged) of row j
  const uint8_t* wt;  // packed weights (nullable: W through the tensor map)
  int wt_nt, wt_KB;   // packed layout: weight tiles per model, 128-k blocks
};

PS_DEV const uint8_t* packed_block(const Args& a, int m, int n, int kb) {
  return a.wt + ((size_t)(m * a.wt_nt + n) * a.wt_KB + kb) * kPackedTileBytes;
}

// The (tile, k-block) iteration space I = ntiles * KB is worked in two parts.
// Data-parallel rounds: when a model has more than one token tile and there
// are at least as many tiles as CTAs, the first R * grid tiles go whole to
// the CTAs, tile b + r * grid to CTA b in round r. Tiles are ordered with the
// token tile innermost, so the token tiles of one weight tile run in the same
// round on neighbouring CTAs and the weight block they share is fetched from
// DRAM once (in back-to-back order on one CTA it would be evicted between the
// two reads). Stream-K: the remaining iterations [base, I) are cut into equal
// contiguous ranges of C, CTA b taking [base + b * C, base + (b + 1) * C).
// With one token tile per model (decode) R = 0: all of it is stream-K.
struct Sched {
  int c0, c1, T0, T1, tiles0, ntiles, KB, nt, I, C, R, base, grid;
};

struct Tile {
  int m, row0, ntok, col0, col1, out0;
  int n;  // weight-column tile of the model (packed weights: tile index)
};



PS_HD int imin(int x, int y) { return x < y ? x : y; }
PS_HD int imax(int x, int y) { return x > y ? x : y; }

// The schedule is host-and-device code: the library's schedule-introspection
// entry points run the same functions on the host.
PS_HD void sched_from_counts(const Args& a, int c0, int c1, int grid, Sched& s) {
  s.c0 = c0;
  s.c1 = c1;
  s.T0 = (c0 + a.tokpad - 1) / a.tokpad;  // token tiles of at most tokpad rows
  s.T1 = (c1 + a.tokpad - 1) / a.tokpad;
  s.nt = a.gated ? (a.ff + 63) / 64 : (a.N + kBM - 1) / kBM;
  s.tiles0 = s.T0 * s.nt;
  s.ntiles = s.tiles0 + s.T1 * s.nt;
  s.KB = (a.K + kBK - 1) / kBK;
  s.I = s.ntiles * s.KB;
  s.grid = grid;
  s.R = ((s.T0 > 1 || s.T1 > 1) && s.ntiles >= grid) ? s.ntiles / grid : 0;
  s.base = s.R * grid * s.KB;
  s.C = imax(1, (s.I - s.base + grid - 1) / grid);
}

// Work segment `seg` (0 <= seg <= s.R) of CTA b as an iteration range:
// seg < s.R is the whole tile b + seg * grid, seg == s.R the stream-K range.
PS_HD void seg_range(const Sched& s, int b, int seg, int& start, int& end) {
  if (seg < s.R) {
    start = (b + seg * s.grid) * s.KB;
    end = start + s.KB;
  } else {
    start = s.base + b * s.C;
    end = imin(start + s.C, s.I);
  }
}

// First tile of CTA b's stream-K range (where its partial goes to slot 0).
PS_HD int sk_first_tile(const Sched& s, int b) { return (s.base + b * s.C) / s.KB; }

// The CTAs [bf, bl] whose stream-K ranges hold iterations of split tile t.
PS_HD void sk_contributors(const Sched& s, int t, int& bf, int& bl) {
  bf = (t * s.KB - s.base) / s.C;
  bl = ((t + 1) * s.KB - 1 - s.base) / s.C;
}

// The schedule of this launch; reads device counts (call after pdl_wait()).
PS_DEV void make_sched(const Args& a, Sched& s) {
  int c0, c1;
  if (a.counts) {
    c0 = a.counts[0];
    c1 = a.counts[1];
  } else {
    c0 = a.split_point;
    c1 = a.M - a.split_point;
  }
  if (c0 < 0 || c1 < 0 || c0 + c1 > a.M) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_status(a.status, PS_ERR_BAD_INDEX);
    c0 = c1 = 0;
  }
  sched_from_counts(a, c0, c1, (int)gridDim.x, s);
}

// A schedule computed without reading device memory: exact for a host split,
// otherwise a guess (tokens spread over both models) used only to prefetch
// static weights into L2 before the dependency wait.
PS_DEV void guess_sched(const Args& a, Sched& s) {
  if (!a.counts)
    sched_from_counts(a, a.split_point, a.M - a.split_point, (int)gridDim.x, s);
  else
    sched_from_counts(a, (a.M + 1) / 2, a.M / 2, (int)gridDim.x, s);
}

// Tiles are ordered model-major, then by weight tile, then by token tile, so
// the token tiles that share one weight tile are adjacent: in a data-parallel
// round they run at the same time on neighbouring CTAs.
PS_HD Tile tile_of(const Args& a, const Sched& s, int t) {
  Tile ti;
  ti.m = t >= s.tiles0 ? 1 : 0;
  const int u = t - (ti.m ? s.tiles0 : 0);
  const int T = ti.m ? s.T1 : s.T0;
  const int cm = ti.m ? s.c1 : s.c0;
  const int ni = u / T, tt = u % T;
  ti.n = ni;
  ti.row0 = (ti.m ? s.c0 : 0) + tt * a.tokpad;
  ti.ntok = imin(a.tokpad, cm - tt * a.tokpad);
  if (a.gated) {
    const int f0 = ni * 64;
    ti.col0 = f0;
    ti.col1 = a.ff + f0;
    ti.out0 = f0;
  } else {
    const int n0 = ni * kBM;
    ti.col0 = n0;
    ti.col1 = n0 + 64;
    ti.out0 = n0;
  }
  return ti;
}

// Per-token values of the current tile, staged in shared memory by the
// epilogue threads (one token each) before the tile's accumulator is ready.
struct TileTokens {
  float rstd[kMaxTok];  // folded RMSNorm: 1/rms of the token (0 past ntok)
  int idx[kMaxTok];     // QKV_ROPE: position; otherwise the scattered output row (-1 past ntok)
  int page[kMaxTok];    // QKV_ROPE: the position's page (paged pools, -1 if out of range)
                        // or the token's slot (contiguous pools)
};

// Output row of token column col (-1: skip) and a bounds check on scattered rows.
PS_DEV int out_row(const Args& a, const Tile& ti, const TileTokens& tk, int col) {
  if (col >= ti.ntok) return -1;
  const int o = a.scatter ? tk.idx[col] : ti.row0 + col;
  if (o < 0 || o >= a.M) {
    set_status(a.status, PS_ERR_BAD_INDEX);
    return -1;
  }
  return o;
}

// Final values of 16 token columns (col0 .. col0 + 15) of the tile -> global
// memory, in the launch's epilogue mode. All 128 epilogue threads call it
// together. Each thread first computes the values of its tile row (feature)
// into a shared-memory stage [16 columns][tile width] of T; after a barrier the
// stage is written out row-contiguously with 16-byte stores (one token's 8
// consecutive features per store), which also yields the sums of squares of
// the stored values by a 16-lane shuffle. The stage reuses the exchange
// buffer: STORE and QKV_ROPE at offset 0 (4 KB; the RoPE exchange is done by
// then), SWIGLU at 4 KB (its gate/up exchange occupies the first 4 KB).
template <typename T>
PS_DEV void finalize(const Args& a, const Sched& s, const Tile& ti, int row, int col0, float* v,
                     float* xchg, const TileTokens& tk, uint32_t tres) {
  const int et = threadIdx.x - 64;
  if (a.in_sumsq) {  // RMSNorm folded into the weights: scale by the token's 1/rms
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] *= tk.rstd[col0 + j];
  }
  if (a.mode == PS_EPI_STORE) {
    T* stg = reinterpret_cast<T*>(xchg);  // [16][128]
    if (a.residual) {  // staged in TMEM while the tile's MMAs ran (stage_residual)
      float rv[16];
      tmem_ld16(tres + col0, rv);
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += rv[j];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) stg[j * kBM + row] = from_f32<T>(v[j]);
    named_bar_sync(2, 128);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = et + k * 128;
      const int jj = i >> 4, piece = i & 15;
      const int n0 = ti.out0 + piece * 8;
      const uint4 val = reinterpret_cast<const uint4*>(stg)[i];
      const int o = (n0 < a.N) ? out_row(a, ti, tk, col0 + jj) : -1;
      if (o >= 0)
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.y) + (size_t)o * a.n_out + n0) = val;
      if (a.out_sumsq) {  // the tile's 128 features of token column jj, fixed order
        const T* h = reinterpret_cast<const T*>(&val);
        float sq = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float f = to_f32<T>(h[e]);
          sq += f * f;
        }
        if (n0 >= a.N) sq = 0.f;
#pragma unroll
        for (int m = 8; m > 0; m >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, m);
        if (piece == 0 && o >= 0) a.out_sumsq[(size_t)o * a.out_parts + ti.out0 / kBM] = sq;
      }
    }
    named_bar_sync(2, 128);
  } else if (a.mode == PS_EPI_SWIGLU) {
    // Tile rows 0..63 hold gate columns f0.., rows 64..127 the matching up columns.
    T* stg = reinterpret_cast<T*>(xchg + 16 * 64);  // [16][64]
    if (row >= 64) {
#pragma unroll
      for (int j = 0; j < 16; ++j) xchg[j * 64 + (row - 64)] = v[j];
    }
    named_bar_sync(2, 128);
    if (row < 64) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float g = v[j];
        const float u = xchg[j * 64 + row];
        stg[j * 64 + row] = from_f32<T>(g / (1.0f + __expf(-g)) * u);
      }
    }
    named_bar_sync(2, 128);
    {
      const int jj = et >> 3, piece = et & 7;
      const int f0 = ti.out0 + piece * 8;
      const int o = (f0 < a.ff) ? out_row(a, ti, tk, col0 + jj) : -1;
      if (o >= 0)
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.y) + (size_t)o * a.n_out + f0) =
            reinterpret_cast<const uint4*>(stg)[et];
    }
    named_bar_sync(2, 128);
  } else {
    // PS_EPI_QKV_ROPE: a 128-column tile is one head of q, k or v.
    const int tile = ti.out0 / kBM;
    const int which = tile / a.n_heads, h = tile % a.n_heads;
    const bool rope = which < 2 && a.apply_rope;
    if (rope) {  // rotate-half pairs (i, i + 64) live in different threads
#pragma unroll
      for (int j = 0; j < 16; ++j) xchg[j * kBM + row] = v[j];
      named_bar_sync(2, 128);
      // rotate in place (no global stores in this pass, so the table loads overlap)
      const int i = row & 63;
      const float sgn = row < 64 ? -1.f : 1.f;
      const int rows = a.bt ? a.max_pages * a.page_size : a.L_cap;  // rows of the cos/sin tables
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int p = min(max(tk.idx[col0 + j], 0), rows - 1);  // table row (checked below)
        v[j] = v[j] * a.rcos[(size_t)p * 64 + i] +
               sgn * xchg[j * kBM + (row ^ 64)] * a.rsin[(size_t)p * 64 + i];
      }
      named_bar_sync(2, 128);  // partners read; the exchange buffer becomes the stage
    }
    T* stg = reinterpret_cast<T*>(xchg);  // [16][128]
#pragma unroll
    for (int j = 0; j < 16; ++j) stg[j * kBM + row] = from_f32<T>(v[j]);
    named_bar_sync(2, 128);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = et + k * 128;
      const int jj = i >> 4, piece = i & 15;
      const int col = col0 + jj;
      if (col >= ti.ntok) continue;
      const int r = ti.row0 + col;
      T* dst;
      if (which == 0) {
        dst = reinterpret_cast<T*>(a.y) + (size_t)r * a.n_out + h * kBM;
      } else {
        T* pool = reinterpret_cast<T*>(which == 1 ? (ti.m ? a.kp1 : a.kp0) : (ti.m ? a.vp1 : a.vp0));
        const int nsl = ti.m ? a.slots1 : a.slots0;
        const int p = tk.idx[col];
        if (a.bt) {  // paged: the position's page (looked up when staged), row p % page_size
          const int pg = tk.page[col];
          if (pg < 0 || pg >= nsl) {
            if (piece == 0) set_status(a.status, PS_ERR_BAD_INDEX);
            continue;
          }
          dst = pool + (((size_t)pg * a.n_heads + h) * a.page_size + (p & (a.page_size - 1))) * kBM;
        } else {
          const int sl = tk.page[col];  // the token's slot
          if (sl < 0 || sl >= nsl || p < 0 || p >= a.L_cap) {
            if (piece == 0) set_status(a.status, PS_ERR_BAD_INDEX);
            continue;
          }
          dst = pool + (((size_t)sl * a.n_heads + h) * a.L_cap + p) * kBM;
        }
      }
      *reinterpret_cast<uint4*>(dst + piece * 8) = reinterpret_cast<const uint4*>(stg)[i];
    }
    named_bar_sync(2, 128);
  }
}

// 1/rms of the tile's tokens (folded RMSNorm), one token per epilogue thread.
// The partials are summed in a fixed order (reproducible results); up to 32
// of them are loaded at once (one L2 round trip for the usual 16 or 32).
PS_DEV void tile_rstd(const Args& a, const Tile& ti, int et, float* rstd) {
  float r = 0.f;
  if (et < ti.ntok) {
    const float* p = a.in_sumsq + (size_t)(ti.row0 + et) * a.in_parts;
    const int n = a.in_parts;
    float t = 0.f;
    int i = 0;
    if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(a.in_sumsq) & 15) == 0) {
      const float4* p4 = reinterpret_cast<const float4*>(p);
      for (; i + 32 <= n; i += 32) {
        float4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = p4[i / 4 + k];
#pragma unroll
        for (int k = 0; k < 8; ++k) t += (v[k].x + v[k].y) + (v[k].z + v[k].w);
      }
      if (i + 16 <= n) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = p4[i / 4 + k];
#pragma unroll
        for (int k = 0; k < 4; ++k) t += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        i += 16;
      }
      for (; i < n; i += 4) {
        const float4 v = p4[i / 4];
        t += (v.x + v.y) + (v.z + v.w);
      }
    } else {
      for (; i < n; ++i) t += p[i];
    }
    r = rsqrtf(t * a.norm_inv_dim + a.eps);
  }
  rstd[et] = r;
}

// Stage the tile's per-token values (thread et handles token column et).
PS_DEV void tile_tokens(const Args& a, const Sched& s, const Tile& ti, int et, TileTokens& tk) {
  if (a.in_sumsq) tile_rstd(a, ti, et, tk.rstd);
  const int r = ti.row0 + et;
  if (a.mode == PS_EPI_QKV_ROPE) {
    const int p = et < ti.ntok ? a.pos[r] : -1;
    tk.idx[et] = p;
    if (a.bt) {
      const int row = et < ti.ntok ? (a.kv_rows ? a.kv_rows[r] : r) : -1;
      const int pi = p >= 0 ? p / a.page_size : -1;
      tk.page[et] = (pi >= 0 && pi < a.max_pages && row >= 0 && row < a.table_rows)
                        ? a.bt[(size_t)row * a.max_pages + pi]
                        : -1;
    } else {
      tk.page[et] = et < ti.ntok ? (a.kv_rows ? a.kv_rows[r] : r - (ti.m ? s.c0 : 0)) : -1;
    }
  } else if (a.scatter)
    tk.idx[et] = et < ti.ntok ? a.scatter[r] : -1;
}

// PS_EPI_STORE with a residual: stage the tile's residual (all token columns)
// in TMEM while the tile's MMAs run, so the epilogue reads it locally once the
// accumulator is ready. 32 token rows at a time are read with 16-byte loads
// (one token's 8 consecutive features each, all issued before any use) into
// the exchange buffer, then transposed: each thread takes its feature for the
// 32 tokens and stores them into its TMEM lane.
// Before the tile's accumulator is ready: if piece [kb0, kb0 + len) is part of
// a split tile whose other contributors have all published (then this CTA
// finishes it), load their partials, in contributor order, into the spare
// TMEM columns (ntok rounded to 16 columns each, up to 128 in all) and return
// true; the arrival counter is reset as the fix-up would. Uniform over the
// 128 epilogue threads.
PS_DEV bool prefetch_partials(const Args& a, const Sched& s, const Tile& ti, int t, int len, int b,
                              int et, int row, uint32_t tspare, volatile int* flags) {
  if (len == s.KB) return false;  // whole tile
  int bf, bl;
  sk_contributors(s, t, bf, bl);
  const int ncols = (ti.ntok + 15) & ~15;
  if ((bl - bf) * ncols > kTmemCols - kTmemSpare) return false;
  if (et == 0) {
    const bool done = ld_acquire_gpu(a.counter + t) + len == s.KB;
    if (done) a.counter[t] = 0;  // nobody else touches it in this launch
    flags[1] = done ? 2 : 0;
  }
  named_bar_sync(1, 128);
  if (flags[1] != 2) return false;
  int k = 0;
  for (int bb = bf; bb <= bl; ++bb) {
    if (bb == b) continue;
    const int wb = (t == sk_first_tile(s, bb)) ? 0 : 1;
    const float* pr = a.partial + (size_t)(bb * 2 + wb) * a.tokpad * kBM + row;
    for (int c = 0; c < ncols; c += 16) {
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (c + j < ti.ntok) ? __ldcg(pr + (size_t)(c + j) * kBM) : 0.f;
      tmem_st16(tspare + k * ncols + c, v);
    }
    ++k;
  }
  tmem_wait_st();
  return true;
}

// The finisher's sum of token columns [c0, c0 + 32) with prefetched partials:
// contributors bf..bl in order (own accumulator for this CTA), the same
// additions as reduce_partials.
PS_DEV void sum_prefetched(int bf, int bl, int self_b, int c0, int ncols, uint32_t tspare,
                           const float* own, float* v) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = 0.f;
  int k = 0;
  for (int bb = bf; bb <= bl; ++bb) {
    if (bb == self_b) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += own[j];
      continue;
    }
    float p[32];
    const uint32_t col = tspare + k * ncols + c0;
    tmem_ld16(col, p);
    if (c0 + 16 < ncols) tmem_ld16(col + 16, p + 16);
    else {
#pragma unroll
      for (int j = 16; j < 32; ++j) p[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += p[j];
    ++k;
  }
}

template <typename T>
PS_DEV void stage_residual(const Args& a, const Tile& ti, int et, int row, uint32_t tres,
                           float* xchg, const TileTokens& tk) {
  const T* res = reinterpret_cast<const T*>(a.residual);
  T* buf = reinterpret_cast<T*>(xchg);  // [32 tokens][128 features]
  if (a.scatter) named_bar_sync(2, 128);  // tk.idx of every token is staged
  for (int c32 = 0; c32 < ti.ntok; c32 += 32) {
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = et + k * 128;
      const int col = c32 + (i >> 4);
      const int n0 = ti.out0 + (i & 15) * 8;
      const int o = col < ti.ntok ? (a.scatter ? tk.idx[col] : ti.row0 + col) : -1;
      v[k] = make_uint4(0u, 0u, 0u, 0u);
      if (o >= 0 && o < a.M && n0 < a.N)
        v[k] = *reinterpret_cast<const uint4*>(res + (size_t)o * a.n_out + n0);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) reinterpret_cast<uint4*>(buf)[et + k * 128] = v[k];
    named_bar_sync(2, 128);
    float f[32];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) f[jj] = to_f32<T>(buf[jj * kBM + row]);
    tmem_st16(tres + c32, f);
    tmem_st16(tres + c32 + 16, f + 16);
    named_bar_sync(2, 128);  // the buffer is reused by the next 32 tokens / the epilogue
  }
  tmem_wait_st();
}

// Sum of the fp32 partials of tile t (contributors bf..bl, summed in that
// order: deterministic) for token columns [c0, c0 + 32) of this thread's tile
// row; ncol (16 or 32) columns are valid. Loads of two contributors x 32
// columns are issued before any add, so the last-arriving CTA pays one L2
// round trip per two contributors.
PS_DEV void reduce_partials(const float* partial, int tokpad, const Sched& s, int t, int bf,
                            int bl, int c0, int ncol, int row, float* v, int self_b,
                            bool use_own, const float* own) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = 0.f;
  for (int b0 = bf; b0 <= bl; b0 += 2) {
    float tv[2][32];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int bb = b0 + u;
      if (bb == self_b && use_own) {  // this CTA's own contribution, still in TMEM
#pragma unroll
        for (int j = 0; j < 32; ++j) tv[u][j] = own[j];
      } else if (bb <= bl) {
        const int wb = (t == sk_first_tile(s, bb)) ? 0 : 1;
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


// ------------------------------------------------------------ host side ----
struct Plan {
  int tokpad, stages, smem, grid, max_tiles;
  size_t counter_bytes, partial_bytes;
};

// Token tiles hold tokpad rows: M rounded to 16 (at most 128), or fewer when
// the caller bounds the rows of either model (`model_rows`, 0 = no bound):
// a narrower x tile per stage leaves room for more weight stages.
inline int tokpad_for(int M, int model_rows) {
  const int rows = model_rows > 0 ? min(M, model_rows) : M;
  return min(kMaxTok, max(16, round_up(rows, 16)));
}

inline Plan plan_for(int M, int N, int gated, int device, int model_rows = 0) {
  Plan p;
  p.tokpad = tokpad_for(M, model_rows);
  const int stage = kABytes + 2 * p.tokpad * 128;
  p.stages = min(kMaxStages, (kSmemLimit - kSmemFixed) / stage);
  p.smem = p.stages * stage + kSmemFixed;
  p.grid = sm_count(device);
  const int nt = gated ? cdiv(N / 2, 64) : cdiv(N, kBM);
  p.max_tiles = nt * (cdiv(max(M, 1), p.tokpad) + 1);
  p.counter_bytes = kCounterRegionBytes;
  p.partial_bytes = (size_t)p.grid * 2 * p.tokpad * kBM * sizeof(float);
  return p;
}

// Packed-weight layout of a [nmat, K, N] weight for an epilogue mode: weight
// tiles per model (128 columns, or 64 gate + 64 up for SwiGLU) and 128-k blocks.
inline void packed_layout(int K, int N, int gated, int* nt, int* KB) {
  *nt = gated ? cdiv(N / 2, 64) : cdiv(N, kBM);
  *KB = cdiv(K, kBK);
}

// Grid for a decode-sized launch (one token tile per model, pure stream-K) of
// `ntiles` output tiles x `KB` k blocks on `sms` SMs, measured on B200 at the
// tensor-parallel shard shapes of Llama-7B (us per launch, 148 SMs vs this
// choice): O 512 x 4096 8.4 vs 5.5 (64 CTAs, whole tiles), down 1376 x 4096
// 12.7 vs 9.7 (64, whole tiles), QKV 4096 x 1536 14.1 vs 12.4 (96, quarter
// tiles); projections with more work than 8 k blocks per SM keep every SM.
inline int auto_grid(int ntiles, int KB, int sms) {
  if (ntiles <= sms && KB <= 12) return max(ntiles, 1);  // whole tiles, no fix-up
  const long long I = (long long)ntiles * KB;
  if (I > 8ll * sms) return sms;
  for (int g = sms; g >= (sms + 1) / 2; --g) {  // equal pieces that split tiles evenly
    if (I % g) continue;
    const long long C = I / g;
    if (C % KB == 0 || KB % C == 0) return g;
  }
  return sms;
}

// Host side of one routed GEMM: argument checks, the launch plan, both tensor
// maps and the kernel arguments (everything but the stream-K workspace).
// PS_OK with *empty = true when M == 0 (nothing to launch).
inline int prepare_gemm(const void* x, const void* W, void* y, int M, int K, int N,
                        int split_point, const int32_t* counts, const ps_gemm_epilogue_t& e,
                        int dtype, int32_t* status, Plan* plan, CUtensorMap* tmw,
                        CUtensorMap* tmx, Args* args, bool* empty) {
  *empty = false;
  PS_CHECK_ARG(M >= 0 && K > 0 && N > 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  PS_CHECK_ARG(e.mode == PS_EPI_STORE || e.mode == PS_EPI_SWIGLU || e.mode == PS_EPI_QKV_ROPE);
  PS_CHECK_ARG(K % 8 == 0 && N % 8 == 0);
  const int gated = e.mode == PS_EPI_SWIGLU;
  const int rope = e.mode == PS_EPI_QKV_ROPE;
  if (gated) PS_CHECK_ARG(N % 16 == 0 && e.residual == nullptr);
  if (e.mode != PS_EPI_STORE) PS_CHECK_ARG(e.out_sumsq == nullptr);
  if (rope) {
    PS_CHECK_ARG(e.n_heads > 0 && N == 3 * e.n_heads * kBM);
    if (e.block_table)
      PS_CHECK_ARG(e.max_pages > 0 && e.page_size >= 8 && e.page_size <= 4096 &&
                   (e.page_size & (e.page_size - 1)) == 0 && (!e.kv_rows || e.table_rows > 0));
    else
      PS_CHECK_ARG(e.L_cap > 0);
    PS_CHECK_ARG(e.scatter_rows == nullptr && e.residual == nullptr && e.pos);
    PS_CHECK_ARG(!e.apply_rope || (e.rope_cos && e.rope_sin));
    PS_CHECK_ARG(e.slots0 >= 0 && e.slots1 >= 0);
    PS_CHECK_ARG((e.k_pool0 && e.v_pool0) || e.slots0 == 0);
    PS_CHECK_ARG((e.k_pool1 && e.v_pool1) || e.slots1 == 0);
  }
  if (e.in_sumsq) PS_CHECK_ARG(e.in_parts > 0 && e.norm_dim > 0 && e.eps >= 0.f);
  if (!counts) PS_CHECK_ARG(split_point >= 0 && split_point <= M);
  if (M == 0) {
    *empty = true;
    return PS_OK;
  }
  PS_CHECK_ARG(x && (W || e.w_packed) && y);
  PS_CHECK_ARG(aligned16(x) && aligned16(y) && (!W || aligned16(W)));
  PS_CHECK_ARG(!e.w_packed || aligned16(e.w_packed));
  PS_CHECK_ARG(!e.residual || aligned16(e.residual));
  if (rope)
    PS_CHECK_ARG((!e.k_pool0 || (aligned16(e.k_pool0) && aligned16(e.v_pool0))) &&
                 (!e.k_pool1 || (aligned16(e.k_pool1) && aligned16(e.v_pool1))));
  const int device = current_device();
  if (!is_sm100(device)) return PS_ERR_UNSUPPORTED;
  PS_CHECK_ARG(e.max_model_rows >= 0 && e.max_ctas >= -1);
  Plan p = plan_for(M, N, gated, device, e.max_model_rows);
  int cap = e.max_ctas;
  if (cap == -1) {  // by shape, for launches with one token tile per model
    const int rows = counts ? min(M, e.max_model_rows > 0 ? e.max_model_rows : M)
                            : max(split_point, M - split_point);
    const int models = counts ? 2 : (split_point > 0) + (split_point < M);
    if (rows <= p.tokpad) {
      const int nt = gated ? cdiv(N / 2, 64) : cdiv(N, kBM);
      cap = auto_grid(nt * models, cdiv(K, kBK), p.grid);
    } else {
      cap = 0;
    }
  }
  if (cap > 0 && cap < p.grid) {
    p.grid = cap;
    p.partial_bytes = (size_t)p.grid * 2 * p.tokpad * kBM * sizeof(float);
  }
  const long long iters = (long long)(gated ? cdiv(N / 2, 64) : cdiv(N, kBM)) *
                          (cdiv(M, p.tokpad) + 1) * cdiv(K, kBK);
  if (iters >= (1ll << 31) || p.max_tiles > kMaxCounters) return PS_ERR_UNSUPPORTED;

  CUtensorMap tw, tx;
  memset(&tw, 0, sizeof(tw));
  if (!e.w_packed) {
    // A single-model call (host split == M) reads W[0] only; W may then be [K, N].
    const uint64_t nmat = (!counts && split_point == M) ? 1 : 2;
    const uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, nmat};
    const uint64_t strides[2] = {(uint64_t)N * 2, (uint64_t)K * N * 2};
    const uint32_t box[3] = {64, (uint32_t)kBK, 1};
    // SwiGLU tiles read two 128-byte column strips that are not adjacent
    // (gate and up), so a 256-byte L2 fill would fetch a neighbour's half.
    if (!make_tmap_16bit(&tw, W, 3, dims, strides, box, dtype == PS_DTYPE_BF16,
                         gated ? 128 : 256))
      return PS_ERR_CUDA;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, (uint32_t)p.tokpad};  // one box per 64-k chunk of a tile
    if (!make_tmap_16bit(&tx, x, 2, dims, strides, box, dtype == PS_DTYPE_BF16))
      return PS_ERR_CUDA;
  }

  Args a{};
  a.y = y;
  a.residual = e.residual;
  a.counts = counts;
  a.scatter = e.scatter_rows;
  a.status = status;
  a.M = M;
  a.K = K;
  a.N = N;
  a.split_point = split_point;
  a.gated = gated;
  a.ff = gated ? N / 2 : 0;
  a.n_out = gated ? N / 2 : rope ? N / 3 : N;
  a.tokpad = p.tokpad;
  a.stages = p.stages;
  a.bf16 = dtype == PS_DTYPE_BF16;
  a.mode = e.mode;
  a.in_sumsq = e.in_sumsq;
  a.in_parts = e.in_parts;
  a.norm_inv_dim = e.in_sumsq ? 1.0f / (float)e.norm_dim : 0.f;
  a.eps = e.eps;
  a.out_sumsq = e.out_sumsq;
  a.out_parts = cdiv(N, kBM);
  a.kp0 = e.k_pool0;
  a.vp0 = e.v_pool0;
  a.kp1 = e.k_pool1;
  a.vp1 = e.v_pool1;
  a.pos = e.pos;
  a.rcos = e.rope_cos;
  a.rsin = e.rope_sin;
  a.n_heads = e.n_heads;
  a.L_cap = e.L_cap;
  a.slots0 = e.slots0;
  a.slots1 = e.slots1;
  a.apply_rope = e.apply_rope;
  a.bt = rope ? e.block_table : nullptr;
  a.max_pages = e.max_pages;
  a.page_size = e.page_size;
  a.table_rows = e.kv_rows ? e.table_rows : (e.table_rows > 0 ? e.table_rows : M);
  a.kv_rows = rope ? e.kv_rows : nullptr;
  a.wt = reinterpret_cast<const uint8_t*>(e.w_packed);
  packed_layout(K, N, gated, &a.wt_nt, &a.wt_KB);
  *plan = p;
  *tmw = tw;
  *tmx = tx;
  *args = a;
  return PS_OK;
}

}  // namespace gemm
}  // namespace ps
