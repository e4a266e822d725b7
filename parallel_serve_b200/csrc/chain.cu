// Projection chain on sm_100a: the routed GEMMs of one decode layer between two
// attentions (O + residual, gate_up + SwiGLU, down + residual, the next
// layer's QKV or the LM head) and, under tensor parallelism, the NVLink
// all-reduces of the row-split ones, in ONE persistent launch.
//
// Replaces the reference's per-projection launches of
// kernel/src/two_model_block_routed.py:138-152 (its routed GEMM,
// kernel/src/routed_gemm.py:60-149, once per projection, with RMSNorm,
// SwiGLU and residual kernels in between). Every GEMM job is computed exactly
// as the per-projection kernel (routed_gemm.cu) computes it — the same
// stream-K cut and summation order, so results are bit-identical — but the
// launch boundaries between projections are gone:
//
//  * dataflow instead of grid-wide waits: every 64-column part of a job's
//    output rows (per model), once final, is published by a release
//    increment of a counter. A later job waits only for what it reads: the
//    TMA producer checks, before loading a 128-k block of x, that the two
//    parts it covers are final; the epilogue waits for the parts its residual
//    tile reads and, for a folded RMSNorm, for all parts of the sums of
//    squares.
//  * weights never wait: the producer keeps two cursors over the CTA's
//    iterations, one issuing weight tiles (which depend on nothing) up to the
//    depth of the stage ring ahead of the other, which issues the x tiles as
//    their inputs become final. The tail of one projection (split-tile
//    fix-up, epilogue) overlaps the next projection's weight stream.
//  * fused all-reduce: an all-reduce job is worked by the epilogue warps, one
//    64-column part of one model's rows at a time: wait for the local partial
//    of that part, signal it to every peer (release store of the launch epoch
//    into the peer's flag), wait for every peer's flag, read the part from
//    every rank's symmetric slot over NVLink with 16-byte loads, sum ranks in
//    order 0..world-1 (bit-identical on every rank), add the residual, store
//    it and its sum of squares, publish the part. The producer and MMA warps
//    meanwhile stream the next GEMM's weights.
//
// All CTAs are resident (one per SM, 227 KB of shared memory each, grid = SM
// count), so a CTA may wait for another. Every wait is bounded by wall time;
// on timeout the kernel records PS_ERR_TIMEOUT, lets its own copies and MMAs
// land, frees TMEM and exits. The last CTA to exit clears the part counters
// and advances the launch epoch (consecutive launches are ordered by the
// stream; the next launch's dependent work starts after this grid completes).
#include <cuda_runtime.h>

#include <cstring>

#include "gemm_core.cuh"
#include "ps_common.cuh"
#include "ps_host.h"
#include "ps_peer.cuh"

namespace ps {
namespace chain {

using namespace gemm;
using ar::kMaxRanks;

constexpr int kMaxJobs = ar::kChainMaxJobs;
constexpr int kMaxUnits = ar::kChainMaxUnits;  // 64-column parts of one output row
constexpr int kMaxTilesPerJob = 4096;          // stream-K arrival counters per job
// Weight tiles the producer warms in L2 while its shared-memory loads are
// blocked behind an x tile that waits for the previous job's last parts: HBM
// keeps streaming the coming weights through that stall (up to 12 x 32 KB per
// SM beyond the loads). In steady state the warm-up cursor only keeps pace.
constexpr int kL2Ahead = 12;
constexpr int kKindGemm = PS_JOB_GEMM;
constexpr int kKindAllReduce = PS_JOB_ALLREDUCE;

// Workspace: [control][tile counters per job][stream-K partials per job]
constexpr size_t kReadyBytes = (size_t)kMaxJobs * 2 * kMaxUnits * 4;
constexpr size_t kTotalOffset = kReadyBytes;                     // int32 [kMaxJobs][2]
constexpr size_t kCtlOffset = kTotalOffset + 256;                // int32 [2]: exited, epoch
constexpr size_t kControlBytes = 32768;
constexpr size_t kCountersBytes = (size_t)kMaxJobs * kMaxTilesPerJob * 4;
constexpr size_t kPartialOffset = kControlBytes + kCountersBytes;
static_assert(kCtlOffset + 8 <= kControlBytes, "control region");

struct Job {
  Args a;  // GEMM: kernel arguments (a.counter / a.partial point at this job's regions)
  int kind;
  int x_from, norm_from, res_from;
  int out_units;  // 64-column parts of this job's output rows
  // all-reduce
  int src, slot, row_elems;
  void* out;
  const void* residual;
  float* out_sumsq;
};

struct Params {
  CUtensorMap tw[kMaxJobs];
  CUtensorMap tx[kMaxJobs];
  Job job[kMaxJobs];
  char* peer[kMaxRanks];
  const int32_t* counts;
  int32_t* status;
  int32_t* ready;        // [kMaxJobs][2][kMaxUnits]
  int32_t* ready_total;  // [kMaxJobs][2]
  int32_t* ctl;          // [0] CTAs exited, [1] launch epoch
  size_t flags_off;
  size_t slot_off[2];
  int n_jobs, M, tokpad, stages, bf16, rank, world;
};

// Kernel parameters are limited to 32764 bytes (4 KB keeps room to spare).
static_assert(sizeof(Params) <= 4096, "chain parameters");

PS_DEV void red_release_gpu_add(int32_t* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's generic-proxy global accesses with later async-proxy
// (TMA) accesses: on the writer before publishing, on the reader before
// issuing the TMA load of what it waited for.
PS_DEV void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

PS_DEV int32_t* ready_ptr(const Params& P, int j, int m) {
  return P.ready + (size_t)(j * 2 + m) * kMaxUnits;
}

PS_DEV int2 ld_acquire_gpu_v2(const int32_t* p) {
  int2 v;
  asm volatile("ld.acquire.gpu.global.v2.s32 {%0, %1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p)
               : "memory");
  return v;
}

// Bounded wait (one thread) until parts [u0, u1) of job j's output (model m) are final.
PS_DEV bool wait_parts(const Params& P, int j, int m, int u0, int u1) {
  const int nu = P.job[j].out_units;
  const int32_t* r = ready_ptr(P, j, m);
  for (int u = u0; u < u1 && u < nu; ++u) {
    if (ld_acquire_gpu(r + u) >= 1) continue;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_gpu(r + u) < 1) {
      __nanosleep(64);
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        set_status(P.status, PS_ERR_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// Bounded wait (one thread) until every part of job j's output (model m) is final.
PS_DEV bool wait_all_parts(const Params& P, int j, int m) {
  const int32_t* r = P.ready_total + j * 2 + m;
  const int nu = P.job[j].out_units;
  if (ld_acquire_gpu(r) >= nu) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_gpu(r) < nu) {
    __nanosleep(64);
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      set_status(P.status, PS_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Publish output columns [c_lo, c_hi) of job j, model m (all 128 epilogue
// threads, after their stores): each thread fences its stores against later
// TMA reads, the barrier gathers them, one thread releases the parts.
PS_DEV void publish_parts(const Params& P, int j, int m, int c_lo, int c_hi, int et) {
  fence_proxy_async_global();
  named_bar_sync(1, 128);
  if (et == 0) {
    fence_acq_rel_gpu();
    const int nu = P.job[j].out_units;
    int n = 0;
    for (int u = c_lo / 64; u * 64 < c_hi && u < nu; ++u) {
      red_release_gpu_add(ready_ptr(P, j, m) + u, 1);
      ++n;
    }
    if (n) red_release_gpu_add(P.ready_total + j * 2 + m, n);
  }
}

// Output columns a GEMM tile finalizes (row-space of y): STORE 128, SwiGLU 64
// (its gate / up column pairs become 64 outputs), QKV_ROPE 128 (q heads only
// land in y; k / v tiles publish parts past the output and nobody waits on them).
PS_DEV int tile_out_cols(const Args& a) { return a.gated ? 64 : kBM; }

// Cursor over one CTA's GEMM iterations across the jobs (the order in which
// the producer, MMA and epilogue roles walk them).
struct Cursor {
  int j, seg, g, end;  // segment [g, end) of job j's iteration space
  int kb, kb1;         // current piece: k-blocks [kb, kb1) of one tile
  int col0, col1, row0, m, n;  // the piece's tile (columns, first token row, model, tile)
  Sched s;
};

// The piece starting at iteration c.g (tile arithmetic once per piece, so
// that the per-stage step of the producer is a few additions).
PS_DEV void cur_piece(const Params& P, Cursor& c) {
  const int t = c.g / c.s.KB;
  c.kb = c.g % c.s.KB;
  c.kb1 = min(c.s.KB, c.kb + (c.end - c.g));
  const Tile ti = tile_of(P.job[c.j].a, c.s, t);
  c.col0 = ti.col0;
  c.col1 = ti.col1;
  c.row0 = ti.row0;
  c.m = ti.m;
  c.n = ti.n;
}

PS_DEV void cur_seek(const Params& P, int c0, int c1, int b, Cursor& c) {
  while (c.j < P.n_jobs) {
    if (P.job[c.j].kind == kKindGemm) {
      while (c.seg <= c.s.R) {
        int st, en;
        seg_range(c.s, b, c.seg, st, en);
        if (st < en) {
          c.g = st;
          c.end = en;
          cur_piece(P, c);
          return;
        }
        ++c.seg;
      }
    }
    ++c.j;
    c.seg = 0;
    if (c.j < P.n_jobs && P.job[c.j].kind == kKindGemm)
      sched_from_counts(P.job[c.j].a, c0, c1, (int)gridDim.x, c.s);
  }
}

PS_DEV void cur_begin(const Params& P, int c0, int c1, int b, Cursor& c) {
  c.j = 0;
  c.seg = 0;
  if (P.job[0].kind == kKindGemm) sched_from_counts(P.job[0].a, c0, c1, (int)gridDim.x, c.s);
  cur_seek(P, c0, c1, b, c);
}

PS_DEV void cur_next(const Params& P, int c0, int c1, int b, Cursor& c) {
  ++c.g;
  if (++c.kb < c.kb1) return;  // same tile
  if (c.g < c.end) {           // next tile of the segment
    cur_piece(P, c);
    return;
  }
  ++c.seg;
  cur_seek(P, c0, c1, b, c);
}

// One all-reduce job, worked by the 128 epilogue threads (et = 0..127). false:
// a wait ran out (status recorded; the decision is uniform over the threads).
template <typename T>
PS_DEV bool allreduce_job(const Params& P, int j, int c0, int c1, int epoch, int et) {
  const Job& J = P.job[j];
  const int upr = J.row_elems / 64;  // parts per row
  const int n0 = c0 > 0 ? upr : 0, n1 = c1 > 0 ? upr : 0;
  const int lane = et & 31;
  const unsigned group = 0xFFu << (lane & 24);  // the 8 lanes of one row's part
  for (int v = blockIdx.x; v < n0 + n1; v += gridDim.x) {
    const int m = v < n0 ? 0 : 1;
    const int u = v < n0 ? v : v - n0;
    const int r0 = m ? c0 : 0, nrows = m ? c1 : c0;
    bool ok = true;
    if (et == 0) {
      ok = wait_parts(P, J.src, m, u, u + 1);  // this rank's partial of the part
      if (ok && J.res_from >= 0 && J.residual) ok = wait_parts(P, J.res_from, m, u, u + 1);
    }
    if (named_bar_or(1, 128, !ok)) return false;
    // Signal the part to every rank, wait for every rank's signal. The release
    // is cumulative: the partial stores this thread acquired above (and the
    // barrier ordered) are visible to a peer that acquires the flag.
    const size_t fidx = ((size_t)(j * 2 + m) * kMaxUnits + u) * kMaxRanks;
    if (et < P.world) {
      const int r = et;
      ar::st_release_sys(reinterpret_cast<int*>(P.peer[r] + P.flags_off) + fidx + P.rank, epoch);
      const int* f = reinterpret_cast<const int*>(P.peer[P.rank] + P.flags_off) + fidx + r;
      if (ar::ld_acquire_sys(f) < epoch) {
        const uint64_t t0 = globaltimer_ns();
        while (ar::ld_acquire_sys(f) < epoch) {
          if (globaltimer_ns() - t0 > ar::kPeerWaitNs) {
            set_status(P.status, PS_ERR_TIMEOUT);
            ok = false;
            break;
          }
        }
      }
    }
    if (named_bar_or(1, 128, !ok)) return false;
    // 8 threads per row: 16 bytes (8 columns) each of the part's 64 columns.
    for (int i = et; i < nrows * 8; i += 128) {
      const int row = r0 + (i >> 3), vec = i & 7;
      const size_t e0 = (size_t)row * J.row_elems + (size_t)u * 64 + vec * 8;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
      if (J.residual)
        ar::add8<T>(acc, *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(J.residual) + e0));
      uint4 pv[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < P.world) pv[r] = ar::ld_cg_v4(P.peer[r] + P.slot_off[J.slot] + e0 * 2);
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < P.world) ar::add8<T>(acc, pv[r]);
      uint4 o;
      T* oh = reinterpret_cast<T*>(&o);
      float sq = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        oh[k] = from_f32<T>(acc[k]);
        const float f = to_f32<T>(oh[k]);
        sq += f * f;
      }
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(J.out) + e0) = o;
      if (J.out_sumsq) {  // fixed order: pairs, quads, the part's 8 vectors
        sq += __shfl_xor_sync(group, sq, 1);
        sq += __shfl_xor_sync(group, sq, 2);
        sq += __shfl_xor_sync(group, sq, 4);
        if (vec == 0) J.out_sumsq[(size_t)row * upr + u] = sq;
      }
    }
    publish_parts(P, j, m, u * 64, u * 64 + 64, et);
  }
  return true;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ Params P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = P.stages;
  const int tokpad = P.tokpad;
  const int xstage = 2 * tokpad * 128;
  uint8_t* sA = smem;
  uint8_t* sX = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + S * xstage);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  // [0] abort [1] split-tile finisher [2] c0 [3] c1 [4] epoch [5] last CTA out.
  // (No static shared memory: the dynamic part may use the whole 227 KB.)
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xchg = reinterpret_cast<float*>(full + 32);
  TileTokens& tk = *reinterpret_cast<TileTokens*>(xchg + 128 * 16);

  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
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
  if (warp == 0 && lane < P.n_jobs && P.job[lane].kind == kKindGemm) {
    if (!P.job[lane].a.wt) tma_prefetch_desc(&P.tw[lane]);
    tma_prefetch_desc(&P.tx[lane]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Before the dependency wait: warm L2 with the first weight tiles of this
  // CTA's range of the first job (weights are never written by a kernel).
  if (warp == 0 && lane == 0 && P.job[0].kind == kKindGemm) {
    Sched gs;
    guess_sched(P.job[0].a, gs);
    int g0, g1;
    seg_range(gs, b, 0, g0, g1);
    for (int g = g0, n = 0; g < g1 && n < kPrefetchStages; ++g, ++n) {
      const Tile ti = tile_of(P.job[0].a, gs, g / gs.KB);
      if (P.job[0].a.wt) {
        bulk_prefetch_l2(packed_block(P.job[0].a, ti.m, ti.n, g % gs.KB), kPackedTileBytes);
      } else {
        tma_prefetch_l2_3d(&P.tw[0], ti.col0, (g % gs.KB) * kBK, ti.m);
        tma_prefetch_l2_3d(&P.tw[0], ti.col1, (g % gs.KB) * kBK, ti.m);
      }
    }
  }
  pdl_wait();
  if (threadIdx.x == 0) {
    pdl_launch_dependents();
    int c0 = P.counts[0], c1 = P.counts[1];
    // one token tile per model: each 64-column part has one producing tile
    if (c0 < 0 || c1 < 0 || c0 + c1 > P.M || c0 > tokpad || c1 > tokpad) {
      if (b == 0) set_status(P.status, PS_ERR_BAD_INDEX);
      c0 = c1 = 0;
    }
    flags[2] = c0;
    flags[3] = c1;
    flags[4] = P.ctl[1] + 1;  // the last CTA of the previous launch advanced it
  }
  __syncthreads();
  const int c0 = flags[2], c1 = flags[3], epoch = flags[4];

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint32_t tx_bytes = kABytes + 2u * (uint32_t)tokpad * 128u;
      Cursor wc, xc, pc;  // weights, x, L2 warm-up
      cur_begin(P, c0, c1, b, wc);
      cur_begin(P, c0, c1, b, xc);
      cur_begin(P, c0, c1, b, pc);
      int w_it = 0, x_it = 0, p_it = 0;
      bool fail = false;
      // Readiness is cached: all_done[m] = the x job whose producer has
      // published every part for model m (one counter read per job in the
      // usual case instead of two L2 round trips per 128-k block).
      int all_done[2] = {-1, -1};
      bool need_fence = false;
      uint64_t idle_since = 0;  // %globaltimer is read only while nothing progresses
      while (xc.j < P.n_jobs) {
        bool prog = false;
        // L2 warm-up: kept level with the weight loads, run ahead of them (up
        // to kL2Ahead stages) only while they are blocked behind x
        if (pc.j < P.n_jobs) {
          if (p_it < w_it) {
            ++p_it;
            cur_next(P, c0, c1, b, pc);
          } else if (w_it >= x_it + S && p_it < w_it + kL2Ahead) {
            const Args& pa = P.job[pc.j].a;
            if (pa.wt) {
              bulk_prefetch_l2(packed_block(pa, pc.m, pc.n, pc.kb), kPackedTileBytes);
            } else {
              tma_prefetch_l2_3d(&P.tw[pc.j], pc.col0, pc.kb * kBK, pc.m);
              tma_prefetch_l2_3d(&P.tw[pc.j], pc.col1, pc.kb * kBK, pc.m);
            }
            ++p_it;
            cur_next(P, c0, c1, b, pc);
          }
        }
        // weights: up to S stages ahead of the x tiles, whatever the x tiles wait for
        if (wc.j < P.n_jobs && w_it < x_it + S) {
          const int st = w_it % S;
          if (mbar_test_wait(empty + st, ((w_it / S) & 1) ^ 1)) {
            mbar_arrive_expect_tx(full + st, tx_bytes);
            uint8_t* dA = sA + st * kABytes;
            const Args& wa = P.job[wc.j].a;
            if (wa.wt) {  // packed: the stage's 32 KB image, one bulk copy
              bulk_load(dA, packed_block(wa, wc.m, wc.n, wc.kb), kPackedTileBytes, full + st,
                        pol_w);
            } else {
              tma_load_3d(dA, &P.tw[wc.j], full + st, wc.col0, wc.kb * kBK, wc.m, pol_w);
              tma_load_3d(dA + kAHalf, &P.tw[wc.j], full + st, wc.col1, wc.kb * kBK, wc.m,
                          pol_w);
            }
            ++w_it;
            cur_next(P, c0, c1, b, wc);
            prog = true;
          }
        }
        // x: once the 128-k block it covers is final
        if (x_it < w_it) {
          const int xf = P.job[xc.j].x_from;
          bool rdy = xf < 0 || all_done[xc.m] == xc.j;
          if (!rdy) {
            // the block's two parts (adjacent counters, one 8-byte load) and
            // the job's total, both in flight at once
            need_fence = true;
            const int nu = P.job[xf].out_units;
            const int2 pr = ld_acquire_gpu_v2(ready_ptr(P, xf, xc.m) + 2 * xc.kb);
            const int tot = ld_acquire_gpu(P.ready_total + xf * 2 + xc.m);
            if (tot >= nu) {
              all_done[xc.m] = xc.j;
              rdy = true;
            } else {
              rdy = (2 * xc.kb >= nu || pr.x >= 1) && (2 * xc.kb + 1 >= nu || pr.y >= 1);
            }
          }
          if (rdy) {
            if (need_fence) {  // what the acquire made visible, before the TMA reads it
              fence_proxy_async_global();
              need_fence = false;
            }
            const int st = x_it % S;
            uint8_t* dX = sX + st * xstage;
            tma_load_2d(dX, &P.tx[xc.j], full + st, xc.kb * kBK, xc.row0, pol_x);
            tma_load_2d(dX + tokpad * 128, &P.tx[xc.j], full + st, xc.kb * kBK + 64, xc.row0,
                        pol_x);
            ++x_it;
            cur_next(P, c0, c1, b, xc);
            prog = true;
          }
        }
        if (prog) {
          idle_since = 0;
        } else if (flags[0]) {  // another role gave up
          fail = true;
          break;
        } else {
          const uint64_t now = globaltimer_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > kWaitLimitNs) {
            set_status(P.status, PS_ERR_TIMEOUT);
            flags[0] = 1;
            fail = true;
            break;
          }
          __nanosleep(32);  // spare the L2 lines being polled
        }
      }
      if (fail) {
        // Stages whose weights are in flight expect their x bytes too: load
        // those x tiles regardless (the contents are not used) so every copy
        // this thread started lands before the CTA exits.
        while (x_it < w_it) {
          const int st = x_it % S;
          uint8_t* dX = sX + st * xstage;
          tma_load_2d(dX, &P.tx[xc.j], full + st, xc.kb * kBK, xc.row0, pol_x);
          tma_load_2d(dX + tokpad * 128, &P.tx[xc.j], full + st, xc.kb * kBK + 64, xc.row0,
                      pol_x);
          ++x_it;
          cur_next(P, c0, c1, b, xc);
        }
        for (int st = 0; st < S && st < w_it; ++st) {
          const int last = st + S * ((w_it - 1 - st) / S);
          mbar_wait(full + st, (last / S) & 1, P.status);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issue
    if (lane == 0) {
      int it = 0, acc_it = 0;
      for (int j = 0; j < P.n_jobs && !flags[0]; ++j) {
        const Job& J = P.job[j];
        if (J.kind != kKindGemm) continue;
        Sched s;
        sched_from_counts(J.a, c0, c1, (int)gridDim.x, s);
        for (int seg = 0; seg <= s.R && !flags[0]; ++seg) {
          int start, end;
          seg_range(s, b, seg, start, end);
          for (int g = start; g < end && !flags[0];) {
            const int t = g / s.KB, kb0 = g % s.KB;
            const int kb1 = min(s.KB, kb0 + (end - g));
            const Tile ti = tile_of(J.a, s, t);
            const int n16 = (ti.ntok + 15) & ~15;
            const uint32_t idesc = idesc_f16(P.bf16, /*A MN-major*/ 1, /*B K-major*/ 0, kBM, n16);
            const int ab = acc_it & 1;
            if (!mbar_wait(acc_empty + ab, ((acc_it >> 1) & 1) ^ 1, P.status)) {
              flags[0] = 1;
              break;
            }
            tc_fence_after();
            const uint32_t d = tmem + ab * kMaxTok;
            for (int kb = kb0; kb < kb1; ++kb) {
              const int st = it % S;
              if (!mbar_wait(full + st, (it / S) & 1, P.status)) {
                flags[0] = 1;
                break;
              }
              tc_fence_after();
              const uint32_t aaddr = smem_u32(sA + st * kABytes);
              const uint32_t xaddr = smem_u32(sX + st * xstage);
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk) {
                const uint64_t ad = smem_desc_sw128(aaddr + kk * 2048, kAHalf, 1024);
                const uint64_t bd =
                    smem_desc_sw128(xaddr + (kk >> 2) * (tokpad * 128) + (kk & 3) * 32, 16, 1024);
                umma_f16(d, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
              }
              umma_commit(empty + st);
              ++it;
            }
            umma_commit(acc_full + ab);
            ++acc_it;
            g += kb1 - kb0;
          }
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, P.status);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int et = threadIdx.x - 64;
    const uint32_t tres = tmem + kTmemResidual + ((uint32_t)(q * 32) << 16);
    const uint32_t tspare = tmem + kTmemSpare + ((uint32_t)(q * 32) << 16);
    int acc_it = 0;
    bool stop = false;  // uniform over the 128 epilogue threads
    for (int j = 0; j < P.n_jobs && !stop; ++j) {
      const Job& J = P.job[j];
      if (J.kind == kKindAllReduce) {
        if (!allreduce_job<T>(P, j, c0, c1, epoch, et)) {
          flags[0] = 1;
          stop = true;
        }
        continue;
      }
      const Args& a = J.a;
      const bool stage_tokens = a.in_sumsq || a.scatter || a.mode == PS_EPI_QKV_ROPE;
      Sched s;
      sched_from_counts(a, c0, c1, (int)gridDim.x, s);
      for (int seg = 0; seg <= s.R && !stop; ++seg) {
        int start, end;
        seg_range(s, b, seg, start, end);
        for (int g = start; g < end;) {
          const int t = g / s.KB, kb0 = g % s.KB;
          const int kb1 = min(s.KB, kb0 + (end - g));
          const Tile ti = tile_of(a, s, t);
          const int nchunk = (ti.ntok + 15) >> 4;
          const int ab = acc_it & 1;
          // Inputs of the epilogue written earlier in this launch: the folded
          // norm's sums of squares (all parts) and the residual tile's parts.
          bool dep_ok = true;
          if (et == 0) {
            if (J.norm_from >= 0 && a.in_sumsq) dep_ok = wait_all_parts(P, J.norm_from, ti.m);
            if (dep_ok && J.res_from >= 0 && a.residual)
              dep_ok = wait_parts(P, J.res_from, ti.m, ti.out0 / 64, (ti.out0 + kBM) / 64);
          }
          if (named_bar_or(1, 128, !dep_ok)) {
            flags[0] = 1;
            stop = true;
            break;
          }
          if (stage_tokens) tile_tokens(a, s, ti, et, tk);
          if (a.residual) stage_residual<T>(a, ti, et, row, tres, xchg, tk);
          // Split tile whose other contributors have all published already: this CTA
          // is the finisher, and their partials are loaded into spare TMEM while this
          // piece's MMAs still run (off the tail's critical path).
          const bool pre = prefetch_partials(a, s, ti, t, kb1 - kb0, b, et, row, tspare, flags);
          const bool ok = !flags[0] && mbar_wait(acc_full + ab, (acc_it >> 1) & 1, P.status);
          if (named_bar_or(1, 128, !ok)) {
            flags[0] = 1;
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem + ab * kMaxTok + ((uint32_t)(q * 32) << 16);
          bool finished = false;
          if (kb0 == 0 && kb1 == s.KB) {
            for (int c = 0; c < nchunk; ++c) {
              float v[16];
              tmem_ld16(taddr + c * 16, v);
              finalize<T>(a, s, ti, row, c * 16, v, xchg, tk, tres);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + ab);
            finished = true;
          } else {
            const int len = kb1 - kb0;
            if (!pre && et == 0) {
              const bool done = ld_acquire_gpu(a.counter + t) + len == s.KB;
              if (done) a.counter[t] = 0;
              flags[1] = done ? 2 : 0;
            }
            if (!pre) named_bar_sync(1, 128);
            const bool fast = flags[1] == 2;
            if (!fast) {
              const int which = (t == sk_first_tile(s, b)) ? 0 : 1;
              const uint64_t keep = l2_policy_evict_last();
              float* pw = a.partial + (size_t)(b * 2 + which) * tokpad * kBM;
              for (int c = 0; c < nchunk; ++c) {
                float v[16];
                tmem_ld16(taddr + c * 16, v);
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                  st_global_keep(pw + (size_t)(c * 16 + jj) * kBM + row, v[jj], keep);
              }
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(acc_empty + ab);
              named_bar_sync(1, 128);
              if (et == 0) {
                fence_acq_rel_gpu();
                const int old = atom_add_acq_rel_gpu(a.counter + t, len);
                const int last = (old + len == s.KB) ? 1 : 0;
                if (last) a.counter[t] = 0;
                flags[1] = last;
              }
              named_bar_sync(1, 128);
            }
            if (fast || flags[1]) {
              int bf, bl;
              sk_contributors(s, t, bf, bl);
              for (int c = 0; c < nchunk; c += 2) {
                float v[32], own[32];
                const int ncol = (c + 1 < nchunk) ? 32 : 16;
                if (fast) {
                  tmem_ld16(taddr + c * 16, own);
                  tmem_ld16(taddr + c * 16 + 16, own + 16);
                } else {
#pragma unroll
                  for (int jj = 0; jj < 32; ++jj) own[jj] = 0.f;
                }
                if (pre)
                  sum_prefetched(bf, bl, b, c * 16, (ti.ntok + 15) & ~15, tspare, own, v);
                else
                  reduce_partials(a.partial, tokpad, s, t, bf, bl, c * 16, ncol, row, v, b, fast,
                                  own);
                finalize<T>(a, s, ti, row, c * 16, v, xchg, tk, tres);
                if (ncol == 32) finalize<T>(a, s, ti, row, c * 16 + 16, v + 16, xchg, tk, tres);
              }
              finished = true;
            }
            if (fast) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(acc_empty + ab);
            }
          }
          if (finished) publish_parts(P, j, ti.m, ti.out0, ti.out0 + tile_out_cols(a), et);
          if (stage_tokens) named_bar_sync(2, 128);  // tk is rewritten for the next tile
          ++acc_it;
          g += kb1 - kb0;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // The last CTA to leave clears the part counters and advances the epoch.
  if (threadIdx.x == 0) {
    fence_acq_rel_gpu();
    flags[5] = atom_add_acq_rel_gpu(P.ctl, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (flags[5]) {
    for (int i = threadIdx.x; i < P.n_jobs * 2 * kMaxUnits; i += blockDim.x) P.ready[i] = 0;
    if (threadIdx.x < P.n_jobs * 2) P.ready_total[threadIdx.x] = 0;
    __syncthreads();
    if (threadIdx.x == 0) {
      P.ctl[0] = 0;
      P.ctl[1] = epoch;
      __threadfence();
    }
  }
}

}  // namespace chain
}  // namespace ps

using namespace ps;

extern "C" size_t ps_routed_chain_workspace_bytes(int M, int n_jobs, int device) {
  if (M <= 0 || n_jobs < 1 || n_jobs > chain::kMaxJobs) return 0;
  const int tokpad = gemm::tokpad_for(M, 0);  // the largest the jobs can ask for
  const size_t per_job = (size_t)sm_count(device) * 2 * tokpad * gemm::kBM * sizeof(float);
  return chain::kPartialOffset + (size_t)n_jobs * per_job;
}

extern "C" int ps_routed_chain(const ps_chain_job_t* jobs, int n_jobs, int M,
                               const int32_t* counts, void* const* peer_bases, int rank,
                               int world, size_t slot_bytes, int dtype, void* workspace,
                               size_t workspace_bytes, int32_t* status, ps_stream_t stream) {
  using namespace chain;
  PS_CHECK_ARG(jobs && n_jobs >= 1 && n_jobs <= kMaxJobs);
  PS_CHECK_ARG(M >= 0 && M <= 2 * gemm::kMaxTok && counts);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  PS_CHECK_ARG(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world);
  if (M == 0) return PS_OK;
  const int device = current_device();
  if (!is_sm100(device)) return PS_ERR_UNSUPPORTED;
  const size_t need = ps_routed_chain_workspace_bytes(M, n_jobs, device);
  if (!workspace || workspace_bytes < need) return PS_ERR_WORKSPACE;
  PS_CHECK_ARG(aligned16(workspace));

  Params P;  // passed by value: the launch copies it
  memset(&P, 0, sizeof(P));
  P.n_jobs = n_jobs;
  P.M = M;
  P.counts = counts;
  P.status = status;
  P.bf16 = dtype == PS_DTYPE_BF16;
  P.rank = rank;
  P.world = world;
  char* ws = reinterpret_cast<char*>(workspace);
  P.ready = reinterpret_cast<int32_t*>(ws);
  P.ready_total = reinterpret_cast<int32_t*>(ws + kTotalOffset);
  P.ctl = reinterpret_cast<int32_t*>(ws + kCtlOffset);
  const bool has_ar = [&] {
    for (int j = 0; j < n_jobs; ++j)
      if (jobs[j].kind == kKindAllReduce) return true;
    return false;
  }();
  if (has_ar) {
    PS_CHECK_ARG(peer_bases && slot_bytes % 256 == 0);
    for (int r = 0; r < world; ++r) {
      PS_CHECK_ARG(peer_bases[r] && aligned16(peer_bases[r]));
      P.peer[r] = reinterpret_cast<char*>(peer_bases[r]);
    }
    P.flags_off = ar::chain_flags_offset(slot_bytes);
    P.slot_off[0] = ar::slot_offset(0, slot_bytes);
    P.slot_off[1] = ar::slot_offset(1, slot_bytes);
  }
  const size_t per_job = (need - kPartialOffset) / n_jobs;
  gemm::Plan plan{};
  bool have_plan = false;
  for (int j = 0; j < n_jobs; ++j) {
    const ps_chain_job_t& in = jobs[j];
    Job& J = P.job[j];
    J.kind = in.kind;
    J.x_from = in.x_from;
    J.norm_from = in.norm_from;
    J.res_from = in.res_from;
    PS_CHECK_ARG(in.x_from >= -1 && in.x_from < j && in.norm_from >= -1 && in.norm_from < j &&
                 in.res_from >= -1 && in.res_from < j);
    if (in.kind == kKindGemm) {
      gemm::Plan p;
      bool empty;
      const int rc = gemm::prepare_gemm(in.x, in.W, in.y, M, in.K, in.N, 0, counts, in.epi, dtype,
                                        status, &p, &P.tw[j], &P.tx[j], &J.a, &empty);
      if (rc != PS_OK) return rc;
      if (p.max_tiles > kMaxTilesPerJob) return PS_ERR_UNSUPPORTED;
      J.out_units = cdiv(J.a.n_out, 64);
      PS_CHECK_ARG(J.out_units <= kMaxUnits && in.epi.scatter_rows == nullptr &&
                   in.epi.max_ctas == 0);  // one grid for the whole chain
      J.a.counter = reinterpret_cast<int32_t*>(ws + kControlBytes) + (size_t)j * kMaxTilesPerJob;
      J.a.partial = reinterpret_cast<float*>(ws + kPartialOffset + (size_t)j * per_job);
      if (have_plan) PS_CHECK_ARG(p.tokpad == plan.tokpad);  // one stage layout per launch
      plan = p;
      have_plan = true;
      if (in.x_from >= 0) {  // x is that job's output: same buffer, K = its row length
        const ps_chain_job_t& src = jobs[in.x_from];
        const void* produced = src.kind == kKindGemm ? src.y : src.out;
        const int width = src.kind == kKindGemm ? P.job[in.x_from].a.n_out : src.row_elems;
        PS_CHECK_ARG(produced == in.x && width == in.K);
      }
    } else {
      PS_CHECK_ARG(in.kind == kKindAllReduce && has_ar);
      PS_CHECK_ARG(in.src >= 0 && in.src < j && jobs[in.src].kind == kKindGemm);
      PS_CHECK_ARG(in.slot == 0 || in.slot == 1);
      PS_CHECK_ARG(in.row_elems > 0 && in.row_elems % 64 == 0 && in.out && aligned16(in.out));
      PS_CHECK_ARG(!in.residual || aligned16(in.residual));
      PS_CHECK_ARG((size_t)M * in.row_elems * 2 <= slot_bytes);
      // the source GEMM writes its partial, row_elems wide, into this rank's slot
      PS_CHECK_ARG(jobs[in.src].y == P.peer[rank] + P.slot_off[in.slot] &&
                   P.job[in.src].a.n_out == in.row_elems);
      J.src = in.src;
      J.slot = in.slot;
      J.row_elems = in.row_elems;
      J.out = in.out;
      J.residual = in.residual;
      J.out_sumsq = in.out_sumsq;
      J.out_units = in.row_elems / 64;
      PS_CHECK_ARG(J.out_units <= kMaxUnits);
    }
  }
  PS_CHECK_ARG(have_plan);
  P.tokpad = plan.tokpad;
  P.stages = plan.stages;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PS_DTYPE_BF16) {
    PS_CUDA_RET(allow_dynamic_smem(chain_kernel<__nv_bfloat16>, gemm::kSmemLimit));
    PS_CUDA_RET(launch(chain_kernel<__nv_bfloat16>, dim3(sm_count(device)),
                       dim3(gemm::kThreads), plan.smem, st, P));
  } else {
    PS_CUDA_RET(allow_dynamic_smem(chain_kernel<__half>, gemm::kSmemLimit));
    PS_CUDA_RET(launch(chain_kernel<__half>, dim3(sm_count(device)), dim3(gemm::kThreads),
                       plan.smem, st, P));
  }
  return PS_OK;
}
