// Routed two-model GEMM on sm_100a: tcgen05 MMA with TMEM accumulators, operands
// staged by TMA, one persistent CTA per SM.
//
// Replaces the Triton `_routed_gemm_kernel` (kernel/src/routed_gemm.py:60-149)
// and its v1 (experiments/routed_linear_n2.py:33-115). Semantics are the same
// — y[:c0] = x[:c0] @ W[0], y[c0:] = x[c0:] @ W[1], fp32 accumulation — but
// the schedule is built for decode-sized M on B200:
//
//  * swap-AB: a tile is 128 weight columns (the MMA M dimension) by up to 128
//    tokens of ONE model (the MMA N dimension, rounded up to 16). W stays in
//    its reference layout [2, K, N] (N contiguous) and is consumed MN-major;
//    x [M, K] is consumed K-major. No tile ever straddles the split, so the
//    reference's two-pass straddle path (routed_gemm.py:112-146) and its
//    double weight read do not exist here.
//  * the split (c0, c1) is read on the device, so a captured CUDA graph serves
//    every split; a model with no tokens contributes no tiles and its weights
//    are not read.
//  * stream-K: the (tile, k-block) iteration space is cut into equal
//    contiguous ranges, one per CTA, so all 148 SMs stream weights even when a
//    projection has only 64 output tiles. A tile split across CTAs is reduced
//    by its last-arriving CTA in fixed contributor order (deterministic).
//    With more than 128 tokens per model (prefill chunks, large batches), the
//    first whole rounds of tiles go data-parallel so that a weight tile's
//    token tiles run side by side and its weights are fetched once (Sched).
//  * warp roles: warp 0 issues TMA, warp 1 issues MMA (one thread each),
//    warps 2-5 drain TMEM (double-buffered accumulators) and run the epilogue
//    (store / residual add / row scatter / fused SwiGLU).
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "ps_common.cuh"
#include "ps_host.h"

#include "gemm_core.cuh"

namespace ps {
namespace gemm {

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    routed_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                       const __grid_constant__ CUtensorMap tmap_x, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  const int xstage = 2 * a.tokpad * 128;  // two 64-wide k chunks of tokpad rows
  uint8_t* sA = smem;
  uint8_t* sX = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + S * xstage);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort [1] last
  float* xchg = reinterpret_cast<float*>(full + 32);
  TileTokens& tk = *reinterpret_cast<TileTokens*>(xchg + 128 * 16);
  const bool stage_tokens = a.in_sumsq || a.scatter || a.mode == PS_EPI_QKV_ROPE;

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
  if (warp == 0 && lane == 0) {
    if (!a.wt) tma_prefetch_desc(&tmap_w);
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

  // Before the dependency wait: warm L2 with the first weight tiles of this
  // CTA's range (weights are never written by a preceding kernel). CTAs that
  // start while the previous kernel finishes its split tiles keep HBM busy
  // through that tail; kPrefetchStages tiles cover its few microseconds.
  //
  // With a host split the schedule is exact before the wait, so the first S
  // stages' weights go straight into shared memory (`early` of them); only
  // their x tiles, written by the preceding kernel, wait for it.
  int early = 0;
  if (warp == 0 && lane == 0) {
    Sched gs;
    guess_sched(a, gs);
    int g0, g1;
    seg_range(gs, b, 0, g0, g1);
    const uint32_t tx = kABytes + 2u * (uint32_t)a.tokpad * 128u;
    const uint64_t pol_w = l2_policy_evict_first();
    for (int g = g0, n = 0; g < g1 && n < kPrefetchStages; ++g, ++n) {
      const Tile ti = tile_of(a, gs, g / gs.KB);
      const int kb = g % gs.KB;
      if (!a.counts && n < S && g - g0 == n) {  // exact schedule: load the stage itself
        mbar_arrive_expect_tx(full + n, tx);
        uint8_t* dA = sA + n * kABytes;
        if (a.wt) {
          bulk_load(dA, packed_block(a, ti.m, ti.n, kb), kPackedTileBytes, full + n, pol_w);
        } else {
          tma_load_3d(dA, &tmap_w, full + n, ti.col0, kb * kBK, ti.m, pol_w);
          tma_load_3d(dA + kAHalf, &tmap_w, full + n, ti.col1, kb * kBK, ti.m, pol_w);
        }
        ++early;
      } else if (a.wt) {
        bulk_prefetch_l2(packed_block(a, ti.m, ti.n, kb), kPackedTileBytes);
      } else {
        tma_prefetch_l2_3d(&tmap_w, ti.col0, kb * kBK, ti.m);
        tma_prefetch_l2_3d(&tmap_w, ti.col1, kb * kBK, ti.m);
      }
    }
  }
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();

  Sched s;
  make_sched(a, s);
  int first_start, first_end;
  seg_range(s, b, 0, first_start, first_end);

  if (first_start >= first_end) {
    // no work for this CTA
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      int it = 0;
      for (int seg = 0; seg <= s.R && !flags[0]; ++seg) {
        int start, end;
        seg_range(s, b, seg, start, end);
        for (int g = start; g < end && !flags[0];) {
          const int t = g / s.KB, kb0 = g % s.KB;
          const int kb1 = min(s.KB, kb0 + (end - g));
          const Tile ti = tile_of(a, s, t);
          // x: one box of tokpad rows per 64-k chunk. Rows past the tile's
          // tokens (the other model's, or zero fill past M) land in columns
          // the MMA's N = ntok rounded to 16 reads at most partly and the
          // epilogue never stores.
          const uint32_t tx = kABytes + 2u * (uint32_t)a.tokpad * 128u;
          for (int kb = kb0; kb < kb1; ++kb) {
            const int st = it % S;
            const uint32_t ph = (it / S) & 1;
            if (it >= early) {  // (the first `early` stages' weights are in flight already)
              if (!mbar_wait(empty + st, ph ^ 1, a.status)) {
                flags[0] = 1;
                break;
              }
              mbar_arrive_expect_tx(full + st, tx);
              uint8_t* dA = sA + st * kABytes;
              if (a.wt) {  // packed: the stage's 32 KB image, one bulk copy
                bulk_load(dA, packed_block(a, ti.m, ti.n, kb), kPackedTileBytes, full + st,
                          pol_w);
              } else {
                tma_load_3d(dA, &tmap_w, full + st, ti.col0, kb * kBK, ti.m, pol_w);
                tma_load_3d(dA + kAHalf, &tmap_w, full + st, ti.col1, kb * kBK, ti.m, pol_w);
              }
            }
            uint8_t* dX = sX + st * xstage;
            tma_load_2d(dX, &tmap_x, full + st, kb * kBK, ti.row0, pol_x);
            tma_load_2d(dX + a.tokpad * 128, &tmap_x, full + st, kb * kBK + 64, ti.row0, pol_x);
            ++it;
          }
          g += kb1 - kb0;
        }
      }
      if (flags[0]) {
        // Let every copy this thread issued land before the CTA exits. Stages
        // whose weights went out before the wait but whose x did not still
        // expect their x bytes: load those x tiles too (contents unused).
        for (int k = it; k < early; ++k) {
          const Tile ti = tile_of(a, s, (first_start + k) / s.KB);
          const int kb = (first_start + k) % s.KB;
          uint8_t* dX = sX + k * xstage;
          tma_load_2d(dX, &tmap_x, full + k, kb * kBK, ti.row0, pol_x);
          tma_load_2d(dX + a.tokpad * 128, &tmap_x, full + k, kb * kBK + 64, ti.row0, pol_x);
        }
        const int issued = it > early ? it : early;
        for (int st = 0; st < S && st < issued; ++st) {
          const int last = st + S * ((issued - 1 - st) / S);
          mbar_wait(full + st, (last / S) & 1, a.status);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issue
    if (lane == 0) {
      int it = 0, acc_it = 0;
      for (int seg = 0; seg <= s.R && !flags[0]; ++seg) {
        int start, end;
        seg_range(s, b, seg, start, end);
        for (int g = start; g < end && !flags[0];) {
          const int t = g / s.KB, kb0 = g % s.KB;
          const int kb1 = min(s.KB, kb0 + (end - g));
          const Tile ti = tile_of(a, s, t);
          const int n16 = (ti.ntok + 15) & ~15;
          const uint32_t idesc = idesc_f16(a.bf16, /*A MN-major*/ 1, /*B K-major*/ 0, kBM, n16);
          const int ab = acc_it & 1;
          if (!mbar_wait(acc_empty + ab, ((acc_it >> 1) & 1) ^ 1, a.status)) {
            flags[0] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + ab * kMaxTok;
          for (int kb = kb0; kb < kb1; ++kb) {
            const int st = it % S;
            if (!mbar_wait(full + st, (it / S) & 1, a.status)) {
              flags[0] = 1;
              break;
            }
            tc_fence_after();
            const uint32_t aaddr = smem_u32(sA + st * kABytes);
            const uint32_t xaddr = smem_u32(sX + st * xstage);
  #pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              // A: MN-major, 128B swizzle; 16 k-rows of 128 B per MMA step,
              //    LBO = distance between the two 64-column boxes.
              const uint64_t ad = smem_desc_sw128(aaddr + kk * 2048, kAHalf, 1024);
              // B: K-major, 128B swizzle; 32 B per 16-element k step inside
              //    a 64-element chunk, chunks tokpad*128 B apart.
              const uint64_t bd =
                  smem_desc_sw128(xaddr + (kk >> 2) * (a.tokpad * 128) + (kk & 3) * 32, 16, 1024);
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
      // Every MMA of this CTA completes before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, a.status);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    const int et = threadIdx.x - 64;
    const uint32_t tres = tmem + kTmemResidual + ((uint32_t)(q * 32) << 16);
    const uint32_t tspare = tmem + kTmemSpare + ((uint32_t)(q * 32) << 16);
    int acc_it = 0;
    bool stop = false;  // uniform over the 128 epilogue threads
    for (int seg = 0; seg <= s.R && !stop; ++seg) {
      int start, end;
      seg_range(s, b, seg, start, end);
      for (int g = start; g < end;) {
        const int t = g / s.KB, kb0 = g % s.KB;
        const int kb1 = min(s.KB, kb0 + (end - g));
        const Tile ti = tile_of(a, s, t);
        const int nchunk = (ti.ntok + 15) >> 4;
        const int ab = acc_it & 1;
        // The previous tile's readers of tk finished at its closing barrier; the
        // barrier below publishes these values before the accumulator is read.
        if (stage_tokens) tile_tokens(a, s, ti, et, tk);
        if (a.residual) stage_residual<T>(a, ti, et, row, tres, xchg, tk);
        // Split tile whose other contributors have all published already: this CTA
        // is the finisher, and their partials are loaded into spare TMEM while this
        // piece's MMAs still run (off the tail's critical path).
        const bool pre = prefetch_partials(a, s, ti, t, kb1 - kb0, b, et, row, tspare, flags);
        const bool ok = !flags[0] && mbar_wait(acc_full + ab, (acc_it >> 1) & 1, a.status);
        // The abort decision must be uniform across the 128 epilogue threads.
        if (named_bar_or(1, 128, !ok)) {
          flags[0] = 1;
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + ab * kMaxTok + ((uint32_t)(q * 32) << 16);
        if (kb0 == 0 && kb1 == s.KB) {
          for (int c = 0; c < nchunk; ++c) {
            float v[16];
            tmem_ld16(taddr + c * 16, v);
            finalize<T>(a, s, ti, row, c * 16, v, xchg, tk, tres);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty + ab);
        } else {
          const int len = kb1 - kb0;
          // Every other contributor of this tile may already have published its
          // partial (their segments usually come first in their CTAs' ranges):
          // then this CTA is certainly the last and finishes the tile from its
          // own accumulator in TMEM, without the round trip through memory.
          if (!pre && et == 0) {
            const bool done = ld_acquire_gpu(a.counter + t) + len == s.KB;
            if (done) a.counter[t] = 0;  // nobody else touches it in this launch
            flags[1] = done ? 2 : 0;
          }
          if (!pre) named_bar_sync(1, 128);
          const bool fast = flags[1] == 2;
          if (!fast) {
            const int which = (t == sk_first_tile(s, b)) ? 0 : 1;
            const uint64_t keep = l2_policy_evict_last();
            float* pw = a.partial + (size_t)(b * 2 + which) * a.tokpad * kBM;
            for (int c = 0; c < nchunk; ++c) {
              float v[16];
              tmem_ld16(taddr + c * 16, v);
  #pragma unroll
              for (int j = 0; j < 16; ++j)
                st_global_keep(pw + (size_t)(c * 16 + j) * kBM + row, v[j], keep);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + ab);
            named_bar_sync(1, 128);
            if (et == 0) {
              fence_acq_rel_gpu();
              const int old = atom_add_acq_rel_gpu(a.counter + t, len);
              const int last = (old + len == s.KB) ? 1 : 0;
              if (last) a.counter[t] = 0;  // leave the workspace zeroed for the next call
              flags[1] = last;
            }
            named_bar_sync(1, 128);
          }
          if (fast || flags[1]) {
            // Contributors are summed in the same order on both paths, so the
            // result does not depend on which path finished the tile.
            int bf, bl;
            sk_contributors(s, t, bf, bl);
            for (int c = 0; c < nchunk; c += 2) {
              float v[32], own[32];
              const int ncol = (c + 1 < nchunk) ? 32 : 16;
              if (fast) {
                tmem_ld16(taddr + c * 16, own);
                tmem_ld16(taddr + c * 16 + 16, own + 16);  // past ntok: unused columns
              } else {
  #pragma unroll
                for (int j = 0; j < 32; ++j) own[j] = 0.f;
              }
              if (pre)
                sum_prefetched(bf, bl, b, c * 16, (ti.ntok + 15) & ~15, tspare, own, v);
              else
                reduce_partials(a.partial, a.tokpad, s, t, bf, bl, c * 16, ncol, row, v, b, fast,
                                own);
              finalize<T>(a, s, ti, row, c * 16, v, xchg, tk, tres);
              if (ncol == 32) finalize<T>(a, s, ti, row, c * 16 + 16, v + 16, xchg, tk, tres);
            }
          }
          if (fast) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + ab);
          }
        }
        if (stage_tokens) named_bar_sync(2, 128);  // tk is rewritten for the next tile
        ++acc_it;
        g += kb1 - kb0;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace gemm
}  // namespace ps

using namespace ps;

namespace ps {
namespace gemm {

// Host copy of a launch's schedule inputs: the schedule depends on the two
// models' token counts, K, N, the epilogue (SwiGLU tiles pair gate and up
// columns) and the grid size only.
static bool host_sched(int c0, int c1, int K, int N, int epilogue, int grid, Sched& s, Args& a) {
  if (c0 < 0 || c1 < 0 || K <= 0 || N <= 0 || grid < 1 || N % 8 != 0) return false;
  if (epilogue == PS_EPI_SWIGLU && N % 16 != 0) return false;
  a = Args{};
  a.M = c0 + c1;
  a.tokpad = tokpad_for(a.M, 0);
  a.K = K;
  a.N = N;
  a.gated = epilogue == PS_EPI_SWIGLU;
  a.ff = a.gated ? N / 2 : 0;
  sched_from_counts(a, c0, c1, grid, s);
  return true;
}

}  // namespace gemm
}  // namespace ps

extern "C" int ps_routed_gemm_schedule(int c0, int c1, int K, int N, int epilogue, int grid,
                                       int32_t* info) {
  gemm::Sched s;
  gemm::Args a;
  PS_CHECK_ARG(info && gemm::host_sched(c0, c1, K, N, epilogue, grid, s, a));
  const int32_t v[10] = {s.T0, s.T1, s.nt, s.ntiles, s.KB, s.I, s.C, s.R, s.base, s.grid};
  for (int i = 0; i < 10; ++i) info[i] = v[i];
  return PS_OK;
}

extern "C" int ps_routed_gemm_cta_work(int c0, int c1, int K, int N, int epilogue, int grid,
                                       int cta, int32_t* pieces, int cap) {
  gemm::Sched s;
  gemm::Args a;
  if (!gemm::host_sched(c0, c1, K, N, epilogue, grid, s, a) || cta < 0 || cta >= grid ||
      cap < 0 || (!pieces && cap > 0))
    return -PS_ERR_INVALID_ARGUMENT;
  // The same walk as the kernel's producer, MMA and epilogue loops.
  int n = 0;
  for (int seg = 0; seg <= s.R; ++seg) {
    int start, end;
    gemm::seg_range(s, cta, seg, start, end);
    for (int g = start; g < end;) {
      const int t = g / s.KB, kb0 = g % s.KB;
      const int kb1 = gemm::imin(s.KB, kb0 + (end - g));
      if (n < cap) {
        int32_t* q = pieces + 6 * n;
        const bool whole = kb0 == 0 && kb1 == s.KB;
        int bf = -1, bl = -1;
        if (!whole) gemm::sk_contributors(s, t, bf, bl);
        q[0] = t;
        q[1] = kb0;
        q[2] = kb1;
        q[3] = whole ? -1 : (t == gemm::sk_first_tile(s, cta) ? 0 : 1);
        q[4] = bf;
        q[5] = bl;
      }
      ++n;
      g += kb1 - kb0;
    }
  }
  return n;
}

extern "C" int ps_routed_gemm_tile(int c0, int c1, int K, int N, int epilogue, int grid, int t,
                                   int32_t* out) {
  gemm::Sched s;
  gemm::Args a;
  PS_CHECK_ARG(out && gemm::host_sched(c0, c1, K, N, epilogue, grid, s, a));
  PS_CHECK_ARG(t >= 0 && t < s.ntiles);
  const gemm::Tile ti = gemm::tile_of(a, s, t);
  const int32_t v[6] = {ti.m, ti.row0, ti.ntok, ti.col0, ti.col1, ti.out0};
  for (int i = 0; i < 6; ++i) out[i] = v[i];
  return PS_OK;
}

extern "C" size_t ps_routed_gemm_workspace_bytes(int M, int N, int epilogue, int device) {
  if (M < 0 || N <= 0) return 0;
  const gemm::Plan p = gemm::plan_for(M, N, epilogue == PS_EPI_SWIGLU, device);
  return p.counter_bytes + p.partial_bytes;
}

namespace ps {
namespace gemm {

static int launch_routed_gemm(const void* x, const void* W, void* y, int M, int K, int N,
                              int split_point, const int32_t* counts,
                              const ps_gemm_epilogue_t& e, int dtype, void* workspace,
                              size_t workspace_bytes, int32_t* status, cudaStream_t st) {
  Plan p;
  CUtensorMap tw, tx;
  Args a;
  bool empty;
  const int rc = prepare_gemm(x, W, y, M, K, N, split_point, counts, e, dtype, status, &p, &tw,
                              &tx, &a, &empty);
  if (rc != PS_OK || empty) return rc;
  if (!workspace || workspace_bytes < p.counter_bytes + p.partial_bytes) return PS_ERR_WORKSPACE;
  PS_CHECK_ARG(aligned16(workspace));
  a.counter = reinterpret_cast<int32_t*>(workspace);
  a.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + p.counter_bytes);

  if (dtype == PS_DTYPE_BF16) {
    PS_CUDA_RET(allow_dynamic_smem(routed_gemm_kernel<__nv_bfloat16>, kSmemLimit));
    PS_CUDA_RET(launch(routed_gemm_kernel<__nv_bfloat16>, dim3(p.grid), dim3(kThreads), p.smem,
                       st, tw, tx, a));
  } else {
    PS_CUDA_RET(allow_dynamic_smem(routed_gemm_kernel<__half>, kSmemLimit));
    PS_CUDA_RET(launch(routed_gemm_kernel<__half>, dim3(p.grid), dim3(kThreads), p.smem, st, tw,
                       tx, a));
  }
  return PS_OK;
}

}  // namespace gemm
}  // namespace ps

extern "C" int ps_routed_gemm(const void* x, const void* W, void* y, int M, int K, int N,
                              int split_point, const int32_t* counts,
                              const int32_t* scatter_rows, const void* residual, int epilogue,
                              int dtype, void* workspace, size_t workspace_bytes,
                              int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(epilogue == PS_EPI_STORE || epilogue == PS_EPI_SWIGLU);
  ps_gemm_epilogue_t e{};
  e.mode = epilogue;
  e.scatter_rows = scatter_rows;
  e.residual = residual;
  return gemm::launch_routed_gemm(x, W, y, M, K, N, split_point, counts, e, dtype, workspace,
                                  workspace_bytes, status, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ps_routed_gemm_ex(const void* x, const void* W, void* y, int M, int K, int N,
                                 int split_point, const int32_t* counts,
                                 const ps_gemm_epilogue_t* epi, int dtype, void* workspace,
                                 size_t workspace_bytes, int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(epi);
  return gemm::launch_routed_gemm(x, W, y, M, K, N, split_point, counts, *epi, dtype, workspace,
                                  workspace_bytes, status, reinterpret_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------- //
// Packed weights: W [nmat, K, N] (N contiguous) -> for every model, weight tile
// and 128-k block, the 32 KB shared-memory image of the stage: two halves of
// 64 columns (SwiGLU: the 64 gate columns, then their 64 up columns), each 128
// k rows of 128 bytes with the 128-byte swizzle applied (16-byte chunk c of row
// r stored at chunk c ^ (r % 8)), zeros past K and N. One thread per 16-byte
// chunk of the output; a one-time conversion at load.
// ------------------------------------------------------------------------- //
namespace ps {
namespace gemm {

__global__ void pack_weights_kernel(const uint4* __restrict__ W, uint4* __restrict__ out, int K,
                                    int N, int gated, int nt, int KB, long long total) {
  const int ff = N / 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int pc = (int)(i & 7);          // physical 16-byte chunk in the row
    const int r = (int)((i >> 3) & 127);  // k row in the block
    const int h = (int)((i >> 10) & 1);   // half
    long long blk = i >> 11;              // (m * nt + n) * KB + kb
    const int kb = (int)(blk % KB);
    blk /= KB;
    const int n = (int)(blk % nt);
    const int m = (int)(blk / nt);
    const int c = pc ^ (r & 7);           // logical chunk = 8 columns
    const int k = kb * kBK + r;
    int col, lim;
    if (gated) {
      col = (h ? ff : 0) + n * 64 + c * 8;
      lim = (h ? ff : 0) + ff;  // gate columns [0, ff), up columns [ff, N)
    } else {
      col = n * kBM + h * 64 + c * 8;
      lim = N;
    }
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (k < K && col < lim) v = W[(((size_t)m * K + k) * N + col) / 8];
    out[i] = v;
  }
}

}  // namespace gemm
}  // namespace ps

extern "C" size_t ps_packed_weights_bytes(int nmat, int K, int N, int epilogue) {
  if (nmat < 1 || K <= 0 || N <= 0) return 0;
  int nt, KB;
  gemm::packed_layout(K, N, epilogue == PS_EPI_SWIGLU, &nt, &KB);
  return (size_t)nmat * nt * KB * gemm::kPackedTileBytes;
}

extern "C" int ps_pack_weights(const void* W, int nmat, int K, int N, int epilogue, void* out,
                               size_t out_bytes, ps_stream_t stream) {
  PS_CHECK_ARG(nmat >= 1 && K > 0 && N > 0 && K % 8 == 0 && N % 8 == 0);
  PS_CHECK_ARG(epilogue == PS_EPI_STORE || epilogue == PS_EPI_SWIGLU ||
               epilogue == PS_EPI_QKV_ROPE);
  const int gated = epilogue == PS_EPI_SWIGLU;
  if (gated) PS_CHECK_ARG(N % 16 == 0);
  PS_CHECK_ARG(W && out && aligned16(W) && aligned16(out));
  const size_t need = ps_packed_weights_bytes(nmat, K, N, epilogue);
  PS_CHECK_ARG(out_bytes >= need);
  int nt, KB;
  gemm::packed_layout(K, N, gated, &nt, &KB);
  const long long total = (long long)(need / 16);
  const int grid = (int)min((total + 255) / 256, (long long)sm_count(current_device()) * 16);
  PS_CUDA_RET(launch(gemm::pack_weights_kernel, dim3(max(grid, 1)), dim3(256), 0,
                     reinterpret_cast<cudaStream_t>(stream), (const uint4*)W, (uint4*)out, K, N,
                     gated, nt, KB, total));
  return PS_OK;
}

// ------------------------------------------------------------------------- //
// Routed GEMM without any allocation by the caller or the library.
//
// Some callers cannot hand this library a workspace: a serving runtime whose
// device memory is fully owned by its own pool (weights and KV cache reserved
// up front, nothing else may allocate), a plugin host that forbids
// allocation inside its execute call, or a latency-bound decode loop that
// cannot afford the device-wide synchronisation cudaMalloc / cudaFree may
// cause. For them ps_routed_gemm_noalloc keeps the stream-K scratch (tile
// arrival counters + partial tiles) in the file-scope array below. The array
// is part of this library's device image: every GPU that loads the library
// holds its 16 MiB until the process exits.
//
// Limits: at most kNoAllocMaxTiles output tiles per call; the grid is capped
// so that the partial tiles fit (full 148-SM grid up to M = 96 rows, fewer
// CTAs above that: a CTA's partial slots are sized by M rounded to 16). Every call shares the one array and leaves it with
// its last contents; the counters are cleared at the start of every call, so
// calls must not overlap on the GPU (calls on different streams race).
// ------------------------------------------------------------------------- //
namespace ps {
namespace gemm {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr size_t kNoAllocCounterBytes = size_t(64) << 10;
constexpr int kNoAllocMaxTiles = (int)(kNoAllocCounterBytes / 4);

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device, resolved once per device
// under g_noalloc_mu (host threads may make first calls at the same time).
static std::atomic<void*> g_noalloc_addr[64];
static std::mutex g_noalloc_mu;

}  // namespace gemm
}  // namespace ps

extern "C" int ps_routed_gemm_noalloc(const void* x, const void* W, void* y, int M, int K,
                                      int N, int split_point, const int32_t* counts,
                                      const int32_t* scatter_rows, const void* residual,
                                      int epilogue, int dtype, int32_t* status,
                                      ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && K > 0 && N > 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  PS_CHECK_ARG(epilogue == PS_EPI_STORE || epilogue == PS_EPI_SWIGLU);
  PS_CHECK_ARG(K % 8 == 0 && N % 8 == 0);
  const int gated = epilogue == PS_EPI_SWIGLU;
  if (gated) PS_CHECK_ARG(N % 16 == 0 && residual == nullptr);
  if (!counts) PS_CHECK_ARG(split_point >= 0 && split_point <= M);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(x && W && y);
  PS_CHECK_ARG(aligned16(x) && aligned16(W) && aligned16(y));
  PS_CHECK_ARG(!residual || aligned16(residual));
  const int device = current_device();
  if (device < 0 || device >= 64 || !is_sm100(device)) return PS_ERR_UNSUPPORTED;

  // Set-up, once per device with that device current: resolve the device
  // address of the scratch array (the host-side name is only a stand-in).
  void* resolved = gemm::g_noalloc_addr[device].load(std::memory_order_acquire);
  if (!resolved) {
    std::lock_guard<std::mutex> lock(gemm::g_noalloc_mu);
    resolved = gemm::g_noalloc_addr[device].load(std::memory_order_relaxed);
    if (!resolved) {
      void* addr = nullptr;
      if (cudaGetSymbolAddress(&addr, gemm::g_noalloc_scratch) != cudaSuccess || !addr)
        return PS_ERR_CUDA;
      PS_CUDA_RET(allow_dynamic_smem(gemm::routed_gemm_kernel<__half>, gemm::kSmemLimit));
      PS_CUDA_RET(allow_dynamic_smem(gemm::routed_gemm_kernel<__nv_bfloat16>, gemm::kSmemLimit));
      gemm::g_noalloc_addr[device].store(addr, std::memory_order_release);
      resolved = addr;
    }
  }
  char* scratch = reinterpret_cast<char*>(resolved);

  gemm::Plan p = gemm::plan_for(M, N, gated, device);
  const size_t per_cta = (size_t)2 * p.tokpad * gemm::kBM * sizeof(float);
  const int fit = (int)((gemm::kNoAllocScratchBytes - gemm::kNoAllocCounterBytes) / per_cta);
  if (fit < p.grid) p.grid = fit;
  const long long iters = (long long)(gated ? cdiv(N / 2, 64) : cdiv(N, gemm::kBM)) *
                          (cdiv(M, p.tokpad) + 1) * cdiv(K, gemm::kBK);
  if (iters >= (1ll << 31) || p.max_tiles > gemm::kNoAllocMaxTiles) return PS_ERR_SCRATCH_LIMIT;

  CUtensorMap tw, tx;
  {
    const uint64_t nmat = (!counts && split_point == M) ? 1 : 2;
    const uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, nmat};
    const uint64_t strides[2] = {(uint64_t)N * 2, (uint64_t)K * N * 2};
    const uint32_t box[3] = {64, (uint32_t)gemm::kBK, 1};
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

  gemm::Args a{};
  a.y = y;
  a.residual = residual;
  a.counts = counts;
  a.scatter = scatter_rows;
  a.counter = reinterpret_cast<int32_t*>(scratch);
  a.partial = reinterpret_cast<float*>(scratch + gemm::kNoAllocCounterBytes);
  a.status = status;
  a.M = M;
  a.K = K;
  a.N = N;
  a.split_point = split_point;
  a.gated = gated;
  a.ff = gated ? N / 2 : 0;
  a.n_out = gated ? N / 2 : N;
  a.tokpad = p.tokpad;
  a.stages = p.stages;
  a.bf16 = dtype == PS_DTYPE_BF16;
  a.mode = epilogue;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The arrival counters must start at zero; a previous call may have been cut
  // short, so clear the ones this call can use.
  PS_CUDA_RET(cudaMemsetAsync(scratch, 0, (size_t)p.max_tiles * 4, st));
  if (dtype == PS_DTYPE_BF16)
    gemm::routed_gemm_kernel<__nv_bfloat16><<<p.grid, gemm::kThreads, p.smem, st>>>(tw, tx, a);
  else
    gemm::routed_gemm_kernel<__half><<<p.grid, gemm::kThreads, p.smem, st>>>(tw, tx, a);
  PS_CUDA_RET(cudaGetLastError());
  return PS_OK;
}
