// One-shot all-reduce over NVLink peer memory for the tensor-parallel decode
// step (the O and down projections are row-split: every rank holds a partial
// [M, H] that must be summed across ranks).
//
// Each rank owns a symmetric region, allocated here and mapped into every peer
// with CUDA IPC:
//   [flags: kMaxBlocks x kMaxRanks int32][slot 0: cap bytes][slot 1: cap bytes]
// A row-split GEMM writes its partial into the local slot of the call's parity.
// ps_allreduce_sum then, in each of its fixed number of blocks b:
//   1. signal: store the block's epoch e into flags[b][my_rank] of every peer
//      (relaxed, system scope: the flag marks arrival and publishes nothing
//      this kernel wrote — the local partial is complete because the GEMM
//      that wrote it finished before this kernel's dependency wait returned);
//   2. wait (bounded by %globaltimer, acquire loads) until every rank's
//      flags[b][r] >= e;
//   3. read its slice of every rank's slot (16-byte loads, ranks summed in
//      order 0..world-1 in fp32, so every rank gets bit-identical results),
//      add the optional residual, store 16-bit output.
// Slots alternate by call parity: a rank rewrites a slot only after its next
// all-reduce passed the wait, i.e. after every peer finished reading it.
//
// Two-shot variant (fewer bytes over NVLink for larger groups): rank r owns
// the r-th 1/world of the vector. After the same first wait it reduces only
// its own part (world reads of count/world elements), adds the residual and
// pushes the result, with its sums of squares, into the gather buffer of
// every rank; a second signal / wait round (per block, release stores after
// the block's barrier) publishes those pushes, then each rank copies the gathered vector
// into `out`. NVLink traffic per rank: 2 (world-1)/world x count elements
// instead of (world-1) x count.
// Low-latency two-shot (PS_AR_TWO_SHOT_LL): the reduced share travels as
// 8-byte {data, epoch} words that receivers poll, so no second round is
// needed (allreduce_ll_kernel below).
// Epochs are per block (block b alone reads and bumps epoch[b]), so the kernel
// needs no grid-wide synchronisation and works under CUDA-graph replay.
#include <cuda_runtime.h>

#include <cstring>

#include "ps_common.cuh"
#include "ps_host.h"
#include "ps_peer.cuh"

namespace ps {
namespace ar {

// Many SMs issue remote loads: NVLink read bandwidth scales with the number of
// SMs in flight, not with threads per SM.
constexpr int kBlocks = 128;
constexpr int kThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kThreads)
    allreduce_kernel(const Peers peers, int rank, int world, int slot, size_t cap, int nvec,
                     T* out, const T* residual, int* epochs, float* sumsq, int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  __shared__ int s_e;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_e = epochs[b] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int e = s_e;
  int* my_flags = reinterpret_cast<int*>(peers.base[rank]);
  if (threadIdx.x < world) {
    const int r = threadIdx.x;
    // The partial being published was written by an earlier kernel on this
    // stream, complete before pdl_wait returned, so the arrival flag needs no
    // release (st_relaxed_sys); the peer's acquire load orders its reads
    // after the flag. The same flag tells this rank that the peer finished
    // its previous call (its reads of the other slot), which allows the slot
    // parity scheme below.
    st_relaxed_sys(reinterpret_cast<int*>(peers.base[r]) + b * kMaxRanks + rank, e);
    // wait for rank r's signal of this epoch
    const int* f = my_flags + b * kMaxRanks + r;
    if (ld_acquire_sys(f) < e) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(f) < e) {
        if (globaltimer_ns() - t0 > kPeerWaitNs) {
          set_status(status, PS_ERR_TIMEOUT);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) epochs[b] = e;
  if (!s_ok) return;

  const size_t data_off = slot_offset(slot, cap);
  for (int i = b * kThreads + threadIdx.x; i < nvec; i += kBlocks * kThreads) {
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    if (residual) add8<T>(acc, reinterpret_cast<const uint4*>(residual)[i]);  // may alias out
    uint4 v[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) v[r] = ld_cg_v4(peers.base[r] + data_off + (size_t)i * 16);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) add8<T>(acc, v[r]);
    uint4 o;
    T* oh = reinterpret_cast<T*>(&o);
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      oh[k] = from_f32<T>(acc[k]);
      const float f = to_f32<T>(oh[k]);
      sq += f * f;
    }
    reinterpret_cast<uint4*>(out)[i] = o;
    if (sumsq) {  // 32 vectors of a warp = one 256-element part of one row
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, s);
      if ((threadIdx.x & 31) == 0) sumsq[i >> 5] = sq;
    }
  }
}

// Signal this block's epoch e on every rank's flag set `set`, then wait
// (bounded) until every rank signalled e for this block. false on timeout.
// `release`: the signal publishes data written by this kernel (the pushes of
// the two-shot's gather); without it the flag only marks arrival.
PS_DEV bool block_barrier(const Peers& peers, int rank, int world, int b, int e, int set,
                          bool release, int32_t* status) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  int* my_flags = reinterpret_cast<int*>(peers.base[rank] + set * kFlagSet);
  if (threadIdx.x < world) {
    const int r = threadIdx.x;
    int* dst = reinterpret_cast<int*>(peers.base[r] + set * kFlagSet) + b * kMaxRanks + rank;
    if (release)
      st_release_sys(dst, e);
    else
      st_relaxed_sys(dst, e);
    const int* f = my_flags + b * kMaxRanks + r;
    if (ld_acquire_sys(f) < e) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(f) < e) {
        if (globaltimer_ns() - t0 > kPeerWaitNs) {
          set_status(status, PS_ERR_TIMEOUT);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return s_ok != 0;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    allreduce2_kernel(const Peers peers, int rank, int world, int slot, size_t cap, int part,
                      T* out, const T* residual, int* epochs, float* sumsq, int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int e = epochs[b] + 1;
  const bool ok1 = block_barrier(peers, rank, world, b, e, 0, false, status);
  if (!ok1) {
    if (threadIdx.x == 0) epochs[b] = e;
    return;
  }
  const size_t data_off = slot_offset(slot, cap);
  const size_t g_off = gather_offset(cap), gsq_off = gather_sq_offset(cap);
  const int own0 = rank * part;  // vectors [own0, own0 + part) are reduced here
  // part % 32 == 0 and the stride is a multiple of 32: every warp has 32
  // consecutive vectors (one 256-element sum-of-squares part) or none.
  for (int i = b * kThreads + threadIdx.x; i < part; i += kBlocks * kThreads) {
    const int g = own0 + i;
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    if (residual) add8<T>(acc, reinterpret_cast<const uint4*>(residual)[g]);
    uint4 v[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) v[r] = ld_cg_v4(peers.base[r] + data_off + (size_t)g * 16);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) add8<T>(acc, v[r]);
    uint4 o;
    T* oh = reinterpret_cast<T*>(&o);
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      oh[k] = from_f32<T>(acc[k]);
      const float f = to_f32<T>(oh[k]);
      sq += f * f;
    }
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) *reinterpret_cast<uint4*>(peers.base[r] + g_off + (size_t)g * 16) = o;
    if (sumsq) {
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, m);
      if ((threadIdx.x & 31) == 0) {
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < world)
            reinterpret_cast<float*>(peers.base[r] + gsq_off)[g >> 5] = sq;
      }
    }
  }
  // The block barrier's __syncthreads orders every thread's pushes before the
  // signalling threads' st.release.sys, whose release is cumulative: the
  // pushes are visible to a rank that acquires the signal.
  const bool ok2 = block_barrier(peers, rank, world, b, e, 1, true, status);
  if (threadIdx.x == 0) epochs[b] = e;
  if (!ok2) return;
  // copy the gathered vector (this block's share of every owner's part)
  for (int r = 0; r < world; ++r) {
    for (int i = b * kThreads + threadIdx.x; i < part; i += kBlocks * kThreads) {
      const int g = r * part + i;
      reinterpret_cast<uint4*>(out)[g] = ld_cg_v4(peers.base[rank] + g_off + (size_t)g * 16);
      if (sumsq && (threadIdx.x & 31) == 0)
        sumsq[g >> 5] = __ldcg(reinterpret_cast<const float*>(peers.base[rank] + gsq_off) + (g >> 5));
    }
  }
}

// Low-latency two-shot (PS_AR_TWO_SHOT_LL). After the same arrival barrier
// as the one-shot, rank r reduces its own 1/world share of the vector (every
// rank's slot, ranks in order 0..world-1, plus the residual), and pushes the
// rounded result, and its sums of squares, to every rank's gather area as
// 8-byte words {4 data bytes, epoch e}. Each rank then polls its own area
// (bounded) until every word of the vector carries e and unpacks it into
// `out`. The gather area can be rewritten at call e + 1 without a second
// barrier: a rank pushes only after the next call's arrival barrier, and a
// rank arrives there only after it finished unpacking call e.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    allreduce_ll_kernel(const Peers peers, int rank, int world, int slot, size_t cap, int part,
                        int nvec, T* out, const T* residual, int* epochs, float* sumsq,
                        int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int e = epochs[b] + 1;
  const bool ok1 = block_barrier(peers, rank, world, b, e, 0, false, status);
  if (!ok1) {
    if (threadIdx.x == 0) epochs[b] = e;
    return;
  }
  const size_t data_off = slot_offset(slot, cap);
  const size_t w_off = ll_offset(cap), sq_off = ll_sq_offset(cap);
  const uint64_t tag = (uint64_t)(uint32_t)e << 32;
  const int own0 = rank * part;
  // reduce this rank's share and push it (part % 32 == 0 and the stride is a
  // multiple of 32: a warp holds 32 consecutive vectors = one 256-element
  // sum-of-squares part, or none)
  for (int i = b * kThreads + threadIdx.x; i < part; i += kBlocks * kThreads) {
    const int g = own0 + i;
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    if (residual) add8<T>(acc, reinterpret_cast<const uint4*>(residual)[g]);
    uint4 v[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) v[r] = ld_cg_v4(peers.base[r] + data_off + (size_t)g * 16);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) add8<T>(acc, v[r]);
    uint4 o;
    T* oh = reinterpret_cast<T*>(&o);
    float sq = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      oh[k] = from_f32<T>(acc[k]);
      const float f = to_f32<T>(oh[k]);
      sq += f * f;
    }
    const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= world) continue;
      uint64_t* dst = reinterpret_cast<uint64_t*>(peers.base[r] + w_off) + (size_t)g * 4;
#pragma unroll
      for (int k = 0; k < 4; ++k) st_relaxed_sys_u64(dst + k, tag | ow[k]);
    }
    if (sumsq) {
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, m);
      if ((threadIdx.x & 31) == 0) {
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r)
          if (r < world)
            st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(peers.base[r] + sq_off) + (g >> 5),
                               tag | __float_as_uint(sq));
      }
    }
  }
  // unpack the whole vector from this rank's gather area
  const uint64_t* words = reinterpret_cast<const uint64_t*>(peers.base[rank] + w_off);
  const uint64_t* sqw = reinterpret_cast<const uint64_t*>(peers.base[rank] + sq_off);
  uint64_t t0 = 0;
  bool ok = true;
  for (int i = b * kThreads + threadIdx.x; i < nvec && ok; i += kBlocks * kThreads) {
    uint64_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = ld_relaxed_sys_u64(words + (size_t)i * 4 + k);
    const bool want_sq = sumsq && (threadIdx.x & 31) == 0;
    uint64_t q = want_sq ? ld_relaxed_sys_u64(sqw + (i >> 5)) : tag;
    while (((w[0] ^ tag) | (w[1] ^ tag) | (w[2] ^ tag) | (w[3] ^ tag) | (q ^ tag)) >> 32) {
      if (t0 == 0) t0 = globaltimer_ns();
      if (globaltimer_ns() - t0 > kPeerWaitNs) {
        set_status(status, PS_ERR_TIMEOUT);
        ok = false;
        break;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if ((w[k] ^ tag) >> 32) w[k] = ld_relaxed_sys_u64(words + (size_t)i * 4 + k);
      if ((q ^ tag) >> 32) q = ld_relaxed_sys_u64(sqw + (i >> 5));
    }
    if (!ok) break;
    reinterpret_cast<uint4*>(out)[i] =
        make_uint4((uint32_t)w[0], (uint32_t)w[1], (uint32_t)w[2], (uint32_t)w[3]);
    if (want_sq) sumsq[i >> 5] = __uint_as_float((uint32_t)q);
  }
  if (threadIdx.x == 0) epochs[b] = e;
}

// Vocab-parallel greedy pick. Block j handles row j: the local (max, index)
// of the row's logits shard (first index on ties), pushed as one 8-byte pair
// into pairs[rank][j] of every rank's region and published with a release
// store of the row's epoch into flags[j][rank]; after a bounded wait for every
// rank's flag, the winner is the largest value, lowest global index on ties
// (ranks hold consecutive vocabulary shards, so this is the first index of
// the whole row), identical on every rank.
template <typename T>
__global__ void __launch_bounds__(512)
    argmax_tp_kernel(const T* __restrict__ logits, const int32_t* __restrict__ perm,
                     int32_t* __restrict__ next, int32_t* __restrict__ tokens_out,
                     int32_t* __restrict__ seq_len, int V, const Peers peers, int rank, int world,
                     size_t pick_off, int* epochs, int32_t* status) {
  __shared__ float sv[16];
  __shared__ int si[16];
  __shared__ int s_ok;
  pdl_wait();
  pdl_launch_dependents();
  const int j = blockIdx.x;
  const T* row = logits + (size_t)j * V;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = to_f32<T>(row[v]);
    if (x > best) {  // strictly greater keeps the first index per thread
      best = x;
      bi = v;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  const int e = epochs[j] + 1;
  if (threadIdx.x < world) {
    const int r = threadIdx.x;
    float b = sv[0];
    int ix = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > b || (sv[w] == b && si[w] < ix)) {
        b = sv[w];
        ix = si[w];
      }
    const int gidx = ix == 0x7fffffff ? 0x7fffffff : rank * V + ix;
    char* base = peers.base[r] + pick_off;
    int2 pair;
    pair.x = __float_as_int(b);
    pair.y = gidx;
    *reinterpret_cast<int2*>(base + kPickFlagBytes + ((size_t)rank * kMaxPickRows + j) * 8) = pair;
    // the release orders this thread's pair store before the flag
    st_release_sys(reinterpret_cast<int*>(base) + j * kMaxRanks + rank, e);
    const int* f = reinterpret_cast<const int*>(peers.base[rank] + pick_off) + j * kMaxRanks + r;
    if (ld_acquire_sys(f) < e) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(f) < e) {
        if (globaltimer_ns() - t0 > kPeerWaitNs) {
          set_status(status, PS_ERR_TIMEOUT);
          s_ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  epochs[j] = e;
  if (!s_ok) return;
  const char* mine = peers.base[rank] + pick_off + kPickFlagBytes;
  float b = -INFINITY;
  int pick = 0x7fffffff;
  for (int r = 0; r < world; ++r) {
    const int2 pr = __ldcg(reinterpret_cast<const int2*>(mine + ((size_t)r * kMaxPickRows + j) * 8));
    const float v = __int_as_float(pr.x);
    if (pr.y != 0x7fffffff && (pick == 0x7fffffff || v > b || (v == b && pr.y < pick))) {
      b = v;
      pick = pr.y;
    }
  }
  if (pick == 0x7fffffff) pick = 0;  // all -inf / NaN row
  const int dst = perm ? perm[j] : j;
  next[dst] = pick;
  if (tokens_out) tokens_out[dst] = pick;
  if (seq_len) seq_len[dst] += 1;
}

}  // namespace ar
}  // namespace ps

using namespace ps;

extern "C" size_t ps_symm_region_bytes(size_t slot_bytes) {
  return ar::region_bytes((slot_bytes + 255) / 256 * 256);
}

extern "C" size_t ps_symm_slot_offset(int slot, size_t slot_bytes) {
  return ar::slot_offset(slot, (slot_bytes + 255) / 256 * 256);
}

extern "C" int ps_symm_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  PS_CHECK_ARG(bytes > 0 && ptr && ipc_handle);
  void* p = nullptr;
  PS_CUDA_RET(cudaMalloc(&p, bytes));
  if (cudaMemset(p, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p) != cudaSuccess) {
    cudaFree(p);
    return PS_ERR_CUDA;
  }
  PS_CUDA_RET(cudaDeviceSynchronize());
  *ptr = p;
  return PS_OK;
}

extern "C" int ps_symm_open(const void* ipc_handle, void** peer_ptr) {
  PS_CHECK_ARG(ipc_handle && peer_ptr);
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  PS_CUDA_RET(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return PS_OK;
}

extern "C" int ps_symm_close(void* peer_ptr) {
  PS_CHECK_ARG(peer_ptr);
  PS_CUDA_RET(cudaIpcCloseMemHandle(peer_ptr));
  return PS_OK;
}

extern "C" int ps_symm_free(void* ptr) {
  PS_CHECK_ARG(ptr);
  PS_CUDA_RET(cudaFree(ptr));
  return PS_OK;
}

extern "C" int ps_allreduce_sum(void* const* peer_bases, int rank, int world, int slot,
                                size_t slot_bytes, size_t count, void* out, const void* residual,
                                int* epochs, int row_elems, float* out_sumsq, int algo,
                                int dtype, int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(world >= 1 && world <= ar::kMaxRanks && rank >= 0 && rank < world);
  PS_CHECK_ARG(slot == 0 || slot == 1);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  PS_CHECK_ARG(count % 8 == 0 && count * 2 <= slot_bytes && slot_bytes % 256 == 0);
  PS_CHECK_ARG(peer_bases && out && epochs && aligned16(out));
  PS_CHECK_ARG(!residual || aligned16(residual));
  PS_CHECK_ARG(!out_sumsq || (row_elems > 0 && row_elems % 256 == 0 && count % row_elems == 0));
  if (count == 0) return PS_OK;
  ar::Peers p;
  for (int r = 0; r < ar::kMaxRanks; ++r) p.base[r] = r < world ? (char*)peer_bases[r] : nullptr;
  for (int r = 0; r < world; ++r) PS_CHECK_ARG(p.base[r] && aligned16(p.base[r]));
  PS_CHECK_ARG(algo >= PS_AR_AUTO && algo <= PS_AR_TWO_SHOT_LL);
  const int nvec = (int)(count / 8);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // two-shot needs whole 32-vector groups per rank (count % (world * 256) == 0)
  const bool two_ok = world > 1 && nvec % (world * 32) == 0;
  // AUTO is one-shot: on 2 GPUs two-shot measured 9 us slower per 512 KB call
  // (its second signal / wait round costs more than the halved reads save).
  const bool two = two_ok && algo == PS_AR_TWO_SHOT;
  if (two_ok && algo == PS_AR_TWO_SHOT_LL) {
    const int part = nvec / world;
    if (dtype == PS_DTYPE_BF16)
      PS_CUDA_RET(launch(ar::allreduce_ll_kernel<__nv_bfloat16>, dim3(ar::kBlocks),
                         dim3(ar::kThreads), 0, st, p, rank, world, slot, slot_bytes, part, nvec,
                         (__nv_bfloat16*)out, (const __nv_bfloat16*)residual, epochs, out_sumsq,
                         status));
    else
      PS_CUDA_RET(launch(ar::allreduce_ll_kernel<__half>, dim3(ar::kBlocks), dim3(ar::kThreads),
                         0, st, p, rank, world, slot, slot_bytes, part, nvec, (__half*)out,
                         (const __half*)residual, epochs, out_sumsq, status));
    return PS_OK;
  }
  if (two) {
    const int part = nvec / world;
    if (dtype == PS_DTYPE_BF16)
      PS_CUDA_RET(launch(ar::allreduce2_kernel<__nv_bfloat16>, dim3(ar::kBlocks),
                         dim3(ar::kThreads), 0, st, p, rank, world, slot, slot_bytes, part,
                         (__nv_bfloat16*)out, (const __nv_bfloat16*)residual, epochs, out_sumsq,
                         status));
    else
      PS_CUDA_RET(launch(ar::allreduce2_kernel<__half>, dim3(ar::kBlocks), dim3(ar::kThreads), 0,
                         st, p, rank, world, slot, slot_bytes, part, (__half*)out,
                         (const __half*)residual, epochs, out_sumsq, status));
    return PS_OK;
  }
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(ar::allreduce_kernel<__nv_bfloat16>, dim3(ar::kBlocks), dim3(ar::kThreads),
                       0, st, p, rank, world, slot, slot_bytes, nvec, (__nv_bfloat16*)out,
                       (const __nv_bfloat16*)residual, epochs, out_sumsq, status));
  else
    PS_CUDA_RET(launch(ar::allreduce_kernel<__half>, dim3(ar::kBlocks), dim3(ar::kThreads), 0, st,
                       p, rank, world, slot, slot_bytes, nvec, (__half*)out,
                       (const __half*)residual, epochs, out_sumsq, status));
  return PS_OK;
}

extern "C" int ps_argmax_tp(const void* logits, const int32_t* perm, int32_t* next_tokens,
                            int32_t* tokens_out, int32_t* seq_len, int M, int V_local,
                            void* const* peer_bases, int rank, int world, size_t slot_bytes,
                            int* epochs, int dtype, int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(world >= 1 && world <= ar::kMaxRanks && rank >= 0 && rank < world);
  PS_CHECK_ARG(M >= 0 && M <= ar::kMaxPickRows && V_local > 0);
  PS_CHECK_ARG((long long)V_local * world < 0x7fffffffll);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  PS_CHECK_ARG(slot_bytes % 256 == 0);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(logits && next_tokens && epochs && peer_bases);
  ar::Peers p;
  for (int r = 0; r < ar::kMaxRanks; ++r) p.base[r] = r < world ? (char*)peer_bases[r] : nullptr;
  for (int r = 0; r < world; ++r) PS_CHECK_ARG(p.base[r] && aligned16(p.base[r]));
  const size_t off = ar::pick_offset(slot_bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(ar::argmax_tp_kernel<__nv_bfloat16>, dim3(M), dim3(512), 0, st,
                       (const __nv_bfloat16*)logits, perm, next_tokens, tokens_out, seq_len,
                       V_local, p, rank, world, off, epochs, status));
  else
    PS_CUDA_RET(launch(ar::argmax_tp_kernel<__half>, dim3(M), dim3(512), 0, st,
                       (const __half*)logits, perm, next_tokens, tokens_out, seq_len, V_local, p,
                       rank, world, off, epochs, status));
  return PS_OK;
}
