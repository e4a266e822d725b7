// Symmetric peer-memory regions for tensor parallelism over NVLink: the
// region layout shared by the all-reduce, the greedy-pick exchange and the
// projection chain's fused all-reduce, and the system-scope signalling
// primitives they use. Each rank allocates one region (cudaMalloc + CUDA IPC,
// mapped by every peer); a kernel reaches a peer's region through plain
// loads and stores over NVLink (no TMA, no multicast).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include "ps_common.cuh"

namespace ps {
namespace ar {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 128;
constexpr size_t kFlagSet = 4096;               // kMaxBlocks x kMaxRanks x 4, padded
constexpr size_t kFlagBytes = 2 * kFlagSet;      // first and second (two-shot) waits
static_assert(kMaxBlocks * kMaxRanks * 4 <= kFlagSet, "flag region");

// Region: [flags][slot 0][slot 1][gather: cap bytes of data, cap / 64 of sums]
//         [greedy-pick exchange: flags kMaxPickRows x kMaxRanks int32,
//                                pairs kMaxRanks x kMaxPickRows x (float value, int index)]
constexpr int kMaxPickRows = 4096;
constexpr size_t kPickFlagBytes = (size_t)kMaxPickRows * kMaxRanks * 4;
constexpr size_t kPickBytes = kPickFlagBytes + (size_t)kMaxRanks * kMaxPickRows * 8;
__host__ __device__ inline size_t slot_offset(int slot, size_t cap) {
  return kFlagBytes + (size_t)slot * cap;
}
__host__ __device__ inline size_t gather_offset(size_t cap) { return kFlagBytes + 2 * cap; }
__host__ __device__ inline size_t gather_sq_offset(size_t cap) { return kFlagBytes + 3 * cap; }
__host__ __device__ inline size_t pick_offset(size_t cap) {
  return gather_sq_offset(cap) + (cap / 64 + 255) / 256 * 256;
}

// 1 s: far beyond any legitimate wait for peers that are executing the same step.
constexpr uint64_t kPeerWaitNs = 1000000000ull;

struct Peers {
  char* base[kMaxRanks];  // symmetric region of every rank (base[rank] is local)
};

PS_DEV void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Arrival signal that publishes nothing written by the signalling kernel.
// A release store costs ~3 us on B200 (it waits for every earlier access of
// the thread at system scope); a relaxed one ~0.4 us. Use it only where the
// data a peer will read after seeing the flag was written by an EARLIER
// kernel on this stream, complete before griddepcontrol.wait returned: those
// writes are in this GPU's memory system, which serves the peers' NVLink
// loads, so no fence of this kernel is needed to order them.
PS_DEV void st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

PS_DEV int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

PS_DEV uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

template <typename T>
PS_DEV void add8(float* acc, uint4 v) {
  const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] += to_f32<T>(h[i]);
}

// Projection-chain all-reduce flags: [job][model][64-column unit][rank] int32,
// written by the rank that published the unit's partial (its launch epoch).
constexpr int kChainMaxJobs = 6;
constexpr int kChainMaxUnits = 512;
constexpr size_t kChainFlagBytes = (size_t)kChainMaxJobs * 2 * kChainMaxUnits * kMaxRanks * 4;
__host__ __device__ inline size_t chain_flags_offset(size_t cap) {
  return pick_offset(cap) + kPickBytes;
}

// Low-latency gather area of the two-shot all-reduce (PS_AR_TWO_SHOT_LL):
// every 4 bytes of data travel as one 8-byte word {data, epoch}, so a receiver
// knows a word has arrived when it carries this call's epoch (an aligned
// 8-byte store is single-copy atomic), with no second barrier and no release
// fence. [words: 2 x cap bytes][sums of squares: 2 x cap / 64 bytes].
__host__ __device__ inline size_t ll_offset(size_t cap) {
  return chain_flags_offset(cap) + kChainFlagBytes;
}
__host__ __device__ inline size_t ll_sq_offset(size_t cap) { return ll_offset(cap) + 2 * cap; }
__host__ __device__ inline size_t region_bytes(size_t cap) {
  return ll_sq_offset(cap) + (2 * (cap / 64) + 255) / 256 * 256;
}

PS_DEV void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

PS_DEV uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace ar
}  // namespace ps
