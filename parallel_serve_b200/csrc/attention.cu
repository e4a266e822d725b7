// Fused two-model decode attention (flash-decoding) and the reference's
// no-KV segment attention, for head_dim 128 on sm_100a.
//
// Decode attention replaces the per-model F.scaled_dot_product_attention calls
// of TwoModelBlockRouted._sdpa_per_model (kernel/src/two_model_block_routed.py:
// 100-120) for the KV-cache decode step: one launch covers the tokens of both
// models; each token reads the pool of its own model (model-id dispatch) at
// its own slot and length.
//
// Work item = (chunk of positions, head, token). KV is streamed HBM -> shared
// memory by cp.async.bulk (each (slot, head) stream is contiguous in the pool
// layout [slots, heads, L_cap, 128]) through a 3-stage mbarrier ring, issued by
// one producer thread; four compute warps each take 16 positions of a 64-position
// stage. q.k uses a 5-step warp-shuffle reduce-scatter (16 sums for 16 shuffles),
// the softmax is online in the log2 domain, and the warps' (m, l, o) are merged
// through shared memory. Chunks of one (token, head) are merged by the
// last-arriving CTA in chunk order (deterministic), so long sequences use all
// SMs. Attention is HBM-bound (1 flop per byte); no tensor cores are used.
#include <cuda_runtime.h>

#include "ps_common.cuh"
#include "ps_host.h"

namespace ps {
namespace attn {

constexpr int kD = 128;
constexpr int kChunkAlign = 128;  // chunk lengths are multiples of every stage size
// Paged KV: page ids of one chunk are staged in shared memory, so a chunk
// spans at most this many pages (the plan caps the chunk length to fit).
constexpr int kMaxChunkPages = 256;

// Pipeline shape: NW compute warps take 16 positions each per stage
// (stage = 16 * NW positions of K and of V), NS stages in the ring.
template <int NW, int NS>
struct Cfg {
  static constexpr int kComputeWarps = NW;
  static constexpr int kStages = NS;
  static constexpr int kStagePos = 16 * NW;
  static constexpr int kThreads = (NW + 1) * 32;
  static constexpr int kStageBytes = kStagePos * kD * 2;  // one K or V stage
  static constexpr int kSmemBytes =
      2 * NS * kStageBytes + 1024 + NW * (kD + 2) * 4 + kMaxChunkPages * 4;
};

struct Args {
  const void* q;
  const void* kp0;
  const void* vp0;
  const void* kp1;
  const void* vp1;
  void* out;
  const int32_t* pos;
  const int32_t* slot;
  const int32_t* counts;
  float* ws_o;
  float* ws_ml;
  int32_t* counter;
  int32_t* status;
  int split_point, M, n_heads, L_cap, slots0, slots1, chunk, max_chunks;
  float scale_log2;
  // Paged KV (block_table != nullptr): pools are [pages, n_heads, page_size,
  // 128]; block_table[j * max_pages + i] = page of model m(j)'s pool holding
  // positions [i * page_size, (i + 1) * page_size) of token j's sequence;
  // slots0 / slots1 are then the page counts of the two pools.
  const int32_t* block_table;
  const int32_t* seq_rows;  // block-table row of token j (nullable: j)
  int table_rows, max_pages, page_size, page_shift;
};

template <typename T>
PS_DEV void load4(const T* p, float* f);
template <>
PS_DEV void load4<__half>(const __half* p, float* f) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}
template <>
PS_DEV void load4<__nv_bfloat16>(const __nv_bfloat16* p, float* f) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

// Sums v[i] over the 32 lanes for 16 different i at once; afterwards lane l
// holds the full sum for i = l >> 1.
PS_DEV float reduce_scatter16(float* v, int lane) {
  {
    const bool hi = lane & 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = hi ? v[i] : v[i + 8];
      const float keep = hi ? v[i + 8] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  {
    const bool hi = lane & 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = hi ? v[i] : v[i + 4];
      const float keep = hi ? v[i + 4] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  {
    const bool hi = lane & 4;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = hi ? v[i] : v[i + 2];
      const float keep = hi ? v[i + 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  }
  {
    const bool hi = lane & 2;
    const float send = hi ? v[0] : v[1];
    const float keep = hi ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

template <typename T, class C>
__global__ void __launch_bounds__(C::kThreads)
    decode_attention_kernel(const Args a) {
  constexpr int kStages = C::kStages, kStagePos = C::kStagePos;
  constexpr int kComputeWarps = C::kComputeWarps, kStageBytes = C::kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  T* sK = reinterpret_cast<T*>(smem);
  T* sV = reinterpret_cast<T*>(smem + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);
  volatile int* last_flag = abort_flag + 1;
  float* cm = reinterpret_cast<float*>(smem + 2 * kStages * kStageBytes + 256);
  float* cl = cm + kComputeWarps;
  float* co = cl + kComputeWarps;  // [warp][128]
  int32_t* pages = reinterpret_cast<int32_t*>(co + kComputeWarps * kD);  // [kMaxChunkPages]
  volatile int* bad_page = last_flag + 1;

  const int c = blockIdx.x, h = blockIdx.y, j = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();
  pdl_launch_dependents();
  const int p = a.pos[j];
  const int c0 = a.counts ? a.counts[0] : a.split_point;
  const int m = j >= c0 ? 1 : 0;
  const bool paged = a.block_table != nullptr;
  const int sl = paged ? 0 : (a.slot ? a.slot[j] : j - (m ? c0 : 0));
  if (p < 0 || p >= a.L_cap || sl < 0 || (!paged && sl >= (m ? a.slots1 : a.slots0))) {
    if (tid == 0 && c == 0) set_status(a.status, PS_ERR_BAD_INDEX);
    return;
  }
  const int L = p + 1;
  if (L > a.max_chunks * a.chunk) {  // beyond the length the grid was sized for
    if (tid == 0 && c == 0) set_status(a.status, PS_ERR_BAD_INDEX);
    return;
  }
  const int cstart = c * a.chunk;
  if (cstart >= L) return;
  const int cend = min(L, cstart + a.chunk);
  const int nsplit = (L + a.chunk - 1) / a.chunk;
  const int nst = (cend - cstart + kStagePos - 1) / kStagePos;
  // contiguous: the (slot, head) stream; paged: the pool base (pages looked up per copy)
  const size_t stream_off = paged ? 0 : ((size_t)sl * a.n_heads + h) * a.L_cap * kD;
  const T* kbase = reinterpret_cast<const T*>(m ? a.kp1 : a.kp0) + stream_off;
  const T* vbase = reinterpret_cast<const T*>(m ? a.vp1 : a.vp0) + stream_off;
  const int first_page = paged ? cstart >> a.page_shift : 0;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kComputeWarps);
    }
    abort_flag[0] = 0;
    bad_page[0] = 0;
    fence_mbar_init();
  }
  if (paged && warp == kComputeWarps) {
    // Stage and check this chunk's page ids before any copy is issued.
    __syncwarp();
    const int npages = ((cend - 1) >> a.page_shift) - first_page + 1;
    const int pool_pages = m ? a.slots1 : a.slots0;
    const int bt_row = a.seq_rows ? a.seq_rows[j] : j;
    // the plan keeps npages in the table; bt_row comes from the caller
    int bad = npages > kMaxChunkPages || bt_row < 0 || bt_row >= a.table_rows;
    for (int i = lane; i < npages && !bad; i += 32) {
      const int pg = a.block_table[(size_t)bt_row * a.max_pages + first_page + i];
      bad |= (pg < 0 || pg >= pool_pages);
      pages[i] = pg;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) {
      bad_page[0] = 1;
      set_status(a.status, PS_ERR_BAD_INDEX);
    }
  }
  __syncthreads();
  if (bad_page[0]) return;

  if (warp == kComputeWarps) {
    // -------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int s = 0;
      for (; s < nst && !abort_flag[0]; ++s) {
        const int st = s % kStages;
        if (!mbar_wait(empty + st, ((s / kStages) & 1) ^ 1, a.status)) {
          abort_flag[0] = 1;
          break;
        }
        const int pos0 = cstart + s * kStagePos;
        const int npos = min(kStagePos, cend - pos0);
        const uint32_t bytes = (uint32_t)npos * kD * 2;
        mbar_arrive_expect_tx(full + st, 2 * bytes);
        if (!paged) {
          bulk_load(sK + st * kStagePos * kD, kbase + (size_t)pos0 * kD, bytes, full + st, pol);
          bulk_load(sV + st * kStagePos * kD, vbase + (size_t)pos0 * kD, bytes, full + st, pol);
        } else {
          // one copy per page run: positions [t, t + n) of one page
          const int ps = a.page_size;
          for (int done = 0; done < npos;) {
            const int t = pos0 + done;
            const int off = t & (ps - 1);
            const int n = min(ps - off, npos - done);
            const size_t src =
                (((size_t)pages[(t >> a.page_shift) - first_page] * a.n_heads + h) * ps + off) * kD;
            const uint32_t nb = (uint32_t)n * kD * 2;
            bulk_load(sK + (st * kStagePos + done) * kD, kbase + src, nb, full + st, pol);
            bulk_load(sV + (st * kStagePos + done) * kD, vbase + src, nb, full + st, pol);
            done += n;
          }
        }
      }
      if (abort_flag[0]) {
        for (int st = 0; st < kStages && st < s; ++st) {
          const int last = st + kStages * ((s - 1 - st) / kStages);
          mbar_wait(full + st, (last / kStages) & 1, a.status);
        }
      }
    }
    return;
  }

  // ---------------------------------------------------------------- compute
  float q4[4];
  load4<T>(reinterpret_cast<const T*>(a.q) + (size_t)j * a.n_heads * kD + h * kD + 4 * lane, q4);
#pragma unroll
  for (int k = 0; k < 4; ++k) q4[k] *= a.scale_log2;
  float m_run = -INFINITY, l_run = 0.f;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  const int kb = warp * 16;

  for (int s = 0; s < nst; ++s) {
    const int st = s % kStages;
    if (abort_flag[0] || !mbar_wait(full + st, (s / kStages) & 1, a.status)) {
      abort_flag[0] = 1;
      break;
    }
    const int npos = min(kStagePos, cend - (cstart + s * kStagePos));
    if (kb < npos) {
      const T* Ks = sK + st * kStagePos * kD + 4 * lane;
      const T* Vs = sV + st * kStagePos * kD + 4 * lane;
      float part[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float kf[4];
        load4<T>(Ks + (kb + i) * kD, kf);
        part[i] = q4[0] * kf[0] + q4[1] * kf[1] + q4[2] * kf[2] + q4[3] * kf[3];
      }
      const float dot = reduce_scatter16(part, lane);
      const int key = kb + (lane >> 1);
      const bool valid = key < npos;
      const float sc = valid ? dot : -INFINITY;
      float mx = sc;
#pragma unroll
      for (int off = 16; off >= 2; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run, mx);
      const float alpha = exp2f(m_run - m_new);
      const float pe = valid ? exp2f(sc - m_new) : 0.f;
      float ps = pe;
#pragma unroll
      for (int off = 16; off >= 2; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      l_run = l_run * alpha + ps;
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] *= alpha;
      m_run = m_new;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (kb + i < npos) {
          const float pi = __shfl_sync(0xffffffffu, pe, 2 * i);
          float vf[4];
          load4<T>(Vs + (kb + i) * kD, vf);
#pragma unroll
          for (int k = 0; k < 4; ++k) o[k] += pi * vf[k];
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + st);
  }

  // Merge the four warps' partial softmax states.
  if (lane == 0) {
    cm[warp] = m_run;
    cl[warp] = l_run;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) co[warp * kD + 4 * lane + k] = o[k];
  named_bar_sync(1, kComputeWarps * 32);
  const int t = tid;  // output dimension (threads >= 128 only join the barriers)
  const bool dim_thread = t < kD;
  float M_ = -INFINITY;
#pragma unroll
  for (int w = 0; w < kComputeWarps; ++w) M_ = fmaxf(M_, cm[w]);
  float Ls = 0.f, Os = 0.f;
#pragma unroll
  for (int w = 0; w < kComputeWarps; ++w) {
    const float sc = (cm[w] == -INFINITY) ? 0.f : exp2f(cm[w] - M_);
    Ls += cl[w] * sc;
    if (dim_thread) Os += co[w * kD + t] * sc;
  }
  T* out = reinterpret_cast<T*>(a.out) + (size_t)j * a.n_heads * kD + h * kD;
  if (nsplit == 1) {
    if (dim_thread) out[t] = from_f32<T>(Os / Ls);
    return;
  }
  const int item = j * a.n_heads + h;
  const size_t slot_idx = (size_t)item * a.max_chunks + c;
  if (dim_thread) __stcg(a.ws_o + slot_idx * kD + t, Os);
  if (t == 0) {
    __stcg(a.ws_ml + slot_idx * 2, M_);
    __stcg(a.ws_ml + slot_idx * 2 + 1, Ls);
  }
  named_bar_sync(1, kComputeWarps * 32);
  if (t == 0) {
    fence_acq_rel_gpu();
    const int old = atom_add_acq_rel_gpu(a.counter + item, 1);
    const int last = (old + 1 == nsplit) ? 1 : 0;
    if (last) a.counter[item] = 0;
    last_flag[0] = last;
  }
  named_bar_sync(1, kComputeWarps * 32);
  if (!last_flag[0]) return;
  const size_t base = (size_t)item * a.max_chunks;
  float Mx = -INFINITY;
  for (int cc = 0; cc < nsplit; ++cc) Mx = fmaxf(Mx, __ldcg(a.ws_ml + (base + cc) * 2));
  if (!dim_thread) return;
  float Lt = 0.f, Ot = 0.f;
  for (int cc = 0; cc < nsplit; ++cc) {
    const float sc = exp2f(__ldcg(a.ws_ml + (base + cc) * 2) - Mx);
    Lt += __ldcg(a.ws_ml + (base + cc) * 2 + 1) * sc;
    Ot += __ldcg(a.ws_o + (base + cc) * kD + t) * sc;
  }
  out[t] = from_f32<T>(Ot / Lt);
}

// Balanced split ("stream-K" over positions): G CTAs (3 per SM, one wave)
// each take an equal contiguous range of the linearised (token, head,
// position) space, so a launch with few (token, head) items — 4 heads per GPU
// under 8-way tensor parallelism — has no partial last wave. A range covers
// the tail of one item, whole items and the head of another: whole items are
// written directly; a CTA's first and last pieces, when partial, go to its
// two partial slots, and the last-arriving contributor of an item merges the
// pieces in CTA order (deterministic). Token lengths and their prefix sums are
// computed by every CTA in shared memory, so the split follows the device
// lengths of this step.
constexpr int kSkMaxTokens = 1024;

struct SkSeg {
  int j, h, cstart, cend, slot, nsplit, b_first;
  long long istart, end;
};

// The piece of this CTA's range that starts at linear position g.
PS_DEV SkSeg sk_segment(const int32_t* P, int M, int nh, long long S, long long g,
                        long long g1, int b) {
  int lo = 0, hi = M - 1;  // largest j with P[j] * nh <= g
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((long long)P[mid] * nh <= g) lo = mid; else hi = mid - 1;
  }
  SkSeg sg;
  sg.j = lo;
  const long long tbase = (long long)P[lo] * nh;
  const int L = P[lo + 1] - P[lo];
  sg.h = (int)((g - tbase) / L);
  const int p0 = (int)((g - tbase) % L);
  sg.istart = tbase + (long long)sg.h * L;
  const long long iend = sg.istart + L;
  sg.end = g1 < iend ? g1 : iend;
  sg.cstart = p0;
  sg.cend = p0 + (int)(sg.end - g);
  sg.b_first = (int)(sg.istart / S);
  sg.nsplit = (int)((iend - 1) / S) - sg.b_first + 1;
  sg.slot = (g == (long long)b * S) ? 0 : 1;
  return sg;
}

template <typename T, class C>
__global__ void __launch_bounds__(C::kThreads)
    decode_attention_sk_kernel(const Args a) {
  constexpr int kStages = C::kStages, kStagePos = C::kStagePos;
  constexpr int kComputeWarps = C::kComputeWarps, kStageBytes = C::kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  T* sK = reinterpret_cast<T*>(smem);
  T* sV = reinterpret_cast<T*>(smem + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);
  volatile int* last_flag = abort_flag + 1;
  int* wsum = const_cast<int*>(last_flag) + 1;  // [8] per-warp scan totals
  volatile int* stage_bad = wsum + 8;           // [kStages] the stage's piece read a bad page
  float* cm = reinterpret_cast<float*>(smem + 2 * kStages * kStageBytes + 256);
  float* cl = cm + kComputeWarps;
  float* co = cl + kComputeWarps;                                         // [warp][128]
  int32_t* pages = reinterpret_cast<int32_t*>(co + kComputeWarps * kD);  // [kMaxChunkPages]
  int32_t* P = pages + kMaxChunkPages;                                  // [kSkMaxTokens + 1]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x;
  const int M = a.M, nh = a.n_heads;
  const bool paged = a.block_table != nullptr;
  pdl_wait();
  pdl_launch_dependents();
  const int c0 = a.counts ? a.counts[0] : a.split_point;
  // token lengths (0 for a token whose position or slot is out of range)
  for (int j = tid; j < M; j += blockDim.x) {
    const int p = a.pos[j];
    const int m = j >= c0 ? 1 : 0;
    const int sl = paged ? 0 : (a.slot ? a.slot[j] : j - (m ? c0 : 0));
    const bool ok = p >= 0 && p < a.L_cap && sl >= 0 && (paged || sl < (m ? a.slots1 : a.slots0));
    if (!ok && b == 0) set_status(a.status, PS_ERR_BAD_INDEX);
    P[j + 1] = ok ? p + 1 : 0;
  }
  if (tid == 0) {
    P[0] = 0;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kComputeWarps);
    }
    abort_flag[0] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  {  // in-place inclusive prefix sums of P[1..M]: per-thread runs, then a block scan
    const int per = (M + blockDim.x - 1) / blockDim.x;
    const int j0 = min(M, tid * per), j1 = min(M, j0 + per);
    int run = 0;
    for (int j = j0; j < j1; ++j) run += P[j + 1];
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += wsum[w];
    int acc = wbase + incl - run;
    __syncthreads();
    for (int j = j0; j < j1; ++j) {
      acc += P[j + 1];
      P[j + 1] = acc;
    }
  }
  __syncthreads();
  const long long W = (long long)P[M] * nh;
  const long long S = (W + gridDim.x - 1) / gridDim.x;
  const long long g0 = (long long)b * S;
  const long long g1 = g0 + S < W ? g0 + S : W;
  if (g0 >= g1) return;

  if (warp == kComputeWarps) {
    // -------------------------------------------------------------- producer
    const uint64_t pol = l2_policy_evict_first();
    int gs = 0;
    for (long long g = g0; g < g1 && !abort_flag[0];) {
      const SkSeg sg = sk_segment(P, M, nh, S, g, g1, b);
      const int m = sg.j >= c0 ? 1 : 0;
      const int sl = paged ? 0 : (a.slot ? a.slot[sg.j] : sg.j - (m ? c0 : 0));
      const size_t stream_off = paged ? 0 : ((size_t)sl * nh + sg.h) * a.L_cap * kD;
      const T* kbase = reinterpret_cast<const T*>(m ? a.kp1 : a.kp0) + stream_off;
      const T* vbase = reinterpret_cast<const T*>(m ? a.vp1 : a.vp0) + stream_off;
      const int first_page = paged ? sg.cstart >> a.page_shift : 0;
      int seg_bad = 0;
      if (paged) {  // this piece's page ids; a bad id reads page 0 and marks the piece
        const int npages = ((sg.cend - 1) >> a.page_shift) - first_page + 1;
        const int pool_pages = m ? a.slots1 : a.slots0;
        const int bt_row = a.seq_rows ? a.seq_rows[sg.j] : sg.j;
        const bool row_ok = bt_row >= 0 && bt_row < a.table_rows && npages <= kMaxChunkPages;
        int bad = !row_ok;
        for (int i = lane; i < npages && i < kMaxChunkPages; i += 32) {
          const int pg = row_ok ? a.block_table[(size_t)bt_row * a.max_pages + first_page + i] : 0;
          const bool good = pg >= 0 && pg < pool_pages;
          bad |= !good;
          pages[i] = good ? pg : 0;
        }
        seg_bad = __any_sync(0xffffffffu, bad) ? 1 : 0;
        if (seg_bad && lane == 0) set_status(a.status, PS_ERR_BAD_INDEX);
        __syncwarp();
      }
      const int nst = (sg.cend - sg.cstart + kStagePos - 1) / kStagePos;
      if (lane == 0) {
        for (int s = 0; s < nst; ++s, ++gs) {
          const int st = gs % kStages;
          if (!mbar_wait(empty + st, ((gs / kStages) & 1) ^ 1, a.status)) {
            abort_flag[0] = 1;
            break;
          }
          const int pos0 = sg.cstart + s * kStagePos;
          const int npos = min(kStagePos, sg.cend - pos0);
          const uint32_t bytes = (uint32_t)npos * kD * 2;
          stage_bad[st] = seg_bad;  // published to the compute warps by the arrive below
          mbar_arrive_expect_tx(full + st, 2 * bytes);
          if (!paged) {
            bulk_load(sK + st * kStagePos * kD, kbase + (size_t)pos0 * kD, bytes, full + st, pol);
            bulk_load(sV + st * kStagePos * kD, vbase + (size_t)pos0 * kD, bytes, full + st, pol);
          } else {
            const int ps = a.page_size;
            for (int done = 0; done < npos;) {
              const int t = pos0 + done;
              const int off = t & (ps - 1);
              const int n = min(ps - off, npos - done);
              const size_t src =
                  (((size_t)pages[(t >> a.page_shift) - first_page] * nh + sg.h) * ps + off) * kD;
              const uint32_t nb = (uint32_t)n * kD * 2;
              bulk_load(sK + (st * kStagePos + done) * kD, kbase + src, nb, full + st, pol);
              bulk_load(sV + (st * kStagePos + done) * kD, vbase + src, nb, full + st, pol);
              done += n;
            }
          }
        }
      }
      gs = __shfl_sync(0xffffffffu, gs, 0);
      __syncwarp();
      g = sg.end;
    }
    if (lane == 0 && abort_flag[0]) {
      for (int st = 0; st < kStages && st < gs; ++st) {
        const int last = st + kStages * ((gs - 1 - st) / kStages);
        mbar_wait(full + st, (last / kStages) & 1, a.status);
      }
    }
    return;
  }

  // ---------------------------------------------------------------- compute
  const int kb = warp * 16;
  const int t = tid;  // output dimension
  int gs = 0;
  for (long long g = g0; g < g1;) {
    const SkSeg sg = sk_segment(P, M, nh, S, g, g1, b);
    const int j = sg.j, h = sg.h;
    float q4[4];
    load4<T>(reinterpret_cast<const T*>(a.q) + (size_t)j * nh * kD + h * kD + 4 * lane, q4);
#pragma unroll
    for (int k = 0; k < 4; ++k) q4[k] *= a.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    bool seg_bad = false;  // the same for every compute thread (same stages)
    const int nst = (sg.cend - sg.cstart + kStagePos - 1) / kStagePos;
    for (int s = 0; s < nst; ++s, ++gs) {
      const int st = gs % kStages;
      if (abort_flag[0] || !mbar_wait(full + st, (gs / kStages) & 1, a.status)) {
        abort_flag[0] = 1;
        break;
      }
      seg_bad |= stage_bad[st] != 0;
      const int npos = min(kStagePos, sg.cend - (sg.cstart + s * kStagePos));
      if (kb < npos) {
        const T* Ks = sK + st * kStagePos * kD + 4 * lane;
        const T* Vs = sV + st * kStagePos * kD + 4 * lane;
        float part[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float kf[4];
          load4<T>(Ks + (kb + i) * kD, kf);
          part[i] = q4[0] * kf[0] + q4[1] * kf[1] + q4[2] * kf[2] + q4[3] * kf[3];
        }
        const float dot = reduce_scatter16(part, lane);
        const int key = kb + (lane >> 1);
        const bool valid = key < npos;
        const float sc = valid ? dot : -INFINITY;
        float mx = sc;
#pragma unroll
        for (int off = 16; off >= 2; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = exp2f(m_run - m_new);
        const float pe = valid ? exp2f(sc - m_new) : 0.f;
        float ps = pe;
#pragma unroll
        for (int off = 16; off >= 2; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l_run = l_run * alpha + ps;
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] *= alpha;
        m_run = m_new;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (kb + i < npos) {
            const float pi = __shfl_sync(0xffffffffu, pe, 2 * i);
            float vf[4];
            load4<T>(Vs + (kb + i) * kD, vf);
#pragma unroll
            for (int k = 0; k < 4; ++k) o[k] += pi * vf[k];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + st);
    }
    // merge the compute warps' softmax states (every compute warp gets here,
    // aborted or not, so the named barriers stay matched)
    if (lane == 0) {
      cm[warp] = m_run;
      cl[warp] = l_run;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) co[warp * kD + 4 * lane + k] = o[k];
    named_bar_sync(1, kComputeWarps * 32);
    const bool stop = abort_flag[0] != 0;
    float M_ = -INFINITY;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) M_ = fmaxf(M_, cm[w]);
    float Ls = 0.f, Os = 0.f;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) {
      const float sc = (cm[w] == -INFINITY) ? 0.f : exp2f(cm[w] - M_);
      Ls += cl[w] * sc;
      Os += co[w * kD + t] * sc;
    }
    T* out = reinterpret_cast<T*>(a.out) + (size_t)j * nh * kD + h * kD;
    if (!stop && sg.nsplit == 1) {
      if (!seg_bad) out[t] = from_f32<T>(Os / Ls);  // a bad page leaves the output unwritten
    } else if (!stop) {
      const size_t idx = (size_t)b * 2 + sg.slot;
      __stcg(a.ws_o + idx * kD + t, Os);
      if (t == 0) {
        __stcg(a.ws_ml + idx * 2, M_);
        __stcg(a.ws_ml + idx * 2 + 1, seg_bad ? -1.f : Ls);  // l < 0 marks a bad piece
      }
      named_bar_sync(1, kComputeWarps * 32);
      const int item = j * nh + h;
      if (t == 0) {
        fence_acq_rel_gpu();
        const int old = atom_add_acq_rel_gpu(a.counter + item, 1);
        const int last = (old + 1 == sg.nsplit) ? 1 : 0;
        if (last) a.counter[item] = 0;
        last_flag[0] = last;
      }
      named_bar_sync(1, kComputeWarps * 32);
      if (last_flag[0]) {  // contributors in CTA order; CTA cb's piece starts at max(istart, cb S)
        float Mx = -INFINITY;
        for (int cc = 0; cc < sg.nsplit; ++cc) {
          const long long cb = sg.b_first + cc;
          const int sl = (sg.istart <= cb * S) ? 0 : 1;
          Mx = fmaxf(Mx, __ldcg(a.ws_ml + ((size_t)cb * 2 + sl) * 2));
        }
        float Lt = 0.f, Ot = 0.f;
        bool any_bad = false;
        for (int cc = 0; cc < sg.nsplit; ++cc) {
          const long long cb = sg.b_first + cc;
          const size_t ix = (size_t)cb * 2 + ((sg.istart <= cb * S) ? 0 : 1);
          const float sc = exp2f(__ldcg(a.ws_ml + ix * 2) - Mx);
          const float lc = __ldcg(a.ws_ml + ix * 2 + 1);
          any_bad |= lc < 0.f;
          Lt += lc * sc;
          Ot += __ldcg(a.ws_o + ix * kD + t) * sc;
        }
        if (!any_bad) out[t] = from_f32<T>(Ot / Lt);
      }
    }
    named_bar_sync(1, kComputeWarps * 32);  // cm / co / last_flag are reused
    if (stop) break;
    g = sg.end;
  }
}

// Reference no-KV semantics: token j of model m attends to every token of
// model m's segment of the batch (non-causal). grid (M, n_heads), 4 warps;
// warp w takes keys w, w+4, ...; one key per step with a full warp reduction.
template <typename T>
__global__ void __launch_bounds__(128)
    segment_attention_kernel(const T* __restrict__ qkv, T* __restrict__ out, int M, int n_heads,
                             int split_point, const int32_t* __restrict__ counts,
                             float scale_log2) {
  __shared__ float cm[4], cl[4], co[4 * kD];
  pdl_wait();
  pdl_launch_dependents();
  const int j = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = n_heads * kD;
  const int c0 = counts ? counts[0] : split_point;
  const int s0 = j >= c0 ? c0 : 0;
  const int s1 = j >= c0 ? M : c0;
  float q4[4];
  load4<T>(qkv + (size_t)j * 3 * H + h * kD + 4 * lane, q4);
#pragma unroll
  for (int k = 0; k < 4; ++k) q4[k] *= scale_log2;
  float m_run = -INFINITY, l_run = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = s0 + warp; i < s1; i += 4) {
    float kf[4], vf[4];
    load4<T>(qkv + (size_t)i * 3 * H + H + h * kD + 4 * lane, kf);
    float d = q4[0] * kf[0] + q4[1] * kf[1] + q4[2] * kf[2] + q4[3] * kf[3];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    const float m_new = fmaxf(m_run, d);
    const float alpha = exp2f(m_run - m_new);
    const float pe = exp2f(d - m_new);
    l_run = l_run * alpha + pe;
    load4<T>(qkv + (size_t)i * 3 * H + 2 * H + h * kD + 4 * lane, vf);
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = o[k] * alpha + pe * vf[k];
    m_run = m_new;
  }
  if (lane == 0) {
    cm[warp] = m_run;
    cl[warp] = l_run;
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) co[warp * kD + 4 * lane + k] = o[k];
  __syncthreads();
  const int t = threadIdx.x;
  float M_ = -INFINITY;
  for (int w = 0; w < 4; ++w) M_ = fmaxf(M_, cm[w]);
  float Ls = 0.f, Os = 0.f;
  for (int w = 0; w < 4; ++w) {
    const float sc = (cm[w] == -INFINITY) ? 0.f : exp2f(cm[w] - M_);
    Ls += cl[w] * sc;
    Os += co[w * kD + t] * sc;
  }
  out[(size_t)j * H + h * kD + t] = from_f32<T>(Os / Ls);
}

// 4 compute warps x 2 stages of 64 positions: 64 KB per CTA, 3 CTAs per SM.
// Measured on B200 (B=64, 32 heads, KV 2049): 6.76 TB/s vs 5.93 for 3 stages
// at 2 CTAs per SM; best or within 2% of best at 4..32 heads per GPU.
using DefaultCfg = Cfg<4, 2>;

template <typename T, class C>
static int launch_cfg(dim3 grid, const Args& a, cudaStream_t st) {
  if (allow_dynamic_smem(decode_attention_kernel<T, C>, C::kSmemBytes) != cudaSuccess)
    return PS_ERR_CUDA;
  return ps::launch(decode_attention_kernel<T, C>, grid, dim3(C::kThreads), C::kSmemBytes, st,
                    a) ==
                 cudaSuccess
             ? PS_OK
             : PS_ERR_CUDA;
}

struct Plan {
  int chunk, max_chunks;
  int sk_grid;  // > 0: balanced split over this many CTAs (decode_attention_sk_kernel)
  size_t counter_bytes, ml_bytes, o_bytes;
};

// CTAs of one balanced-split launch: three per SM (one wave); more when the
// pieces would otherwise span more pages than a CTA's page table holds.
static int sk_grid_for(int M, int n_heads, int max_len, int device, int page_size) {
  long long g = 3ll * sm_count(device);
  if (page_size > 0) {
    const long long cap = (long long)(kMaxChunkPages - 2) * page_size;  // positions per piece
    const long long need = ((long long)M * n_heads * max_len + cap - 1) / cap;
    if (need > g) g = need;
  }
  return (int)g;
}

// chunk > 0: that many positions per CTA; chunk == 0: automatic — one CTA per
// (token, head) when they cover the SMs several times, else the balanced
// split; chunk == -1: the balanced split.
static Plan plan_for(int M, int n_heads, int max_len, int chunk, int device, int page_size = 0) {
  Plan p;
  p.sk_grid = 0;
  const long long pairs = (long long)M * n_heads;
  if ((chunk == -1 || (chunk == 0 && pairs < 8ll * sm_count(device))) && M <= kSkMaxTokens) {
    p.sk_grid = sk_grid_for(M, n_heads, max_len, device, page_size);
    p.chunk = 0;
    p.max_chunks = 0;
    p.counter_bytes = kCounterRegionBytes;
    p.ml_bytes = ((size_t)p.sk_grid * 2 * 2 * 4 + 255) / 256 * 256;
    p.o_bytes = (size_t)p.sk_grid * 2 * kD * 4;
    return p;
  }
  if (chunk <= 0) {
    // Enough CTAs to cover every SM a few times over; 2 CTAs fit per SM.
    const long long target = 8ll * sm_count(device);
    long long nsplit = pairs >= target ? 1 : (target + pairs - 1) / pairs;
    const long long max_split = cdiv(max_len, kChunkAlign);
    if (nsplit > max_split) nsplit = max_split;
    if (nsplit < 1) nsplit = 1;
    chunk = round_up(cdiv(max_len, (int)nsplit), kChunkAlign);
  }
  p.chunk = round_up(chunk, kChunkAlign);
  if (p.chunk < kChunkAlign) p.chunk = kChunkAlign;
  if (page_size > 0) {  // a chunk's page ids must fit the shared-memory table
    const long long cap = (long long)(kMaxChunkPages - 1) * page_size / kChunkAlign * kChunkAlign;
    if (cap >= kChunkAlign && p.chunk > cap) p.chunk = (int)cap;
  }
  p.max_chunks = cdiv(max_len, p.chunk);
  const size_t items = (size_t)M * n_heads;
  if (p.max_chunks <= 1) {
    p.counter_bytes = p.ml_bytes = p.o_bytes = 0;
  } else {
    p.counter_bytes = kCounterRegionBytes;
    p.ml_bytes = (items * p.max_chunks * 2 * 4 + 255) / 256 * 256;
    p.o_bytes = items * p.max_chunks * kD * 4;
  }
  return p;
}

}  // namespace attn
}  // namespace ps

using namespace ps;

namespace ps {
namespace attn {

struct Paging {
  const int32_t* block_table = nullptr;
  const int32_t* seq_rows = nullptr;
  int table_rows = 0, max_pages = 0, page_size = 0;
};

static int decode_attention(const void* q, const void* k_pool0, const void* v_pool0,
                            const void* k_pool1, const void* v_pool1, void* out,
                            const int32_t* pos, const int32_t* slot, const int32_t* counts,
                            int split_point, int M, int n_heads, int L_cap, int slots0, int slots1,
                            int max_len, int chunk, float scale, int dtype, const Paging& pg,
                            void* workspace, size_t workspace_bytes, int32_t* status,
                            cudaStream_t st) {
  PS_CHECK_ARG(M >= 0 && n_heads > 0 && L_cap > 0 && max_len > 0 && max_len <= L_cap);
  PS_CHECK_ARG(slots0 >= 0 && slots1 >= 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (!counts) PS_CHECK_ARG(split_point >= 0 && split_point <= M);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(M <= 65535 && chunk >= -1);
  PS_CHECK_ARG(q && out && pos);
  PS_CHECK_ARG((k_pool0 && v_pool0 && aligned16(k_pool0) && aligned16(v_pool0)) || slots0 == 0);
  PS_CHECK_ARG((k_pool1 && v_pool1 && aligned16(k_pool1) && aligned16(v_pool1)) || slots1 == 0);
  const int device = current_device();
  const Plan p = plan_for(M, n_heads, max_len, chunk, device, pg.page_size);
  const size_t need = p.counter_bytes + p.ml_bytes + p.o_bytes;
  if (need > 0 && (!workspace || workspace_bytes < need)) return PS_ERR_WORKSPACE;
  if (need > 0 && (size_t)M * n_heads > (size_t)kMaxCounters) return PS_ERR_UNSUPPORTED;

  Args a{};
  a.q = q;
  a.kp0 = k_pool0;
  a.vp0 = v_pool0;
  a.kp1 = k_pool1;
  a.vp1 = v_pool1;
  a.out = out;
  a.pos = pos;
  a.slot = slot;
  a.counts = counts;
  char* ws = reinterpret_cast<char*>(workspace);
  a.counter = need ? reinterpret_cast<int32_t*>(ws) : nullptr;
  a.ws_ml = need ? reinterpret_cast<float*>(ws + p.counter_bytes) : nullptr;
  a.ws_o = need ? reinterpret_cast<float*>(ws + p.counter_bytes + p.ml_bytes) : nullptr;
  a.status = status;
  a.split_point = split_point;
  a.M = M;
  a.n_heads = n_heads;
  a.L_cap = L_cap;
  a.slots0 = slots0;
  a.slots1 = slots1;
  a.chunk = p.chunk;
  a.max_chunks = p.max_chunks;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.block_table = pg.block_table;
  a.seq_rows = pg.seq_rows;
  a.table_rows = pg.table_rows;
  a.max_pages = pg.max_pages;
  a.page_size = pg.page_size;
  a.page_shift = 0;
  while (pg.page_size > 0 && (1 << a.page_shift) < pg.page_size) ++a.page_shift;

  if (p.sk_grid > 0) {
    constexpr int smem = DefaultCfg::kSmemBytes + (kSkMaxTokens + 1) * 4;
    if (dtype == PS_DTYPE_BF16) {
      if (allow_dynamic_smem(decode_attention_sk_kernel<__nv_bfloat16, DefaultCfg>, smem) !=
          cudaSuccess)
        return PS_ERR_CUDA;
      return ps::launch(decode_attention_sk_kernel<__nv_bfloat16, DefaultCfg>, dim3(p.sk_grid),
                        dim3(DefaultCfg::kThreads), smem, st, a) == cudaSuccess
                 ? PS_OK
                 : PS_ERR_CUDA;
    }
    if (allow_dynamic_smem(decode_attention_sk_kernel<__half, DefaultCfg>, smem) != cudaSuccess)
      return PS_ERR_CUDA;
    return ps::launch(decode_attention_sk_kernel<__half, DefaultCfg>, dim3(p.sk_grid),
                      dim3(DefaultCfg::kThreads), smem, st, a) == cudaSuccess
               ? PS_OK
               : PS_ERR_CUDA;
  }
  dim3 grid(p.max_chunks, n_heads, M);
  if (dtype == PS_DTYPE_BF16) return launch_cfg<__nv_bfloat16, DefaultCfg>(grid, a, st);
  return launch_cfg<__half, DefaultCfg>(grid, a, st);
}

static bool valid_page_size(int ps) { return ps >= 8 && ps <= 4096 && (ps & (ps - 1)) == 0; }

}  // namespace attn
}  // namespace ps

extern "C" size_t ps_decode_attention_workspace_bytes(int M, int n_heads, int max_len, int chunk) {
  if (M <= 0 || n_heads <= 0 || max_len <= 0) return 0;
  const attn::Plan p = attn::plan_for(M, n_heads, max_len, chunk, current_device());
  return p.counter_bytes + p.ml_bytes + p.o_bytes;
}

extern "C" int ps_decode_attention(const void* q, const void* k_pool0, const void* v_pool0,
                                   const void* k_pool1, const void* v_pool1, void* out,
                                   const int32_t* pos, const int32_t* slot, const int32_t* counts,
                                   int split_point, int M, int n_heads, int L_cap, int slots0,
                                   int slots1, int max_len, int chunk, float scale, int dtype,
                                   void* workspace, size_t workspace_bytes, int32_t* status,
                                   ps_stream_t stream) {
  return attn::decode_attention(q, k_pool0, v_pool0, k_pool1, v_pool1, out, pos, slot, counts,
                                split_point, M, n_heads, L_cap, slots0, slots1, max_len, chunk,
                                scale, dtype, attn::Paging{}, workspace, workspace_bytes, status,
                                (cudaStream_t)stream);
}

extern "C" size_t ps_paged_decode_attention_workspace_bytes(int M, int n_heads, int max_len,
                                                            int chunk, int page_size) {
  if (M <= 0 || n_heads <= 0 || max_len <= 0 || !attn::valid_page_size(page_size)) return 0;
  const attn::Plan p = attn::plan_for(M, n_heads, max_len, chunk, current_device(), page_size);
  return p.counter_bytes + p.ml_bytes + p.o_bytes;
}

extern "C" int ps_paged_decode_attention(const void* q, const void* k_pages0,
                                         const void* v_pages0, const void* k_pages1,
                                         const void* v_pages1, void* out, const int32_t* pos,
                                         const int32_t* block_table, int table_rows,
                                         const int32_t* seq_rows, int max_pages, int page_size,
                                         const int32_t* counts, int split_point,
                                         int M, int n_heads, int pages0, int pages1, int max_len,
                                         int chunk, float scale, int dtype, void* workspace,
                                         size_t workspace_bytes, int32_t* status,
                                         ps_stream_t stream) {
  PS_CHECK_ARG(attn::valid_page_size(page_size) && max_pages > 0);
  PS_CHECK_ARG((long long)max_pages * page_size <= (1ll << 30));
  PS_CHECK_ARG(M == 0 || (block_table && table_rows > 0));
  PS_CHECK_ARG(seq_rows || table_rows >= M);
  attn::Paging pg;
  pg.table_rows = table_rows;
  pg.block_table = block_table;
  pg.seq_rows = seq_rows;
  pg.max_pages = max_pages;
  pg.page_size = page_size;
  return attn::decode_attention(q, k_pages0, v_pages0, k_pages1, v_pages1, out, pos, nullptr,
                                counts, split_point, M, n_heads, max_pages * page_size, pages0,
                                pages1, max_len, chunk, scale, dtype, pg, workspace,
                                workspace_bytes, status, (cudaStream_t)stream);
}

extern "C" int ps_segment_attention(const void* qkv, void* out, int M, int n_heads,
                                    int split_point, const int32_t* counts, float scale,
                                    int dtype, int32_t* status, ps_stream_t stream) {
  (void)status;
  PS_CHECK_ARG(M >= 0 && n_heads > 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (!counts) PS_CHECK_ARG(split_point >= 0 && split_point <= M);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(qkv && out);
  dim3 grid(M, n_heads);
  const float sl2 = scale * 1.4426950408889634f;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(attn::segment_attention_kernel<__nv_bfloat16>, grid, dim3(128), 0, st,
                       (const __nv_bfloat16*)qkv, (__nv_bfloat16*)out, M, n_heads, split_point,
                       counts, sl2));
  else
    PS_CUDA_RET(launch(attn::segment_attention_kernel<__half>, grid, dim3(128), 0, st,
                       (const __half*)qkv, (__half*)out, M, n_heads, split_point, counts, sl2));
  return PS_OK;
}
