// Causal prefill attention on the 5th-generation tensor cores (sm_100a).
//
// The reference only measures decode; its prefill plan is a varlen causal
// attention over the prompt (docs/routing_kernel_design.md:229-232). Here the
// prompt tokens of a routed prefill chunk already wrote their k / v into the
// KV cache (QKV epilogue), so attention for a query at position p reads the
// cache positions [0, p] of its own sequence: causal by position, varlen by
// construction, both models in one launch (each block reads its model's pool).
//
// Work item = (query block, head): up to 128 consecutive prompt tokens of one
// sequence (positions p0 .. p0+nq-1) against key blocks of 128 positions.
//   warp 0     TMA: Q once, then K and V blocks through a 2-stage ring
//   warp 1     MMA: S = Q K^T (M=128 queries, N=128 keys, K=128 dims) into one
//              of two TMEM S buffers; O += P V (A = P in shared memory, B = V
//              MN-major) into the TMEM O accumulator
//   warps 2-5  softmax, one thread per query row (its TMEM lane): row max,
//              exp2, row sum, P (16-bit, 128-byte swizzle) into shared memory,
//              rescale of the O row in TMEM only when the running max grows
//              by more than 2^8 (the result is exact either way: P and l use
//              the same stale max), final O / l to global memory.
// Every wait is bounded (%globaltimer); on a timeout the kernel sets
// PS_ERR_TIMEOUT, drains its copies and MMAs, frees TMEM and returns.
#include <cuda_runtime.h>

#include "ps_common.cuh"
#include "ps_host.h"

namespace ps {
namespace pfa {

constexpr int kQ = 128;                 // queries per work item
constexpr int kKeys = 128;              // keys per block
constexpr int kD = 128;                 // head dim
constexpr int kThreads = 192;
constexpr int kTile = kQ * kD * 2;      // 32 KB: Q, P, one K or one V block
constexpr int kHalf = kTile / 2;        // one 64-column box (128 rows x 128 B)
constexpr int kStages = 2;
constexpr int kSmem = 1024 + kTile * (2 + 2 * kStages) + 256;
constexpr int kTmemCols = 512;          // S buffers [0, 256), O [256, 384)
constexpr int kTmemO = 256;
constexpr float kRescaleLog2 = 8.f;     // rescale O only when the max grows by > 2^8

struct Args {
  void* out;
  const int32_t* blocks;  // [nblocks][5]: row0, nq, p0, model, slot (paged: block-table row)
  int nblocks, n_heads, T, L_cap, slots0, slots1, bf16;
  float scale_log2;
  int32_t* status;
  // paged pools (bt != nullptr): pools are [pages, n_heads, page_size, 128];
  // K / V of a 128-key block arrive as runs of box_rows = min(page_size, 128)
  const int32_t* bt;
  int table_rows, max_pages, page_size, box_rows;
};

// 16 consecutive keys (kcol % 16 == 0) of query row r into the P tile: two
// 16-byte chunks of a 128-byte swizzled row.
template <typename T>
PS_DEV void store_p16(uint8_t* sP, int r, int kcol, const float* p) {
  uint4 c[2];
  T* h = reinterpret_cast<T*>(c);
#pragma unroll
  for (int i = 0; i < 16; ++i) h[i] = from_f32<T>(p[i]);
  uint8_t* row = sP + (kcol >> 6) * kHalf + r * 128;
  const int ch = (kcol & 63) >> 3;
  *reinterpret_cast<uint4*>(row + (((ch) ^ (r & 7)) << 4)) = c[0];
  *reinterpret_cast<uint4*>(row + (((ch + 1) ^ (r & 7)) << 4)) = c[1];
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap tq,
                             const __grid_constant__ CUtensorMap tk0,
                             const __grid_constant__ CUtensorMap tv0,
                             const __grid_constant__ CUtensorMap tk1,
                             const __grid_constant__ CUtensorMap tv1, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem =
      reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sP = sQ + kTile;
  uint8_t* sK = sP + kTile;               // [kStages] K blocks
  uint8_t* sV = sK + kStages * kTile;     // [kStages] V blocks
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kStages * kTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(kv_full + i, 1);
      mbar_init(kv_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full + i, 1);
      mbar_init(s_empty + i, 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    flags[0] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  if (threadIdx.x == 0) pdl_launch_dependents();

  const int h = blockIdx.y;
  const int32_t* blk = a.blocks + (size_t)blockIdx.x * 5;
  const int row0 = blk[0], nq = blk[1], p0 = blk[2], m = blk[3], slot = blk[4];
  const int slots = m ? a.slots1 : a.slots0;
  const bool valid = nq >= 1 && nq <= kQ && row0 >= 0 && row0 + nq <= a.T && p0 >= 0 &&
                     p0 + nq <= a.L_cap && (m == 0 || m == 1) && slot >= 0 &&
                     (a.bt ? slot < a.table_rows : slot < slots);
  if (!valid && threadIdx.x == 0) set_status(a.status, PS_ERR_BAD_INDEX);
  const int nkb = valid ? (p0 + nq + kKeys - 1) / kKeys : 0;
  const int kv_row0 = (slot * a.n_heads + h) * a.L_cap;  // first pool row of (slot, head)
  const CUtensorMap* tk = m ? &tk1 : &tk0;
  const CUtensorMap* tv = m ? &tv1 : &tv0;

  if (nkb == 0) {
    // nothing to do (invalid item)
  } else if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();  // a sequence's K / V serve all its blocks
      mbar_arrive_expect_tx(q_full, kTile);
      tma_load_2d(sQ, &tq, q_full, h * kD, row0, pol);
      tma_load_2d(sQ + kHalf, &tq, q_full, h * kD + 64, row0, pol);
      int j = 0;
      for (; j < nkb && !flags[0]; ++j) {
        const int st = j & 1;
        if (!mbar_wait(kv_empty + st, ((j >> 1) & 1) ^ 1, a.status)) {
          flags[0] = 1;
          break;
        }
        if (!a.bt) {
          const int r = kv_row0 + j * kKeys;
          mbar_arrive_expect_tx(kv_full + st, 2 * kTile);
          tma_load_2d(sK + st * kTile, tk, kv_full + st, 0, r, pol);
          tma_load_2d(sK + st * kTile + kHalf, tk, kv_full + st, 64, r, pol);
          tma_load_2d(sV + st * kTile, tv, kv_full + st, 0, r, pol);
          tma_load_2d(sV + st * kTile + kHalf, tv, kv_full + st, 64, r, pol);
        } else {
          // one run of box_rows positions per page slice; runs past the
          // prompt are skipped (their keys are masked, their V rows cleared)
          const int nrun = kKeys / a.box_rows;
          int rows[kKeys / 8];
          int nissue = 0;
          for (int i = 0; i < nrun; ++i) {
            const int p = j * kKeys + i * a.box_rows;
            rows[i] = -1;
            if (p >= p0 + nq) continue;
            const int pi = p / a.page_size;
            const int pg = pi < a.max_pages ? a.bt[(size_t)slot * a.max_pages + pi] : -1;
            if (pg < 0 || pg >= slots) {
              set_status(a.status, PS_ERR_BAD_INDEX);
              continue;
            }
            rows[i] = (pg * a.n_heads + h) * a.page_size + (p % a.page_size);
            ++nissue;
          }
          const uint32_t run_bytes = (uint32_t)a.box_rows * 128;
          if (nissue > 0) {
            mbar_arrive_expect_tx(kv_full + st, 4 * run_bytes * nissue);
          } else {
            mbar_arrive(kv_full + st);  // nothing to load: complete the phase
          }
          for (int i = 0; i < nrun; ++i) {
            if (rows[i] < 0) continue;
            const int off = i * a.box_rows * 128;
            tma_load_2d(sK + st * kTile + off, tk, kv_full + st, 0, rows[i], pol);
            tma_load_2d(sK + st * kTile + kHalf + off, tk, kv_full + st, 64, rows[i], pol);
            tma_load_2d(sV + st * kTile + off, tv, kv_full + st, 0, rows[i], pol);
            tma_load_2d(sV + st * kTile + kHalf + off, tv, kv_full + st, 64, rows[i], pol);
          }
        }
      }
      if (flags[0]) {  // let every issued copy land before the CTA exits
        mbar_wait(q_full, 0, a.status);
        for (int st = 0; st < kStages && st < j; ++st) {
          const int last = st + kStages * ((j - 1 - st) / kStages);
          mbar_wait(kv_full + st, (last >> 1) & 1, a.status);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t idesc_s = idesc_f16(a.bf16, 0, 0, kQ, kKeys);  // Q, K both K-major
      const uint32_t idesc_o = idesc_f16(a.bf16, 0, 1, kQ, kD);     // P K-major, V MN-major
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, a.status);
      for (int j = 0; ok && j <= nkb && !flags[0]; ++j) {
        if (j < nkb) {
          const int st = j & 1;
          if (!mbar_wait(kv_full + st, (j >> 1) & 1, a.status) ||
              !mbar_wait(s_empty + st, ((j >> 1) & 1) ^ 1, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + st * kTile);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(q_addr + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(k_addr + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
            umma_f16(tmem + st * kKeys, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(s_full + st);
        }
        if (j >= 1) {  // O += P_{j-1} V_{j-1}
          const int jp = j - 1, st = jp & 1;
          if (!mbar_wait(p_full, jp & 1, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + st * kTile);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(p_addr + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(v_addr + kk * 2048, kHalf, 1024);
            umma_f16(tmem + kTmemO, ad, bd, idesc_o, (jp > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(o_done);
          umma_commit(kv_empty + st);
        }
      }
      if (!ok) flags[0] = 1;
      // Every MMA of this CTA completes before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, a.status);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int q = warp & 3;          // TMEM lane quadrant of this warp
    const int r = q * 32 + lane;     // query row = TMEM lane
    const int qp = p0 + r;           // its position
    const bool live = r < nq;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    float mrow = -INFINITY, lrow = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int st = j & 1;
      const bool got = !flags[0] && mbar_wait(s_full + st, (j >> 1) & 1, a.status);
      if (!__all_sync(0xffffffffu, got)) {  // the warp leaves together (collective TMEM ops)
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tmem + st * kKeys + lane_off;
      const int k0 = j * kKeys;
      // pass 1: row max of the visible keys
      float smax = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kKeys / 16; ++c) {
        float v[16];
        tmem_ld16(s_addr + c * 16, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (live && k0 + c * 16 + i <= qp) smax = fmaxf(smax, v[i] * a.scale_log2);
      }
      float muse = mrow;
      if (mrow == -INFINITY || smax > mrow + kRescaleLog2) muse = smax;
      // O and the P tile are free once P_{j-1} V_{j-1} completed
      if (j >= 1) {
        if (!__all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, a.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Rescale O rows whose max moved (lazy: rare after the first blocks).
        // tcgen05.ld / st are warp-collective (.sync.aligned): the whole warp
        // takes the branch when any of its rows needs it, the others scale by 1.
        const bool moved = muse != mrow;
        if (__any_sync(0xffffffffu, moved)) {
          const float alpha = moved ? exp2f(mrow - muse) : 1.f;
          lrow *= alpha;
#pragma unroll 1
          for (int c = 0; c < kD / 16; ++c) {
            float o[16];
            tmem_ld16(tmem + kTmemO + lane_off + c * 16, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= alpha;
            tmem_st16(tmem + kTmemO + lane_off + c * 16, o);
          }
          tmem_wait_st();
        }
      }
      mrow = muse;
      // pass 2: P = exp2(s - m) (0 for hidden keys and padding rows) and its row sum
      float lsum = 0.f;
#pragma unroll 1
      for (int c = 0; c < kKeys / 16; ++c) {
        float v[16];
        tmem_ld16(s_addr + c * 16, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const bool vis = live && k0 + c * 16 + i <= qp && mrow != -INFINITY;
          v[i] = vis ? exp2f(v[i] * a.scale_log2 - mrow) : 0.f;
          lsum += v[i];
        }
        store_p16<T>(sP, r, c * 16, v);
      }
      lrow += lsum;
      // keys past the prompt in the last block: their V rows may hold anything
      // (NaN would survive P = 0), so clear them for P V
      if (j == nkb - 1 && k0 + r >= p0 + nq) {
        uint4* vr0 = reinterpret_cast<uint4*>(sV + st * kTile + r * 128);
        uint4* vr1 = reinterpret_cast<uint4*>(sV + st * kTile + kHalf + r * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          vr0[c] = make_uint4(0u, 0u, 0u, 0u);
          vr1[c] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();  // P and cleared V rows -> the tensor core's view
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(s_empty + st);
        mbar_arrive(p_full);
      }
    }
    const bool fin = ok && !flags[0] && mbar_wait(o_done, (nkb - 1) & 1, a.status);
    if (__all_sync(0xffffffffu, fin)) {
      tc_fence_after();
      const float inv = lrow > 0.f ? 1.f / lrow : 0.f;
      T* orow = reinterpret_cast<T*>(a.out) + (size_t)(row0 + r) * a.n_heads * kD + h * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 16; ++c) {
        float o[16];
        tmem_ld16(tmem + kTmemO + lane_off + c * 16, o);
        if (live) {
          uint4 w[2];
          T* hw = reinterpret_cast<T*>(w);
#pragma unroll
          for (int i = 0; i < 16; ++i) hw[i] = from_f32<T>(o[i] * inv);
          reinterpret_cast<uint4*>(orow + c * 16)[0] = w[0];
          reinterpret_cast<uint4*>(orow + c * 16)[1] = w[1];
        }
      }
    } else {
      flags[0] = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace pfa
}  // namespace ps

using namespace ps;

extern "C" int ps_prefill_attention(const void* q, const void* k_pool0, const void* v_pool0,
                                    const void* k_pool1, const void* v_pool1, void* out,
                                    const int32_t* blocks, int nblocks, int T, int n_heads,
                                    int L_cap, int slots0, int slots1, const int32_t* block_table,
                                    int table_rows, int max_pages, int page_size, float scale,
                                    int dtype, int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(nblocks >= 0 && T >= 0 && n_heads > 0 && L_cap > 0 && slots0 >= 0 && slots1 >= 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (nblocks == 0 || T == 0) return PS_OK;
  PS_CHECK_ARG(q && out && blocks && aligned16(q) && aligned16(out));
  PS_CHECK_ARG((k_pool0 && v_pool0 && aligned16(k_pool0) && aligned16(v_pool0)) || slots0 == 0);
  PS_CHECK_ARG((k_pool1 && v_pool1 && aligned16(k_pool1) && aligned16(v_pool1)) || slots1 == 0);
  PS_CHECK_ARG(slots0 + slots1 > 0 && nblocks <= (1 << 30) && n_heads <= 65535);
  if (block_table) {
    PS_CHECK_ARG(table_rows > 0 && max_pages > 0 && page_size >= 8 && page_size <= 4096 &&
                 (page_size & (page_size - 1)) == 0);
    PS_CHECK_ARG((long long)max_pages * page_size >= L_cap);
  }
  const int box_rows = block_table ? (page_size < pfa::kKeys ? page_size : pfa::kKeys) : pfa::kQ;
  const int pool_rows_per = block_table ? page_size : L_cap;  // rows of one (slot|page, head)
  const int device = current_device();
  if (!is_sm100(device)) return PS_ERR_UNSUPPORTED;
  const bool bf = dtype == PS_DTYPE_BF16;
  const uint32_t box[2] = {64, (uint32_t)pfa::kQ};
  const uint32_t kv_box[2] = {64, (uint32_t)box_rows};
  CUtensorMap tq, tk[2], tv[2];
  {
    const uint64_t dims[2] = {(uint64_t)n_heads * pfa::kD, (uint64_t)T};
    const uint64_t strides[1] = {(uint64_t)n_heads * pfa::kD * 2};
    if (!make_tmap_16bit(&tq, q, 2, dims, strides, box, bf)) return PS_ERR_CUDA;
  }
  const void* kp[2] = {k_pool0, k_pool1};
  const void* vp[2] = {v_pool0, v_pool1};
  const int sl[2] = {slots0, slots1};
  for (int m = 0; m < 2; ++m) {
    // a model without slots gets the other model's maps (no block reads them)
    const int src = sl[m] > 0 ? m : 1 - m;
    const uint64_t rows = (uint64_t)sl[src] * n_heads * pool_rows_per;
    const uint64_t dims[2] = {(uint64_t)pfa::kD, rows};
    const uint64_t strides[1] = {(uint64_t)pfa::kD * 2};
    if (!make_tmap_16bit(&tk[m], kp[src], 2, dims, strides, kv_box, bf) ||
        !make_tmap_16bit(&tv[m], vp[src], 2, dims, strides, kv_box, bf))
      return PS_ERR_CUDA;
  }
  pfa::Args a;
  a.out = out;
  a.blocks = blocks;
  a.nblocks = nblocks;
  a.n_heads = n_heads;
  a.T = T;
  a.L_cap = L_cap;
  a.slots0 = slots0;
  a.slots1 = slots1;
  a.bf16 = bf ? 1 : 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.status = status;
  a.bt = block_table;
  a.table_rows = table_rows;
  a.max_pages = max_pages;
  a.page_size = page_size;
  a.box_rows = box_rows;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(nblocks, n_heads);
  if (bf) {
    PS_CUDA_RET(allow_dynamic_smem(pfa::prefill_attention_kernel<__nv_bfloat16>, pfa::kSmem));
    PS_CUDA_RET(launch(pfa::prefill_attention_kernel<__nv_bfloat16>, grid, dim3(pfa::kThreads),
                       pfa::kSmem, st, tq, tk[0], tv[0], tk[1], tv[1], a));
  } else {
    PS_CUDA_RET(allow_dynamic_smem(pfa::prefill_attention_kernel<__half>, pfa::kSmem));
    PS_CUDA_RET(launch(pfa::prefill_attention_kernel<__half>, grid, dim3(pfa::kThreads),
                       pfa::kSmem, st, tq, tk[0], tv[0], tk[1], tv[1], a));
  }
  return PS_OK;
}
