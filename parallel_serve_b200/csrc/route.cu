// Route bookkeeping and decode-step glue: stable model-id partition, row
// gather / scatter, routed embedding lookup, greedy argmax, positions.
//
// The reference routes by a host integer split_point
// (kernel/src/routed_gemm.py:157, 176-179): the caller pre-sorts tokens so
// model 0 comes first. Here the partition is computed on the device from
// per-token model ids, so decode batches with interleaved ids (model_id[i] =
// i % 2) need no host round trip and one CUDA graph serves any split.
#include <cuda_runtime.h>

#include "ps_common.cuh"
#include "ps_host.h"

namespace ps {
namespace route {

constexpr int kPartThreads = 1024;

// One CTA. Pass 1 counts model-0 tokens; pass 2 walks the ids in order in
// chunks of 1024 and places each token with a ballot/popc scan, which keeps
// both groups in original order (a stable partition).
__global__ void __launch_bounds__(kPartThreads)
    partition_kernel(const int32_t* __restrict__ ids, int M, int32_t* __restrict__ perm,
                     int32_t* __restrict__ counts, int32_t* status) {
  __shared__ int warp_tot[32];
  __shared__ int s_c0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_launch_dependents();

  int local = 0;
  for (int i = tid; i < M; i += kPartThreads) {
    const int id = ids[i];
    if (id != 0 && id != 1) set_status(status, PS_ERR_BAD_MODEL_ID);
    local += (id == 0);
  }
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  if (lane == 0) warp_tot[warp] = local;
  __syncthreads();
  if (tid == 0) {
    int c = 0;
    for (int w = 0; w < kPartThreads / 32; ++w) c += warp_tot[w];
    s_c0 = c;
    counts[0] = c;
    counts[1] = M - c;
  }
  __syncthreads();
  const int c0 = s_c0;

  int off0 = 0, off1 = 0;  // model-0 / model-1 tokens before this chunk
  for (int base = 0; base < M; base += kPartThreads) {
    const int i = base + tid;
    const bool valid = i < M;
    const bool is0 = valid && ids[i] == 0;
    const unsigned bal = __ballot_sync(0xffffffffu, is0);
    const int in_warp = __popc(bal & ((1u << lane) - 1u));
    __syncthreads();
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    int before = 0, chunk0 = 0;
    for (int w = 0; w < kPartThreads / 32; ++w) {
      const int v = warp_tot[w];
      before += (w < warp) ? v : 0;
      chunk0 += v;
    }
    const int rank0 = before + in_warp;  // model-0 tokens before i within the chunk
    if (valid) {
      const int local_i = tid;
      const int pos = is0 ? off0 + rank0 : c0 + off1 + (local_i - rank0);
      perm[pos] = i;
    }
    const int len = min(kPartThreads, M - base);
    off0 += chunk0;
    off1 += len - chunk0;
  }
}

__global__ void gather_rows_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ perm,
                                   uint4* __restrict__ dst, int M, int row_vec, int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int j = blockIdx.x;
  const int r = perm[j];
  if (r < 0 || r >= M) {
    if (threadIdx.x == 0) set_status(status, PS_ERR_BAD_INDEX);
    return;
  }
  const uint4* s = src + (size_t)r * row_vec;
  uint4* d = dst + (size_t)j * row_vec;
  for (int i = threadIdx.x; i < row_vec; i += blockDim.x) d[i] = s[i];
}

__global__ void scatter_rows_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ perm,
                                    uint4* __restrict__ dst, int M, int row_vec, int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int j = blockIdx.x;
  const int r = perm[j];
  if (r < 0 || r >= M) {
    if (threadIdx.x == 0) set_status(status, PS_ERR_BAD_INDEX);
    return;
  }
  const uint4* s = src + (size_t)j * row_vec;
  uint4* d = dst + (size_t)r * row_vec;
  for (int i = threadIdx.x; i < row_vec; i += blockDim.x) d[i] = s[i];
}

// x[j] = emb[m(j)][tokens[perm[j]]]; optionally sumsq[j] = sum(x[j]^2).
template <typename T>
__global__ void embed_kernel(const uint4* __restrict__ emb, const int32_t* __restrict__ tokens,
                             const int32_t* __restrict__ perm, const int32_t* __restrict__ counts,
                             uint4* __restrict__ x, int M, int row_vec, int vocab,
                             float* __restrict__ sumsq, int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int j = blockIdx.x;
  const int c0 = counts ? counts[0] : M;
  const int m = j >= c0 ? 1 : 0;
  const int src = perm ? perm[j] : j;
  if (src < 0 || src >= M) {
    if (threadIdx.x == 0) set_status(status, PS_ERR_BAD_INDEX);
    return;
  }
  const int tok = tokens[src];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) set_status(status, PS_ERR_BAD_INDEX);
    return;
  }
  const uint4* s = emb + ((size_t)m * vocab + tok) * row_vec;
  uint4* d = x + (size_t)j * row_vec;
  float sq = 0.f;
  for (int i = threadIdx.x; i < row_vec; i += blockDim.x) {
    const uint4 v = s[i];
    d[i] = v;
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float f = to_f32<T>(e[k]);
      sq += f * f;
    }
  }
  if (!sumsq) return;
  __shared__ float part[32];
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    sumsq[j] = t;
  }
}

template <typename T>
__global__ void argmax_kernel(const T* __restrict__ logits, const int32_t* __restrict__ perm,
                              int32_t* __restrict__ next, int32_t* __restrict__ seq_len, int M,
                              int V) {
  __shared__ float sv[32];
  __shared__ int si[32];
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
  __syncthreads();
  if (threadIdx.x == 0) {
    const int nw = blockDim.x >> 5;
    for (int w = 1; w < nw; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    if (bi == 0x7fffffff) bi = 0;  // all -inf / NaN row
    const int dst = perm ? perm[j] : j;
    next[dst] = bi;
    if (seq_len) seq_len[dst] += 1;
  }
}

__global__ void positions_kernel(const int32_t* __restrict__ seq_len,
                                 const int32_t* __restrict__ perm, int32_t* __restrict__ pos,
                                 int M) {
  pdl_wait();
  pdl_launch_dependents();
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < M; j += gridDim.x * blockDim.x)
    pos[j] = seq_len[perm ? perm[j] : j];
}

}  // namespace route
}  // namespace ps

using namespace ps;

extern "C" int ps_route_partition(const int32_t* model_id, int M, int32_t* perm, int32_t* counts,
                                  int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && counts);
  PS_CHECK_ARG(M == 0 || (model_id && perm));
  PS_CUDA_RET(launch(route::partition_kernel, dim3(1), dim3(route::kPartThreads), 0,
                     (cudaStream_t)stream, model_id, M, perm, counts, status));
  return PS_OK;
}

extern "C" int ps_gather_rows(const void* src, const int32_t* perm, void* dst, int M,
                              int row_bytes, int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && row_bytes > 0 && row_bytes % 16 == 0);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(src && perm && dst && aligned16(src) && aligned16(dst));
  PS_CUDA_RET(launch(route::gather_rows_kernel, dim3(M), dim3(128), 0, (cudaStream_t)stream,
                     (const uint4*)src, perm, (uint4*)dst, M, row_bytes / 16, status));
  return PS_OK;
}

extern "C" int ps_scatter_rows(const void* src, const int32_t* perm, void* dst, int M,
                               int row_bytes, int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && row_bytes > 0 && row_bytes % 16 == 0);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(src && perm && dst && aligned16(src) && aligned16(dst));
  PS_CUDA_RET(launch(route::scatter_rows_kernel, dim3(M), dim3(128), 0, (cudaStream_t)stream,
                     (const uint4*)src, perm, (uint4*)dst, M, row_bytes / 16, status));
  return PS_OK;
}

extern "C" int ps_embed_routed(const void* emb, const int32_t* tokens, const int32_t* perm,
                               const int32_t* counts, void* x, int M, int H, int vocab,
                               float* out_sumsq, int dtype, int32_t* status,
                               ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && H > 0 && (H * 2) % 16 == 0 && vocab > 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(emb && tokens && x && aligned16(emb) && aligned16(x));
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(route::embed_kernel<__nv_bfloat16>, dim3(M), dim3(128), 0,
                       (cudaStream_t)stream, (const uint4*)emb, tokens, perm, counts, (uint4*)x, M,
                       H * 2 / 16, vocab, out_sumsq, status));
  else
    PS_CUDA_RET(launch(route::embed_kernel<__half>, dim3(M), dim3(128), 0, (cudaStream_t)stream,
                       (const uint4*)emb, tokens, perm, counts, (uint4*)x, M, H * 2 / 16, vocab,
                       out_sumsq, status));
  return PS_OK;
}

extern "C" int ps_argmax_rows(const void* logits, const int32_t* perm, int32_t* next_tokens,
                              int32_t* seq_len, int M, int V, int dtype, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && V > 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(logits && next_tokens);
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(route::argmax_kernel<__nv_bfloat16>, dim3(M), dim3(512), 0,
                       (cudaStream_t)stream, (const __nv_bfloat16*)logits, perm, next_tokens,
                       seq_len, M, V));
  else
    PS_CUDA_RET(launch(route::argmax_kernel<__half>, dim3(M), dim3(512), 0, (cudaStream_t)stream,
                       (const __half*)logits, perm, next_tokens, seq_len, M, V));
  return PS_OK;
}

extern "C" int ps_positions_routed(const int32_t* seq_len, const int32_t* perm, int32_t* pos_out,
                                   int M, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(seq_len && pos_out);
  PS_CUDA_RET(launch(route::positions_kernel, dim3(1), dim3(256), 0, (cudaStream_t)stream,
                     seq_len, perm, pos_out, M));
  return PS_OK;
}
