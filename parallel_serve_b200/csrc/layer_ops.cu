// Per-layer element-wise / row-reduction kernels of the two-model decoder:
// per-model RMSNorm, SwiGLU, and RoPE + KV-cache append.
//
// Rounding follows the reference's torch ops so that the fp16 results agree
// with the serial per-model path:
//   F.rms_norm (experiments/two_model_block.py:56,69): fp32 x * rsqrt(mean(x^2)
//     + eps) rounded to the 16-bit type, then times the weight, rounded again.
//   F.silu(gate) * up (experiments/two_model_block.py:71-72): silu rounded to
//     the 16-bit type, product rounded again.
#include <cuda_runtime.h>

#include "ps_common.cuh"
#include "ps_host.h"

namespace ps {
namespace ops {

template <typename T>
struct Vec8 {
  T v[8];
};

// One CTA per row; 8 elements (16 bytes) per thread per step.
template <typename T>
__global__ void __launch_bounds__(256)
    rmsnorm_routed_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                          int M, int H, int split_point, const int32_t* __restrict__ counts,
                          float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int j = blockIdx.x;
  const int c0 = counts ? counts[0] : split_point;
  const int m = j >= c0 ? 1 : 0;
  const T* xr = x + (size_t)j * H;
  const T* wr = w + (size_t)m * H;
  T* yr = y + (size_t)j * H;
  const int nvec = H / 8;

  float ss = 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    const Vec8<T> a = reinterpret_cast<const Vec8<T>*>(xr)[i];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float f = to_f32<T>(a.v[k]);
      ss += f * f;
    }
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[0] / (float)H + eps);
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    const Vec8<T> a = reinterpret_cast<const Vec8<T>*>(xr)[i];
    const Vec8<T> g = reinterpret_cast<const Vec8<T>*>(wr)[i];
    Vec8<T> o;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float nrm = to_f32<T>(from_f32<T>(to_f32<T>(a.v[k]) * rstd));
      o.v[k] = from_f32<T>(nrm * to_f32<T>(g.v[k]));
    }
    reinterpret_cast<Vec8<T>*>(yr)[i] = o;
  }
}

template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ gu, T* __restrict__ out, int M, int FF) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t total = (size_t)M * FF;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t j = idx / FF, f = idx % FF;
    const float g = to_f32<T>(gu[j * 2 * FF + f]);
    const float u = to_f32<T>(gu[j * 2 * FF + FF + f]);
    const float s = to_f32<T>(from_f32<T>(g / (1.0f + __expf(-g))));
    out[idx] = from_f32<T>(s * u);
  }
}

// grid (M, n_heads), 64 threads: thread i rotates the pair (i, i + 64) of q
// and k (rotate-half convention) and copies v elements i and i + 64.
template <typename T>
__global__ void rope_kv_append_kernel(const T* __restrict__ qkv, T* __restrict__ q_out,
                                      T* k_pool0, T* v_pool0, T* k_pool1, T* v_pool1,
                                      const float* __restrict__ rc, const float* __restrict__ rs,
                                      const int32_t* __restrict__ pos,
                                      const int32_t* __restrict__ slot,
                                      const int32_t* __restrict__ counts, int split_point, int M,
                                      int n_heads, int L_cap, int slots0, int slots1,
                                      int apply_rope, int32_t* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int j = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
  const int H = n_heads * 128;
  const int c0 = counts ? counts[0] : split_point;
  const int m = j >= c0 ? 1 : 0;
  const int sl = slot ? slot[j] : j - (m ? c0 : 0);
  const int p = pos[j];
  const int nslots = m ? slots1 : slots0;
  if (sl < 0 || sl >= nslots || p < 0 || p >= L_cap) {
    if (i == 0) set_status(status, PS_ERR_BAD_INDEX);
    return;
  }
  const T* row = qkv + (size_t)j * 3 * H;
  const T* q = row + h * 128;
  const T* k = row + H + h * 128;
  const T* v = row + 2 * H + h * 128;
  T* kp = (m ? k_pool1 : k_pool0) + (((size_t)sl * n_heads + h) * L_cap + p) * 128;
  T* vp = (m ? v_pool1 : v_pool0) + (((size_t)sl * n_heads + h) * L_cap + p) * 128;
  T* qo = q_out + (size_t)j * H + h * 128;
  const float q1 = to_f32<T>(q[i]), q2 = to_f32<T>(q[i + 64]);
  const float k1 = to_f32<T>(k[i]), k2 = to_f32<T>(k[i + 64]);
  if (apply_rope) {
    const float c = rc[(size_t)p * 64 + i], s = rs[(size_t)p * 64 + i];
    qo[i] = from_f32<T>(q1 * c - q2 * s);
    qo[i + 64] = from_f32<T>(q2 * c + q1 * s);
    kp[i] = from_f32<T>(k1 * c - k2 * s);
    kp[i + 64] = from_f32<T>(k2 * c + k1 * s);
  } else {
    qo[i] = q[i];
    qo[i + 64] = q[i + 64];
    kp[i] = k[i];
    kp[i + 64] = k[i + 64];
  }
  vp[i] = v[i];
  vp[i + 64] = v[i + 64];
}

}  // namespace ops
}  // namespace ps

using namespace ps;

extern "C" int ps_rmsnorm_routed(const void* x, const void* w, void* y, int M, int H,
                                 int split_point, const int32_t* counts, float eps, int dtype,
                                 int32_t* status, ps_stream_t stream) {
  (void)status;
  PS_CHECK_ARG(M >= 0 && H > 0 && H % 8 == 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (!counts) PS_CHECK_ARG(split_point >= 0 && split_point <= M);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(x && w && y && aligned16(x) && aligned16(w) && aligned16(y));
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(ops::rmsnorm_routed_kernel<__nv_bfloat16>, dim3(M), dim3(256), 0, st,
                       (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, M, H,
                       split_point, counts, eps));
  else
    PS_CUDA_RET(launch(ops::rmsnorm_routed_kernel<__half>, dim3(M), dim3(256), 0, st,
                       (const __half*)x, (const __half*)w, (__half*)y, M, H, split_point, counts,
                       eps));
  return PS_OK;
}

extern "C" int ps_swiglu(const void* gu, void* out, int M, int FF, int dtype, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && FF > 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(gu && out);
  const size_t total = (size_t)M * FF;
  const size_t want = (total + 255) / 256;
  const int blocks = (int)(want < 4096 ? want : 4096);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(ops::swiglu_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st,
                       (const __nv_bfloat16*)gu, (__nv_bfloat16*)out, M, FF));
  else
    PS_CUDA_RET(launch(ops::swiglu_kernel<__half>, dim3(blocks), dim3(256), 0, st,
                       (const __half*)gu, (__half*)out, M, FF));
  return PS_OK;
}

extern "C" int ps_rope_kv_append(const void* qkv, void* q_out, void* k_pool0, void* v_pool0,
                                 void* k_pool1, void* v_pool1, const float* rope_cos,
                                 const float* rope_sin, const int32_t* pos, const int32_t* slot,
                                 const int32_t* counts, int split_point, int M, int n_heads,
                                 int L_cap, int slots0, int slots1, int apply_rope, int dtype,
                                 int32_t* status, ps_stream_t stream) {
  PS_CHECK_ARG(M >= 0 && n_heads > 0 && L_cap > 0 && slots0 >= 0 && slots1 >= 0);
  PS_CHECK_ARG(dtype == PS_DTYPE_F16 || dtype == PS_DTYPE_BF16);
  if (!counts) PS_CHECK_ARG(split_point >= 0 && split_point <= M);
  if (M == 0) return PS_OK;
  PS_CHECK_ARG(qkv && q_out && pos);
  PS_CHECK_ARG(!apply_rope || (rope_cos && rope_sin));
  PS_CHECK_ARG((k_pool0 && v_pool0) || slots0 == 0);
  PS_CHECK_ARG((k_pool1 && v_pool1) || slots1 == 0);
  dim3 grid(M, n_heads);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == PS_DTYPE_BF16)
    PS_CUDA_RET(launch(ops::rope_kv_append_kernel<__nv_bfloat16>, grid, dim3(64), 0, st,
                       (const __nv_bfloat16*)qkv, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_pool0,
                       (__nv_bfloat16*)v_pool0, (__nv_bfloat16*)k_pool1, (__nv_bfloat16*)v_pool1,
                       rope_cos, rope_sin, pos, slot, counts, split_point, M, n_heads, L_cap,
                       slots0, slots1, apply_rope, status));
  else
    PS_CUDA_RET(launch(ops::rope_kv_append_kernel<__half>, grid, dim3(64), 0, st,
                       (const __half*)qkv, (__half*)q_out, (__half*)k_pool0, (__half*)v_pool0,
                       (__half*)k_pool1, (__half*)v_pool1, rope_cos, rope_sin, pos, slot, counts,
                       split_point, M, n_heads, L_cap, slots0, slots1, apply_rope, status));
  return PS_OK;
}
