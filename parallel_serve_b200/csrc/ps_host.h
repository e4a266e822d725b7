// Host-side helpers shared by the C-ABI entry points: argument checks, device
// properties, and the driver's tensor-map encoder fetched through the runtime
// (so the library does not link libcuda directly).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <utility>

#include "parallel_serve.h"

namespace ps {

// Workspaces of kernels with arrival counters start with a fixed-size counter
// region (zero at rest) followed by the shape-dependent scratch, so one buffer
// can be reused across calls of different shapes without re-zeroing.
constexpr size_t kCounterRegionBytes = 256 * 1024;
constexpr int kMaxCounters = (int)(kCounterRegionBytes / 4);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }
inline int cdiv(int a, int b) { return (a + b - 1) / b; }

int current_device();
int sm_count(int device);
bool is_sm100(int device);

// cuTensorMapEncodeTiled resolved at first use; nullptr if unavailable.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// 2-D / 3-D row-major 16-bit tensor maps with 128-byte swizzle.
// dims[0] is the contiguous dimension; strides_bytes[i] is the stride of
// dims[i+1].
// `l2_promo_bytes` (128 or 256) sets how much a miss fills in L2: 256 when a
// CTA reads both 128-byte halves of an aligned 256-byte span together.
bool make_tmap_16bit(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int bf16,
                     int l2_promo_bytes = 256);

// Programmatic dependent launch (overlap of a kernel's prologue with the tail
// of the previous kernel on the stream). On by default; PS_PDL=0 disables.
bool pdl_enabled();

// Raise `func`'s dynamic shared memory limit to `bytes` on the current device.
// A function attribute belongs to one device's context, so this is done once
// per (function, device, bytes); the record is guarded by a mutex, so host
// threads may make first calls on several devices at once.
cudaError_t allow_dynamic_smem(const void* func, int bytes);

template <typename... KArgs>
cudaError_t allow_dynamic_smem(void (*kernel)(KArgs...), int bytes) {
  return allow_dynamic_smem(reinterpret_cast<const void*>(kernel), bytes);
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace ps

#define PS_CHECK_ARG(cond) \
  do {                     \
    if (!(cond)) return PS_ERR_INVALID_ARGUMENT; \
  } while (0)

#define PS_CUDA_RET(expr)                            \
  do {                                               \
    cudaError_t e_ = (expr);                         \
    if (e_ != cudaSuccess) return PS_ERR_CUDA;       \
  } while (0)
