// Host helpers and library-wide C entry points (error strings, version,
// device queries, tensor-map encoding).
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <set>
#include <tuple>

#include "ps_host.h"

namespace ps {

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int sm_count(int device) {
  static std::atomic<int> cache[64];
  if (device < 0 || device >= 64) return 0;
  int v = cache[device].load(std::memory_order_relaxed);
  if (v == 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      return 0;
    cache[device].store(v, std::memory_order_relaxed);
  }
  return v;
}

bool is_sm100(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return false;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  return major == 10 && minor == 0;
}

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PS_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

cudaError_t allow_dynamic_smem(const void* func, int bytes) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int>> done;
  const int device = current_device();
  const auto key = std::make_tuple(func, device, bytes);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_tmap_16bit(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box, int bf16,
                     int l2_promo_bytes) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) {
      if (strides_bytes[i] % 16 != 0) return false;
      gstride[i] = strides_bytes[i];
    }
  }
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   l2_promo_bytes >= 256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                                         : CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace ps

extern "C" const char* ps_error_string(int code) {
  switch (code) {
    case PS_OK: return "ok";
    case PS_ERR_INVALID_ARGUMENT: return "invalid argument (shape, pointer or alignment)";
    case PS_ERR_WORKSPACE: return "workspace missing or too small";
    case PS_ERR_CUDA: return "CUDA runtime or driver call failed";
    case PS_ERR_UNSUPPORTED: return "unsupported device or size";
    case PS_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the library's static no-allocation buffer holds";
    default: return "unknown error";
  }
}

extern "C" const char* ps_version(void) { return "parallel-serve-b200 0.1 (sm_100a)"; }

extern "C" int ps_device_sm_count(int device) { return ps::sm_count(device); }
