// Host-side helpers shared by the C-ABI entry points: device properties, TMA descriptor encoding
// through the driver entry point (no link against libcuda), argument checks.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/solort_attn.h"

namespace solort {

struct DeviceInfo {
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int max_smem_optin = 0;
};

// Properties of the current device, cached per device ordinal.
inline int current_device_info(DeviceInfo* info, int* device_out = nullptr) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool valid[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SOLORT_ERR_NO_DEVICE;
  if (dev < 0 || dev >= 64) return SOLORT_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (!valid[dev]) {
    DeviceInfo d;
    if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                               dev) != cudaSuccess) {
      return SOLORT_ERR_NO_DEVICE;
    }
    cache[dev] = d;
    valid[dev] = true;
  }
  *info = cache[dev];
  if (device_out) *device_out = dev;
  if (info->cc_major != 10) return SOLORT_ERR_NO_DEVICE;  // built for sm_100a only
  return SOLORT_OK;
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// Encode a bf16 tiled tensor map. dims/strides are innermost-first; strides_bytes has rank-1
// entries (dimension 1..rank-1). The innermost box extent must be 64 (128 bytes) for
// SWIZZLE_128B.
inline int encode_bf16_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                           const uint64_t* strides_bytes, const uint32_t* box,
                           CUtensorMapSwizzle swizzle) {
  auto fn = tensor_map_encoder();
  if (!fn) return SOLORT_ERR_TENSOR_MAP;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return SOLORT_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < rank - 1; ++i) {
    if ((strides_bytes[i] & 15u) != 0 || strides_bytes[i] >= (1ull << 40))
      return SOLORT_ERR_INVALID_ARGUMENT;
  }
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || dims[i] > (1ull << 32) || box[i] == 0 || box[i] > 256)
      return SOLORT_ERR_INVALID_ARGUMENT;
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gstride[i] = strides_bytes[i];
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                  const_cast<void*>(base), gdim, gstride, bdim, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SOLORT_OK : SOLORT_ERR_TENSOR_MAP;
}

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SOLORT_OK : SOLORT_ERR_CUDA;
}

}  // namespace solort
