// Host-side helpers shared by the C-ABI entry points: TMA tensor-map encoding through
// the driver entry point (no -lcuda link), status codes and SM-count caching.
#pragma once

#include <atomic>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <mutex>
#include <set>
#include <stdint.h>
#include <tuple>

namespace vdn {

// C-ABI status codes (the host wrapper maps them to Python exceptions).
enum : int {
  kOk = 0,
  kBadArgument = -1,      // ValueError
  kUnsupported = -2,      // ValueError (geometry outside what the kernels handle)
  kTensorMapFailed = -3,  // RuntimeError
  kLaunchFailed = -4,     // RuntimeError (cudaGetLastError after launch)
  kMisaligned = -5,       // ValueError (pointer / stride not 16-byte aligned)
  kTooLarge = -6,         // ValueError (problem exceeds a fixed-size device scratch area)
};

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  }
  return fn;
}

// 2-D row-major tensor [outer][inner] with a row pitch of `row_stride_elems`.
inline int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                        int elem_bytes, uint64_t inner, uint64_t outer,
                        uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                        CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = tensor_map_encoder();
  if (!enc) return kTensorMapFailed;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((row_stride_elems * elem_bytes) & 15))
    return kMisaligned;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kTensorMapFailed;
}

// 3-D row-major tensor [groups][outer][inner]: rows `row_stride_elems` apart, groups
// `group_stride_elems` apart; box {box_inner, box_outer, 1}.
inline int make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                        uint64_t inner, uint64_t outer, uint64_t groups, uint64_t row_stride_elems,
                        uint64_t group_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  auto enc = tensor_map_encoder();
  if (!enc) return kTensorMapFailed;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((row_stride_elems * elem_bytes) & 15) ||
      ((group_stride_elems * elem_bytes) & 15))
    return kMisaligned;
  cuuint64_t dims[3] = {inner, outer, groups};
  cuuint64_t strides[2] = {row_stride_elems * (uint64_t)elem_bytes, group_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = enc(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kTensorMapFailed;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

// Set a function attribute of `kernel` on the current device (smem_optin: `bytes` of dynamic
// shared memory).  The attribute belongs to the device that is current at the call, so each
// (kernel, device, attribute, value) is set once per process -- a process driving several
// GPUs sets it on every one of them -- under a lock, since entry points may be called from
// several host threads.  False if CUDA refused.
inline bool func_attr(const void* kernel, cudaFuncAttribute attr, int value) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const auto key = std::make_tuple(kernel, dev, (int)attr, value);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return true;
  if (cudaFuncSetAttribute(kernel, attr, value) != cudaSuccess) {
    cudaGetLastError();  // the caller reports the failure; later calls must not see it again
    return false;
  }
  done.insert(key);
  return true;
}

inline bool smem_optin(const void* kernel, int bytes) {
  return func_attr(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Kernel launches made by this library since it was loaded: every <<<>>> site is followed
// by count_launch() (host side, so the count is exact without touching the device).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> n{0};
  return n;
}
inline void count_launch() { launch_counter().fetch_add(1, std::memory_order_relaxed); }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace vdn
