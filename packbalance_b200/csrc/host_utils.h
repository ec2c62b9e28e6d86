// Host-side helpers shared by the extension's .cu files: CUDA error checks, TMA
// descriptor encoding (driver entry point fetched through the runtime, so the
// extension does not link libcuda), SM counts and the per-device status word that
// device code reports bounded-wait timeouts into.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <c10/util/Exception.h>

#include <mutex>
#include <set>
#include <utility>

#define PB_CUDA_CHECK(expr)                                                              \
  do {                                                                                   \
    cudaError_t _e = (expr);                                                             \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", #expr); \
  } while (0)

namespace pb {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    PB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map, 128-byte swizzle.  ``inner`` is the contiguous extent,
// ``outer`` the row count, ``row_bytes`` the row pitch.  Out-of-range elements of a
// box read as zero.
inline CUtensorMap make_tmap_bf16_2d(const void* ptr, int64_t inner, int64_t outer, int64_t row_bytes,
                                     uint32_t box_inner, uint32_t box_outer) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tmap_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ") inner=", inner,
              " outer=", outer, " pitch=", row_bytes, " box=", box_inner, "x", box_outer);
  return m;
}

// General 2-D tensor map (epilogue staging boxes): dtype, swizzle chosen by caller.
inline CUtensorMap make_tmap_2d(const void* ptr, CUtensorMapDataType dtype, int64_t inner, int64_t outer,
                                int64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                                CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tmap_encoder()(&m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ") inner=", inner,
              " outer=", outer, " pitch=", row_bytes);
  return m;
}

inline int num_sms(int dev) {
  static int cache[64] = {0};
  if (cache[dev] == 0) PB_CUDA_CHECK(cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev));
  return cache[dev];
}

// One int per device, zero-initialised; kernels atomically record the first error.
inline int* status_ptr(int dev) {
  static int* ptrs[64] = {nullptr};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    int prev = 0;
    PB_CUDA_CHECK(cudaGetDevice(&prev));
    PB_CUDA_CHECK(cudaSetDevice(dev));
    PB_CUDA_CHECK(cudaMalloc(&ptrs[dev], sizeof(int)));
    PB_CUDA_CHECK(cudaMemset(ptrs[dev], 0, sizeof(int)));
    PB_CUDA_CHECK(cudaSetDevice(prev));
  }
  return ptrs[dev];
}

// Kernels whose shared-memory carveouts differ cannot be resident on one SM at the same
// time.  The collectives that run beside the tensor-core kernels (and those kernels,
// which need ~225 KB anyway) ask for the largest carveout, so a collective CTA never
// switches an SM to a configuration a GEMM or attention CTA cannot share.  (What keeps a
// collective from holding back the compute kernels in practice is its width: see
// parallel/comm.py.)  Returns ``value``, used as the first launch argument:
// ``k<<<pb::smem_max(k, grid), ...>>>``; one attribute call per (device, kernel).
template <typename K, typename V>
inline V smem_max(K* kernel, V value) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return value;
  const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
  std::lock_guard<std::mutex> lock(mu);
  if (done.insert(key).second)
    PB_CUDA_CHECK(cudaFuncSetAttribute(reinterpret_cast<const void*>(kernel),
                                       cudaFuncAttributePreferredSharedMemoryCarveout,
                                       cudaSharedmemCarveoutMaxShared));
  return value;
}

}  // namespace pb
