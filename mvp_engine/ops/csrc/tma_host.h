// Host-side helpers: TMA tensor-map encoding through the driver entry point
// (no link-time dependency on libcuda) and a cached SM count per device.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <c10/util/Exception.h>

#include <array>
#include <mutex>

namespace mvp {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "mvp_engine: cuTensorMapEncodeTiled is unavailable");
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

// The driver's tensor-map encoder needs a current context on the calling
// thread.  Worker threads (autograd's backward thread, Python threads) may
// have none yet, so make the device's primary context current once per thread.
inline void ensure_thread_context() {
  thread_local bool done = false;
  if (done) return;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(dev);  // CUDA >= 12: initialises and binds the primary context
  cudaFree(nullptr);
  done = true;
}

// 2-D bf16 tensor map: dim0 (contiguous, `inner` elements) x dim1 (`outer`
// rows, `row_stride` elements apart), box = box0 x box1, 128-byte swizzle.
inline void make_tmap_2d_bf16(CUtensorMap* map, void* base, int64_t inner, int64_t outer, int64_t row_stride,
                              uint32_t box0, uint32_t box1,
                              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  ensure_thread_context();
  TORCH_CHECK((row_stride * 2) % 16 == 0, "TMA: row stride must be a multiple of 16 bytes");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA: base must be 16-byte aligned");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = encode_tiled_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estride,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r), " (inner=", inner,
              ", outer=", outer, ", stride=", row_stride, ", box=", box0, "x", box1, ")");
}

inline int num_sms(int device) {
  static std::array<int, 64> cache{};
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 64) device = 0;
  if (cache[device] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cache[device] = v > 0 ? v : 148;
  }
  return cache[device];
}

}  // namespace mvp
