// RMSNorm backward that allocates no device memory: exported C entry point
// `mvp_rmsnorm_bwd_noalloc`.
//
// This entry point has no counterpart in the reference (MVP Engine has no
// native code); it is an addition of this library.
//
// Who needs it.  Some callers cannot allocate device memory at the point where
// they run a kernel: a host runtime that plans every device buffer ahead of
// time and forbids allocation while executing (inference / training graph
// executors, plugin interfaces of other frameworks), code running while a
// CUDA stream is being captured into a graph (where an allocation would have
// to be captured too), or real-time threads that must not block in the
// allocator.  The regular `rmsnorm_bwd` allocates its output and a scratch
// buffer for the weight-gradient partial sums through PyTorch's allocator, so
// those callers cannot use it.  This variant takes inputs and outputs from the
// caller and keeps its scratch in a file-scope device array instead.
//
// Contract.
//   * Inputs: dy, h [rows, H] bf16 (row-major, contiguous), rstd [rows] fp32
//     (the forward's 1 / RMS), w [H] bf16.  Outputs (caller-allocated):
//     dx [rows, H] bf16, dw [H] fp32 (overwritten, not accumulated).
//   * Limits: 1 <= H <= kMaxHidden (16384), H % 8 == 0, rows >= 1.  The scratch
//     holds kMaxSplits (64) partial rows of H floats: 4 MiB, reserved on every
//     GPU that loads this library for the life of the process.  Larger sizes are
//     rejected with kNoAllocTooLarge; nothing is launched then.
//   * No cudaMalloc / cudaFree / library allocation happens on any path.  The
//     first call on each device looks up the device address of the scratch
//     array with cudaGetSymbolAddress (with that device current) and caches it;
//     make that first call before any stream capture begins.
//   * All calls share the one scratch array.  Every partial slot a call reads
//     is written by the same call first, so nothing needs zeroing between calls,
//     but two calls whose kernels overlap on the GPU (different streams, or
//     different host threads on one device) race on the scratch: serialise them.
//   * An error already pending on the calling thread (from an earlier launch of
//     the caller) is returned as kNoAllocPendingError without launching anything
//     and without clearing it.
//   * Returns 0 on success, or a kNoAlloc* code; the launches are asynchronous
//     on `stream` (cudaStream_t, may be null for the legacy default stream).
#include "noalloc_rmsnorm.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace mvp {
namespace noalloc {

constexpr int kMaxSplits = 64;
constexpr int kMaxHidden = 16384;
constexpr int kMaxDevices = 64;

enum Code : int {
  kNoAllocOk = 0,
  kNoAllocTooLarge = 1,
  kNoAllocBadArgument = 2,
  kNoAllocSetupFailed = 3,
  kNoAllocLaunchFailed = 4,
  kNoAllocPendingError = 5,
};

// Weight-gradient partial sums: [kMaxSplits][kMaxHidden] fp32.
static __device__ __align__(256) float g_dw_partials[kMaxSplits * kMaxHidden];

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// dx = rstd * (w * dy - xhat * mean(xhat * w * dy)), xhat = h * rstd; one warp per row.
__global__ void dx_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ h,
                          const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ w,
                          __nv_bfloat16* __restrict__ dx, int rows, int H) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const int64_t off = static_cast<int64_t>(row) * H;
  const float r = rstd[row];
  float dot = 0.f;
  for (int c = lane; c < H; c += 32) {
    dot += __bfloat162float(dy[off + c]) * __bfloat162float(w[c]) * __bfloat162float(h[off + c]) * r;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  dot /= static_cast<float>(H);
  for (int c = lane; c < H; c += 32) {
    const float hv = __bfloat162float(h[off + c]);
    const float g = __bfloat162float(dy[off + c]) * __bfloat162float(w[c]);
    dx[off + c] = __float2bfloat16_rn(r * (g - hv * r * dot));
  }
}

// partials[split][c] = sum over the split's rows of dy * bf16(h * rstd); block = 256 columns.
__global__ void dw_partial_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ h,
                                  const float* __restrict__ rstd, float* __restrict__ partials, int64_t rows, int H,
                                  int64_t rows_per_split) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t split = blockIdx.y;
  if (c >= H) return;
  const int64_t r0 = split * rows_per_split;
  const int64_t r1 = r0 + rows_per_split < rows ? r0 + rows_per_split : rows;
  float acc = 0.f;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t off = static_cast<int64_t>(r) * H + c;
    acc += __bfloat162float(dy[off]) * bf16r(__bfloat162float(h[off]) * rstd[r]);
  }
  partials[static_cast<int64_t>(split) * H + c] = acc;
}

__global__ void dw_reduce_kernel(const float* __restrict__ partials, float* __restrict__ dw, int splits, int H) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int k = 0; k < splits; ++k) s += partials[static_cast<int64_t>(k) * H + c];
  dw[c] = s;
}

std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kNoAllocSetupFailed;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dw_partials) != cudaSuccess || p == nullptr) return kNoAllocSetupFailed;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return kNoAllocOk;
}

}  // namespace noalloc
}  // namespace mvp

extern "C" __attribute__((visibility("default"))) int mvp_rmsnorm_bwd_noalloc(
    const void* dy, const void* h, const float* rstd, const void* w, void* dx, float* dw, int rows, int hidden,
    void* stream) {
  using namespace mvp::noalloc;
  if (dy == nullptr || h == nullptr || rstd == nullptr || w == nullptr || dx == nullptr || dw == nullptr)
    return kNoAllocBadArgument;
  if (rows < 1 || hidden < 1 || hidden % 8 != 0) return kNoAllocBadArgument;
  if (hidden > kMaxHidden) return kNoAllocTooLarge;
  // An error left by an earlier launch of the caller is reported, not cleared: nothing is launched
  // and the caller's own error handling still sees it.
  if (cudaPeekAtLastError() != cudaSuccess) return kNoAllocPendingError;
  float* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch); rc != kNoAllocOk) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nrows = rows;  // int64 grid arithmetic: rows may be any positive int
  const int splits = rows < kMaxSplits ? rows : kMaxSplits;
  const int64_t rows_per_split = (nrows + splits - 1) / splits;
  const auto* dy_b = static_cast<const __nv_bfloat16*>(dy);
  const auto* h_b = static_cast<const __nv_bfloat16*>(h);
  const auto* w_b = static_cast<const __nv_bfloat16*>(w);
  const unsigned dx_blocks = static_cast<unsigned>((nrows + 7) / 8);  // <= 2^28, under the grid limit
  dx_kernel<<<dx_blocks, 256, 0, s>>>(dy_b, h_b, rstd, w_b, static_cast<__nv_bfloat16*>(dx), rows, hidden);
  if (cudaGetLastError() != cudaSuccess) return kNoAllocLaunchFailed;
  dim3 grid((hidden + 255) / 256, splits);
  dw_partial_kernel<<<grid, 256, 0, s>>>(dy_b, h_b, rstd, scratch, nrows, hidden, rows_per_split);
  if (cudaGetLastError() != cudaSuccess) return kNoAllocLaunchFailed;
  dw_reduce_kernel<<<(hidden + 255) / 256, 256, 0, s>>>(scratch, dw, splits, hidden);
  return cudaGetLastError() == cudaSuccess ? kNoAllocOk : kNoAllocLaunchFailed;
}
