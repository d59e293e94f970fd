// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-gen tensor core.
//
//   C[M, N] (+)= A[M, K] * B[N, K]^T        (fp32 accumulation in TMEM)
//
// Each operand may be K-major (contiguous along the reduction dimension) or
// MN-major (contiguous along M resp. N), so the same kernel serves the three
// GEMMs of a linear layer without any transpose copies:
//   forward   Y  = X  W^T : A = X  (K-major),  B = W (K-major)
//   input grad dX = dY W  : A = dY (K-major),  B = W (N-major)
//   weight grad dW = dY^T X: A = dY (M-major), B = X (N-major)
//
// Pipeline (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: streams BM x 64 A and BN x 64 B tiles into a
//               STAGES-deep ring of 128-byte-swizzled shared-memory buffers.
//   warp 1      allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16) from
//               one elected thread; tcgen05.commit releases ring slots and
//               publishes finished accumulators.
//   warps 2..   epilogue: tcgen05.ld the fp32 accumulator (one TMEM lane per
//               output row), convert and store to global memory.
// Two tile shapes:
//   BM=128: two accumulator buffers in TMEM (2 x BN columns) let the epilogue
//           of tile i overlap the MMAs of tile i+1; 4 epilogue warps.
//   BM=256 (BN=256): each k-step issues two M=128 MMAs that share the B tile,
//           so a CTA moves 1.5x fewer operand bytes per FLOP through L2 and
//           shared memory (3-stage ring of 64 KB); the two M-halves fill all
//           512 TMEM columns, so the epilogue (8 warps, one per half and lane
//           quarter) does not overlap the next tile.  The host picks the shape
//           from the reduction length.
// All waits are bounded (see common.cuh).
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"

#include <cstdio>
#include <cstdlib>

static bool gemm_trace() {
  static const bool on = std::getenv("MVP_GEMM_TRACE") != nullptr;
  return on;
}
#define GEMM_TRACE(...)                        \
  do {                                         \
    if (gemm_trace()) {                        \
      std::fprintf(stderr, "[gemm] " __VA_ARGS__); \
      std::fflush(stderr);                     \
    }                                          \
  } while (0)

namespace mvp {
namespace gemm {

constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row

enum Epilogue : int { kStoreBf16 = 0, kStoreF32 = 1, kAccumF32 = 2 };

struct Params {
  int M, N, K;
  void* C;
  int64_t ldc;
  int* status;
  int group_m;
};

template <int BN, int BM>
struct Config {
  static_assert(BM == 128 || (BM == 256 && BN == 256), "tile shapes: 128 x {128, 256} or 256 x 256");
  static constexpr int STAGES = BM == 256 ? 3 : (BN == 256 ? 4 : 6);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NACC = BM == 256 ? 1 : 2;      // accumulator buffers (M-halves fill TMEM at BM=256)
  static constexpr int TMEM_COLS = 2 * BN;            // 512 or 256 columns
  static constexpr int EPI_WARPS = BM == 256 ? 8 : 4;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group_m, int& tm, int& tn) {
  // Grouped raster: `group_m` M-tiles sweep all N-tiles before the next group,
  // so concurrently running CTAs share A panels and B panels in L2.
  const int per_group = group_m * num_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gm = min(group_m, num_m - first_m);
  const int r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

template <int BN, int BM, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(Config<BN, BM>::THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  using Cfg = Config<BN, BM>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint64_t* done_bar = tempty_bar + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 32 * Cfg::EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, num_m, num_n, p.group_m, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, abort_flag, p.status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full_bar[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * 64 * BK * 2, &tmA, &full_bar[stage], m0 + 64 * j, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full_bar[stage], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * 64 * BK * 2, &tmB, &full_bar[stage], n0 + 64 * j, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: after an abort, wait (bounded) until the last load issued into
      // every ring slot has landed, so no bulk copy still writes shared memory
      // when the CTA exits.
      if (!ok || *abort_flag) {
        for (int s = 0; s < STAGES; ++s) {
          if (!((issued_mask >> s) & 1u)) continue;
          const uint32_t par = (issued_phase >> s) & 1u;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(&full_bar[s], par)) {
            if (globaltimer() - t0 > 200000000ull) {
              record_status(p.status, kTimeoutDrain);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (elect_one_sync()) {
      constexpr uint32_t idesc = make_idesc_bf16(128, BN, A_MN, B_MN);  // every MMA is M=128 (cta_group::1)
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = Cfg::NACC == 2 ? (local & 1) : 0;
        const uint32_t acc_phase = Cfg::NACC == 2 ? ((local >> 1) & 1) : (local & 1);
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.status, kTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag, p.status, kTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t bdesc;
            if constexpr (!B_MN) bdesc = make_smem_desc_sw128(b_base + k * 32, 16, 1024);
            else bdesc = make_smem_desc_sw128(b_base + k * 2048, 64 * BK * 2, 1024);
#pragma unroll
            for (int half = 0; half < BM / 128; ++half) {
              // rows 128*half.. of the A tile: 16 KB further in both layouts (K-major: 128 rows of
              // 128 B; MN-major: two 64-row chunks of 8 KB)
              const uint32_t a_half = a_base + half * 16384;
              uint64_t adesc;
              if constexpr (!A_MN) adesc = make_smem_desc_sw128(a_half + k * 32, 16, 1024);
              else adesc = make_smem_desc_sw128(a_half + k * 2048, 64 * BK * 2, 1024);
              mma_bf16_ss(d_tmem + half * BN, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
          mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&tfull_bar[acc]);
      }
      // All previously issued MMAs must retire before TMEM is released.
      mma_commit(done_bar);
      mbar_wait_bounded(done_bar, 0, abort_flag, p.status, kTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    const int mhalf = (warp - 2) >> 2;  // BM=256: which M-half (accumulator) this warpgroup drains
    const int row_in_tile = mhalf * 128 + sub * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(t, num_m, num_n, p.group_m, tm, tn);
      const int acc = Cfg::NACC == 2 ? (local & 1) : 0;
      const uint32_t acc_phase = Cfg::NACC == 2 ? ((local >> 1) & 1) : (local & 1);
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&tfull_bar[acc], acc_phase, abort_flag, p.status, kTimeoutEpilogue))) break;
      tc_fence_after();
      const int m = tm * BM + row_in_tile;
      const bool row_ok = m < p.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + (acc + mhalf) * BN + c * 32, r);
        tmem_wait_ld();
        const int n = tn * BN + c * 32;
        if (!row_ok || n >= p.N) continue;
        const bool full_chunk = (n + 32 <= p.N);
        if constexpr (EPI == kStoreBf16) {
          __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(m) * p.ldc + n;
          if (full_chunk && ((reinterpret_cast<uintptr_t>(C) & 15) == 0)) {
            uint4* dst = reinterpret_cast<uint4*>(C);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 q;
              q.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
              q.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
              q.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
              q.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
              dst[v] = q;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)  // constant indices keep r[] in registers
              if (n + j < p.N) C[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
          }
        } else {
          float* C = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(m) * p.ldc + n;
          if (full_chunk && ((reinterpret_cast<uintptr_t>(C) & 15) == 0)) {
            float4* dst = reinterpret_cast<float4*>(C);
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float4 q = make_float4(__uint_as_float(r[4 * v + 0]), __uint_as_float(r[4 * v + 1]),
                                     __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
              if constexpr (EPI == kAccumF32) {
                const float4 o = dst[v];
                q.x += o.x;
                q.y += o.y;
                q.z += o.z;
                q.w += o.w;
              }
              dst[v] = q;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (n + j >= p.N) continue;
              float val = __uint_as_float(r[j]);
              if constexpr (EPI == kAccumF32) val += C[j];
              C[j] = val;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int BN, int BM, bool A_MN, bool B_MN, int EPI>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int num_sms, cudaStream_t stream) {
  using Cfg = Config<BN, BM>;
  auto kern = gemm_bf16_kernel<BN, BM, A_MN, B_MN, EPI>;
  static bool configured = false;  // per instantiation
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    configured = true;
  }
  const int num_tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(num_tiles, num_sms));
  kern<<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN, int BM, int EPI>
void dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int sms,
                    cudaStream_t s) {
  if (!a_mn && !b_mn) launch<BN, BM, false, false, EPI>(ta, tb, p, sms, s);
  else if (!a_mn && b_mn) launch<BN, BM, false, true, EPI>(ta, tb, p, sms, s);
  else if (a_mn && !b_mn) launch<BN, BM, true, false, EPI>(ta, tb, p, sms, s);
  else launch<BN, BM, true, true, EPI>(ta, tb, p, sms, s);
}

// BM=256 only when the reduction is long (K >= 8192): its epilogue does not overlap the next tile's
// MMAs, which costs more than the operand-traffic saving buys on short reductions (measured on
// the Qwen3-8B linear shapes: forward / input-grad GEMMs with K = 4096 run faster at BM=128,
// weight-grad GEMMs with K = 8192 tokens and K >= 12288 ones at BM=256).
// MVP_GEMM_BM=128/256 forces one shape.
inline int choose_bm(int64_t M, int64_t N, int64_t K, int BN) {
  static const char* force = std::getenv("MVP_GEMM_BM");
  if (force != nullptr) return std::atoi(force) == 256 && BN == 256 ? 256 : 128;
  return (BN == 256 && M >= 256 && K >= 8192) ? 256 : 128;
}

}  // namespace gemm
}  // namespace mvp

void gemm_sm100_pair(const torch::Tensor& a, bool a_mn, const torch::Tensor& b, bool b_mn, torch::Tensor& c,
                     bool accumulate, int64_t status_ptr);

// The two-SM 256 x 256 kernel (gemm2sm_sm100.cu) takes every GEMM with M, N >= 256;
// MVP_GEMM_PAIR=0 keeps the single-SM kernels.
static bool use_pair_kernel(int64_t M, int64_t N) {
  static const char* env = std::getenv("MVP_GEMM_PAIR");
  static const bool on = env == nullptr || std::atoi(env) != 0;
  return on && M >= 256 && N >= 256;
}

// Host entry point.
//   a: if a_mn == false, an [M, K] view with unit stride along K;
//      if a_mn == true,  a [K, M] view with unit stride along M.
//   b: if b_mn == false, an [N, K] view (unit stride along K);
//      if b_mn == true,  a [K, N] view (unit stride along N).
//   c: [M, N] output with unit column stride; bf16 or fp32.
//   accumulate: c += result (fp32 output only).
void gemm_sm100(const torch::Tensor& a, bool a_mn, const torch::Tensor& b, bool b_mn, torch::Tensor& c,
                bool accumulate, int64_t status_ptr) {
  using namespace mvp::gemm;
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm_sm100: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_sm100: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm_sm100: 2-D operands");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "gemm_sm100: unit inner stride required");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm_sm100: reduction sizes differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(c.size(0) == M && c.size(1) == N, "gemm_sm100: output shape mismatch");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "gemm_sm100: row strides must be multiples of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(b.data_ptr()) & 15) == 0,
              "gemm_sm100: operands must be 16-byte aligned");
  const bool out_f32 = c.scalar_type() == at::kFloat;
  TORCH_CHECK(out_f32 || c.scalar_type() == at::kBFloat16, "gemm_sm100: output must be bf16 or fp32");
  TORCH_CHECK(!accumulate || out_f32, "gemm_sm100: accumulate needs an fp32 output");
  if (M == 0 || N == 0) return;
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (K == 0) {
    if (!accumulate) c.zero_();
    return;
  }

  GEMM_TRACE("enter M=%lld N=%lld K=%lld a_mn=%d b_mn=%d acc=%d f32=%d\n", (long long)M, (long long)N,
             (long long)K, (int)a_mn, (int)b_mn, (int)accumulate, (int)out_f32);
  if (use_pair_kernel(M, N)) {
    gemm_sm100_pair(a, a_mn, b, b_mn, c, accumulate, status_ptr);
    return;
  }
  const int BN = N >= 256 ? 256 : 128;
  const int sms = mvp::num_sms(a.get_device());
  const int BM = choose_bm(M, N, K, BN);
  // Tensor maps: dim0 is the contiguous dimension.
  CUtensorMap ta, tb;
  if (!a_mn) mvp::make_tmap_2d_bf16(&ta, a.data_ptr(), K, M, a.stride(0), 64, BM);
  else mvp::make_tmap_2d_bf16(&ta, a.data_ptr(), M, K, a.stride(0), 64, 64);
  if (!b_mn) mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), K, N, b.stride(0), 64, BN);
  else mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), N, K, b.stride(0), 64, 64);

  GEMM_TRACE("tensor maps encoded\n");
  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.status = reinterpret_cast<int*>(status_ptr);
  p.group_m = BM == 256 ? 8 : 16;
  GEMM_TRACE("launch sms=%d BM=%d BN=%d\n", sms, BM, BN);
  const int epi = out_f32 ? (accumulate ? kAccumF32 : kStoreF32) : kStoreBf16;
  if (BN == 256 && BM == 256) {
    if (epi == kStoreBf16) dispatch_major<256, 256, kStoreBf16>(a_mn, b_mn, ta, tb, p, sms, stream);
    else if (epi == kStoreF32) dispatch_major<256, 256, kStoreF32>(a_mn, b_mn, ta, tb, p, sms, stream);
    else dispatch_major<256, 256, kAccumF32>(a_mn, b_mn, ta, tb, p, sms, stream);
  } else if (BN == 256) {
    if (epi == kStoreBf16) dispatch_major<256, 128, kStoreBf16>(a_mn, b_mn, ta, tb, p, sms, stream);
    else if (epi == kStoreF32) dispatch_major<256, 128, kStoreF32>(a_mn, b_mn, ta, tb, p, sms, stream);
    else dispatch_major<256, 128, kAccumF32>(a_mn, b_mn, ta, tb, p, sms, stream);
  } else {
    if (epi == kStoreBf16) dispatch_major<128, 128, kStoreBf16>(a_mn, b_mn, ta, tb, p, sms, stream);
    else if (epi == kStoreF32) dispatch_major<128, 128, kStoreF32>(a_mn, b_mn, ta, tb, p, sms, stream);
    else dispatch_major<128, 128, kAccumF32>(a_mn, b_mn, ta, tb, p, sms, stream);
  }
}
