// Collectives over NVLink peer memory for the native data-parallel runtime.
//
// Gradient reduce-scatter by pulling (replaces NCCL's reduce-scatter of the
// flat fp32 gradient buffer of one unit):
//   * every rank keeps the full fp32 gradient of every unit in one symmetric
//     allocation (same offsets on every rank, peers mapped into this process);
//   * when a unit's backward is done, the kernel on each rank first publishes
//     "unit ready, sequence s" into every peer's signal slots (system-scope
//     release after a system fence), then waits until every peer has
//     published s into its own slots (system-scope acquire, bounded by
//     %globaltimer), then sums its shard slice over all ranks with 16-byte
//     loads straight from peer memory and writes the fp32 gradient shard,
//     optionally scaled, and its sum of squares (for the global-norm clip).
// The wire traffic equals a ring reduce-scatter's ((W-1)/W of the unit per
// rank) but there is no intermediate buffer, no extra pass over HBM and the
// squared norm comes for free.
//
// A wait that runs out (a peer that never arrives) sets the status word to
// kTimeoutPeer and returns without reading peer memory; the host raises.
// The bound (timeout_ns) is a launch argument: 10 s in training, far above
// the millisecond skew between ranks that run the same unit order.
#include <cuda_runtime.h>
#include <cstdlib>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "peer_host.h"

namespace mvp {
namespace comm {

constexpr int kMaxRanks = 8;

struct RsParams {
  const float* peers[kMaxRanks];        // base of the symmetric gradient buffer on each rank
  unsigned long long* peer_slots[kMaxRanks];  // base of each rank's signal slots [kMaxRanks]
  unsigned long long* my_slots;         // this rank's slots, written by the peers
  int64_t offset;                        // element offset of the unit in the buffer
  int64_t shard;                         // elements per rank (multiple of 4)
  int rank, world;
  unsigned long long seq;
  float scale;
  float* out;                            // [shard] fp32
  float* sumsq;                          // optional [1] fp32 accumulator
  int* status;
  unsigned long long timeout_ns;         // bound of every wait for a peer
};

__global__ void __launch_bounds__(256) rs_pull_kernel(RsParams p) {
  __shared__ int s_ok;
  __shared__ float s_red[8];
  // 1. publish: this rank's unit is complete (its producing kernels finished before this one started)
  if (blockIdx.x == 0 && threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.peer_slots[threadIdx.x] + p.rank, p.seq);
  }
  // 2. wait for every peer's publication, bounded
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < p.world && ok; ++r) {
      while (ld_acquire_sys(p.my_slots + r) < p.seq) {
        if (globaltimer() - t0 > p.timeout_ns) {
          atomicCAS(p.status, 0, kTimeoutPeer);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  // 3. pull and sum this rank's slice: kUnroll float4 per rank in flight per thread so that enough
  //    bytes are outstanding to cover the NVLink round trip
  constexpr int kUnroll = 4;
  const int64_t base = p.offset + static_cast<int64_t>(p.rank) * p.shard;
  const int64_t n4 = p.shard / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  float local_sq = 0.f;
  for (int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i0 < n4; i0 += stride * kUnroll) {
    float4 acc[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < p.world) {
        const float4* src = reinterpret_cast<const float4*>(p.peers[r] + base);
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t i = i0 + u * stride;
          v[u] = i < n4 ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          acc[u].x += v[u].x;
          acc[u].y += v[u].y;
          acc[u].z += v[u].z;
          acc[u].w += v[u].w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n4) {
        float4 a = acc[u];
        a.x *= p.scale;
        a.y *= p.scale;
        a.z *= p.scale;
        a.w *= p.scale;
        reinterpret_cast<float4*>(p.out)[i] = a;
        local_sq += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
      }
    }
  }
  if (p.sumsq != nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) local_sq += __shfl_xor_sync(0xffffffffu, local_sq, o);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = local_sq;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < blockDim.x / 32; ++w) t += s_red[w];
      atomicAdd(p.sumsq, t);
    }
  }
}

// Device-side barrier over the same slots (used before gradient buffers are reused): publish
// seq to every peer, wait for every peer's seq.  One block.
__global__ void slots_barrier_kernel(RsParams p) {
  if (threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.peer_slots[threadIdx.x] + p.rank, p.seq);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < p.world; ++r) {
      while (ld_acquire_sys(p.my_slots + r) < p.seq) {
        if (globaltimer() - t0 > p.timeout_ns) {
          atomicCAS(p.status, 0, kTimeoutPeer);
          return;
        }
        __nanosleep(64);
      }
    }
  }
}

RsParams make_params(const std::vector<int64_t>& peer_bufs, const std::vector<int64_t>& peer_slots,
                     int64_t my_slots, int rank, int64_t seq, int64_t status_ptr, int64_t timeout_ns) {
  TORCH_CHECK(timeout_ns > 0, "peer collectives need a positive wait bound");
  const int world = static_cast<int>(peer_bufs.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "peer collectives support 1..8 ranks");
  TORCH_CHECK(static_cast<int>(peer_slots.size()) == world, "one signal base per rank");
  TORCH_CHECK(rank >= 0 && rank < world, "rank out of range");
  RsParams p{};
  for (int r = 0; r < world; ++r) {
    p.peers[r] = reinterpret_cast<const float*>(peer_bufs[r]);
    p.peer_slots[r] = reinterpret_cast<unsigned long long*>(peer_slots[r]);
  }
  p.my_slots = reinterpret_cast<unsigned long long*>(my_slots);
  p.rank = rank;
  p.world = world;
  p.seq = static_cast<unsigned long long>(seq);
  p.status = reinterpret_cast<int*>(status_ptr);
  p.timeout_ns = static_cast<unsigned long long>(timeout_ns);
  return p;
}

}  // namespace comm
}  // namespace mvp

// out[i] = scale * sum_r peer_r[offset + rank*shard + i]; optional sumsq += ||out||^2.
void peer_reduce_scatter(const std::vector<int64_t>& peer_bufs, const std::vector<int64_t>& peer_slots,
                         int64_t my_slots, int64_t rank, int64_t offset, int64_t shard, int64_t seq, double scale,
                         torch::Tensor& out, const c10::optional<torch::Tensor>& sumsq, int64_t status_ptr,
                         int64_t timeout_ns) {
  using namespace mvp::comm;
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() >= shard,
              "peer_reduce_scatter: fp32 contiguous output of at least `shard` elements");
  TORCH_CHECK(shard % 4 == 0 && offset % 4 == 0, "peer_reduce_scatter: 16-byte aligned slices");
  const at::cuda::CUDAGuard guard(out.device());
  RsParams p = make_params(peer_bufs, peer_slots, my_slots, static_cast<int>(rank), seq, status_ptr, timeout_ns);
  p.offset = offset;
  p.shard = shard;
  p.scale = static_cast<float>(scale);
  p.out = out.data_ptr<float>();
  p.sumsq = sumsq.has_value() ? sumsq->data_ptr<float>() : nullptr;
  // CTAs per SM (MVP_RS_CTAS_PER_SM, default 2): two keep ~10 MB of loads in flight, enough for NVLink.
  // The kernel runs beside the backward's GEMM / attention CTAs, and at 126 registers per thread two of its
  // CTAs fill an SM's register file, so fewer CTAs trade reduce-scatter speed for co-residency.
  static const int per_sm = [] {
    const char* env = std::getenv("MVP_RS_CTAS_PER_SM");
    const int v = env != nullptr ? std::atoi(env) : 2;
    return v < 1 ? 1 : (v > 4 ? 4 : v);
  }();
  const int64_t n4 = shard / 4;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  const int blocks =
      static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(static_cast<int64_t>(per_sm) * sms, (n4 + 1023) / 1024)));
  rs_pull_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_barrier(const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                  int64_t status_ptr, int64_t timeout_ns) {
  using namespace mvp::comm;
  std::vector<int64_t> dummy(peer_slots.size(), 0);
  RsParams p = make_params(dummy, peer_slots, my_slots, static_cast<int>(rank), seq, status_ptr, timeout_ns);
  slots_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------------------------------
// Tensor-parallel all-gather / reduce-scatter halves around the two-SM GEMM.
//
// All-gather by pushing: every rank copies its row slice into the gather buffer of every rank
// (same offsets; peers' buffers are mapped), then publishes a sequence number; the consuming
// GEMM waits per row slice (gemm_pair_tp), so it starts on the rows it already holds.
// Reduce-scatter by routing: the producing GEMM writes row block d of its partial result into
// rank d's slot buffer (slot = source rank); rank d then publishes, waits for every source and
// sums its slots.
namespace mvp {
namespace comm {

// Destination bases travel in p.peers (the ranks' gather buffers).
__global__ void __launch_bounds__(256) push_rows_kernel(RsParams p, const uint4* __restrict__ src, int64_t n16,
                                                        int64_t dst_off16) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 v = src[i];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < p.world) reinterpret_cast<uint4*>(const_cast<float*>(p.peers[r]))[dst_off16 + i] = v;
  }
  __threadfence_system();
}

__global__ void publish_kernel(RsParams p) {
  if (threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.peer_slots[threadIdx.x] + p.rank, p.seq);
  }
}

__global__ void wait_all_kernel(RsParams p) {
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < p.world; ++r) {
      while (ld_acquire_sys(p.my_slots + r) < p.seq) {
        if (globaltimer() - t0 > p.timeout_ns) {
          atomicCAS(p.status, 0, kTimeoutPeer);
          return;
        }
        __nanosleep(64);
      }
    }
  }
}

// out[i] = sum over sources s of slots[s * n + i] (bf16 in, fp32 sum, bf16 out), after publishing this
// rank's routed writes and seeing every source's.
__global__ void __launch_bounds__(256) slot_reduce_kernel(RsParams p, const __nv_bfloat16* __restrict__ slots,
                                                          __nv_bfloat16* __restrict__ out, int64_t n) {
  __shared__ int s_ok;
  if (blockIdx.x == 0 && threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.peer_slots[threadIdx.x] + p.rank, p.seq);
  }
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < p.world && ok; ++r) {
      while (ld_acquire_sys(p.my_slots + r) < p.seq) {
        if (globaltimer() - t0 > p.timeout_ns) {
          atomicCAS(p.status, 0, kTimeoutPeer);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int64_t n8 = n / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < p.world; ++s) {
      const uint4 v = reinterpret_cast<const uint4*>(slots + static_cast<int64_t>(s) * n)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(h[t]);
        acc[2 * t] += f.x;
        acc[2 * t + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

}  // namespace comm
}  // namespace mvp

// Copy src (contiguous bf16, `rows` x `cols`) to rows [dst_row0, dst_row0 + rows) of every rank's
// buffer (bases in `dsts`, row stride `cols`), then publish `seq` to every rank.
void peer_push_rows(const torch::Tensor& src, const std::vector<int64_t>& dsts, int64_t dst_row0,
                    const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                    int64_t status_ptr, int64_t timeout_ns) {
  using namespace mvp::comm;
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.dim() == 2,
              "peer_push_rows: contiguous 2-D bf16 source");
  TORCH_CHECK((src.size(1) * 2) % 16 == 0, "peer_push_rows: rows must be multiples of 16 bytes");
  const at::cuda::CUDAGuard guard(src.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  RsParams p = make_params(dsts, peer_slots, my_slots, static_cast<int>(rank), seq, status_ptr, timeout_ns);
  const int64_t n16 = src.numel() * 2 / 16;
  const int64_t off16 = dst_row0 * src.size(1) * 2 / 16;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(2 * 148, (n16 + 255) / 256)));
  push_rows_kernel<<<blocks, 256, 0, stream>>>(p, reinterpret_cast<const uint4*>(src.data_ptr()), n16, off16);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  publish_kernel<<<1, 32, 0, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void peer_wait_all(const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                   int64_t status_ptr, int64_t timeout_ns) {
  using namespace mvp::comm;
  std::vector<int64_t> dummy(peer_slots.size(), 0);
  RsParams p = make_params(dummy, peer_slots, my_slots, static_cast<int>(rank), seq, status_ptr, timeout_ns);
  wait_all_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out = sum over the `world` slot blocks of `slots` (contiguous [world, rows, cols] bf16) after the
// publish / wait handshake on `seq`.
void peer_slot_reduce(const torch::Tensor& slots, torch::Tensor& out, const std::vector<int64_t>& peer_slots,
                      int64_t my_slots, int64_t rank, int64_t seq, int64_t status_ptr, int64_t timeout_ns) {
  using namespace mvp::comm;
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == at::kBFloat16 && slots.is_contiguous(),
              "peer_slot_reduce: contiguous bf16 slots");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() % 8 == 0,
              "peer_slot_reduce: contiguous bf16 output, 8-element multiple");
  std::vector<int64_t> dummy(peer_slots.size(), 0);
  RsParams p = make_params(dummy, peer_slots, my_slots, static_cast<int>(rank), seq, status_ptr, timeout_ns);
  TORCH_CHECK(slots.numel() == out.numel() * p.world, "peer_slot_reduce: slots = world x output");
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t n = out.numel();
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(2 * 148, (n / 8 + 255) / 256)));
  slot_reduce_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p, reinterpret_cast<const __nv_bfloat16*>(slots.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------------------------------
// Stand-alone peer pull (the compute kernels carry the same copy in extra CTAs).
namespace mvp {

__global__ void __launch_bounds__(256) peer_pull_kernel(PeerPull j, int* status) {
  __shared__ int flag;
  peer_pull_cta(j, status, &flag);
}

void launch_peer_pull(const PeerPull& j, int* status, cudaStream_t stream) {
  if (j.rows == 0) return;
  PeerPull k = j;
  k.rows = 1;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(148, (j.n16 + 2047) / 2048)));
  peer_pull_kernel<<<dim3(blocks, 1), 256, 0, stream>>>(k, status);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mvp

// ----------------------------------------------------------------------------
// Routed fp32 partial sums (ring attention dK / dV): every source rank writes its partial into
// slot [source] of the owner's symmetric buffer; the owner publishes, waits for every source's
// publication of the same sequence number and sums the slots into bf16.
namespace mvp {
namespace comm {

__global__ void __launch_bounds__(256) slot_sum_f32_kernel(RsParams p, const float* __restrict__ slots,
                                                           __nv_bfloat16* __restrict__ out, int64_t n) {
  __shared__ int s_ok;
  if (blockIdx.x == 0 && threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.peer_slots[threadIdx.x] + p.rank, p.seq);
  }
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < p.world && ok; ++r) {
      while (ld_acquire_sys(p.my_slots + r) < p.seq) {
        if (globaltimer() - t0 > p.timeout_ns) {
          atomicCAS(p.status, 0, kTimeoutPeer);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int64_t n4 = n / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < p.world; ++s) {
      const float4 v = reinterpret_cast<const float4*>(slots + static_cast<int64_t>(s) * n)[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    uint2 o;
    o.x = pack_bf16x2(acc.x, acc.y);
    o.y = pack_bf16x2(acc.z, acc.w);
    reinterpret_cast<uint2*>(out)[i] = o;
  }
}

}  // namespace comm
}  // namespace mvp

void peer_publish(const std::vector<int64_t>& peer_slots, int64_t my_slots, int64_t rank, int64_t seq,
                  int64_t status_ptr, int64_t timeout_ns) {
  using namespace mvp::comm;
  std::vector<int64_t> dummy(peer_slots.size(), 0);
  RsParams p = make_params(dummy, peer_slots, my_slots, static_cast<int>(rank), seq, status_ptr, timeout_ns);
  publish_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out [n] (bf16) = sum over the `world` fp32 slots of `slots` [world, n], after the publish / wait
// handshake on `seq` (every source's routed writes into this rank's slots are complete).
void peer_slot_sum_f32(const torch::Tensor& slots, torch::Tensor& out, const std::vector<int64_t>& peer_slots,
                       int64_t my_slots, int64_t rank, int64_t seq, int64_t status_ptr, int64_t timeout_ns) {
  using namespace mvp::comm;
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == at::kFloat && slots.is_contiguous(),
              "peer_slot_sum_f32: contiguous fp32 slots");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() % 4 == 0,
              "peer_slot_sum_f32: contiguous bf16 output, 4-element multiple");
  std::vector<int64_t> dummy(peer_slots.size(), 0);
  RsParams p = make_params(dummy, peer_slots, my_slots, static_cast<int>(rank), seq, status_ptr, timeout_ns);
  TORCH_CHECK(slots.numel() == out.numel() * p.world, "peer_slot_sum_f32: slots = world x output");
  const at::cuda::CUDAGuard guard(out.device());
  const int64_t n = out.numel();
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(2 * 148, (n / 4 + 255) / 256)));
  slot_sum_f32_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p, slots.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------------------------------
// FSDP parameter gather (resharded units): stand-alone launch of the shard pull, and the epoch
// publication that tells the peers this rank's shards are final for the coming step.
namespace mvp {
namespace comm {

constexpr int kGatherKernelStages = 6;
constexpr int kGatherKernelSmem = kGatherKernelStages * kGatherChunk + 1024 + 64;

__global__ void __launch_bounds__(128) shard_gather_kernel(ShardGather g, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  shard_gather_cta_bulk(g, blockIdx.x, status, smem, kGatherKernelStages);
}

__global__ void publish_epoch_kernel(unsigned long long* flag, unsigned long long epoch) {
  if (threadIdx.x == 0) {
    __threadfence_system();  // the optimizer's shard writes (earlier kernels) before the flag
    st_release_sys(flag, epoch);
  }
}

}  // namespace comm
}  // namespace mvp

void peer_gather_shards(const std::vector<int64_t>& peer_bufs, const std::vector<int64_t>& peer_flags,
                        int64_t offset, int64_t shard, int64_t epoch, torch::Tensor& out, int64_t status_ptr,
                        int64_t timeout_ns) {
  using namespace mvp;
  const int world = static_cast<int>(peer_bufs.size());
  TORCH_CHECK(world >= 1 && world <= kMaxGatherRanks && static_cast<int>(peer_flags.size()) == world,
              "peer_gather_shards: 1..8 ranks, one flag per rank");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.element_size() == 2 && out.numel() == world * shard,
              "peer_gather_shards: contiguous 16-bit output of world x shard elements");
  TORCH_CHECK((shard * 2) % 16 == 0 && (offset * 2) % 16 == 0, "peer_gather_shards: 16-byte aligned shards");
  ShardGather g{};
  for (int r = 0; r < world; ++r) {
    g.src[r] = reinterpret_cast<const uint4*>(peer_bufs[r] + offset * 2);
    g.flags[r] = reinterpret_cast<const unsigned long long*>(peer_flags[r]);
  }
  g.dst = reinterpret_cast<uint4*>(out.data_ptr());
  g.n16 = shard * 2 / 16;
  g.world = world;
  g.epoch = static_cast<unsigned long long>(epoch);
  g.timeout_ns = static_cast<unsigned long long>(timeout_ns);
  // Bulk copies: each CTA keeps up to 5 x 32 KB loads in flight; 32 CTAs (~5 MB outstanding) cover
  // NVLink's bandwidth-delay product with room to spare.
  const int64_t chunks = world * ((shard * 2 + kGatherChunk - 1) / kGatherChunk);
  g.ctas = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(32, chunks)));
  const at::cuda::CUDAGuard guard(out.device());
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(mvp::comm::shard_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        mvp::comm::kGatherKernelSmem));
    configured = true;
  }
  mvp::comm::shard_gather_kernel<<<g.ctas, 128, mvp::comm::kGatherKernelSmem, at::cuda::getCurrentCUDAStream()>>>(
      g, reinterpret_cast<int*>(status_ptr));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void publish_epoch(int64_t flag_ptr, int64_t epoch) {
  mvp::comm::publish_epoch_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<unsigned long long*>(flag_ptr), static_cast<unsigned long long>(epoch));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
