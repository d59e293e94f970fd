// Pair-of-SMs bf16 GEMM for sm_100a: one 256 x 256 output tile per cluster of two CTAs.
//
//   C[M, N] (+)= A[M, K] * B[N, K]^T   (same operand conventions as gemm_sm100.cu)
//
// tcgen05.mma with cta_group::2 computes a 256 x 256 x 16 product across the two
// SMs of a cluster: CTA r of the pair holds rows 128r..128r+127 of the A tile and
// rows 128r..128r+127 of the B tile (half of N) in its own shared memory, and its
// own tensor memory receives rows 128r..128r+127 of the accumulator (all 256
// columns).  Per SM and k-block that is 32 KB of operands for 2 x 128 x 256 x 64
// FLOPs -- half the B traffic of a single-SM 128 x 256 tile -- while each SM still
// holds two 256-column accumulators, so the epilogue of one tile overlaps the MMAs
// of the next.
//
// Roles (both CTAs run the same warp layout):
//   warp 0      TMA: each CTA loads its own A and B halves; the copies report
//               their bytes to the leader CTA's full barrier (cta_group::2 copy,
//               plain -- never multicast).
//   warp 1      allocates TMEM in both CTAs (cta_group::2); in the leader CTA one
//               thread issues the MMAs and commits with a two-CTA multicast
//               arrive, releasing ring slots and publishing accumulators in both.
//   warps 2..5  epilogue of this CTA's 128 rows; releases the accumulator by
//               arriving on the leader's barrier.
// Work: whole 256 x 256 tiles, tile t on cluster t % clusters.  For the fp32
// accumulate epilogue (weight gradients) a last, partial wave of tiles is instead
// cut along k and its k-blocks spread evenly over all clusters (WorkList); the
// pieces of a cut tile are added with vector reductions, whole tiles with a
// read-add-write.
// Every wait is bounded; every thread of both CTAs reaches the final cluster
// barrier, after which both MMA warps free the tensor memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tma_host.h"

namespace mvp {
namespace gemm2 {

constexpr int BK = 64;
constexpr int TILE = 256;      // output tile per cluster: 256 x 256
constexpr int HALF = 128;      // rows of A and of B held by each CTA
constexpr int STAGES = 6;
constexpr int A_BYTES = HALF * BK * 2;   // 16 KB
constexpr int B_BYTES = HALF * BK * 2;   // 16 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;           // two 256-column accumulators
constexpr int THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;

enum Epilogue : int { kStoreBf16 = 0, kStoreF32 = 1, kAccumF32 = 2 };

struct Params {
  int M, N, K;
  void* C;
  int64_t ldc;
  int* status;
  int group_m;
  // Tensor-parallel fusion (both optional):
  //  * rows of a K-major A arrive from other ranks: rows [j*a_rows, (j+1)*a_rows) are usable once
  //    a_slots[j] >= a_seq (published by rank j after pushing them here); tiles start at row
  //    a_first_row so a rank begins with the rows it already holds.
  const unsigned long long* a_slots;
  unsigned long long a_seq;
  int a_rows;
  int a_first_row;
  unsigned long long wait_ns;
  //  * bf16 output rows are routed to other ranks: row m goes to row (dst_row0 + m % dst_rows) of
  //    the buffer at dst[m / dst_rows] (a peer's memory), row stride ldc.
  void* dst[8];
  int dst_rows;
  int dst_row0;
  //  * Ulysses sequence -> head routing (u_world > 0): output row m (this rank's local token) goes to
  //    global row ulysses_global_row(m) of dst[d], where column n of section s (u_sec[s] heads of
  //    u_hd columns, each section split evenly over the u_world ranks) belongs to rank
  //    d = head / (u_sec[s] / u_world); on rank d the sections are packed side by side (this rank's
  //    share of section 0, then of section 1, ...), row stride ldc.
  int u_world, u_rank, u_chunk, u_hd;
  int u_sec[3];
  // FSDP parameter gather carried by this GEMM (optional, gather.ctas > 0): CTAs with
  // blockIdx.x >= 2 * gemm_clusters pull the next unit's shards into its staging slot while the
  // other CTAs compute this GEMM's tiles.  Nothing in the GEMM reads the gathered buffer.
  ShardGather gather{};
  int gemm_clusters = 0;  // clusters that compute tiles (set at launch)
  // Work split (set at launch): tiles [0, dp_tiles) are whole-tile units, tile t on cluster
  // t % gemm_clusters; the k-blocks of tiles [dp_tiles, tiles) are spread evenly over clusters
  // 0 .. sk_clusters-1 (stream-K tail; only for the fp32 accumulate epilogue, whose split tiles are
  // summed with vector reductions).  sk_clusters == 0: every tile is a whole-tile unit.
  int dp_tiles = 0;
  int sk_clusters = 0;
};

// The units of work of one cluster, in the order all three roles walk them: its whole tiles first,
// then its contiguous share of the tail's (tile, k-block) iterations, cut at tile boundaries.
struct WorkList {
  int clusters, dp_tiles, num_kb;
  int t;                 // next whole tile
  long long it, it_end;  // next / end tail iteration
  __device__ WorkList(const Params& p, int cluster, int num_kb_)
      : clusters(p.gemm_clusters), dp_tiles(p.dp_tiles), num_kb(num_kb_), t(cluster), it(0), it_end(0) {
    if (cluster < p.sk_clusters) {
      const int num_m = (p.M + TILE - 1) / TILE, num_n = (p.N + TILE - 1) / TILE;
      const long long total = static_cast<long long>(num_m * num_n - p.dp_tiles) * num_kb;
      it = total * cluster / p.sk_clusters;
      it_end = total * (cluster + 1) / p.sk_clusters;
    }
  }
  // Next unit: tile index and k-block range [kb0, kb1); false when the cluster is done.
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (t < dp_tiles) {
      tile = t;
      kb0 = 0;
      kb1 = num_kb;
      t += clusters;
      return true;
    }
    if (it < it_end) {
      tile = dp_tiles + static_cast<int>(it / num_kb);
      kb0 = static_cast<int>(it % num_kb);
      kb1 = static_cast<int>(min(static_cast<long long>(num_kb), kb0 + (it_end - it)));
      it += kb1 - kb0;
      return true;
    }
    return false;
  }
};

// Fire-and-forget fp32 x4 reduction into global memory (split tiles of the accumulate epilogue).
__device__ __forceinline__ void red_add_f32x4(float* addr, float4 v) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared-memory address of the same variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_bar_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar_addr) : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion is reported to the
// barrier at cluster address `bar` (the leader CTA's).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at this offset in both CTAs of the pair when the MMAs issued so far are done.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Arrive on this CTA's barrier when the pair MMAs issued so far are done.
__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group_m, int& tm, int& tn) {
  const int per_group = group_m * num_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gm = min(group_m, num_m - first_m);
  const int r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);  // used in the leader
  uint64_t* empty_bar = full_bar + STAGES;                                         // both CTAs
  uint64_t* tfull_bar = empty_bar + STAGES;                                        // [2] both CTAs
  uint64_t* tempty_bar = tfull_bar + 2;                                            // [2] used in the leader
  uint64_t* done_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (p.gather.ctas > 0 && static_cast<int>(blockIdx.x) >= 2 * p.gemm_clusters) {
    // copy CTA (both CTAs of its cluster are copy CTAs): no barriers, no tensor memory
    // 5 x 32 KB stages of bulk copies fit in the GEMM's shared-memory footprint (6 operand stages)
    shard_gather_cta_bulk(p.gather, static_cast<int>(blockIdx.x) - 2 * p.gemm_clusters, p.status, smem, 5);
    return;
  }
  const uint32_t crank = cluster_ctarank();  // 0 = leader
  const int cluster_id = blockIdx.x >> 1;
  const int num_m = (p.M + TILE - 1) / TILE;
  const int num_n = (p.N + TILE - 1) / TILE;
  const int num_kb = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * 128);  // epilogue threads of both CTAs
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
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive / copy
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one_sync()) {
      const uint32_t leader_full0 = mapa_shared(smem_u32(&full_bar[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      uint32_t ready = 0;  // A row slices already seen published
      bool ok = true;
      WorkList work(p, cluster_id, num_kb);
      int t, kb0, kb1;
      while (ok && work.next(t, kb0, kb1)) {
        int tm, tn;
        tile_coords(t, num_m, num_n, p.group_m, tm, tn);
        tm = (tm + p.a_first_row / TILE) % num_m;
        const int m0 = tm * TILE + crank * HALF, n0 = tn * TILE + crank * HALF;
        if (p.a_slots != nullptr) {
          const int j = (tm * TILE) / p.a_rows;
          if (!((ready >> j) & 1u)) {
            const uint64_t t0 = globaltimer();
            while (ld_acquire_sys_u64(p.a_slots + j) < p.a_seq) {
              if (*abort_flag || globaltimer() - t0 > p.wait_ns) {
                if (!*abort_flag) record_status(p.status, kTimeoutPeer);
                *abort_flag = 1;
                ok = false;
                break;
              }
              __nanosleep(128);
            }
            if (!ok) break;
            asm volatile("fence.proxy.async.global;" ::: "memory");  // peer-written rows, read by TMA
            ready |= 1u << j;
          }
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, abort_flag, p.status, kTimeoutProducer)) {
            ok = false;
            break;
          }
          if (crank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * STAGE_BYTES);
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          const uint32_t bar = leader_full0 + stage * 8;
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, bar, k0, m0);
          } else {
            tma_load_2d_pair(a_dst, &tmA, bar, m0, k0);
            tma_load_2d_pair(a_dst + 64 * BK * 2, &tmA, bar, m0 + 64, k0);
          }
          if constexpr (!B_MN) {
            tma_load_2d_pair(b_dst, &tmB, bar, k0, n0);
          } else {
            tma_load_2d_pair(b_dst, &tmB, bar, n0, k0);
            tma_load_2d_pair(b_dst + 64 * BK * 2, &tmB, bar, n0 + 64, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // After an abort, let copies already issued into this CTA's ring land (bounded) before exit.
      if ((!ok || *abort_flag) && issued_mask) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 200000000ull) {
        }
        (void)issued_phase;
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA (leader only)
    if (crank == 0 && elect_one_sync()) {
      constexpr uint32_t idesc = make_idesc_bf16(TILE, TILE, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      WorkList work(p, cluster_id, num_kb);
      int t, kb0, kb1;
      for (; ok && work.next(t, kb0, kb1); ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, abort_flag, p.status, kTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * TILE;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag, p.status, kTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t adesc, bdesc;
            if constexpr (!A_MN) adesc = make_smem_desc_sw128(a_base + k * 32, 16, 1024);
            else adesc = make_smem_desc_sw128(a_base + k * 2048, 64 * BK * 2, 1024);
            if constexpr (!B_MN) bdesc = make_smem_desc_sw128(b_base + k * 32, 16, 1024);
            else bdesc = make_smem_desc_sw128(b_base + k * 2048, 64 * BK * 2, 1024);
            mma_pair(d_tmem, adesc, bdesc, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          mma_commit_pair(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit_pair(&tfull_bar[acc]);
      }
      mma_commit_pair_local(done_bar);
      mbar_wait_bounded(done_bar, 0, abort_flag, p.status, kTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int sub = warp & 3;
    const int row_in_tile = crank * HALF + sub * 32 + lane;
    const uint32_t leader_tempty0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
    int local = 0;
    WorkList work(p, cluster_id, num_kb);
    int t, kb0, kb1;
    for (; work.next(t, kb0, kb1); ++local) {
      int tm, tn;
      tile_coords(t, num_m, num_n, p.group_m, tm, tn);
      tm = (tm + p.a_first_row / TILE) % num_m;
      // a tile split over several units is summed with reductions; a whole tile is read, added, written
      const bool split = kb0 != 0 || kb1 != num_kb;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!__all_sync(0xffffffffu,
                      mbar_wait_bounded(&tfull_bar[acc], acc_phase, abort_flag, p.status, kTimeoutEpilogue)))
        break;
      tc_fence_after();
      const int m = tm * TILE + row_in_tile;
      const bool row_ok = m < p.M;
#pragma unroll 1
      for (int c = 0; c < TILE / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + acc * TILE + c * 32, r);
        tmem_wait_ld();
        const int n = tn * TILE + c * 32;
        if (!row_ok || n >= p.N) continue;
        const bool full_chunk = (n + 32 <= p.N);
        if constexpr (EPI == kStoreBf16) {
          __nv_bfloat16* C = p.dst_rows > 0
                                 ? reinterpret_cast<__nv_bfloat16*>(p.dst[m / p.dst_rows]) +
                                       static_cast<int64_t>(p.dst_row0 + m % p.dst_rows) * p.ldc + n
                                 : reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(m) * p.ldc + n;
          if (p.u_world > 0) {  // a 32-column chunk never straddles a head (u_hd % 32 == 0)
            int col = n, prefix = 0, s = 0;
            while (s < 2 && col >= p.u_sec[s] * p.u_hd) {
              col -= p.u_sec[s] * p.u_hd;
              prefix += (p.u_sec[s] / p.u_world) * p.u_hd;
              ++s;
            }
            const int per = p.u_sec[s] / p.u_world;
            const int head = col / p.u_hd;
            const int d = head / per;
            const int g = ulysses_global_row(p.u_world, p.u_rank, p.u_chunk, m);
            C = reinterpret_cast<__nv_bfloat16*>(p.dst[d]) + static_cast<int64_t>(g) * p.ldc + prefix +
                (head - d * per) * p.u_hd + col % p.u_hd;
          }
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
                if (split) {
                  red_add_f32x4(reinterpret_cast<float*>(dst + v), q);
                  continue;
                }
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
              if constexpr (EPI == kAccumF32) {
                if (split) {
                  atomicAdd(C + j, val);
                  continue;
                }
                val += C[j];
              }
              C[j] = val;
            }
          }
        }
      }
      tc_fence_before();
      remote_arrive(leader_tempty0 + acc * 8);
    }
    if (p.dst_rows > 0 || p.u_world > 0) __threadfence_system();  // routed rows visible before the publish
  }

  // Both CTAs: every role is done (the leader's MMAs have retired); then free the pair's TMEM.
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

constexpr int kMinSkBlocks = 8;  // smallest stream-K piece, in k-blocks of BK

// Stream-K tail for the accumulate epilogue; MVP_GEMM_STREAMK=0 turns it off (whole tiles only).
inline bool stream_k_enabled() {
  static const bool on = [] {
    const char* env = std::getenv("MVP_GEMM_STREAMK");
    return env == nullptr || env[0] != '0';
  }();
  return on;
}

template <bool A_MN, bool B_MN, int EPI>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int num_sms, cudaStream_t stream) {
  auto kern = gemm2sm_kernel<A_MN, B_MN, EPI>;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured = true;
  }
  const int num_tiles = ((p.M + TILE - 1) / TILE) * ((p.N + TILE - 1) / TILE);
  const int num_kb = (p.K + BK - 1) / BK;
  const int copy_ctas = p.gather.ctas;  // even: copy CTAs come in clusters of two
  const int max_clusters = std::max(1, (num_sms - copy_ctas) / 2);
  int clusters = std::min(num_tiles, max_clusters);
  int dp_tiles = num_tiles, sk_clusters = 0;
  if (EPI == kAccumF32 && stream_k_enabled()) {
    // The last, partial wave of whole tiles would leave clusters idle: spread its k-blocks over
    // all clusters instead (pieces of at least kMinSkBlocks), when that wave is at most 7/8 full.
    const int tail = num_tiles % max_clusters;
    if (tail > 0 && 8 * tail <= 7 * max_clusters) {
      const long long tail_blocks = static_cast<long long>(tail) * num_kb;
      const int sk = static_cast<int>(std::min<long long>(max_clusters, tail_blocks / kMinSkBlocks));
      if (sk > tail) {
        dp_tiles = num_tiles - tail;
        sk_clusters = sk;
        clusters = std::max(std::min(dp_tiles, max_clusters), sk);
      }
    }
  }
  Params q = p;
  q.gemm_clusters = clusters;
  q.dp_tiles = dp_tiles;
  q.sk_clusters = sk_clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters + copy_ctas);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, q));
}

template <int EPI>
void dispatch(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int sms,
              cudaStream_t s) {
  if (!a_mn && !b_mn) launch<false, false, EPI>(ta, tb, p, sms, s);
  else if (!a_mn && b_mn) launch<false, true, EPI>(ta, tb, p, sms, s);
  else if (a_mn && !b_mn) launch<true, false, EPI>(ta, tb, p, sms, s);
  else launch<true, true, EPI>(ta, tb, p, sms, s);
}

}  // namespace gemm2
}  // namespace mvp

// Same contract as gemm_sm100 (operands already validated by the caller); `gather` (optional) is an
// FSDP shard pull carried by extra CTAs of the launch.
static void pair_gemm_impl(const torch::Tensor& a, bool a_mn, const torch::Tensor& b, bool b_mn, torch::Tensor& c,
                           bool accumulate, int64_t status_ptr, const mvp::ShardGather* gather) {
  using namespace mvp::gemm2;
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const bool out_f32 = c.scalar_type() == at::kFloat;
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  CUtensorMap ta, tb;
  // Each CTA loads 128 rows of A and 128 rows of B (K-major: one 64 x 128 box; MN-major: two 64 x 64 boxes).
  if (!a_mn) mvp::make_tmap_2d_bf16(&ta, a.data_ptr(), K, M, a.stride(0), 64, HALF);
  else mvp::make_tmap_2d_bf16(&ta, a.data_ptr(), M, K, a.stride(0), 64, 64);
  if (!b_mn) mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), K, N, b.stride(0), 64, HALF);
  else mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), N, K, b.stride(0), 64, 64);
  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.status = reinterpret_cast<int*>(status_ptr);
  p.group_m = 8;
  p.a_slots = nullptr;
  p.a_seq = 0;
  p.a_rows = 0;
  p.a_first_row = 0;
  p.wait_ns = 0;
  for (int j = 0; j < 8; ++j) p.dst[j] = nullptr;
  p.dst_rows = 0;
  p.dst_row0 = 0;
  p.u_world = p.u_rank = p.u_chunk = p.u_hd = 0;
  p.u_sec[0] = p.u_sec[1] = p.u_sec[2] = 0;
  if (gather != nullptr) p.gather = *gather;
  const int sms = mvp::num_sms(a.get_device());
  const int epi = out_f32 ? (accumulate ? kAccumF32 : kStoreF32) : kStoreBf16;
  if (epi == kStoreBf16) dispatch<kStoreBf16>(a_mn, b_mn, ta, tb, p, sms, stream);
  else if (epi == kStoreF32) dispatch<kStoreF32>(a_mn, b_mn, ta, tb, p, sms, stream);
  else dispatch<kAccumF32>(a_mn, b_mn, ta, tb, p, sms, stream);
}

void gemm_sm100_pair(const torch::Tensor& a, bool a_mn, const torch::Tensor& b, bool b_mn, torch::Tensor& c,
                     bool accumulate, int64_t status_ptr) {
  pair_gemm_impl(a, a_mn, b, b_mn, c, accumulate, status_ptr, nullptr);
}

// Two-SM GEMM (operands as gemm_sm100, M, N >= 256) that also carries the FSDP parameter gather of
// another unit: `copy_ctas` (even, < SM count) extra CTAs pull peer_bufs[r] + offset (bf16 elements, one
// shard of `shard` elements per rank, after every rank published `epoch` into peer_flags[r]) into
// `slot` [world * shard].  The GEMM never reads `slot`; the caller orders the gathered unit's use after
// this launch on the same stream.
void gemm_pair_gather(const torch::Tensor& a, bool a_mn, const torch::Tensor& b, bool b_mn, torch::Tensor& c,
                      bool accumulate, int64_t status_ptr, const std::vector<int64_t>& peer_bufs,
                      const std::vector<int64_t>& peer_flags, int64_t offset, int64_t shard, int64_t epoch,
                      torch::Tensor& slot, int64_t copy_ctas, int64_t timeout_ns) {
  using namespace mvp;
  const int world = static_cast<int>(peer_bufs.size());
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && c.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16 && a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1 &&
                  a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0,
              "gemm_pair_gather: bf16 operands with unit inner stride and 8-element row strides");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(b.data_ptr()) & 15) == 0,
              "gemm_pair_gather: operands must be 16-byte aligned");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK(K == (b_mn ? b.size(0) : b.size(1)) && c.size(0) == M && c.size(1) == N && M >= 256 && N >= 256 && K > 0,
              "gemm_pair_gather: shapes (M, N >= 256)");
  TORCH_CHECK(c.scalar_type() == at::kBFloat16 || c.scalar_type() == at::kFloat, "gemm_pair_gather: bf16/fp32 out");
  TORCH_CHECK(!accumulate || c.scalar_type() == at::kFloat, "gemm_pair_gather: accumulate needs fp32 output");
  TORCH_CHECK(world >= 1 && world <= kMaxGatherRanks && static_cast<int>(peer_flags.size()) == world,
              "gemm_pair_gather: 1..8 ranks, one flag per rank");
  TORCH_CHECK(slot.is_cuda() && slot.is_contiguous() && slot.element_size() == 2 && slot.numel() == world * shard,
              "gemm_pair_gather: contiguous 16-bit slot of world x shard elements");
  TORCH_CHECK((shard * 2) % 16 == 0 && (offset * 2) % 16 == 0, "gemm_pair_gather: 16-byte aligned shards");
  const int sms = num_sms(a.get_device());
  TORCH_CHECK(copy_ctas >= 2 && copy_ctas % 2 == 0 && copy_ctas <= sms - 2, "gemm_pair_gather: even copy_ctas < SMs");
  ShardGather g{};
  for (int r = 0; r < world; ++r) {
    g.src[r] = reinterpret_cast<const uint4*>(peer_bufs[r] + offset * 2);
    g.flags[r] = reinterpret_cast<const unsigned long long*>(peer_flags[r]);
  }
  g.dst = reinterpret_cast<uint4*>(slot.data_ptr());
  g.n16 = shard * 2 / 16;
  g.world = world;
  g.epoch = static_cast<unsigned long long>(epoch);
  g.timeout_ns = static_cast<unsigned long long>(timeout_ns);
  g.ctas = static_cast<int>(copy_ctas);
  pair_gemm_impl(a, a_mn, b, b_mn, c, accumulate, status_ptr, &g);
}

// Tensor-parallel GEMM on the two-SM kernel, bf16 out, K-major A [M, K] and B [N, K]
// (or N-major B [K, N] when b_mn).
//   a_slots != 0: A's rows arrive in slices of a_rows rows (slice j usable once slot j >= a_seq);
//                 the rank owning slice a_first_row / a_rows starts there.
//   dst non-empty: output row m is written to row dst_row0 + m % dst_rows of dst[m / dst_rows]
//                  (row stride ldc); otherwise to c.
void gemm_pair_tp(const torch::Tensor& a, const torch::Tensor& b, bool b_mn, const c10::optional<torch::Tensor>& c,
                  int64_t ldc, int64_t a_slots, int64_t a_seq, int64_t a_rows, int64_t a_first_row,
                  const std::vector<int64_t>& dst, int64_t dst_rows, int64_t dst_row0, int64_t status_ptr,
                  int64_t wait_ns) {
  using namespace mvp::gemm2;
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "gemm_pair_tp: bf16 CUDA operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 && a.stride(0) % 8 == 0 &&
                  b.stride(0) % 8 == 0,
              "gemm_pair_tp: row-major operands with 16-byte row strides");
  const int64_t M = a.size(0), K = a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm_pair_tp: reduction sizes differ");
  TORCH_CHECK(M >= TILE && N >= TILE && M % TILE == 0, "gemm_pair_tp: M, N >= 256 and M % 256 == 0");
  TORCH_CHECK(a_slots == 0 || (a_rows % TILE == 0 && M % a_rows == 0 && M / a_rows <= 32 && a_first_row % TILE == 0),
              "gemm_pair_tp: A slices must be whole 256-row tiles");
  TORCH_CHECK(dst.empty() || (dst.size() <= 8 && dst_rows > 0 && M == dst_rows * static_cast<int64_t>(dst.size())),
              "gemm_pair_tp: output routing covers M with <= 8 destinations");
  TORCH_CHECK(!dst.empty() || (c.has_value() && c->scalar_type() == at::kBFloat16 && c->size(0) == M &&
                               c->size(1) == N && c->stride(1) == 1),
              "gemm_pair_tp: bf16 output [M, N]");
  TORCH_CHECK(ldc % 8 == 0 && ldc >= N, "gemm_pair_tp: ldc");
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  CUtensorMap ta, tb;
  mvp::make_tmap_2d_bf16(&ta, a.data_ptr(), K, M, a.stride(0), 64, HALF);
  if (!b_mn) mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), K, N, b.stride(0), 64, HALF);
  else mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), N, K, b.stride(0), 64, 64);
  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = dst.empty() ? c->data_ptr() : nullptr;
  p.ldc = ldc;
  p.status = reinterpret_cast<int*>(status_ptr);
  p.group_m = 8;
  p.a_slots = reinterpret_cast<const unsigned long long*>(a_slots);
  p.a_seq = static_cast<unsigned long long>(a_seq);
  p.a_rows = static_cast<int>(a_rows);
  p.a_first_row = static_cast<int>(a_first_row);
  p.wait_ns = static_cast<unsigned long long>(wait_ns);
  for (int j = 0; j < 8; ++j) p.dst[j] = j < static_cast<int>(dst.size()) ? reinterpret_cast<void*>(dst[j]) : nullptr;
  p.dst_rows = static_cast<int>(dst_rows);
  p.dst_row0 = static_cast<int>(dst_row0);
  p.u_world = p.u_rank = p.u_chunk = p.u_hd = 0;
  p.u_sec[0] = p.u_sec[1] = p.u_sec[2] = 0;
  const int sms = mvp::num_sms(a.get_device());
  dispatch<kStoreBf16>(false, b_mn, ta, tb, p, sms, stream);
}

// Ulysses projection on the two-SM kernel: Y = A[M = 2 x chunk local tokens, K] * B^T (B [N, K], or
// N-major [K, N] when b_mn), bf16, with every output element written straight into the buffer of the
// rank that owns its head (dst[d], [world x 2 x chunk tokens, ld]; see Params).  `secs` gives the heads
// of each column section (e.g. q, k, v); N = head_dim x sum(secs).
void gemm_ulysses(const torch::Tensor& a, const torch::Tensor& b, bool b_mn, const std::vector<int64_t>& dst,
                  int64_t ld, int64_t rank, int64_t chunk, int64_t head_dim, const std::vector<int64_t>& secs,
                  int64_t status_ptr) {
  using namespace mvp::gemm2;
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "gemm_ulysses: bf16 CUDA operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 && a.stride(0) % 8 == 0 &&
                  b.stride(0) % 8 == 0,
              "gemm_ulysses: row-major operands with 16-byte row strides");
  const int64_t M = a.size(0), K = a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t W = static_cast<int64_t>(dst.size());
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm_ulysses: reduction sizes differ");
  TORCH_CHECK(W >= 1 && W <= 8 && rank >= 0 && rank < W, "gemm_ulysses: 1..8 ranks");
  TORCH_CHECK(M == 2 * chunk && M >= TILE && N >= TILE, "gemm_ulysses: M = 2 x chunk >= 256, N >= 256");
  TORCH_CHECK(head_dim % 32 == 0 && secs.size() == 3, "gemm_ulysses: head_dim % 32 == 0, three sections");
  int64_t heads = 0, per_rank = 0;
  for (int64_t s : secs) {
    TORCH_CHECK(s >= 0 && s % W == 0, "gemm_ulysses: every section's heads divisible by the ranks");
    heads += s;
    per_rank += s / W;
  }
  TORCH_CHECK(N == heads * head_dim, "gemm_ulysses: N = head_dim x heads");
  TORCH_CHECK(ld % 8 == 0 && ld >= per_rank * head_dim, "gemm_ulysses: destination row stride");
  for (int64_t d : dst) TORCH_CHECK(d != 0 && d % 16 == 0, "gemm_ulysses: 16-byte aligned destinations");
  const at::cuda::CUDAGuard guard(a.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  CUtensorMap ta, tb;
  mvp::make_tmap_2d_bf16(&ta, a.data_ptr(), K, M, a.stride(0), 64, HALF);
  if (!b_mn) mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), K, N, b.stride(0), 64, HALF);
  else mvp::make_tmap_2d_bf16(&tb, b.data_ptr(), N, K, b.stride(0), 64, 64);
  Params p;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = nullptr;
  p.ldc = ld;
  p.status = reinterpret_cast<int*>(status_ptr);
  p.group_m = 8;
  p.a_slots = nullptr;
  p.a_seq = 0;
  p.a_rows = 0;
  p.a_first_row = 0;
  p.wait_ns = 0;
  for (int j = 0; j < 8; ++j) p.dst[j] = j < W ? reinterpret_cast<void*>(dst[j]) : nullptr;
  p.dst_rows = 0;
  p.dst_row0 = 0;
  p.u_world = static_cast<int>(W);
  p.u_rank = static_cast<int>(rank);
  p.u_chunk = static_cast<int>(chunk);
  p.u_hd = static_cast<int>(head_dim);
  for (int s = 0; s < 3; ++s) p.u_sec[s] = static_cast<int>(secs[s]);
  const int sms = mvp::num_sms(a.get_device());
  dispatch<kStoreBf16>(false, b_mn, ta, tb, p, sms, stream);
}
