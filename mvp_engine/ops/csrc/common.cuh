// Shared device helpers for the sm_100a kernels of mvp_engine.
//
// Everything here is written directly against the PTX ISA for Blackwell
// (sm_100a): mbarriers, TMA tensor copies (cp.async.bulk.tensor), the
// 5th-generation tensor core (tcgen05.mma with accumulators in TMEM) and the
// TMEM load path (tcgen05.ld).  Every wait on an mbarrier is bounded by a
// wall-clock budget read from %globaltimer: when the budget runs out the
// waiting thread raises a CTA-wide abort flag in shared memory and records an
// error code in a global status word, so a broken pipeline returns to the host
// with an error instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#ifndef MVP_WAIT_TIMEOUT_NS
#define MVP_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: far above any legitimate wait
#endif

namespace mvp {

// Error codes written into the global status word (first writer wins).
enum StatusCode : int {
  kOk = 0,
  kTimeoutProducer = 1,
  kTimeoutMma = 2,
  kTimeoutEpilogue = 3,
  kTimeoutDrain = 4,
  kTimeoutPeer = 5,
  kBadArgument = 6,
  kBoundsCheck = 7,  // debug builds only: an index derived from metadata left its tensor; the access was skipped
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// Bounds checks of the debug build (``MVP_DEBUG=1 python setup.py build_ext --inplace`` defines
// MVP_DEBUG_BOUNDS): MVP_BOUNDS_OK(status, cond) is `cond`, and a false `cond` also records kBoundsCheck so
// that the host raises after the step; the caller then skips the access (never a trap).  Release builds
// compile it to `true`.
#ifdef MVP_DEBUG_BOUNDS
#define MVP_BOUNDS_OK(status, cond) ((cond) ? true : (::mvp::record_status((status), ::mvp::kBoundsCheck), false))
#else
#define MVP_BOUNDS_OK(status, cond) true
#endif

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false
// when the CTA is aborting (another role gave up) or when this wait ran past
// its budget, in which case it raises the abort flag and records `code`.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > MVP_WAIT_TIMEOUT_NS) {
        *abort_flag = 1;
        record_status(status, code);
        return false;
      }
    }
  }
}

// -------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory; completion is reported as
// transaction bytes on `bar`.  c0 is the innermost (contiguous) coordinate and
// must be a multiple of 8 for 16-bit data (16-byte rule of the TMA unit).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
// Shared-memory matrix descriptor (Blackwell format, version field = 1).
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4
//   bits 32-45 stride-dimension byte offset >> 4
//   bits 46-47 version (1 on sm_100)
//   bits 61-63 swizzle mode (2 = 128-byte swizzle)
__device__ __forceinline__ uint64_t make_smem_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 inputs and fp32 accumulate.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format,
//   bit 15/16 A/B major (0 = K-major, 1 = MN-major), 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(N) >> 3) << 17) | ((static_cast<uint32_t>(M) >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by a single thread.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T (A operand read from tensor memory).
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane
// (base_lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive columns written from registers (used to stage P in TMEM).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "selp.b32 %0, 1, 0, px;\n\t}"
      : "=r"(pred)
      : "r"(0xFFFFFFFFu));
  return pred;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------- peer memory (NVLink)
// Release / acquire at system scope: a flag another GPU reads (or writes) orders the data around it.
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// A copy of another rank's buffer into this GPU's memory, carried by extra CTAs of a compute
// kernel (grid rows blockIdx.y < rows) so that the transfer overlaps the kernel's own tiles.
// The copy starts once the owner has published `seq` into `ready` (a slot in this GPU's memory
// that the owner writes with a system-scope release); the wait is bounded by timeout_ns, after
// which the status word records kTimeoutPeer and nothing is read.
struct PeerPull {
  const uint4* src;  // the owner's buffer, mapped into this process
  uint4* dst;        // this GPU's buffer
  int64_t n16;       // 16-byte units
  const unsigned long long* ready;
  unsigned long long seq;
  unsigned long long timeout_ns;
  int rows;  // grid rows given to the copy (0: no copy)
};

// FSDP parameter gather by pulling: the full weights of one unit are rebuilt in this GPU's staging
// slot from every rank's bf16 shard, read straight out of the ranks' symmetric shard buffers (rank r's
// shard lands at r * n16).  Each rank publishes an epoch into its own flag after its optimizer step has
// written its shard; a copy CTA waits (bounded) until every rank's epoch reaches `epoch`, so a rank
// that runs ahead never reads a peer's shard of the previous step.  Shards do not change between
// two optimizer steps, so nothing else needs ordering: the copy is safe at any point of the step.
constexpr int kMaxGatherRanks = 8;
struct ShardGather {
  const uint4* src[kMaxGatherRanks];                 // rank r's shard of the unit (peer mapping; own: local)
  const unsigned long long* flags[kMaxGatherRanks];  // rank r's published epoch
  uint4* dst;                                        // the unit's full buffer in this GPU's staging slot
  int64_t n16;                                       // 16-byte units per shard
  int world;
  unsigned long long epoch;
  unsigned long long timeout_ns;
  int ctas;  // CTAs that carry the copy (0: no copy)
};

// One copy CTA of `g`: CTA `cta` of g.ctas copies every (g.ctas)-th chunk (all threads call it).
__device__ __forceinline__ void shard_gather_cta(const ShardGather& g, int cta, int* status, int* flag) {
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < g.world && ok; ++r) {
      while (ld_acquire_sys(g.flags[r]) < g.epoch) {
        if (globaltimer() - t0 > g.timeout_ns) {
          record_status(status, kTimeoutPeer);
          ok = 0;
          break;
        }
        __nanosleep(128);
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    *flag = ok;
  }
  __syncthreads();
  if (!*flag) return;
  constexpr int kUnroll = 8;  // 16-byte loads in flight per thread: covers the NVLink round trip
  const int64_t total = g.n16 * g.world;
  const int64_t stride = static_cast<int64_t>(g.ctas) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(cta) * blockDim.x + threadIdx.x; i0 < total; i0 += stride * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < total) {
        const int64_t r = i / g.n16;
        v[u] = g.src[r][i - r * g.n16];
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < total) g.dst[i] = v[u];
    }
  }
}

// Bulk-copy (TMA, non-tensor) variant of shard_gather_cta: one elected thread moves the CTA's chunks
// with cp.async.bulk, peer (or local) global memory -> this CTA's shared memory -> the staging slot,
// `stages` chunks of kGatherChunk bytes in flight at a time.  A handful of CTAs then saturates NVLink:
// each keeps stages x 32 KB of loads outstanding instead of a few KB of register loads.  Never a
// multicast load.  `smem` holds the stages and, after them, `stages` mbarriers.
constexpr int kGatherChunk = 32768;

__device__ __forceinline__ void bulk_load_to_smem(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(sdst)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_store_from_smem(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_one_pending() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ bool mbar_spin_bounded(uint64_t* bar, uint32_t parity, uint64_t t0, uint64_t limit_ns) {
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}

__device__ __forceinline__ void shard_gather_cta_bulk(const ShardGather& g, int cta, int* status, uint8_t* smem,
                                                      int stages) {
  __shared__ int ok_flag;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * kGatherChunk);
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer();
    for (int r = 0; r < g.world && ok; ++r) {
      while (ld_acquire_sys(g.flags[r]) < g.epoch) {
        if (globaltimer() - t0 > g.timeout_ns) {
          record_status(status, kTimeoutPeer);
          ok = 0;
          break;
        }
        __nanosleep(128);
      }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_mbarrier_init();
    ok_flag = ok;
  }
  __syncthreads();
  if (!ok_flag || threadIdx.x != 0) return;
  const int64_t shard_bytes = g.n16 * 16;
  const int64_t per_rank = (shard_bytes + kGatherChunk - 1) / kGatherChunk;
  const int64_t total = per_rank * g.world;
  const int64_t mine = total > cta ? (total - cta + g.ctas - 1) / g.ctas : 0;  // chunks cta, cta+ctas, ...
  uint8_t* dst_base = reinterpret_cast<uint8_t*>(g.dst);
  // Ring of `stages` chunk buffers: chunk i lives in stage i % stages.  Loads run `stages` chunks ahead;
  // a stage is refilled as soon as the store of its previous chunk has read it, so stages - 1 loads stay in
  // flight while each store drains (a load's round trip over NVLink is the long pole).
  auto chunk_of = [&](int64_t i, int64_t& off, uint32_t& len) -> const uint8_t* {
    const int64_t q = cta + i * g.ctas;
    const int64_t r = q / per_rank, b0 = (q - r * per_rank) * kGatherChunk;
    len = static_cast<uint32_t>(shard_bytes - b0 < kGatherChunk ? shard_bytes - b0 : kGatherChunk);
    off = r * shard_bytes + b0;
    return reinterpret_cast<const uint8_t*>(g.src[r]) + b0;
  };
  auto issue_load = [&](int64_t i) {
    int64_t off;
    uint32_t len;
    const uint8_t* src = chunk_of(i, off, len);
    const int st = static_cast<int>(i % stages);
    mbar_arrive_expect_tx(&bars[st], len);
    bulk_load_to_smem(smem + static_cast<size_t>(st) * kGatherChunk, src, len, &bars[st]);
  };
  for (int64_t i = 0; i < mine && i < stages; ++i) issue_load(i);
  const uint64_t t0 = globaltimer();
  for (int64_t i = 0; i < mine; ++i) {
    const int st = static_cast<int>(i % stages);
    const uint32_t parity = static_cast<uint32_t>((i / stages) & 1);
    if (!mbar_spin_bounded(&bars[st], parity, t0, g.timeout_ns)) {
      record_status(status, kTimeoutPeer);
      // let the loads already issued land (bounded) before the CTA's shared memory goes away
      const uint64_t t1 = globaltimer();
      for (int64_t w = i; w < mine && w < i + stages; ++w)
        mbar_spin_bounded(&bars[w % stages], static_cast<uint32_t>((w / stages) & 1), t1, 200000000ull);
      break;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    int64_t off;
    uint32_t len;
    chunk_of(i, off, len);
    bulk_store_from_smem(dst_base + off, smem + static_cast<size_t>(st) * kGatherChunk, len);
    bulk_commit();
    // Refill the stage of the previous chunk once its store has read it (the store just issued may still
    // be reading): stores overlap each other and stages - 1 loads stay in flight.
    if (i > 0 && i - 1 + stages < mine) {
      bulk_wait_read_one_pending();
      issue_load(i - 1 + stages);
    }
  }
  bulk_wait_all();
}

// Body of one copy CTA (all threads of the CTA call it; `flag` is one int of shared memory).
__device__ __forceinline__ void peer_pull_cta(const PeerPull& j, int* status, int* flag) {
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(j.ready) < j.seq) {
      if (globaltimer() - t0 > j.timeout_ns) {
        record_status(status, kTimeoutPeer);
        ok = 0;
        break;
      }
      __nanosleep(128);
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    *flag = ok;
  }
  __syncthreads();
  if (!*flag) return;
  constexpr int kUnroll = 8;  // 16-byte loads in flight per thread: covers the NVLink round trip
  const int64_t cta = static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x;
  const int64_t stride = static_cast<int64_t>(j.rows) * gridDim.x * blockDim.x;
  for (int64_t i0 = cta * blockDim.x + threadIdx.x; i0 < j.n16; i0 += stride * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < j.n16) v[u] = j.src[i];
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < j.n16) j.dst[i] = v[u];
    }
  }
}

// ---------------------------------------------- Ulysses (sequence <-> head) routing
// Context-parallel ranks hold a packed row in zig-zag order: with W ranks the row is cut into 2W chunks
// of `chunk` tokens and rank r keeps chunks r and 2W-1-r (its local rows 0..chunk-1 and chunk..2chunk-1).
// Head-parallel tensors ([T tokens, this rank's heads]) are written back to the token's rank by a
// producing kernel through this descriptor.
struct UlyssesRoute {
  void* dst[8];  // every rank's destination buffer (peer-mapped); dst[0] == nullptr: no routing
  int64_t ld;    // destination row stride in elements
  int world, rank, chunk;
  int col0;      // destination column of this rank's first head (first section)
  int col0_k;    // same for a second section (kernels writing q and k)
};

// Rank and local row of global token i.
__device__ __forceinline__ void ulysses_home(const UlyssesRoute& u, int i, int& owner, int& row) {
  const int c = i / u.chunk;
  owner = c < u.world ? c : 2 * u.world - 1 - c;
  row = (c < u.world ? 0 : u.chunk) + (i - c * u.chunk);
}

// Global token of local row m on `rank`.
__device__ __forceinline__ int ulysses_global_row(int world, int rank, int chunk, int m) {
  return m < chunk ? rank * chunk + m : (2 * world - 1 - rank) * chunk + (m - chunk);
}

// Named barrier among a subset of warps (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace mvp
