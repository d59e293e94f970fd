// Varlen (packed-document) flash attention for sm_100a on tcgen05.
//
// Layout: tokens of all documents are packed into one stream of T rows;
// cu_seqlens[d] .. cu_seqlens[d+1] delimit document d.  Row i attends to keys
// j with start(i) <= j <= i (causal) or start(i) <= j < end(i) (bidirectional,
// used by the vision tower).  No mask tensor is ever built.
//
// Separate key documents: with cu_seqlens_k, query rows cu_q[d] .. cu_q[d+1]
// attend keys cu_k[d] .. cu_k[d+1] of a key stream of Tk rows (document d may
// be empty on either side).  Causal masking is then aligned to the end of the
// document (query row t of Lq sees key u of Lk iff u <= t + Lk - Lq), which is
// plain causal masking when cu_k == cu_q.  Ring context parallelism uses this
// to attend a local query chunk to another rank's key chunk.
//
// q: [T, Hq, 128], k: [T, Hkv, 128], v: [T, Hkv, 128] (any row strides that
// are multiples of 8 elements), o: [T, Hq, 128] bf16, lse: [Hq, T] fp32
// (natural-log LSE of the scaled logits, for the backward pass).
//
// Forward CTA = one 128-row query block of one head (grid = q blocks x Hq):
//   warps 0-7  softmax, two warpgroups: thread (warp % 4, lane) owns query row
//              r = TMEM lane, warpgroup h its keys 64h .. 64h+63 of each
//              block, with its own running max, sum and O accumulator (the two
//              partial softmaxes are merged once, in the epilogue, so the
//              halves never wait for each other per block).  Each reads its
//              half of S from TMEM, applies the document mask (skipped for
//              blocks entirely inside the row's window), rescales its O only
//              when its max grows by more than 2^8 (lazy rescale), and writes
//              P (bf16 pairs) back into the first 32 columns of its half of S,
//              where the PV MMA reads it as a tensor-memory A operand.
//   warp 8     TMA producer: Q once, then K/V blocks into a 3-deep ring.
//   warp 9     MMA issuer: S_{j+1} = Q K_{j+1}^T is issued before waiting for
//              P_j so the tensor core overlaps the softmax; then, per half,
//              O_h += P_j,h V_j,h as soon as that half's P is in place.
// TMEM: S double buffer (2 x 128 columns, P aliased) + two O accumulators
// (2 x 128 columns).
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "peer_host.h"
#include "tma_host.h"

namespace mvp {
namespace attn {

constexpr int D = 128;
constexpr int BLK = 128;               // query rows and keys per block
constexpr int TILE_BYTES = BLK * D * 2;  // 32 KB: [128 rows][128 d] as two 64-wide swizzled chunks
constexpr int CHUNK_BYTES = BLK * 64 * 2;  // 16 KB
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FwdParams {
  __nv_bfloat16* o;
  int64_t o_row_stride;
  float* lse;
  const int* cu_seqlens;    // query-side documents
  const int* cu_seqlens_k;  // key-side documents (== cu_seqlens for self-attention)
  int n_docs;
  int T, Tk, Hq, Hkv;
  float scale_log2;
  int causal;
  int* status;
  PeerPull pull;  // optional copy of the next ring hop's K/V, carried by grid rows 0 .. pull.rows-1
  UlyssesRoute route;  // optional: O rows also written to the token's rank (o_proj input layout)
};

// Largest d with cu[d] <= i (cu has n_docs + 1 entries): the non-empty document holding row i.
__device__ __forceinline__ int doc_index(const int* cu, int n_docs, int i) {
  int lo = 0, hi = n_docs;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(cu + mid) <= i) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Key range [lo, hi] (inclusive) visible to query row i.
__device__ __forceinline__ void key_range(const int* cu_q, const int* cu_k, int n_docs, int causal, int i, int& lo,
                                          int& hi) {
  const int d = doc_index(cu_q, n_docs, i);
  const int ks = __ldg(cu_k + d), ke = __ldg(cu_k + d + 1);
  lo = ks;
  hi = ke - 1;
  if (causal) {
    const int qs = __ldg(cu_q + d), qe = __ldg(cu_q + d + 1);
    hi = min(hi, ks + (i - qs) + (ke - ks) - (qe - qs));
  }
}

// Query range [lo, hi) that sees key row k.
__device__ __forceinline__ void query_range(const int* cu_q, const int* cu_k, int n_docs, int causal, int k, int& lo,
                                            int& hi) {
  const int d = doc_index(cu_k, n_docs, k);
  const int qs = __ldg(cu_q + d), qe = __ldg(cu_q + d + 1);
  lo = qs;
  hi = qe;
  if (causal) {
    const int ks = __ldg(cu_k + d), ke = __ldg(cu_k + d + 1);
    lo = qs + max(0, (k - ks) - ((ke - ks) - (qe - qs)));
  }
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// K-major operand descriptor for a [128 rows][128 k] tile stored as two 64-wide
// 128-byte-swizzled chunks; k-step s covers k = 16s .. 16s+15.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int s) {
  return make_smem_desc_sw128(base + (s >> 2) * CHUNK_BYTES + (s & 3) * 32, 16, 1024);
}
// MN-major operand descriptor for V ([keys][128 d], d contiguous) used as B with
// N = d and K = keys; k-step s covers keys 16s .. 16s+15.
__device__ __forceinline__ uint64_t vmajor_desc(uint32_t base, int s) {
  return make_smem_desc_sw128(base + s * 2048, CHUNK_BYTES, 1024);
}

constexpr int kFwdThreads = 320;  // 8 softmax warps + TMA warp + MMA warp
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kKvStages = 3;  // K/V ring depth

// 2^x with the MUFU.EX2 instruction (PTX ex2.approx.ftz.f32: relative error ~2^-22, 2^-inf = 0); the
// result is rounded to bf16 right after, so the approximation is far below the storage precision.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// D[tmem] (+)= A[tmem] * B[smem]: tcgen05.mma with the A operand (P) read from tensor memory.
__device__ __forceinline__ void mma_p_tmem(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  mma_bf16_ts(d_tmem, a_tmem, b_desc, idesc, accumulate);
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + TILE_BYTES;                 // [kKvStages]
  uint8_t* sV = sK + kKvStages * TILE_BYTES;     // [kKvStages]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kKvStages * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                   // [kKvStages]
  uint64_t* v_full = k_full + kKvStages;         // [kKvStages]
  uint64_t* kv_empty = v_full + kKvStages;       // [kKvStages]
  uint64_t* s_full = kv_empty + kKvStages;       // [2]
  uint64_t* p_full = s_full + 2;                 // [2 halves] (128 arrivals each)
  uint64_t* o_ready = p_full + 2;                // [2 halves]
  uint64_t* done_bar = o_ready + 2;
  uint64_t* lsum_bar = done_bar + 1;             // the halves exchanged (max, sum) once (256 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lsum_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [2 halves][2 (max, sum)][128 rows], exchanged in the epilogue once every MMA (and so every K/V load
  // it waited for) has retired: it reuses the first K stage.
  float* xml = reinterpret_cast<float*>(sK);

  if (static_cast<int>(blockIdx.y) < p.pull.rows) {  // copy CTA: pull the next hop's K/V, no attention
    peer_pull_cta(p.pull, p.status, reinterpret_cast<int*>(smem));
    return;
  }
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int qb = blockIdx.x;
  const int h = blockIdx.y - p.pull.rows;
  const int hk = h / (p.Hq / p.Hkv);
  const int q0 = qb * BLK;

  // KV range of this query block.
  const int q_last = min(q0 + BLK, p.T) - 1;
  int kv_lo, first_hi, last_lo, last_hi;
  key_range(p.cu_seqlens, p.cu_seqlens_k, p.n_docs, p.causal, q0, kv_lo, first_hi);
  key_range(p.cu_seqlens, p.cu_seqlens_k, p.n_docs, p.causal, q_last, last_lo, last_hi);
  const int kv_hi = last_hi + 1;
  // debug builds: document boundaries (cu_seqlens) that point outside the key stream skip the block
  const bool kv_in_bounds = MVP_BOUNDS_OK(p.status, kv_hi <= kv_lo || (kv_lo >= 0 && kv_hi <= p.Tk));
  const int n_blocks = (kv_hi > kv_lo && kv_in_bounds) ? (kv_hi - kv_lo + BLK - 1) / BLK : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int b = 0; b < kKvStages; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&v_full[b], 1);
      mbar_init(&kv_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&o_ready[b], 1);
    }
    mbar_init(done_bar, 1);
    mbar_init(lsum_bar, 256);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;         // [2] x 128 columns; P_j (bf16 pairs) overwrites S_j's first 32 columns per half
  const uint32_t tO = tmem + 256;   // [2 halves] x 128 columns

  if (warp == kTmaWarp) {
    // --------------------------------------------------------------- TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, h * D, q0);
      tma_load_2d(sQ + CHUNK_BYTES, &tmQ, q_full, h * D + 64, q0);
      uint32_t issued = 0;  // bit b: a load into slot b has been issued
      uint32_t issued_phase = 0;
      bool ok = true;
      for (int j = 0; j < n_blocks; ++j) {
        const int b = j % kKvStages;
        const uint32_t ph = (j / kKvStages) & 1;
        if (!mbar_wait_bounded(&kv_empty[b], ph ^ 1, abort_flag, p.status, kTimeoutProducer)) {
          ok = false;
          break;
        }
        const int k0 = kv_lo + j * BLK;
        mbar_arrive_expect_tx(&k_full[b], TILE_BYTES);
        tma_load_2d(sK + b * TILE_BYTES, &tmK, &k_full[b], hk * D, k0);
        tma_load_2d(sK + b * TILE_BYTES + CHUNK_BYTES, &tmK, &k_full[b], hk * D + 64, k0);
        mbar_arrive_expect_tx(&v_full[b], TILE_BYTES);
        tma_load_2d(sV + b * TILE_BYTES, &tmV, &v_full[b], hk * D, k0);
        tma_load_2d(sV + b * TILE_BYTES + CHUNK_BYTES, &tmV, &v_full[b], hk * D + 64, k0);
        issued |= 1u << b;
        issued_phase = (issued_phase & ~(1u << b)) | (ph << b);
      }
      if (!ok || *abort_flag) {
        // Let in-flight copies land before the CTA can exit.
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(q_full, 0) && globaltimer() - t0 < 200000000ull) {
        }
        for (int b = 0; b < kKvStages; ++b) {
          if (!((issued >> b) & 1u)) continue;
          const uint32_t par = (issued_phase >> b) & 1u;
          const uint64_t t1 = globaltimer();
          while ((!mbar_try_wait(&k_full[b], par) || !mbar_try_wait(&v_full[b], par)) &&
                 globaltimer() - t1 < 200000000ull) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // --------------------------------------------------------------- MMA
    // tcgen05.mma operations of this thread execute in issue order, so S_{j+2} (written into the
    // columns that hold P_j) is issued only after PV_j, which reads P_j.
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BLK, BLK, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BLK, D, false, true);
      const uint32_t q_base = smem_u32(sQ);
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, p.status, kTimeoutMma);
      auto issue_s = [&](int j) -> bool {
        const int st = j % kKvStages;
        const uint32_t ph = (j / kKvStages) & 1;
        if (!mbar_wait_bounded(&k_full[st], ph, abort_flag, p.status, kTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + st * TILE_BYTES);
#pragma unroll
        for (int s = 0; s < D / 16; ++s)
          mma_bf16_ss(tS + (j & 1) * BLK, kmajor_desc(q_base, s), kmajor_desc(k_base, s), idesc_s, s > 0 ? 1u : 0u);
        mma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok && n_blocks > 0) ok = issue_s(0);
      for (int j = 0; j < n_blocks && ok; ++j) {
        if (j + 1 < n_blocks && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        const int st = j % kKvStages;
        const uint32_t ph = (j / kKvStages) & 1;
        if (!mbar_wait_bounded(&v_full[st], ph, abort_flag, p.status, kTimeoutMma)) {
          ok = false;
          break;
        }
        const uint32_t v_base = smem_u32(sV + st * TILE_BYTES);
        for (int hf = 0; hf < 2 && ok; ++hf) {
          // O_hf += P_j[:, keys 64hf..64hf+63] V_j[keys 64hf.., :], P from tensor memory
          if (!mbar_wait_bounded(&p_full[hf], j & 1, abort_flag, p.status, kTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int s = 0; s < 4; ++s)
            mma_p_tmem(tO + hf * D, tS + (j & 1) * BLK + hf * 64 + s * 8, vmajor_desc(v_base, 4 * hf + s), idesc_o,
                       (j > 0 || s > 0) ? 1u : 0u);
          mma_commit(&o_ready[hf]);
        }
        if (!ok) break;
        mma_commit(&kv_empty[st]);
      }
      // Retire everything issued before TMEM is released (the epilogue waits on the same barrier).
      mma_commit(done_bar);
      mbar_wait_bounded(done_bar, 0, abort_flag, p.status, kTimeoutDrain);
    }
  } else {
    // ----------------------------------------------------------- softmax
    // Warpgroup `half` owns keys 64*half .. +63 of every block with its own running max, sum and
    // O accumulator, so the halves never wait for each other until the final merge.
    const int r = (warp & 3) * 32 + lane;  // query row = TMEM lane
    const int half = warp >> 2;
    const int i = q0 + r;
    const bool valid = i < p.T;
    int start_i = 0, hi_i = -1;  // allowed keys start_i .. hi_i
    if (valid) key_range(p.cu_seqlens, p.cu_seqlens_k, p.n_docs, p.causal, i, start_i, hi_i);
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tOh = tO + half * D + lane_addr;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_blocks; ++j) {
      const int b = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s_full[b], ph, abort_flag, p.status, kTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tSh = tS + b * BLK + lane_addr + half * 64;
      float s[64];  // raw logits; scaled inside the exponent
      {
        uint32_t rr[64];
        tmem_ld_32x32b_x32(tSh, *reinterpret_cast<uint32_t(*)[32]>(rr));
        tmem_ld_32x32b_x32(tSh + 32, *reinterpret_cast<uint32_t(*)[32]>(rr + 32));
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 64; ++t) s[t] = __uint_as_float(rr[t]);
      }
      const int k0 = kv_lo + j * BLK + half * 64;
      if (!(valid && k0 >= start_i && k0 + 63 <= hi_i)) {  // some keys of this half-block are masked
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int key = k0 + c;
          s[c] = (valid && key >= start_i && key <= hi_i) ? s[c] : -INFINITY;
        }
      }
      // row max as an 8-way tree (a 64-long dependent chain would serialise the warp)
      float mx8[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mx8[t] = fmaxf(s[t], s[t + 8]);
#pragma unroll
      for (int c = 16; c < 64; c += 8) {
#pragma unroll
        for (int t = 0; t < 8; ++t) mx8[t] = fmaxf(mx8[t], s[c + t]);
      }
      const float mb = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * p.scale_log2;
      const float m_new = fmaxf(m, mb);
      float m_use = m, alpha = 1.f;
      if (m_new > m + kRescaleThreshold || (m == -INFINITY && m_new != -INFINITY)) {
        m_use = m_new;
        alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
      }
      // PV_{j-1} of this half must have retired before O is rescaled, and before P_j is published
      // (so p_full never runs two phases ahead of the MMA warp).  s_full_j implies PV_{j-2} has
      // retired, so o_ready is at most one phase behind and its parity is unambiguous.
      bool waited = false;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(&o_ready[half], (j - 1) & 1, abort_flag, p.status, kTimeoutEpilogue));
        if (!ok) break;
        waited = true;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t rr[16];
          tmem_ld_32x32b_x16(tOh + c * 16, rr);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) rr[t] = __float_as_uint(__uint_as_float(rr[t]) * alpha);
          tmem_st_32x32b_x16(tOh + c * 16, rr);
        }
        tmem_wait_st();
      }
      m = m_use;
      // P = 2^(s * scale_log2 - m) as bf16 pairs over S_j's first 32 columns of this half (A operand
      // of PV_j); masked keys (s = -inf) give 0.  A dead row (m = -inf) writes zeros.
      const float neg_m = (m != -INFINITY) ? -m : -INFINITY;
      float rs8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float e0 = ex2_approx(fmaf(s[c * 32 + 2 * t], p.scale_log2, neg_m));
          const float e1 = ex2_approx(fmaf(s[c * 32 + 2 * t + 1], p.scale_log2, neg_m));
          rs8[(2 * t) & 7] += e0;
          rs8[(2 * t + 1) & 7] += e1;
          pk[t] = pack_bf16x2(e0, e1);
        }
        tmem_st_32x32b_x16(tSh + c * 16, pk);
      }
      const float rowsum = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      tmem_wait_st();
      if (j > 0 && !waited) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait_bounded(&o_ready[half], (j - 1) & 1, abort_flag, p.status, kTimeoutEpilogue));
        if (!ok) break;
      }
      l = l * alpha + rowsum;
      tc_fence_before();
      mbar_arrive(&p_full[half]);
    }
    // ------------------------------------------------------------ epilogue
    // Every MMA has retired once done_bar completes; merge the two halves' (max, sum, O).
    if (ok && n_blocks > 0)
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(done_bar, 0, abort_flag, p.status, kTimeoutEpilogue));
    xml[(half * 2 + 0) * 128 + r] = m;
    xml[(half * 2 + 1) * 128 + r] = l;
    mbar_arrive(lsum_bar);
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(lsum_bar, 0, abort_flag, p.status, kTimeoutEpilogue));
    if (ok) {
      tc_fence_after();
      const float m0 = xml[0 * 128 + r], l0 = xml[1 * 128 + r];
      const float m1 = xml[2 * 128 + r], l1 = xml[3 * 128 + r];
      const float mx = fmaxf(m0, m1);
      const float f0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - mx);
      const float f1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - mx);
      const float lt = l0 * f0 + l1 * f1;
      const float inv = (lt > 0.f) ? 1.f / lt : 0.f;
      const float w0 = f0 * inv, w1 = f1 * inv;
      __nv_bfloat16* orow = p.o + static_cast<int64_t>(i) * p.o_row_stride + h * D + half * 64;
      __nv_bfloat16* urow = nullptr;  // the same row in the token rank's o_proj input (Ulysses)
      if (p.route.dst[0] != nullptr && valid) {
        int owner, lrow;
        ulysses_home(p.route, i, owner, lrow);
        urow = reinterpret_cast<__nv_bfloat16*>(p.route.dst[owner]) + static_cast<int64_t>(lrow) * p.route.ld +
               p.route.col0 + h * D + half * 64;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t a0[32], a1[32];
        if (n_blocks > 0) {
          tmem_ld_32x32b_x32(tO + lane_addr + half * 64 + c * 32, a0);
          tmem_ld_32x32b_x32(tO + D + lane_addr + half * 64 + c * 32, a1);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) a0[t] = a1[t] = 0u;
        }
        if (valid) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            float o8[8];
#pragma unroll
            for (int t = 0; t < 8; ++t)
              o8[t] = __uint_as_float(a0[8 * v + t]) * w0 + __uint_as_float(a1[8 * v + t]) * w1;
            uint4 pk;
            pk.x = pack_bf16x2(o8[0], o8[1]);
            pk.y = pack_bf16x2(o8[2], o8[3]);
            pk.z = pack_bf16x2(o8[4], o8[5]);
            pk.w = pack_bf16x2(o8[6], o8[7]);
            *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = pk;
            if (urow != nullptr) *reinterpret_cast<uint4*>(urow + c * 32 + v * 8) = pk;
          }
        }
      }
      if (urow != nullptr) __threadfence_system();
      if (valid && half == 0)
        p.lse[static_cast<int64_t>(h) * p.T + i] = (lt > 0.f) ? (mx + log2f(lt)) / kLog2e : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// tiles, align, barriers (9 + 3 * stages), TMEM slot / abort flag
constexpr int kFwdSmem = (1 + 2 * kKvStages) * TILE_BYTES + 1024 + (9 + 3 * kKvStages) * 8 + 16;
static_assert(kFwdSmem <= 232448, "forward kernel exceeds 227 KB of shared memory");

}  // namespace attn
}  // namespace mvp

// q [T, Hq, 128], k/v [Tk, Hkv, 128] (row strides multiple of 8, unit head/dim
// strides), cu_seqlens int32 [n+1] on device (and cu_seqlens_k [n+1] when the key
// stream has its own documents; Tk == T otherwise).  Returns (o [T, Hq, 128], lse [Hq, T]).
std::vector<torch::Tensor> flash_attn_fwd(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                                          const torch::Tensor& cu_seqlens, double softmax_scale, bool causal,
                                          int64_t status_ptr, const c10::optional<torch::Tensor>& cu_seqlens_k,
                                          const c10::optional<std::vector<int64_t>>& pull,
                                          const c10::optional<std::vector<int64_t>>& route) {
  using namespace mvp::attn;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "flash_attn_fwd: bf16 inputs");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3 && q.size(2) == D && k.size(2) == D && v.size(2) == D,
              "flash_attn_fwd: [T, H, 128] inputs");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1 && v.stride(2) == 1 && q.stride(1) == D && k.stride(1) == D &&
                  v.stride(1) == D,
              "flash_attn_fwd: heads must be contiguous within a token");
  TORCH_CHECK(cu_seqlens.scalar_type() == at::kInt && cu_seqlens.is_cuda(), "flash_attn_fwd: int32 cu_seqlens");
  const int T = static_cast<int>(q.size(0));
  const int Tk = static_cast<int>(k.size(0));
  const int Hq = static_cast<int>(q.size(1));
  const int Hkv = static_cast<int>(k.size(1));
  TORCH_CHECK(Hq % Hkv == 0, "flash_attn_fwd: Hq must be a multiple of Hkv");
  TORCH_CHECK(v.size(0) == Tk && v.size(1) == Hkv, "flash_attn_fwd: k/v shapes differ");
  const torch::Tensor& cu_k = cu_seqlens_k.has_value() ? *cu_seqlens_k : cu_seqlens;
  TORCH_CHECK(cu_k.scalar_type() == at::kInt && cu_k.is_cuda() && cu_k.numel() == cu_seqlens.numel(),
              "flash_attn_fwd: cu_seqlens_k must be int32 with as many documents as cu_seqlens");
  TORCH_CHECK(cu_seqlens_k.has_value() || Tk == T, "flash_attn_fwd: Tk != T needs cu_seqlens_k");
  const at::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty({T, Hq, D}, q.options());
  auto lse = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  const mvp::PeerPull pj = mvp::make_peer_pull(pull);
  if (T == 0 || Tk == 0) {  // nothing to attend: zero output, -inf LSE (the copy still runs)
    o.zero_();
    lse.fill_(-INFINITY);
    mvp::launch_peer_pull(pj, reinterpret_cast<int*>(status_ptr), at::cuda::getCurrentCUDAStream());
    return {o, lse};
  }
  CUtensorMap tq, tk, tv;
  mvp::make_tmap_2d_bf16(&tq, q.data_ptr(), static_cast<int64_t>(Hq) * D, T, q.stride(0), 64, BLK);
  mvp::make_tmap_2d_bf16(&tk, k.data_ptr(), static_cast<int64_t>(Hkv) * D, Tk, k.stride(0), 64, BLK);
  mvp::make_tmap_2d_bf16(&tv, v.data_ptr(), static_cast<int64_t>(Hkv) * D, Tk, v.stride(0), 64, BLK);
  FwdParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.o_row_stride = o.stride(0);
  p.lse = lse.data_ptr<float>();
  p.cu_seqlens = cu_seqlens.data_ptr<int>();
  p.cu_seqlens_k = cu_k.data_ptr<int>();
  p.n_docs = static_cast<int>(cu_seqlens.numel() - 1);
  p.T = T;
  p.Tk = Tk;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = static_cast<float>(softmax_scale) * kLog2e;
  p.causal = causal ? 1 : 0;
  p.status = reinterpret_cast<int*>(status_ptr);
  p.pull = pj;
  p.route = mvp::make_ulysses_route(route);
  TORCH_CHECK(p.route.dst[0] == nullptr || T == 2 * p.route.world * p.route.chunk,
              "flash_attn_fwd: routed rows need T = 2 x world x chunk");
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
    configured = true;
  }
  dim3 grid((T + BLK - 1) / BLK, Hq + pj.rows);
  fwd_kernel<<<grid, kFwdThreads, kFwdSmem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {o, lse};
}

// ============================================================== backward
//
// CTA = one 128-key block of one KV head (grid = kv blocks x Hkv).  It loops
// over the Hq/Hkv query heads of its group and over every 128-row query block
// that can see its keys, keeping dK and dV in TMEM for the whole loop:
//   S^T  = K Q^T          (TMEM, lane = key)       dP^T = V dO^T (TMEM)
//   P^T  = exp(S^T*scale - lse),  dS^T = P^T * (dP^T - delta) * scale
//   dV  += P^T dO,  dK += dS^T Q   (TMEM accumulators)
//   dQ   = dS K  -> TMEM (lane = query row) -> fp32 vector atomics into dq_acc
// P^T is written back into S^T's TMEM columns (bf16 pairs) and read from there
// as the A operand of dV; dS^T goes once into a 128-byte-swizzled smem tile
// that serves both as the K-major A operand of dK and, read MN-major, as the A
// operand of dQ.  Q/dO tiles (a 2-deep ring, so the next query block loads
// while this one computes) serve as K-major B (S^T, dP^T) and as MN-major B
// (dK, dV).  TMEM: S^T | dP^T | dV | dK (4 x 128 columns); dQ goes into dP^T's
// columns and is issued before dV / dK so its read-out overlaps them.
namespace mvp {
namespace attn {

struct BwdParams {
  float* dq_acc;  // [T, Hq, 128] fp32, zero-initialised
  __nv_bfloat16* dk;
  int64_t dk_row_stride;
  __nv_bfloat16* dv;
  int64_t dv_row_stride;
  const float* lse;    // [Hq, T]
  const float* delta;  // [Hq, T]
  const int* cu_seqlens;
  const int* cu_seqlens_k;
  int n_docs;
  int T, Tk, Hq, Hkv;
  float scale, scale_log2;
  int causal;
  int* status;
  PeerPull pull;       // optional copy of the next ring hop's K/V, carried by grid rows 0 .. pull.rows-1
  float* dk_f32;       // optional fp32 dK / dV destination (may be another rank's memory): written, or
  float* dv_f32;       // added to when f32_accumulate, instead of the bf16 dk / dv
  int64_t f32_row_stride;
  int f32_accumulate;
  UlyssesRoute route;  // optional: dV rows written to the token's rank (dqkv layout) instead of dv
};

// Fire-and-forget fp32 x4 reduction into global memory (no return value, so no scoreboard wait).
__device__ __forceinline__ void red_add_v4(float* addr, const uint32_t* v) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(__uint_as_float(v[0])),
               "f"(__uint_as_float(v[1])), "f"(__uint_as_float(v[2])), "f"(__uint_as_float(v[3]))
               : "memory");
}

constexpr int kBwdThreads = 320;  // 8 gradient warps + TMA warp + MMA warp
constexpr int kQdStages = 2;       // Q / dO ring depth

__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO, BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE_BYTES;
  uint8_t* sQ = sV + TILE_BYTES;                  // [kQdStages]
  uint8_t* sdO = sQ + kQdStages * TILE_BYTES;     // [kQdStages]
  uint8_t* sdSt = sdO + kQdStages * TILE_BYTES;
  float* s_lse = reinterpret_cast<float*>(sdSt + TILE_BYTES);  // [128] LSE (log2 units) of this query block
  float* s_delta = s_lse + BLK;                                 // [128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_delta + BLK);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;                   // [kQdStages]
  uint64_t* qd_empty = bars + 1 + kQdStages;      // [kQdStages] dV / dK of the stage's iteration retired
  uint64_t* s_full = bars + 1 + 2 * kQdStages;    // S^T, dP^T in TMEM
  uint64_t* p_full = s_full + 1;                  // P^T in TMEM, dS^T in smem (256 arrivals)
  uint64_t* dq_full = s_full + 2;                 // dQ in TMEM
  uint64_t* dq_read = s_full + 3;                 // dQ read out of TMEM (256 arrivals)
  uint64_t* done_bar = s_full + 4;
  uint64_t* stg_full = s_full + 5;                // LSE / delta of this query block staged (256 arrivals)
  uint64_t* stg_free = s_full + 6;                // ... and no longer read (256 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  if (static_cast<int>(blockIdx.y) < p.pull.rows) {  // copy CTA: pull the next hop's K/V, no gradients
    peer_pull_cta(p.pull, p.status, reinterpret_cast<int*>(smem));
    return;
  }
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int hk = blockIdx.y - p.pull.rows;
  const int rep = p.Hq / p.Hkv;
  const int k0 = blockIdx.x * BLK;
  const int k_last = min(k0 + BLK, p.Tk) - 1;
  int q_lo, q_hi0, ql_lo, q_hi;
  query_range(p.cu_seqlens, p.cu_seqlens_k, p.n_docs, p.causal, k0, q_lo, q_hi0);
  query_range(p.cu_seqlens, p.cu_seqlens_k, p.n_docs, p.causal, k_last, ql_lo, q_hi);
  const bool q_in_bounds = MVP_BOUNDS_OK(p.status, q_hi <= q_lo || (q_lo >= 0 && q_hi <= p.T));
  const int nq = (q_hi > q_lo && q_in_bounds) ? (q_hi - q_lo + BLK - 1) / BLK : 0;
  const int n_iter = nq * rep;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int st = 0; st < kQdStages; ++st) {
      mbar_init(&qd_full[st], 1);
      mbar_init(&qd_empty[st], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_read, 256);
    mbar_init(done_bar, 1);
    mbar_init(stg_full, 256);
    mbar_init(stg_free, 256);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S^T (then P^T as bf16 pairs) | dP^T (then dQ) | dV | dK
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_2d(sK, &tmK, kv_full, hk * D, k0);
      tma_load_2d(sK + CHUNK_BYTES, &tmK, kv_full, hk * D + 64, k0);
      tma_load_2d(sV, &tmV, kv_full, hk * D, k0);
      tma_load_2d(sV + CHUNK_BYTES, &tmV, kv_full, hk * D + 64, k0);
      int issued = 0;
      for (int n = 0; n < n_iter; ++n) {
        const int st = n % kQdStages;
        const uint32_t ph = (n / kQdStages) & 1;
        if (!mbar_wait_bounded(&qd_empty[st], ph ^ 1, abort_flag, p.status, kTimeoutProducer)) break;
        const int h = hk * rep + n / nq;
        const int q0 = q_lo + (n % nq) * BLK;
        mbar_arrive_expect_tx(&qd_full[st], 2 * TILE_BYTES);
        tma_load_2d(sQ + st * TILE_BYTES, &tmQ, &qd_full[st], h * D, q0);
        tma_load_2d(sQ + st * TILE_BYTES + CHUNK_BYTES, &tmQ, &qd_full[st], h * D + 64, q0);
        tma_load_2d(sdO + st * TILE_BYTES, &tmdO, &qd_full[st], h * D, q0);
        tma_load_2d(sdO + st * TILE_BYTES + CHUNK_BYTES, &tmdO, &qd_full[st], h * D + 64, q0);
        issued = n + 1;
      }
      if (*abort_flag) {  // let copies already issued land (bounded) before the CTA can exit
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(kv_full, 0) && globaltimer() - t0 < 200000000ull) {
        }
        for (int n = max(0, issued - kQdStages); n < issued; ++n) {
          const uint64_t t1 = globaltimer();
          while (!mbar_try_wait(&qd_full[n % kQdStages], (n / kQdStages) & 1) && globaltimer() - t1 < 200000000ull) {
          }
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA
    // tcgen05.mma operations of this thread execute in issue order: S^T(n+1) overwrites P^T(n) only
    // after dV(n) (issued before it) has read it.
    if (elect_one_sync()) {
      constexpr uint32_t id_kk = make_idesc_bf16(BLK, BLK, false, false);
      constexpr uint32_t id_km = make_idesc_bf16(BLK, D, false, true);
      constexpr uint32_t id_mm = make_idesc_bf16(BLK, D, true, true);
      const uint32_t bK = smem_u32(sK), bV = smem_u32(sV), bdSt = smem_u32(sdSt);
      bool ok = mbar_wait_bounded(kv_full, 0, abort_flag, p.status, kTimeoutMma);
      for (int n = 0; n < n_iter && ok; ++n) {
        const int st = n % kQdStages;
        ok = mbar_wait_bounded(&qd_full[st], (n / kQdStages) & 1, abort_flag, p.status, kTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t bQ = smem_u32(sQ + st * TILE_BYTES), bdO = smem_u32(sdO + st * TILE_BYTES);
#pragma unroll
        for (int s = 0; s < D / 16; ++s) mma_bf16_ss(tS, kmajor_desc(bK, s), kmajor_desc(bQ, s), id_kk, s > 0);
        // dP^T goes where dQ(n-1) was: wait until it has been read out
        if (n > 0) {
          ok = mbar_wait_bounded(dq_read, (n - 1) & 1, abort_flag, p.status, kTimeoutMma);
          if (!ok) break;
          tc_fence_after();
        }
#pragma unroll
        for (int s = 0; s < D / 16; ++s) mma_bf16_ss(tdP, kmajor_desc(bV, s), kmajor_desc(bdO, s), id_kk, s > 0);
        mma_commit(s_full);
        ok = mbar_wait_bounded(p_full, n & 1, abort_flag, p.status, kTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        // dQ = dS K first (the gradient warps wait for it), into dP^T's columns
#pragma unroll
        for (int s = 0; s < BLK / 16; ++s) mma_bf16_ss(tdP, vmajor_desc(bdSt, s), vmajor_desc(bK, s), id_mm, s > 0);
        mma_commit(dq_full);
        // dV += P^T dO with P^T from tensor memory (query columns 64h.. of half h at S^T column 64h)
#pragma unroll
        for (int s = 0; s < BLK / 16; ++s)
          mma_bf16_ts(tdV, tS + (s >> 2) * 64 + (s & 3) * 8, vmajor_desc(bdO, s), id_km, (n > 0 || s > 0) ? 1u : 0u);
#pragma unroll
        for (int s = 0; s < BLK / 16; ++s)
          mma_bf16_ss(tdK, kmajor_desc(bdSt, s), vmajor_desc(bQ, s), id_km, (n > 0 || s > 0) ? 1u : 0u);
        mma_commit(&qd_empty[st]);
      }
      mma_commit(done_bar);
      mbar_wait_bounded(done_bar, 0, abort_flag, p.status, kTimeoutDrain);
    }
  } else {
    // warps 0-7, two warpgroups: thread (warp % 4, lane) owns key row c (S^T / dP^T / dK / dV lane) and
    // query row c of the dQ tile; warpgroup `half` takes query columns 64*half .. +63 of S^T / dP^T
    // and d columns 64*half .. +63 of dQ / dK / dV.
    const int c = (warp & 3) * 32 + lane;
    const int half = warp >> 2;
    const int kc = k0 + c;
    const bool kvalid = kc < p.Tk;
    int lo_c = 0, ke = 0;  // query rows lo_c .. ke-1 see key kc
    if (kvalid) query_range(p.cu_seqlens, p.cu_seqlens_k, p.n_docs, p.causal, kc, lo_c, ke);
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    // LSE (warpgroup 0) or delta (warpgroup 1) of query row c of block n: loaded one block ahead, so the
    // global-memory latency is not on the per-block critical path
    auto row_stat = [&](int n_) -> float {
      const int h_ = hk * rep + n_ / nq;
      const int qi = min(q_lo + (n_ % nq) * BLK + c, p.T - 1);
      const int64_t at = static_cast<int64_t>(h_) * p.T + qi;
      return half == 0 ? p.lse[at] * kLog2e : p.delta[at];
    };
    float next_stat = n_iter > 0 ? row_stat(0) : 0.f;
    for (int n = 0; n < n_iter; ++n) {
      const int h = hk * rep + n / nq;
      const int q0 = q_lo + (n % nq) * BLK;
      // stage this query block's LSE (log2 units) and delta once the previous block's are no longer read
      if (n > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(stg_free, (n - 1) & 1, abort_flag, p.status, kTimeoutEpilogue));
        if (!ok) break;
      }
      if (half == 0) s_lse[c] = next_stat;
      else s_delta[c] = next_stat;
      if (n + 1 < n_iter) next_stat = row_stat(n + 1);  // in flight while this block is processed
      mbar_arrive(stg_full);
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(stg_full, n & 1, abort_flag, p.status, kTimeoutEpilogue));
      if (!ok) break;
      // s_full(n) also means dK(n-1) and dQ(n-1) have retired, so the dS^T tile is free again.
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(s_full, n & 1, abort_flag, p.status, kTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        const int col0 = half * 64 + ch * 32;
        uint32_t sr[32], dr[32];
        tmem_ld_32x32b_x32(tS + lane_addr + col0, sr);
        tmem_ld_32x32b_x32(tdP + lane_addr + col0, dr);
        tmem_wait_ld();
        float pv[32], ds[32];
        const int qc = q0 + col0;
        if (kvalid && qc >= lo_c && qc + 31 < ke && qc + 31 < p.T) {  // all 32 queries see this key
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int r = col0 + t;
            const float pe = ex2_approx(fmaf(__uint_as_float(sr[t]), p.scale_log2, -s_lse[r]));
            pv[t] = pe;
            ds[t] = pe * (__uint_as_float(dr[t]) - s_delta[r]) * p.scale;
          }
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int r = col0 + t;
            const int qr = q0 + r;
            const bool allowed = kvalid && qr >= lo_c && qr < ke && qr < p.T;
            const float pe = allowed ? ex2_approx(fmaf(__uint_as_float(sr[t]), p.scale_log2, -s_lse[r])) : 0.f;
            pv[t] = pe;
            ds[t] = pe * (__uint_as_float(dr[t]) - s_delta[r]) * p.scale;
          }
        }
        // P^T (bf16 pairs) back into this half's S^T columns (already read): A operand of dV
        {
          uint32_t pk[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) pk[t] = pack_bf16x2(pv[2 * t], pv[2 * t + 1]);
          tmem_st_32x32b_x16(tS + lane_addr + half * 64 + ch * 16, pk);
        }
        // dS^T: 32 q columns = half of one 64-wide swizzled chunk = four 16-byte units.
        uint8_t* drow = sdSt + half * CHUNK_BYTES + c * 128;
        const int u0 = ch * 4;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 b;
          b.x = pack_bf16x2(ds[8 * u + 0], ds[8 * u + 1]);
          b.y = pack_bf16x2(ds[8 * u + 2], ds[8 * u + 3]);
          b.z = pack_bf16x2(ds[8 * u + 4], ds[8 * u + 5]);
          b.w = pack_bf16x2(ds[8 * u + 6], ds[8 * u + 7]);
          *reinterpret_cast<uint4*>(drow + (((u0 + u) ^ (c & 7)) << 4)) = b;
        }
      }
      mbar_arrive(stg_free);
      tmem_wait_st();
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(p_full);
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(dq_full, n & 1, abort_flag, p.status, kTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
      // dQ rows: thread c now owns query row q0 + c, d columns 64*half .. +63.  Both chunks are read
      // out of TMEM first, so the MMA warp can reuse the columns while the reductions are issued.
      const int qi = q0 + c;
      float* dst = p.dq_acc + (static_cast<int64_t>(qi) * p.Hq + h) * D + half * 64;
      uint32_t rq[64];
      tmem_ld_32x32b_x32(tdP + lane_addr + half * 64, *reinterpret_cast<uint32_t(*)[32]>(rq));
      tmem_ld_32x32b_x32(tdP + lane_addr + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(rq + 32));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(dq_read);
      if (qi < p.T) {
#pragma unroll
        for (int v = 0; v < 16; ++v) red_add_v4(dst + 4 * v, rq + 4 * v);
      }
    }
    // dK / dV are final once every MMA has retired
    if (ok && n_iter > 0)
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(done_bar, 0, abort_flag, p.status, kTimeoutEpilogue));
    if (ok) {  // keys no query sees (n_iter == 0) get zero gradients
      tc_fence_after();
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t tacc = which == 0 ? tdK : tdV;
        __nv_bfloat16* out = which == 0 ? p.dk + static_cast<int64_t>(kc) * p.dk_row_stride + hk * D + half * 64
                                        : p.dv + static_cast<int64_t>(kc) * p.dv_row_stride + hk * D + half * 64;
        if (which == 1 && p.route.dst[0] != nullptr && kvalid) {
          int owner, lrow;
          ulysses_home(p.route, kc, owner, lrow);
          out = reinterpret_cast<__nv_bfloat16*>(p.route.dst[owner]) + static_cast<int64_t>(lrow) * p.route.ld +
                p.route.col0 + hk * D + half * 64;
        }
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint32_t rr[32];
          if (n_iter > 0) {
            tmem_ld_32x32b_x32(tacc + lane_addr + half * 64 + ch * 32, rr);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int t = 0; t < 32; ++t) rr[t] = 0u;
          }
          if (kvalid && p.dk_f32 != nullptr) {  // fp32 partial sums, possibly into the owner's memory
            float* dst = (which == 0 ? p.dk_f32 : p.dv_f32) + static_cast<int64_t>(kc) * p.f32_row_stride + hk * D +
                         half * 64 + ch * 32;
            float4 acc[8];
#pragma unroll
            for (int v = 0; v < 8; ++v)
              acc[v] = make_float4(__uint_as_float(rr[4 * v]), __uint_as_float(rr[4 * v + 1]),
                                   __uint_as_float(rr[4 * v + 2]), __uint_as_float(rr[4 * v + 3]));
            if (p.f32_accumulate) {
              float4 old[8];
#pragma unroll
              for (int v = 0; v < 8; ++v) old[v] = reinterpret_cast<const float4*>(dst)[v];
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                acc[v].x += old[v].x;
                acc[v].y += old[v].y;
                acc[v].z += old[v].z;
                acc[v].w += old[v].w;
              }
            }
#pragma unroll
            for (int v = 0; v < 8; ++v) reinterpret_cast<float4*>(dst)[v] = acc[v];
          } else if (kvalid) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 pk;
              pk.x = pack_bf16x2(__uint_as_float(rr[8 * v + 0]), __uint_as_float(rr[8 * v + 1]));
              pk.y = pack_bf16x2(__uint_as_float(rr[8 * v + 2]), __uint_as_float(rr[8 * v + 3]));
              pk.z = pack_bf16x2(__uint_as_float(rr[8 * v + 4]), __uint_as_float(rr[8 * v + 5]));
              pk.w = pack_bf16x2(__uint_as_float(rr[8 * v + 6]), __uint_as_float(rr[8 * v + 7]));
              *reinterpret_cast<uint4*>(out + ch * 32 + v * 8) = pk;
            }
          }
        }
      }
    }
  }

  if (p.route.dst[0] != nullptr) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[h, i] = sum_d dO[i, h, d] * O[i, h, d]; one warp per (i, h).
__global__ void bwd_delta_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                 float* __restrict__ delta, int T, int Hq) {
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (item >= static_cast<int64_t>(T) * Hq) return;
  const int i = static_cast<int>(item / Hq), h = static_cast<int>(item % Hq);
  const int64_t off = item * D + lane * 4;
  const uint2 a = *reinterpret_cast<const uint2*>(dout + off);
  const uint2 b = *reinterpret_cast<const uint2*>(out + off);
  const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
  const float2 a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
  const float2 b0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.x));
  const float2 b1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.y));
  float s = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) delta[static_cast<int64_t>(h) * T + i] = s;
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  for (int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 4; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    uint2 u;
    u.x = pack_bf16x2(v.x, v.y);
    u.y = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(y + i) = u;
  }
}

// tiles (K, V, Q and dO rings, dS^T), LSE / delta, align, barriers + TMEM slot
constexpr int kBwdSmem = (3 + 2 * kQdStages) * TILE_BYTES + 2 * BLK * 4 + 1024 + 256;
static_assert(kBwdSmem <= 232448, "backward kernel exceeds 227 KB of shared memory");

}  // namespace attn
}  // namespace mvp

// Returns (dq [T, Hq, 128], dk, dv); dk/dv are written into the given buffers when
// provided (e.g. the k/v column slices of a fused dqkv gradient).
std::vector<torch::Tensor> flash_attn_bwd(const torch::Tensor& dout, const torch::Tensor& q, const torch::Tensor& k,
                                          const torch::Tensor& v, const torch::Tensor& out, const torch::Tensor& lse,
                                          const torch::Tensor& cu_seqlens, double softmax_scale, bool causal,
                                          int64_t status_ptr, const c10::optional<torch::Tensor>& dk_out,
                                          const c10::optional<torch::Tensor>& dv_out,
                                          const c10::optional<torch::Tensor>& cu_seqlens_k,
                                          const c10::optional<std::vector<int64_t>>& pull,
                                          const c10::optional<torch::Tensor>& dq_accum,
                                          const c10::optional<std::vector<int64_t>>& dkv_f32,
                                          const c10::optional<std::vector<int64_t>>& route) {
  using namespace mvp::attn;
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous() && q.is_contiguous(), "flash_attn_bwd: contiguous q/o/do");
  TORCH_CHECK(k.stride(2) == 1 && v.stride(2) == 1 && k.stride(1) == D && v.stride(1) == D,
              "flash_attn_bwd: k/v head layout");
  const int T = static_cast<int>(q.size(0));
  const int Tk = static_cast<int>(k.size(0));
  const int Hq = static_cast<int>(q.size(1));
  const int Hkv = static_cast<int>(k.size(1));
  const torch::Tensor& cu_k = cu_seqlens_k.has_value() ? *cu_seqlens_k : cu_seqlens;
  TORCH_CHECK(cu_k.scalar_type() == at::kInt && cu_k.is_cuda() && cu_k.numel() == cu_seqlens.numel(),
              "flash_attn_bwd: cu_seqlens_k must be int32 with as many documents as cu_seqlens");
  TORCH_CHECK(cu_seqlens_k.has_value() || Tk == T, "flash_attn_bwd: Tk != T needs cu_seqlens_k");
  const at::cuda::CUDAGuard guard(q.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  // dq_accum: the caller's fp32 [T, Hq, 128] accumulator (dq is added to it and returned as is);
  // dkv_f32 = [dk_ptr, dv_ptr, row_stride, accumulate]: fp32 dK / dV destinations (e.g. another
  // rank's accumulator slot), written or added to, instead of bf16 outputs.
  const bool ext_dq = dq_accum.has_value();
  if (ext_dq)
    TORCH_CHECK(dq_accum->scalar_type() == at::kFloat && dq_accum->is_contiguous() && dq_accum->dim() == 3 &&
                    dq_accum->size(0) == T && dq_accum->size(1) == Hq && dq_accum->size(2) == D,
                "flash_attn_bwd: dq_accum must be contiguous fp32 [T, Hq, 128]");
  const bool f32_kv = dkv_f32.has_value() && !dkv_f32->empty();
  if (f32_kv) {
    TORCH_CHECK(dkv_f32->size() == 4, "dkv_f32 = [dk_ptr, dv_ptr, row_stride, accumulate]");
    TORCH_CHECK((*dkv_f32)[0] % 16 == 0 && (*dkv_f32)[1] % 16 == 0 && (*dkv_f32)[2] % 4 == 0 &&
                    (*dkv_f32)[2] >= static_cast<int64_t>(Hkv) * D,
                "dkv_f32: 16-byte aligned rows of at least Hkv x 128 floats");
  }
  auto dq_acc = ext_dq ? *dq_accum : torch::zeros({T, Hq, D}, q.options().dtype(at::kFloat));
  auto delta = torch::empty({Hq, T}, q.options().dtype(at::kFloat));
  torch::Tensor dk = f32_kv ? torch::empty({0, Hkv, D}, q.options())
                            : (dk_out.has_value() ? *dk_out : torch::empty({Tk, Hkv, D}, q.options()));
  const mvp::UlyssesRoute uroute = mvp::make_ulysses_route(route);
  const bool routed_dv = uroute.dst[0] != nullptr;
  TORCH_CHECK(!routed_dv || (!f32_kv && Tk == 2 * uroute.world * uroute.chunk),
              "flash_attn_bwd: routed dV rows need bf16 outputs and Tk = 2 x world x chunk");
  torch::Tensor dv = (f32_kv || routed_dv)
                         ? torch::empty({0, Hkv, D}, q.options())
                         : (dv_out.has_value() ? *dv_out : torch::empty({Tk, Hkv, D}, q.options()));
  TORCH_CHECK(dk.stride(2) == 1 && dv.stride(2) == 1 && dk.stride(1) == D && dv.stride(1) == D,
              "flash_attn_bwd: dk/dv head layout");
  auto dq = ext_dq ? dq_acc : torch::empty({T, Hq, D}, q.options());
  const mvp::PeerPull pj = mvp::make_peer_pull(pull);
  if (T == 0 || Tk == 0) {
    TORCH_CHECK(!f32_kv || Tk == 0, "flash_attn_bwd: fp32 dK / dV destinations with no queries");
    if (!ext_dq) dq.zero_();
    dk.zero_();
    dv.zero_();
    mvp::launch_peer_pull(pj, reinterpret_cast<int*>(status_ptr), stream);
    return {dq, dk, dv};
  }
  {
    const int64_t items = static_cast<int64_t>(T) * Hq;
    bwd_delta_kernel<<<static_cast<int>((items + 7) / 8), 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
        delta.data_ptr<float>(), T, Hq);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  CUtensorMap tq, tk, tv, tdo;
  mvp::make_tmap_2d_bf16(&tq, q.data_ptr(), static_cast<int64_t>(Hq) * D, T, q.stride(0), 64, BLK);
  mvp::make_tmap_2d_bf16(&tk, k.data_ptr(), static_cast<int64_t>(Hkv) * D, Tk, k.stride(0), 64, BLK);
  mvp::make_tmap_2d_bf16(&tv, v.data_ptr(), static_cast<int64_t>(Hkv) * D, Tk, v.stride(0), 64, BLK);
  mvp::make_tmap_2d_bf16(&tdo, dout.data_ptr(), static_cast<int64_t>(Hq) * D, T, dout.stride(0), 64, BLK);
  BwdParams p;
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dk_row_stride = dk.stride(0);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.dv_row_stride = dv.stride(0);
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.cu_seqlens = cu_seqlens.data_ptr<int>();
  p.cu_seqlens_k = cu_k.data_ptr<int>();
  p.n_docs = static_cast<int>(cu_seqlens.numel() - 1);
  p.T = T;
  p.Tk = Tk;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = static_cast<float>(softmax_scale);
  p.scale_log2 = static_cast<float>(softmax_scale) * kLog2e;
  p.causal = causal ? 1 : 0;
  p.status = reinterpret_cast<int*>(status_ptr);
  p.pull = pj;
  p.dk_f32 = f32_kv ? reinterpret_cast<float*>((*dkv_f32)[0]) : nullptr;
  p.dv_f32 = f32_kv ? reinterpret_cast<float*>((*dkv_f32)[1]) : nullptr;
  p.f32_row_stride = f32_kv ? (*dkv_f32)[2] : 0;
  p.f32_accumulate = f32_kv ? static_cast<int>((*dkv_f32)[3] != 0) : 0;
  p.route = uroute;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem));
    configured = true;
  }
  dim3 grid((Tk + BLK - 1) / BLK, Hkv + pj.rows);
  bwd_kernel<<<grid, kBwdThreads, kBwdSmem, stream>>>(tq, tk, tv, tdo, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (ext_dq) return {dq, dk, dv};
  const int64_t n = static_cast<int64_t>(T) * Hq * D;
  f32_to_bf16_kernel<<<static_cast<int>(std::min<int64_t>((n / 4 + 255) / 256, 148 * 16)), 256, 0, stream>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dq, dk, dv};
}
