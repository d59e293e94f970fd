// Bandwidth-bound transformer kernels for sm_100a: RMSNorm (with the residual
// add fused in), per-head QK-RMSNorm fused with RoPE / interleaved M-RoPE, and
// SwiGLU.  All read and write bf16 with fp32 math; each forward saves only the
// per-row reciprocal RMS needed by its backward.
//
// Numerics follow the Hugging Face Qwen3 modules the reference trains
// (transformers Qwen3RMSNorm / apply_rotary_pos_emb / Qwen3MLP): the
// normalised activation is rounded to bf16 before the weight multiply, and
// RoPE uses cos/sin rounded to bf16.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "peer_host.h"

namespace mvp {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// ------------------------------------------------------------------ RMSNorm
// One warp per row.  If `res` is given, h = x + res is formed first and
// written to `h_out` (the updated residual stream).
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                   __nv_bfloat16* __restrict__ h_out, float* __restrict__ rstd_out, int rows, int H,
                                   float eps) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(row) * H;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8];
    load8(xr + c, f);
    if (res != nullptr) {
      float r[8];
      load8(res + static_cast<int64_t>(row) * H + c, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = bf16r(f[i] + r[i]);
      store8(h_out + static_cast<int64_t>(row) * H + c, f);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / static_cast<float>(H) + eps);
  if (lane == 0) rstd_out[row] = rstd;
  const __nv_bfloat16* src = res != nullptr ? h_out + static_cast<int64_t>(row) * H : xr;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8], wf[8];
    load8(src + c, f);
    load8(w + c, wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = wf[i] * bf16r(f[i] * rstd);
    store8(y + static_cast<int64_t>(row) * H + c, f);
  }
}

// dx = rstd * (w*dy - xhat * mean(xhat * w * dy)) (+ dres)
__global__ void rmsnorm_bwd_dx_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ h,
                                      const float* __restrict__ rstd_in, const __nv_bfloat16* __restrict__ w,
                                      const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx, int rows,
                                      int H) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const int64_t off = static_cast<int64_t>(row) * H;
  const float rstd = rstd_in[row];
  float dot = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    float g[8], hv[8], wf[8];
    load8(dy + off + c, g);
    load8(h + off + c, hv);
    load8(w + c, wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) dot += g[i] * wf[i] * hv[i] * rstd;
  }
  dot = warp_sum(dot) / static_cast<float>(H);
  for (int c = lane * 8; c < H; c += 256) {
    float g[8], hv[8], wf[8], o[8];
    load8(dy + off + c, g);
    load8(h + off + c, hv);
    load8(w + c, wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = rstd * (wf[i] * g[i] - hv[i] * rstd * dot);
    if (dres != nullptr) {
      float r[8];
      load8(dres + off + c, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += r[i];
    }
    store8(dx + off + c, o);
  }
}

// Column partial sums of dy * bf16(h * rstd): block (32 x 8) covers 64 columns
// of a row strip; partial[blockIdx.y, col].
// Row-resident variants for H = CH x 1024: one 128-thread CTA per row, each thread keeps its CH x 8
// elements in registers between the reduction and the output pass, so every input is read once.
__device__ __forceinline__ float block_sum_128(float v, float* part) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  return (part[0] + part[1]) + (part[2] + part[3]);
}

template <int CH>
__global__ void __launch_bounds__(128) rmsnorm_fwd_row_kernel(const __nv_bfloat16* __restrict__ x,
                                                              const __nv_bfloat16* __restrict__ res,
                                                              const __nv_bfloat16* __restrict__ w,
                                                              __nv_bfloat16* __restrict__ y,
                                                              __nv_bfloat16* __restrict__ h_out,
                                                              float* __restrict__ rstd_out, int H, float eps) {
  __shared__ float part[4];
  const int64_t off = static_cast<int64_t>(blockIdx.x) * H;
  float f[CH][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = (k * 128 + threadIdx.x) * 8;
    load8(x + off + c, f[k]);
    if (res != nullptr) {
      float r[8];
      load8(res + off + c, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[k][i] = bf16r(f[k][i] + r[i]);
      store8(h_out + off + c, f[k]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[k][i] * f[k][i];
  }
  const float rstd = rsqrtf(block_sum_128(ss, part) / static_cast<float>(H) + eps);
  if (threadIdx.x == 0) rstd_out[blockIdx.x] = rstd;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = (k * 128 + threadIdx.x) * 8;
    float wf[8], o[8];
    load8(w + c, wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = wf[i] * bf16r(f[k][i] * rstd);
    store8(y + off + c, o);
  }
}

template <int CH>
__global__ void __launch_bounds__(128) rmsnorm_bwd_dx_row_kernel(const __nv_bfloat16* __restrict__ dy,
                                                                 const __nv_bfloat16* __restrict__ h,
                                                                 const float* __restrict__ rstd_in,
                                                                 const __nv_bfloat16* __restrict__ w,
                                                                 const __nv_bfloat16* __restrict__ dres,
                                                                 __nv_bfloat16* __restrict__ dx, int H) {
  __shared__ float part[4];
  const int64_t off = static_cast<int64_t>(blockIdx.x) * H;
  const float rstd = rstd_in[blockIdx.x];
  float g[CH][8], hv[CH][8];
  float dot = 0.f;
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = (k * 128 + threadIdx.x) * 8;
    float wf[8];
    load8(dy + off + c, g[k]);
    load8(h + off + c, hv[k]);
    load8(w + c, wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) dot += g[k][i] * wf[i] * hv[k][i] * rstd;
  }
  dot = block_sum_128(dot, part) / static_cast<float>(H);
#pragma unroll
  for (int k = 0; k < CH; ++k) {
    const int c = (k * 128 + threadIdx.x) * 8;
    float wf[8], o[8];
    load8(w + c, wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = rstd * (wf[i] * g[k][i] - hv[k][i] * rstd * dot);
    if (dres != nullptr) {
      float r[8];
      load8(dres + off + c, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] += r[i];
    }
    store8(dx + off + c, o);
  }
}

__global__ void rmsnorm_bwd_dw_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ h,
                                      const float* __restrict__ rstd_in, float* __restrict__ partial, int rows, int H,
                                      int rows_per_split, int accumulate) {
  __shared__ float red[8][64];
  const int col = blockIdx.x * 64 + threadIdx.x * 2;
  const int r0 = blockIdx.y * rows_per_split;
  const int r1 = min(rows, r0 + rows_per_split);
  float a0 = 0.f, a1 = 0.f;
  if (col < H) {
    for (int r = r0 + threadIdx.y; r < r1; r += 8) {
      const int64_t off = static_cast<int64_t>(r) * H + col;
      const float2 g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dy + off));
      const float2 hv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(h + off));
      const float rs = rstd_in[r];
      a0 += g.x * bf16r(hv.x * rs);
      a1 += g.y * bf16r(hv.y * rs);
    }
  }
  red[threadIdx.y][threadIdx.x * 2] = a0;
  red[threadIdx.y][threadIdx.x * 2 + 1] = a1;
  __syncthreads();
  if (threadIdx.y == 0 && col < H) {
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s0 += red[j][threadIdx.x * 2];
      s1 += red[j][threadIdx.x * 2 + 1];
    }
    if (accumulate) {  // straight into the caller's fp32 gradient accumulator
      atomicAdd(partial + col, s0);
      atomicAdd(partial + col + 1, s1);
    } else {
      partial[static_cast<int64_t>(blockIdx.y) * H + col] = s0;
      partial[static_cast<int64_t>(blockIdx.y) * H + col + 1] = s1;
    }
  }
}

// --------------------------------------------------------- QK-norm + RoPE
// One warp per (token, head) of q and k; lane l owns elements [4l, 4l+4) of a
// 128-wide head and exchanges the rotate-half partner with lane l ^ 16.
// `pos` is [n_axes, T]; `axis_of` maps each of the 64 frequencies to the
// position axis it reads (all zeros for plain RoPE; t/h/w interleave for the
// Qwen3-VL multimodal RoPE).  cos/sin tables are [P, 64] fp32.
struct QKRopeArgs {
  const __nv_bfloat16* qkv;  // [T, ld_qkv]; q at col 0, k at col Hq*D
  int64_t ld_qkv;
  const __nv_bfloat16* wq;
  const __nv_bfloat16* wk;
  const int* pos;
  int64_t pos_stride;
  const int8_t* axis_of;
  const float* cos_tab;
  const float* sin_tab;
  __nv_bfloat16* q_out;  // [T, Hq, D]
  __nv_bfloat16* k_out;  // [T, Hkv, D]
  float* rstd;           // [T, Hq + Hkv]
  int T, Hq, Hkv;
  float eps;
  int tab_rows;          // rows of cos_tab / sin_tab; positions are clamped into [0, tab_rows)
};

__device__ __forceinline__ int clamp_pos(int p, int rows) { return min(max(p, 0), rows - 1); }

// One warp per token: the lane's cos / sin (four frequencies) and norm weights are loaded once and
// reused for every head of the token; heads are processed four at a time for independent reductions.
__global__ void qk_norm_rope_fwd_kernel(QKRopeArgs a) {
  constexpr int D = 128;
  const int warps = blockDim.x / 32;
  const int t = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= a.T) return;
  const int heads = a.Hq + a.Hkv;
  float c[4], sn[4], wq[4], wk[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int f = (lane * 4 + i) & 63;
    const int p = clamp_pos(a.pos[a.axis_of[f] * a.pos_stride + t], a.tab_rows);
    c[i] = bf16r(a.cos_tab[static_cast<int64_t>(p) * 64 + f]);
    sn[i] = bf16r(a.sin_tab[static_cast<int64_t>(p) * 64 + f]);
    wq[i] = __bfloat162float(a.wq[lane * 4 + i]);
    wk[i] = __bfloat162float(a.wk[lane * 4 + i]);
  }
  const bool lo = lane < 16;
  const __nv_bfloat16* row = a.qkv + static_cast<int64_t>(t) * a.ld_qkv + lane * 4;
  // Heads in groups of kGroup: every load of a group is issued before the group's first store (the
  // compiler cannot move a load above a store to a possibly aliasing output), so kGroup row loads are in
  // flight per warp instead of one.
  constexpr int kGroup = 8;
  for (int h0 = 0; h0 < heads; h0 += kGroup) {
    uint2 raw[kGroup];
#pragma unroll
    for (int j = 0; j < kGroup; ++j)
      raw[j] = h0 + j < heads ? *reinterpret_cast<const uint2*>(row + static_cast<int64_t>(h0 + j) * D)
                              : make_uint2(0u, 0u);
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      const int hd = h0 + j;
      if (hd >= heads) break;
      const bool is_q = hd < a.Hq;
      float x[4];
      {
        const uint2 u = raw[j];
        const float2 p0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 p1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        x[0] = p0.x; x[1] = p0.y; x[2] = p1.x; x[3] = p1.y;
      }
      float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
      ss = warp_sum(ss);
      const float rstd = rsqrtf(ss / D + a.eps);
      if (lane == 0) a.rstd[static_cast<int64_t>(t) * heads + hd] = rstd;
      float y[4], partner[4], o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = bf16r((is_q ? wq[i] : wk[i]) * bf16r(x[i] * rstd));
#pragma unroll
      for (int i = 0; i < 4; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = lo ? (y[i] * c[i] - partner[i] * sn[i]) : (y[i] * c[i] + partner[i] * sn[i]);
      __nv_bfloat16* dst = is_q ? a.q_out + (static_cast<int64_t>(t) * a.Hq + hd) * D
                                : a.k_out + (static_cast<int64_t>(t) * a.Hkv + (hd - a.Hq)) * D;
      uint2 u;
      u.x = pack_bf16x2(o[0], o[1]);
      u.y = pack_bf16x2(o[2], o[3]);
      *reinterpret_cast<uint2*>(dst + lane * 4) = u;
    }
  }
}

struct QKRopeBwdArgs {
  const __nv_bfloat16* dq;  // [T, Hq, D]
  const __nv_bfloat16* dk;  // [T, Hkv, D]
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  const __nv_bfloat16* wq;
  const __nv_bfloat16* wk;
  const int* pos;
  int64_t pos_stride;
  const int8_t* axis_of;
  const float* cos_tab;
  const float* sin_tab;
  const float* rstd;
  __nv_bfloat16* dqkv;  // [T, ld_dqkv]: q and k parts written
  int64_t ld_dqkv;
  float* dw_partial;  // [gridDim.x, 2, D], or with dw_accumulate the fp32 accumulators dwq, dwk
  float* dwk_acc;
  int dw_accumulate;
  int T, Hq, Hkv;
  int tab_rows;
  UlyssesRoute route;  // optional: dq / dk rows written to the token's rank (its dqkv) instead of dqkv
};

__device__ __forceinline__ void load_bf16x4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 p0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 p1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  v[0] = p0.x; v[1] = p0.y; v[2] = p1.x; v[3] = p1.y;
}

// One warp per token (grid-stride): cos / sin and the norm weights of the lane's four elements are
// loaded once per token and reused for every head; 8-byte loads and stores per lane.
__global__ void qk_norm_rope_bwd_kernel(QKRopeBwdArgs a) {
  constexpr int D = 128;
  __shared__ float red[2][D];
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) (&red[0][0])[i] = 0.f;
  __syncthreads();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int heads = a.Hq + a.Hkv;
  const bool lo = lane < 16;
  float wq[4], wk[4];
  load_bf16x4(a.wq + lane * 4, wq);
  load_bf16x4(a.wk + lane * 4, wk);
  float accq[4] = {0.f, 0.f, 0.f, 0.f}, acck[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t = blockIdx.x * warps + threadIdx.x / 32; t < a.T; t += gridDim.x * warps) {
    float c[4], sn[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = (lane * 4 + i) & 63;
      const int p = clamp_pos(a.pos[a.axis_of[f] * a.pos_stride + t], a.tab_rows);
      c[i] = bf16r(a.cos_tab[static_cast<int64_t>(p) * 64 + f]);
      sn[i] = bf16r(a.sin_tab[static_cast<int64_t>(p) * 64 + f]);
    }
    int owner = 0, lrow = 0;
    if (a.route.dst[0] != nullptr) ulysses_home(a.route, t, owner, lrow);
    // Heads in groups of kGroup, all loads of a group (gradient, input row, row scale) before its first
    // store: the stores may alias the inputs as far as the compiler knows, so without this each head would
    // wait for its own loads.
    constexpr int kGroup = 8;
    for (int h0 = 0; h0 < heads; h0 += kGroup) {
      float gs[kGroup][4], xs[kGroup][4], rs[kGroup];
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        const int hd = min(h0 + j, heads - 1);  // a repeated head past the end is loaded but not used
        const bool is_q = hd < a.Hq;
        load_bf16x4(is_q ? a.dq + (static_cast<int64_t>(t) * a.Hq + hd) * D + lane * 4
                         : a.dk + (static_cast<int64_t>(t) * a.Hkv + (hd - a.Hq)) * D + lane * 4, gs[j]);
        load_bf16x4(a.qkv + static_cast<int64_t>(t) * a.ld_qkv + static_cast<int64_t>(hd) * D + lane * 4, xs[j]);
        rs[j] = a.rstd[static_cast<int64_t>(t) * heads + hd];
      }
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        const int hd = h0 + j;
        if (hd >= heads) break;
        const bool is_q = hd < a.Hq;
        float g[4], x[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          g[i] = gs[j][i];
          x[i] = xs[j][i];
        }
        float gp[4], dy[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) gp[i] = __shfl_xor_sync(0xffffffffu, g[i], 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) dy[i] = lo ? (g[i] * c[i] + gp[i] * sn[i]) : (g[i] * c[i] - gp[i] * sn[i]);
        const float rstd = rs[j];
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) dot += dy[i] * (is_q ? wq[i] : wk[i]) * x[i] * rstd;
        dot = warp_sum(dot) / D;
        float dx[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dx[i] = rstd * ((is_q ? wq[i] : wk[i]) * dy[i] - x[i] * rstd * dot);
          const float xh = bf16r(x[i] * rstd);
          if (is_q) accq[i] += dy[i] * xh;
          else acck[i] += dy[i] * xh;
        }
        __nv_bfloat16* dst = a.dqkv + static_cast<int64_t>(t) * a.ld_dqkv + static_cast<int64_t>(hd) * D + lane * 4;
        if (a.route.dst[0] != nullptr)  // Ulysses: back to the token's rank, global head columns
          dst = reinterpret_cast<__nv_bfloat16*>(a.route.dst[owner]) + static_cast<int64_t>(lrow) * a.route.ld +
                (is_q ? a.route.col0 + hd * D : a.route.col0_k + (hd - a.Hq) * D) + lane * 4;
        uint2 u;
        u.x = pack_bf16x2(dx[0], dx[1]);
        u.y = pack_bf16x2(dx[2], dx[3]);
        *reinterpret_cast<uint2*>(dst) = u;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    atomicAdd(&red[0][lane * 4 + i], accq[i]);
    atomicAdd(&red[1][lane * 4 + i], acck[i]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) {
    if (a.dw_accumulate) atomicAdd(i < D ? a.dw_partial + i : a.dwk_acc + (i - D), (&red[0][0])[i]);
    else a.dw_partial[static_cast<int64_t>(blockIdx.x) * 2 * D + i] = (&red[0][0])[i];
  }
  if (a.route.dst[0] != nullptr) __threadfence_system();
}

// ------------------------------------------------------------------ SwiGLU
// gu = [T, 2F] with gate in columns [0, F) and up in [F, 2F); out = silu(g)*u.
// One thread per 8 columns of one row (grid.x = row, grid.y = column block): no index division, 16-byte accesses, the
// sigmoid through the fast exp / divide intrinsics.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out, int64_t T,
                                  int F) {
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  const int64_t t = blockIdx.x;
  if (c >= F) return;
  float g[8], u[8], o[8];
  load8(gu + t * 2 * F + c, g);
  load8(gu + t * 2 * F + F + c, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float s = __fdividef(g[j], 1.f + __expf(-g[j]));
    o[j] = bf16r(s) * u[j];
  }
  store8(out + t * F + c, o);
}
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dout,
                                  __nv_bfloat16* __restrict__ dgu, int64_t T, int F) {
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  const int64_t t = blockIdx.x;
  if (c >= F) return;
  float g[8], u[8], d[8], dg[8], du[8];
  load8(gu + t * 2 * F + c, g);
  load8(gu + t * 2 * F + F + c, u);
  load8(dout + t * F + c, d);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float sig = __fdividef(1.f, 1.f + __expf(-g[j]));
    const float s = g[j] * sig;
    du[j] = d[j] * bf16r(s);
    dg[j] = d[j] * u[j] * sig * (1.f + g[j] * (1.f - sig));
  }
  store8(dgu + t * 2 * F + c, dg);
  store8(dgu + t * 2 * F + F + c, du);
}

inline int grid_for(int64_t n, int threads) {
  const int64_t g = (n + threads - 1) / threads;
  return static_cast<int>(std::min<int64_t>(std::max<int64_t>(g, 1), 148 * 16));
}

}  // namespace
}  // namespace mvp

using mvp::grid_for;

#define CHECK_BF16(t) TORCH_CHECK((t).scalar_type() == at::kBFloat16 && (t).is_contiguous(), #t " must be contiguous bf16")

std::vector<torch::Tensor> rmsnorm_fwd(const torch::Tensor& x, const c10::optional<torch::Tensor>& res,
                                       const torch::Tensor& w, double eps) {
  CHECK_BF16(x);
  CHECK_BF16(w);
  const int H = static_cast<int>(x.size(-1));
  TORCH_CHECK(H % 8 == 0 && w.numel() == H, "rmsnorm: hidden size must be a multiple of 8 and match the weight");
  const int rows = static_cast<int>(x.numel() / H);
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  torch::Tensor h;
  const __nv_bfloat16* rp = nullptr;
  if (res.has_value()) {
    CHECK_BF16(*res);
    h = torch::empty_like(x);
    rp = reinterpret_cast<const __nv_bfloat16*>(res->data_ptr());
  }
  const int threads = 256, per = threads / 32;
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  auto* hp = h.defined() ? reinterpret_cast<__nv_bfloat16*>(h.data_ptr()) : nullptr;
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto fwd_rows = [&](auto kern) {
    kern<<<rows, 128, 0, stream>>>(xp, rp, wp, yp, hp, rstd.data_ptr<float>(), H, static_cast<float>(eps));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  };
  if (rows == 0) {
  } else if (H == 4096) {
    fwd_rows(mvp::rmsnorm_fwd_row_kernel<4>);
  } else if (H == 5120) {
    fwd_rows(mvp::rmsnorm_fwd_row_kernel<5>);
  } else if (H == 2048) {
    fwd_rows(mvp::rmsnorm_fwd_row_kernel<2>);
  } else {
    mvp::rmsnorm_fwd_kernel<<<(rows + per - 1) / per, threads, 0, stream>>>(xp, rp, wp, yp, hp, rstd.data_ptr<float>(),
                                                                          rows, H, static_cast<float>(eps));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (h.defined()) return {y, rstd, h};
  return {y, rstd};
}

std::vector<torch::Tensor> rmsnorm_bwd(const torch::Tensor& dy, const torch::Tensor& h, const torch::Tensor& rstd,
                                       const torch::Tensor& w, const c10::optional<torch::Tensor>& dres,
                                       bool need_dw, const c10::optional<torch::Tensor>& dw_acc) {
  CHECK_BF16(dy);
  CHECK_BF16(h);
  CHECK_BF16(w);
  const int H = static_cast<int>(h.size(-1));
  const int rows = static_cast<int>(h.numel() / H);
  const at::cuda::CUDAGuard guard(h.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto dx = torch::empty_like(h);
  const __nv_bfloat16* dr = nullptr;
  if (dres.has_value()) {
    CHECK_BF16(*dres);
    dr = reinterpret_cast<const __nv_bfloat16*>(dres->data_ptr());
  }
  const int threads = 256, per = threads / 32;
  auto* dyp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto* hp = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto* dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  auto bwd_rows = [&](auto kern) {
    kern<<<rows, 128, 0, stream>>>(dyp, hp, rstd.data_ptr<float>(), wp, dr, dxp, H);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  };
  if (rows == 0) {
  } else if (H == 4096) {
    bwd_rows(mvp::rmsnorm_bwd_dx_row_kernel<4>);
  } else if (H == 5120) {
    bwd_rows(mvp::rmsnorm_bwd_dx_row_kernel<5>);
  } else if (H == 2048) {
    bwd_rows(mvp::rmsnorm_bwd_dx_row_kernel<2>);
  } else {
    mvp::rmsnorm_bwd_dx_kernel<<<(rows + per - 1) / per, threads, 0, stream>>>(dyp, hp, rstd.data_ptr<float>(), wp, dr,
                                                                             dxp, rows, H);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (!need_dw) return {dx};
  const int splits = std::max(1, std::min(64, rows / 64));
  const int rows_per_split = (rows + splits - 1) / splits;
  dim3 grid((H + 63) / 64, splits), block(32, 8);
  if (dw_acc.has_value()) {  // dW added to the caller's fp32 accumulator [H]: no partials, no reduction
    TORCH_CHECK(dw_acc->scalar_type() == at::kFloat && dw_acc->is_contiguous() && dw_acc->numel() == H,
                "rmsnorm_bwd: dw_acc must be contiguous fp32 [H]");
    mvp::rmsnorm_bwd_dw_kernel<<<grid, block, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()),
        rstd.data_ptr<float>(), dw_acc->data_ptr<float>(), rows, H, rows_per_split, 1);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {dx, *dw_acc};
  }
  auto partial = torch::empty({splits, H}, h.options().dtype(at::kFloat));
  mvp::rmsnorm_bwd_dw_kernel<<<grid, block, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                                                         reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()),
                                                         rstd.data_ptr<float>(), partial.data_ptr<float>(), rows, H,
                                                         rows_per_split, 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dx, partial.sum(0)};
}

std::vector<torch::Tensor> qk_norm_rope_fwd(const torch::Tensor& qkv, int64_t Hq, int64_t Hkv,
                                            const torch::Tensor& wq, const torch::Tensor& wk,
                                            const torch::Tensor& pos, const torch::Tensor& axis_of,
                                            const torch::Tensor& cos_tab, const torch::Tensor& sin_tab, double eps) {
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.stride(-1) == 1, "qk_norm_rope: bf16 qkv");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.dim() == 2 && pos.stride(1) == 1, "qk_norm_rope: pos [A, T] int32");
  TORCH_CHECK(axis_of.scalar_type() == at::kChar && axis_of.numel() == 64, "qk_norm_rope: axis_of int8[64]");
  CHECK_BF16(wq);
  CHECK_BF16(wk);
  const int T = static_cast<int>(qkv.size(0));
  const at::cuda::CUDAGuard guard(qkv.device());
  auto q = torch::empty({T, Hq, 128}, qkv.options());
  auto k = torch::empty({T, Hkv, 128}, qkv.options());
  auto rstd = torch::empty({T, Hq + Hkv}, qkv.options().dtype(at::kFloat));
  mvp::QKRopeArgs a;
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.ld_qkv = qkv.stride(0);
  a.wq = reinterpret_cast<const __nv_bfloat16*>(wq.data_ptr());
  a.wk = reinterpret_cast<const __nv_bfloat16*>(wk.data_ptr());
  a.pos = pos.data_ptr<int>();
  a.pos_stride = pos.stride(0);
  a.axis_of = axis_of.data_ptr<int8_t>();
  a.cos_tab = cos_tab.data_ptr<float>();
  a.sin_tab = sin_tab.data_ptr<float>();
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q.data_ptr());
  a.k_out = reinterpret_cast<__nv_bfloat16*>(k.data_ptr());
  a.rstd = rstd.data_ptr<float>();
  a.T = T;
  a.Hq = static_cast<int>(Hq);
  a.Hkv = static_cast<int>(Hkv);
  a.eps = static_cast<float>(eps);
  a.tab_rows = static_cast<int>(cos_tab.size(0));
  TORCH_CHECK(a.tab_rows > 0 && sin_tab.size(0) == cos_tab.size(0), "qk_norm_rope: cos/sin tables");
  const int threads = 256;  // 8 tokens per block
  mvp::qk_norm_rope_fwd_kernel<<<static_cast<int>((T + 7) / 8), threads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {q, k, rstd};
}

// Writes the q/k parts of `dqkv` in place and returns (dwq, dwk).
std::vector<torch::Tensor> qk_norm_rope_bwd(const torch::Tensor& dq, const torch::Tensor& dk,
                                            const torch::Tensor& qkv, torch::Tensor& dqkv, int64_t Hq, int64_t Hkv,
                                            const torch::Tensor& wq, const torch::Tensor& wk,
                                            const torch::Tensor& pos, const torch::Tensor& axis_of,
                                            const torch::Tensor& cos_tab, const torch::Tensor& sin_tab,
                                            const torch::Tensor& rstd,
                                            const c10::optional<std::vector<int64_t>>& route,
                                            const c10::optional<torch::Tensor>& dwq_acc,
                                            const c10::optional<torch::Tensor>& dwk_acc) {
  CHECK_BF16(dq);
  CHECK_BF16(dk);
  TORCH_CHECK(dqkv.stride(-1) == 1 && qkv.stride(-1) == 1, "qk_norm_rope_bwd: unit inner stride");
  const int T = static_cast<int>(qkv.size(0));
  const at::cuda::CUDAGuard guard(qkv.device());
  const int threads = 256;
  const int blocks = 148 * 4;
  // dwq_acc / dwk_acc (both or neither): the norm-weight gradients are added straight into these fp32
  // accumulators [128] and returned as they are.
  const bool acc = dwq_acc.has_value() && dwk_acc.has_value();
  if (acc)
    TORCH_CHECK(dwq_acc->scalar_type() == at::kFloat && dwk_acc->scalar_type() == at::kFloat &&
                    dwq_acc->is_contiguous() && dwk_acc->is_contiguous() && dwq_acc->numel() == 128 &&
                    dwk_acc->numel() == 128,
                "qk_norm_rope_bwd: fp32 [128] accumulators");
  auto partial = acc ? torch::Tensor() : torch::empty({blocks, 2, 128}, qkv.options().dtype(at::kFloat));
  mvp::QKRopeBwdArgs a;
  a.dq = reinterpret_cast<const __nv_bfloat16*>(dq.data_ptr());
  a.dk = reinterpret_cast<const __nv_bfloat16*>(dk.data_ptr());
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.ld_qkv = qkv.stride(0);
  a.wq = reinterpret_cast<const __nv_bfloat16*>(wq.data_ptr());
  a.wk = reinterpret_cast<const __nv_bfloat16*>(wk.data_ptr());
  a.pos = pos.data_ptr<int>();
  a.pos_stride = pos.stride(0);
  a.axis_of = axis_of.data_ptr<int8_t>();
  a.cos_tab = cos_tab.data_ptr<float>();
  a.sin_tab = sin_tab.data_ptr<float>();
  a.rstd = rstd.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.ld_dqkv = dqkv.stride(0);
  a.dw_partial = acc ? dwq_acc->data_ptr<float>() : partial.data_ptr<float>();
  a.dwk_acc = acc ? dwk_acc->data_ptr<float>() : nullptr;
  a.dw_accumulate = acc ? 1 : 0;
  a.T = T;
  a.Hq = static_cast<int>(Hq);
  a.Hkv = static_cast<int>(Hkv);
  a.tab_rows = static_cast<int>(cos_tab.size(0));
  a.route = mvp::make_ulysses_route(route);
  TORCH_CHECK(a.route.dst[0] == nullptr || T == 2 * a.route.world * a.route.chunk,
              "qk_norm_rope_bwd: routed rows need T = 2 x world x chunk");
  mvp::qk_norm_rope_bwd_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (acc) return {*dwq_acc, *dwk_acc};
  auto dw = partial.sum(0);
  return {dw[0], dw[1]};
}

torch::Tensor swiglu_fwd(const torch::Tensor& gu) {
  CHECK_BF16(gu);
  const int64_t T = gu.size(0);
  const int F = static_cast<int>(gu.size(1) / 2);
  TORCH_CHECK(F % 8 == 0, "swiglu: F must be a multiple of 8");
  const at::cuda::CUDAGuard guard(gu.device());
  auto out = torch::empty({T, F}, gu.options());
  if (T == 0) return out;
  TORCH_CHECK(T <= 0x7fffffff && (F / 8 + 255) / 256 <= 65535, "swiglu: shape beyond the launch grid");
  mvp::swiglu_fwd_kernel<<<dim3(static_cast<unsigned>(T), (F / 8 + 255) / 256), 256, 0,
                           at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

torch::Tensor swiglu_bwd(const torch::Tensor& gu, const torch::Tensor& dout) {
  CHECK_BF16(gu);
  CHECK_BF16(dout);
  const int64_t T = gu.size(0);
  const int F = static_cast<int>(gu.size(1) / 2);
  const at::cuda::CUDAGuard guard(gu.device());
  auto dgu = torch::empty_like(gu);
  if (T == 0) return dgu;
  TORCH_CHECK(F % 8 == 0 && T <= 0x7fffffff && (F / 8 + 255) / 256 <= 65535, "swiglu: shape beyond the launch grid");
  mvp::swiglu_bwd_kernel<<<dim3(static_cast<unsigned>(T), (F / 8 + 255) / 256), 256, 0,
                           at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), T, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dgu;
}
