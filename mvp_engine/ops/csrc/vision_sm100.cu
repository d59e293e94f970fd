// Bandwidth-bound kernels of the vision tower (Qwen3-VL ViT): LayerNorm with
// bias, bias + GELU (tanh or erf form) after the first MLP GEMM, and the
// vision RoPE (rotate-half form) that also pads q / k / v to the head_dim-128
// attention kernel's layout.  bf16 in and out, fp32 math, one bf16 rounding
// per output as PyTorch's eager ops round (transformers Qwen3VLVisionBlock /
// Qwen3VLVisionMLP / apply_rotary_pos_emb_vision, the modules the reference's
// qwen3_vl recipe trains; it patches only the patch embedding of that HF model,
// recipes/qwen3_vl/model/qwen3_vl.py:151-171).
//
// Parameter gradients (LayerNorm weight / bias, GELU bias) are column sums over
// rows: each CTA sums its rows into fp32 partials, a second kernel sums the
// partials, optionally adding into caller-owned fp32 accumulators.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace mvp {
namespace {

__device__ __forceinline__ float vwarp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void vload8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void vstore8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float rbf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

constexpr int kLnWarps = 4;

// ---------------------------------------------------------------- LayerNorm
// One warp per row, 8 columns per lane access.  Mean first, then the variance
// about it (two-pass, as PyTorch computes it, not E[x^2] - mean^2); the row is
// re-read from L1 for each pass.
__global__ void __launch_bounds__(kLnWarps * 32) layernorm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ b,
    __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int H,
    float eps) {
  const int row = blockIdx.x * kLnWarps + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(row) * H;
  const int nv = H / 8;
  float s = 0.f;
  for (int v = lane; v < nv; v += 32) {
    float f[8];
    vload8(xr + v * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += f[i];
  }
  const float mean = vwarp_sum(s) / H;
  float q = 0.f;
  for (int v = lane; v < nv; v += 32) {
    float f[8];
    vload8(xr + v * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) q += (f[i] - mean) * (f[i] - mean);
  }
  const float rstd = rsqrtf(vwarp_sum(q) / H + eps);
  __nv_bfloat16* yr = y + static_cast<int64_t>(row) * H;
  for (int v = lane; v < nv; v += 32) {
    float f[8], wf[8], bf[8];
    vload8(xr + v * 8, f);
    vload8(w + v * 8, wf);
    vload8(b + v * 8, bf);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = (f[i] - mean) * rstd * wf[i] + bf[i];
    vstore8(yr + v * 8, f);
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// dx = rstd * (g - mean(g) - xhat * mean(g * xhat)), g = dy * w, xhat = (x - mean) * rstd;
// dw = sum_rows dy * xhat and db = sum_rows dy.  Each warp sums its rows into its own 2H-float region
// of shared memory (a lane always owns the same columns, so no atomics); the CTA then adds its warps'
// regions and writes part[blockIdx.x, 0:H] (dw) and part[blockIdx.x, H:2H] (db).
__global__ void __launch_bounds__(256) layernorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, const float* __restrict__ mean_in,
    const float* __restrict__ rstd_in, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ part, int rows, int H) {
  extern __shared__ float sacc[];  // (blockDim.x / 32) regions of 2H floats
  const int warps = blockDim.x / 32;
  for (int i = threadIdx.x; i < 2 * H * warps; i += blockDim.x) sacc[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x % 32;
  const int nv = H / 8;
  float* wacc = sacc + (threadIdx.x / 32) * 2 * H;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += gridDim.x * warps) {
    const __nv_bfloat16* xr = x + static_cast<int64_t>(row) * H;
    const __nv_bfloat16* gr = dy + static_cast<int64_t>(row) * H;
    const float mean = mean_in[row], rstd = rstd_in[row];
    float sg = 0.f, sgx = 0.f;
#pragma unroll 4
    for (int v = lane; v < nv; v += 32) {
      float f[8], g[8], wf[8];
      vload8(xr + v * 8, f);
      vload8(gr + v * 8, g);
      vload8(w + v * 8, wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float gw = g[i] * wf[i];
        sg += gw;
        sgx += gw * (f[i] - mean) * rstd;
      }
    }
    const float mg = vwarp_sum(sg) / H, mgx = vwarp_sum(sgx) / H;
    __nv_bfloat16* dxr = dx + static_cast<int64_t>(row) * H;
#pragma unroll 4
    for (int v = lane; v < nv; v += 32) {
      float f[8], g[8], wf[8], o[8];
      vload8(xr + v * 8, f);
      vload8(gr + v * 8, g);
      vload8(w + v * 8, wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = (f[i] - mean) * rstd;
        o[i] = rstd * (g[i] * wf[i] - mg - xh * mgx);
        wacc[i * nv + v] += g[i] * xh;  // column v * 8 + i, stored element-major: no bank conflicts
        wacc[H + i * nv + v] += g[i];
      }
      vstore8(dxr + v * 8, o);
    }
  }
  __syncthreads();
  float* pr = part + static_cast<int64_t>(blockIdx.x) * 2 * H;
  for (int c = threadIdx.x; c < 2 * H; c += blockDim.x) {
    const int half = c >= H ? H : 0, col = c - half;
    const int idx = half + (col % 8) * nv + col / 8;
    float t = 0.f;
    for (int k = 0; k < warps; ++k) t += sacc[k * 2 * H + idx];
    pr[c] = t;
  }
}

// out[c] (+)= sum_g part[g, c] for c < n; one thread per column.
__global__ void colsum_kernel(const float* __restrict__ part, int G, int n, int ld, float* __restrict__ out,
                              bool accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float s = 0.f;
  for (int g = 0; g < G; ++g) s += part[static_cast<int64_t>(g) * ld + c];
  out[c] = accumulate ? out[c] + s : s;
}

// -------------------------------------------------------------- bias + GELU
// h = bf16(x + b) (the eager bias add rounds), y = bf16(gelu(h)).
// tanh form: 0.5 h (1 + tanh(sqrt(2/pi) (h + 0.044715 h^3)));  erf form: 0.5 h (1 + erf(h / sqrt(2))).
constexpr float kSqrt2OverPi = 0.7978845608028654f;
constexpr float kInvSqrt2 = 0.7071067811865476f;
constexpr float kInvSqrt2Pi = 0.3989422804014327f;

// tanh(u) = 1 - 2 / (exp(2u) + 1): saturates to +-1 when exp over- or underflows; its absolute error
// (about 1e-7) is far below the bf16 rounding of the GELU result.
__device__ __forceinline__ float tanh_exp(float u) { return 1.f - __fdividef(2.f, __expf(2.f * u) + 1.f); }

template <bool kTanh>
__device__ __forceinline__ float gelu_f(float h) {
  if (kTanh) return 0.5f * h * (1.f + tanh_exp(kSqrt2OverPi * (h + 0.044715f * h * h * h)));
  return 0.5f * h * (1.f + erff(h * kInvSqrt2));
}

template <bool kTanh>
__device__ __forceinline__ float gelu_grad(float h) {
  if (kTanh) {
    const float t = tanh_exp(kSqrt2OverPi * (h + 0.044715f * h * h * h));
    return 0.5f * (1.f + t) + 0.5f * h * (1.f - t * t) * kSqrt2OverPi * (1.f + 3.f * 0.044715f * h * h);
  }
  return 0.5f * (1.f + erff(h * kInvSqrt2)) + h * kInvSqrt2Pi * expf(-0.5f * h * h);
}

// grid: x over column blocks of 8 * blockDim.x columns, y over row groups (rows stride gridDim.y)
template <bool kTanh>
__global__ void __launch_bounds__(128) bias_gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ b,
                                                            __nv_bfloat16* __restrict__ y, int rows, int F) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v * 8 >= F) return;
  float bf[8];
  vload8(b + v * 8, bf);
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const int64_t off = static_cast<int64_t>(r) * F + v * 8;
    float f[8];
    vload8(x + off, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = gelu_f<kTanh>(rbf16(f[i] + bf[i]));
    vstore8(y + off, f);
  }
}

// dh = bf16(dy * gelu'(h)); dx = dh (the bias add passes it through); db partials per row group.
template <bool kTanh>
__global__ void __launch_bounds__(128) bias_gelu_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                            const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ b,
                                                            __nv_bfloat16* __restrict__ dx, float* __restrict__ part,
                                                            int rows, int F) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v * 8 >= F) return;
  float bf[8], acc[8];
  vload8(b + v * 8, bf);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const int64_t off = static_cast<int64_t>(r) * F + v * 8;
    float f[8], g[8];
    vload8(x + off, f);
    vload8(dy + off, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      f[i] = rbf16(g[i] * gelu_grad<kTanh>(rbf16(f[i] + bf[i])));
      acc[i] += f[i];
    }
    vstore8(dx + off, f);
  }
  float* pr = part + static_cast<int64_t>(blockIdx.y) * F + v * 8;
#pragma unroll
  for (int i = 0; i < 8; ++i) pr[i] = acc[i];
}

// ------------------------------------------------------ bias + residual add
// out = bf16(x + bf16(y + b)): the projection's bias add and the residual add, rounded as the two eager
// adds round.  grid as bias_gelu_fwd_kernel.
__global__ void __launch_bounds__(128) bias_residual_fwd_kernel(const __nv_bfloat16* __restrict__ y,
                                                                const __nv_bfloat16* __restrict__ b,
                                                                const __nv_bfloat16* __restrict__ x,
                                                                __nv_bfloat16* __restrict__ out, int rows, int F) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v * 8 >= F) return;
  float bf[8];
  vload8(b + v * 8, bf);
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    const int64_t off = static_cast<int64_t>(r) * F + v * 8;
    float f[8], g[8];
    vload8(y + off, f);
    vload8(x + off, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = g[i] + rbf16(f[i] + bf[i]);
    vstore8(out + off, f);
  }
}

// Per-row-group column sums of a bf16 matrix (the bias gradient): part[blockIdx.y, F].
__global__ void __launch_bounds__(128) col_partial_kernel(const __nv_bfloat16* __restrict__ g,
                                                          float* __restrict__ part, int rows, int F) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v * 8 >= F) return;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll 4
  for (int r = blockIdx.y; r < rows; r += gridDim.y) {
    float f[8];
    vload8(g + static_cast<int64_t>(r) * F + v * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += f[i];
  }
  float* pr = part + static_cast<int64_t>(blockIdx.y) * F + v * 8;
#pragma unroll
  for (int i = 0; i < 8; ++i) pr[i] = acc[i];
}

// ------------------------------------------------------------- vision RoPE
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// qkv: [N, 3, nh, D] bf16; cos / sin: [N, D/2] fp32.  One warp per (token, head).
// q_out / k_out / v_out: [N, nh, DP] bf16 with columns D..DP-1 zero.
// rotate-half: out[i] = x[i] c_i - x[i+h] s_i, out[i+h] = x[i+h] c_i + x[i] s_i (h = D/2).
__global__ void __launch_bounds__(256) vision_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                              const float* __restrict__ cosv,
                                                              const float* __restrict__ sinv,
                                                              __nv_bfloat16* __restrict__ qo,
                                                              __nv_bfloat16* __restrict__ ko,
                                                              __nv_bfloat16* __restrict__ vo, int64_t N, int nh, int D,
                                                              int DP, const __nv_bfloat16* __restrict__ bias) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (wid >= N * nh) return;
  const int64_t n = wid / nh;
  const int hd = static_cast<int>(wid % nh);
  const int h = D / 2;
  const __nv_bfloat16* src = qkv + (n * 3 * nh + hd) * D;
  const int64_t dst = wid * DP;
  // qkv + bias (optional, [3 * nh * D]), rounded to bf16 as a separate bias add would round it
  auto in = [&](int t, int i) {
    const float x = __bfloat162float(src[static_cast<int64_t>(t) * nh * D + i]);
    return bias == nullptr ? x : bf16_round(x + __bfloat162float(bias[(t * nh + hd) * D + i]));
  };
  for (int t = 0; t < 2; ++t) {
    __nv_bfloat16* o = (t == 0 ? qo : ko) + dst;
    for (int i = lane; i < h; i += 32) {
      const float c = cosv[n * h + i], sn = sinv[n * h + i];
      const float a = in(t, i), bb = in(t, i + h);
      o[i] = __float2bfloat16_rn(a * c - bb * sn);
      o[i + h] = __float2bfloat16_rn(bb * c + a * sn);
    }
    for (int i = D + lane; i < DP; i += 32) o[i] = __float2bfloat16_rn(0.f);
  }
  for (int i = lane; i < DP; i += 32) vo[dst + i] = i < D ? __float2bfloat16_rn(in(2, i)) : __float2bfloat16_rn(0.f);
}

// Inverse rotation of dq / dk and the dv slice, written into dqkv [N, 3, nh, D]:
// dx[i] = d[i] c_i + d[i+h] s_i, dx[i+h] = d[i+h] c_i - d[i] s_i.
__global__ void __launch_bounds__(256) vision_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dq,
                                                              const __nv_bfloat16* __restrict__ dk,
                                                              const __nv_bfloat16* __restrict__ dv,
                                                              const float* __restrict__ cosv,
                                                              const float* __restrict__ sinv,
                                                              __nv_bfloat16* __restrict__ dqkv, int64_t N, int nh,
                                                              int D, int DP) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (wid >= N * nh) return;
  const int64_t n = wid / nh;
  const int hd = static_cast<int>(wid % nh);
  const int h = D / 2;
  __nv_bfloat16* dst = dqkv + (n * 3 * nh + hd) * D;
  const int64_t src = wid * DP;
  for (int t = 0; t < 2; ++t) {
    const __nv_bfloat16* d = (t == 0 ? dq : dk) + src;
    __nv_bfloat16* o = dst + static_cast<int64_t>(t) * nh * D;
    for (int i = lane; i < h; i += 32) {
      const float c = cosv[n * h + i], sn = sinv[n * h + i];
      const float a = __bfloat162float(d[i]), bb = __bfloat162float(d[i + h]);
      o[i] = __float2bfloat16_rn(a * c + bb * sn);
      o[i + h] = __float2bfloat16_rn(bb * c - a * sn);
    }
  }
  __nv_bfloat16* ov = dst + static_cast<int64_t>(2) * nh * D;
  for (int i = lane; i < D; i += 32) ov[i] = dv[src + i];
}

// Row-vectorised RoPE for head dims that are multiples of 8 (64, 72): one thread per [q|k|v] row of one
// (token, head), 16-byte loads and stores, the row held in registers.  Thread i handles the i-th row of qkv
// in memory order ([N, 3, nh, D]), so neighbouring threads touch neighbouring rows.
template <int D>
__global__ void __launch_bounds__(128) vision_rope_fwd_vec_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                  const float* __restrict__ cosv,
                                                                  const float* __restrict__ sinv,
                                                                  __nv_bfloat16* __restrict__ qo,
                                                                  __nv_bfloat16* __restrict__ ko,
                                                                  __nv_bfloat16* __restrict__ vo, int64_t N, int nh,
                                                                  int DP, const __nv_bfloat16* __restrict__ bias) {
  constexpr int h = D / 2;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= N * 3 * nh) return;
  const int64_t n = idx / (3 * nh);
  const int rem = static_cast<int>(idx - n * 3 * nh);
  const int t = rem / nh, hd = rem % nh;
  float x[D];
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    float f[8];
    vload8(qkv + idx * D + c * 8, f);
    if (bias != nullptr) {  // the qkv bias (row `rem` of [3 * nh, D]), rounded as a separate add would round it
      float bf[8];
      vload8(bias + static_cast<int64_t>(rem) * D + c * 8, bf);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = bf16_round(f[i] + bf[i]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) x[c * 8 + i] = f[i];
  }
  if (t < 2) {
    const float* cr = cosv + n * h;
    const float* sr = sinv + n * h;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float c = cr[i], sn = sr[i], a = x[i], b = x[i + h];
      x[i] = a * c - b * sn;
      x[i + h] = b * c + a * sn;
    }
  }
  __nv_bfloat16* o = (t == 0 ? qo : (t == 1 ? ko : vo)) + (n * nh + hd) * DP;
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    float f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = x[c * 8 + i];
    vstore8(o + c * 8, f);
  }
  for (int c = D; c < DP; c += 8) *reinterpret_cast<uint4*>(o + c) = make_uint4(0u, 0u, 0u, 0u);
}

template <int D>
__global__ void __launch_bounds__(128) vision_rope_bwd_vec_kernel(const __nv_bfloat16* __restrict__ dq,
                                                                  const __nv_bfloat16* __restrict__ dk,
                                                                  const __nv_bfloat16* __restrict__ dv,
                                                                  const float* __restrict__ cosv,
                                                                  const float* __restrict__ sinv,
                                                                  __nv_bfloat16* __restrict__ dqkv, int64_t N, int nh,
                                                                  int DP) {
  constexpr int h = D / 2;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= N * 3 * nh) return;
  const int64_t n = idx / (3 * nh);
  const int rem = static_cast<int>(idx - n * 3 * nh);
  const int t = rem / nh, hd = rem % nh;
  const __nv_bfloat16* src = (t == 0 ? dq : (t == 1 ? dk : dv)) + (n * nh + hd) * DP;
  float x[D];
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    float f[8];
    vload8(src + c * 8, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[c * 8 + i] = f[i];
  }
  if (t < 2) {
    const float* cr = cosv + n * h;
    const float* sr = sinv + n * h;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float c = cr[i], sn = sr[i], a = x[i], b = x[i + h];
      x[i] = a * c + b * sn;
      x[i + h] = b * c - a * sn;
    }
  }
#pragma unroll
  for (int c = 0; c < D / 8; ++c) {
    float f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = x[c * 8 + i];
    vstore8(dqkv + idx * D + c * 8, f);
  }
}

void check_bf16_2d(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.is_contiguous(), what,
              ": expected a contiguous 2-D bf16 CUDA tensor");
}

void check_vec(const torch::Tensor& t, int64_t n, c10::ScalarType st, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == st && t.numel() == n && t.is_contiguous(), what,
              ": bad vector (dtype, size or layout)");
}

void launch_colsum(const torch::Tensor& part, int G, int n, int ld, int64_t col0, torch::Tensor& out, bool acc) {
  colsum_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      part.data_ptr<float>() + col0, G, n, ld, out.data_ptr<float>(), acc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int num_sms(const torch::Tensor& t) {
  return at::cuda::getDeviceProperties(t.device().index())->multiProcessorCount;
}

}  // namespace
}  // namespace mvp

using namespace mvp;

std::vector<torch::Tensor> layernorm_fwd(const torch::Tensor& x, const torch::Tensor& w, const torch::Tensor& b,
                                         double eps) {
  check_bf16_2d(x, "layernorm_fwd x");
  const int64_t rows = x.size(0), H = x.size(1);
  check_vec(w, H, at::kBFloat16, "layernorm_fwd w");
  check_vec(b, H, at::kBFloat16, "layernorm_fwd b");
  TORCH_CHECK(H % 8 == 0 && rows <= 0x7fffffff, "layernorm_fwd: H must be a multiple of 8");
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  auto mean = torch::empty({rows}, x.options().dtype(at::kFloat));
  auto rstd = torch::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, mean, rstd};
  const int grid = static_cast<int>((rows + kLnWarps - 1) / kLnWarps);
  layernorm_fwd_kernel<<<grid, kLnWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
      mean.data_ptr<float>(), rstd.data_ptr<float>(), static_cast<int>(rows), static_cast<int>(H),
      static_cast<float>(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, mean, rstd};
}

// Returns (dx, dw, db).  With dw_acc / db_acc (fp32, H) the sums are added there instead and the
// returned dw / db alias them.
std::vector<torch::Tensor> layernorm_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& mean,
                                         const torch::Tensor& rstd, const torch::Tensor& w,
                                         const c10::optional<torch::Tensor>& dw_acc,
                                         const c10::optional<torch::Tensor>& db_acc) {
  check_bf16_2d(dy, "layernorm_bwd dy");
  check_bf16_2d(x, "layernorm_bwd x");
  const int64_t rows = x.size(0), H = x.size(1);
  TORCH_CHECK(dy.sizes() == x.sizes(), "layernorm_bwd: dy / x shapes differ");
  check_vec(w, H, at::kBFloat16, "layernorm_bwd w");
  check_vec(mean, rows, at::kFloat, "layernorm_bwd mean");
  check_vec(rstd, rows, at::kFloat, "layernorm_bwd rstd");
  TORCH_CHECK(H % 8 == 0 && 2 * H * 4 <= 200 * 1024, "layernorm_bwd: H must be a multiple of 8 and <= 25600");
  const at::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  torch::Tensor dw, db;
  if (dw_acc.has_value()) {
    check_vec(*dw_acc, H, at::kFloat, "layernorm_bwd dw_acc");
    dw = *dw_acc;
  } else {
    dw = torch::empty({H}, x.options().dtype(at::kFloat));
  }
  if (db_acc.has_value()) {
    check_vec(*db_acc, H, at::kFloat, "layernorm_bwd db_acc");
    db = *db_acc;
  } else {
    db = torch::empty({H}, x.options().dtype(at::kFloat));
  }
  if (rows == 0) {
    if (!dw_acc.has_value()) dw.zero_();
    if (!db_acc.has_value()) db.zero_();
    return {dx, dw, db};
  }
  // warps per CTA: as many private 2H-float regions as fit in ~100 KB (two CTAs per SM), 1..8
  const int64_t region = 2 * H * static_cast<int64_t>(sizeof(float));
  const int warps = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(8, (100 * 1024) / region)));
  const int64_t want = (rows + warps - 1) / warps;
  const int G = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(num_sms(x)) * 2));
  auto part = torch::empty({G, 2 * H}, x.options().dtype(at::kFloat));
  const size_t smem = static_cast<size_t>(region) * warps;
  if (smem > 48 * 1024)
    C10_CUDA_CHECK(cudaFuncSetAttribute(layernorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
  auto stream = at::cuda::getCurrentCUDAStream();
  layernorm_bwd_kernel<<<G, warps * 32, smem, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      mean.data_ptr<float>(), rstd.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), part.data_ptr<float>(), static_cast<int>(rows),
      static_cast<int>(H));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  launch_colsum(part, G, static_cast<int>(H), static_cast<int>(2 * H), 0, dw, dw_acc.has_value());
  launch_colsum(part, G, static_cast<int>(H), static_cast<int>(2 * H), H, db, db_acc.has_value());
  return {dx, dw, db};
}

torch::Tensor bias_gelu_fwd(const torch::Tensor& x, const torch::Tensor& b, bool tanh_form) {
  check_bf16_2d(x, "bias_gelu_fwd x");
  const int64_t rows = x.size(0), F = x.size(1);
  check_vec(b, F, at::kBFloat16, "bias_gelu_fwd b");
  TORCH_CHECK(F % 8 == 0 && rows <= 0x7fffffff, "bias_gelu: F must be a multiple of 8");
  const at::cuda::CUDAGuard guard(x.device());
  auto y = torch::empty_like(x);
  if (rows == 0) return y;
  const dim3 grid(static_cast<unsigned>((F / 8 + 127) / 128), static_cast<unsigned>(std::min<int64_t>(rows, 65535)));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto bp = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (tanh_form)
    bias_gelu_fwd_kernel<true><<<grid, 128, 0, stream>>>(xp, bp, yp, static_cast<int>(rows), static_cast<int>(F));
  else
    bias_gelu_fwd_kernel<false><<<grid, 128, 0, stream>>>(xp, bp, yp, static_cast<int>(rows), static_cast<int>(F));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return y;
}

// Returns (dx, db); with db_acc (fp32, F) the bias gradient is added there and db aliases it.
std::vector<torch::Tensor> bias_gelu_bwd(const torch::Tensor& dy, const torch::Tensor& x, const torch::Tensor& b,
                                         bool tanh_form, const c10::optional<torch::Tensor>& db_acc) {
  check_bf16_2d(dy, "bias_gelu_bwd dy");
  check_bf16_2d(x, "bias_gelu_bwd x");
  TORCH_CHECK(dy.sizes() == x.sizes(), "bias_gelu_bwd: dy / x shapes differ");
  const int64_t rows = x.size(0), F = x.size(1);
  check_vec(b, F, at::kBFloat16, "bias_gelu_bwd b");
  TORCH_CHECK(F % 8 == 0 && rows <= 0x7fffffff, "bias_gelu: F must be a multiple of 8");
  const at::cuda::CUDAGuard guard(x.device());
  auto dx = torch::empty_like(x);
  torch::Tensor db;
  if (db_acc.has_value()) {
    check_vec(*db_acc, F, at::kFloat, "bias_gelu_bwd db_acc");
    db = *db_acc;
  } else {
    db = torch::empty({F}, x.options().dtype(at::kFloat));
  }
  if (rows == 0) {
    if (!db_acc.has_value()) db.zero_();
    return {dx, db};
  }
  const int col_blocks = static_cast<int>((F / 8 + 127) / 128);
  // enough row groups for ~8 CTAs per SM, each group a few dozen rows at least
  const int64_t want = std::max<int64_t>(1, static_cast<int64_t>(num_sms(x)) * 16 / col_blocks);
  const int G = static_cast<int>(std::min<int64_t>({rows, want, 65535}));
  auto part = torch::empty({G, F}, x.options().dtype(at::kFloat));
  const dim3 grid(static_cast<unsigned>(col_blocks), static_cast<unsigned>(G));
  auto stream = at::cuda::getCurrentCUDAStream();
  auto gp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto bp = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr());
  auto dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  if (tanh_form)
    bias_gelu_bwd_kernel<true><<<grid, 128, 0, stream>>>(gp, xp, bp, dxp, part.data_ptr<float>(),
                                                         static_cast<int>(rows), static_cast<int>(F));
  else
    bias_gelu_bwd_kernel<false><<<grid, 128, 0, stream>>>(gp, xp, bp, dxp, part.data_ptr<float>(),
                                                          static_cast<int>(rows), static_cast<int>(F));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  launch_colsum(part, G, static_cast<int>(F), static_cast<int>(F), 0, db, db_acc.has_value());
  return {dx, db};
}

torch::Tensor bias_residual_fwd(const torch::Tensor& y, const torch::Tensor& b, const torch::Tensor& x) {
  check_bf16_2d(y, "bias_residual_fwd y");
  check_bf16_2d(x, "bias_residual_fwd x");
  TORCH_CHECK(y.sizes() == x.sizes(), "bias_residual_fwd: y / x shapes differ");
  const int64_t rows = y.size(0), F = y.size(1);
  check_vec(b, F, at::kBFloat16, "bias_residual_fwd b");
  TORCH_CHECK(F % 8 == 0 && rows <= 0x7fffffff, "bias_residual: F must be a multiple of 8");
  const at::cuda::CUDAGuard guard(y.device());
  auto out = torch::empty_like(y);
  if (rows == 0) return out;
  const dim3 grid(static_cast<unsigned>((F / 8 + 127) / 128), static_cast<unsigned>(std::min<int64_t>(rows, 65535)));
  bias_residual_fwd_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      static_cast<int>(rows), static_cast<int>(F));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Column sums of g [rows, F] in fp32 (a bias gradient); with acc (fp32, F) they are added there.
torch::Tensor bias_grad(const torch::Tensor& g, const c10::optional<torch::Tensor>& acc) {
  check_bf16_2d(g, "bias_grad g");
  const int64_t rows = g.size(0), F = g.size(1);
  TORCH_CHECK(F % 8 == 0 && rows <= 0x7fffffff, "bias_grad: F must be a multiple of 8");
  const at::cuda::CUDAGuard guard(g.device());
  torch::Tensor db;
  if (acc.has_value()) {
    check_vec(*acc, F, at::kFloat, "bias_grad acc");
    db = *acc;
  } else {
    db = torch::empty({F}, g.options().dtype(at::kFloat));
  }
  if (rows == 0) {
    if (!acc.has_value()) db.zero_();
    return db;
  }
  const int col_blocks = static_cast<int>((F / 8 + 127) / 128);
  // few row groups: the column-sum pass over the partials is one thread per column
  const int64_t want = std::max<int64_t>(1, static_cast<int64_t>(num_sms(g)) * 4 / col_blocks);
  const int G = static_cast<int>(std::min<int64_t>({rows, want, 65535}));
  auto part = torch::empty({G, F}, g.options().dtype(at::kFloat));
  col_partial_kernel<<<dim3(static_cast<unsigned>(col_blocks), static_cast<unsigned>(G)), 128, 0,
                       at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
                                                           part.data_ptr<float>(), static_cast<int>(rows),
                                                           static_cast<int>(F));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  launch_colsum(part, G, static_cast<int>(F), static_cast<int>(F), 0, db, acc.has_value());
  return db;
}

// Returns (q, k, v), each [N, nh, DP] bf16 with the head columns past D zero.
std::vector<torch::Tensor> vision_rope_fwd(const torch::Tensor& qkv, int64_t nh, const torch::Tensor& cosv,
                                           const torch::Tensor& sinv, int64_t DP,
                                           const c10::optional<torch::Tensor>& bias) {
  check_bf16_2d(qkv, "vision_rope_fwd qkv");
  const int64_t N = qkv.size(0);
  TORCH_CHECK(nh > 0 && qkv.size(1) % (3 * nh) == 0, "vision_rope_fwd: qkv width is not 3 * nh * D");
  const int64_t D = qkv.size(1) / (3 * nh);
  TORCH_CHECK(D % 2 == 0 && D <= DP, "vision_rope_fwd: D must be even and <= DP");
  check_vec(cosv, N * (D / 2), at::kFloat, "vision_rope_fwd cos");
  check_vec(sinv, N * (D / 2), at::kFloat, "vision_rope_fwd sin");
  const __nv_bfloat16* bp = nullptr;
  if (bias.has_value()) {
    check_vec(*bias, 3 * nh * D, at::kBFloat16, "vision_rope_fwd bias");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(bias->data_ptr()) % 16 == 0, "vision_rope_fwd: 16-byte aligned bias");
    bp = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  const at::cuda::CUDAGuard guard(qkv.device());
  auto q = torch::empty({N, nh, DP}, qkv.options());
  auto k = torch::empty_like(q);
  auto v = torch::empty_like(q);
  if (N == 0) return {q, k, v};
  const bool vec = DP % 8 == 0 && reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0;
  if (vec && (D == 64 || D == 72)) {
    const int64_t rows = N * 3 * nh;
    TORCH_CHECK((rows + 127) / 128 <= 0x7fffffff, "vision_rope_fwd: too many rows");
    const unsigned grid = static_cast<unsigned>((rows + 127) / 128);
    const auto* src = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
    auto* qp = reinterpret_cast<__nv_bfloat16*>(q.data_ptr());
    auto* kp = reinterpret_cast<__nv_bfloat16*>(k.data_ptr());
    auto* vp = reinterpret_cast<__nv_bfloat16*>(v.data_ptr());
    auto stream = at::cuda::getCurrentCUDAStream();
    const int nhi = static_cast<int>(nh), dpi = static_cast<int>(DP);
    if (D == 64)
      vision_rope_fwd_vec_kernel<64><<<grid, 128, 0, stream>>>(src, cosv.data_ptr<float>(), sinv.data_ptr<float>(),
                                                               qp, kp, vp, N, nhi, dpi, bp);
    else
      vision_rope_fwd_vec_kernel<72><<<grid, 128, 0, stream>>>(src, cosv.data_ptr<float>(), sinv.data_ptr<float>(),
                                                               qp, kp, vp, N, nhi, dpi, bp);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {q, k, v};
  }
  const int64_t threads = N * nh * 32;
  TORCH_CHECK((threads + 255) / 256 <= 0x7fffffff, "vision_rope_fwd: too many rows");
  vision_rope_fwd_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), cosv.data_ptr<float>(), sinv.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(q.data_ptr()), reinterpret_cast<__nv_bfloat16*>(k.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(v.data_ptr()), N, static_cast<int>(nh), static_cast<int>(D),
      static_cast<int>(DP), bp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {q, k, v};
}

torch::Tensor vision_rope_bwd(const torch::Tensor& dq, const torch::Tensor& dk, const torch::Tensor& dv,
                              const torch::Tensor& cosv, const torch::Tensor& sinv, int64_t D) {
  for (const auto* t : {&dq, &dk, &dv})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 3 && t->is_contiguous() &&
                    t->sizes() == dq.sizes(),
                "vision_rope_bwd: dq / dk / dv must be contiguous bf16 [N, nh, DP] of one shape");
  const int64_t N = dq.size(0), nh = dq.size(1), DP = dq.size(2);
  TORCH_CHECK(D % 2 == 0 && D <= DP, "vision_rope_bwd: D must be even and <= DP");
  check_vec(cosv, N * (D / 2), at::kFloat, "vision_rope_bwd cos");
  check_vec(sinv, N * (D / 2), at::kFloat, "vision_rope_bwd sin");
  const at::cuda::CUDAGuard guard(dq.device());
  auto dqkv = torch::empty({N, 3 * nh * D}, dq.options());
  if (N == 0) return dqkv;
  const bool vec = DP % 8 == 0 && reinterpret_cast<uintptr_t>(dq.data_ptr()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(dk.data_ptr()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(dv.data_ptr()) % 16 == 0;
  if (vec && (D == 64 || D == 72)) {
    const int64_t rows = N * 3 * nh;
    TORCH_CHECK((rows + 127) / 128 <= 0x7fffffff, "vision_rope_bwd: too many rows");
    const unsigned grid = static_cast<unsigned>((rows + 127) / 128);
    const auto* a = reinterpret_cast<const __nv_bfloat16*>(dq.data_ptr());
    const auto* b = reinterpret_cast<const __nv_bfloat16*>(dk.data_ptr());
    const auto* c = reinterpret_cast<const __nv_bfloat16*>(dv.data_ptr());
    auto* o = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
    auto stream = at::cuda::getCurrentCUDAStream();
    const int nhi = static_cast<int>(nh), dpi = static_cast<int>(DP);
    if (D == 64)
      vision_rope_bwd_vec_kernel<64><<<grid, 128, 0, stream>>>(a, b, c, cosv.data_ptr<float>(), sinv.data_ptr<float>(),
                                                               o, N, nhi, dpi);
    else
      vision_rope_bwd_vec_kernel<72><<<grid, 128, 0, stream>>>(a, b, c, cosv.data_ptr<float>(), sinv.data_ptr<float>(),
                                                               o, N, nhi, dpi);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return dqkv;
  }
  const int64_t threads = N * nh * 32;
  vision_rope_bwd_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dq.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dk.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(dv.data_ptr()), cosv.data_ptr<float>(), sinv.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), N, static_cast<int>(nh), static_cast<int>(D),
      static_cast<int>(DP));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}
