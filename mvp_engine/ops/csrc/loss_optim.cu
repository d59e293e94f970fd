// Token cross-entropy over a vocabulary chunk of logits, the flat-buffer
// AdamW update (with the token-normalisation scale and the global-norm clip
// folded in), sum-of-squares for grad-norm clipping, and the embedding
// gather / scatter-add.  All sm_100a, bandwidth-bound.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace mvp {
namespace {

constexpr int kIgnoreIndex = -100;

template <int THREADS>
__device__ __forceinline__ void block_max_sum(float& m, float& s) {
  // Merge (max, sum-of-exp) pairs across the block.
  __shared__ float sm[THREADS / 32], ss[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < THREADS / 32 ? sm[lane] : -INFINITY;
    s = lane < THREADS / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (lane == 0) {
      sm[0] = m;
      ss[0] = s;
    }
  }
  __syncthreads();
  m = sm[0];
  s = ss[0];
}

// One block per row.  loss[i] = logsumexp(x_i) - x_i[label_i] (0 if ignored).
template <int THREADS>
__global__ void __launch_bounds__(THREADS) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                                                         const int64_t* __restrict__ labels, float* __restrict__ loss,
                                                         float* __restrict__ lse) {
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + static_cast<int64_t>(row) * ld;
  float m = -INFINITY, s = 0.f;
  const int V8 = V / 8;
  for (int i = threadIdx.x; i < V8; i += THREADS) {
    const uint4 u = reinterpret_cast<const uint4*>(x)[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(h[j]);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
    float lm = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, f[j]);
    const float nm = fmaxf(m, lm);
    float acc = (m == -INFINITY) ? 0.f : s * __expf(m - nm);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += __expf(f[j] - nm);
    s = acc;
    m = nm;
  }
  for (int i = V8 * 8 + threadIdx.x; i < V; i += THREADS) {
    const float f = __bfloat162float(x[i]);
    const float nm = fmaxf(m, f);
    s = ((m == -INFINITY) ? 0.f : s * __expf(m - nm)) + __expf(f - nm);
    m = nm;
  }
  block_max_sum<THREADS>(m, s);
  if (threadIdx.x == 0) {
    const float l = m + logf(s);
    lse[row] = l;
    const int64_t lab = labels[row];
    loss[row] = (lab == kIgnoreIndex || lab < 0 || lab >= V) ? 0.f : l - __bfloat162float(x[lab]);
  }
}

// In place: x_i <- g_i * (softmax(x_i) - onehot(label_i)); zero rows for ignored labels.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) ce_bwd_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, int V,
                                                         const int64_t* __restrict__ labels,
                                                         const float* __restrict__ lse, const float* __restrict__ g,
                                                         int64_t g_stride) {
  const int row = blockIdx.x;
  __nv_bfloat16* x = logits + static_cast<int64_t>(row) * ld;
  const int64_t lab = labels[row];
  const bool ignored = (lab == kIgnoreIndex || lab < 0 || lab >= V);
  const float gi = ignored ? 0.f : g[row * g_stride];
  const float l = lse[row];
  const int V8 = V / 8;
  for (int i = threadIdx.x; i < V8; i += THREADS) {
    uint4 u = reinterpret_cast<uint4*>(x)[i];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(h[j]);
      const int c = i * 8 + 2 * j;
      float a = __expf(t.x - l) - (c == lab ? 1.f : 0.f);
      float b = __expf(t.y - l) - (c + 1 == lab ? 1.f : 0.f);
      h[j] = __floats2bfloat162_rn(gi * a, gi * b);
    }
    reinterpret_cast<uint4*>(x)[i] = u;
  }
  for (int i = V8 * 8 + threadIdx.x; i < V; i += THREADS) {
    const float f = __bfloat162float(x[i]);
    x[i] = __float2bfloat16_rn(gi * (__expf(f - l) - (i == lab ? 1.f : 0.f)));
  }
}

// --------------------------------------------------------------- AdamW
struct AdamWArgs {
  float* p;
  const float* g;
  float* m;
  float* v;
  __nv_bfloat16* p_bf16;  // optional shadow copy for the next forward
  int64_t n;
  float lr, beta1, beta2, eps, wd;
  float bc1, bc2_sqrt;
  float grad_scale;
  const float* norm_sq;  // optional: sum of squares of the unscaled grads (global)
  float max_norm;
};

__global__ void adamw_kernel(AdamWArgs a) {
  float scale = a.grad_scale;
  if (a.norm_sq != nullptr) {
    const float total = sqrtf(*a.norm_sq) * a.grad_scale;
    const float coef = a.max_norm / (total + 1e-6f);
    scale *= fminf(coef, 1.f);
  }
  const float step_size = a.lr / a.bc1;
  const float decay = 1.f - a.lr * a.wd;
  const int64_t n4 = a.n / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 p = reinterpret_cast<float4*>(a.p)[i];
    const float4 g4 = reinterpret_cast<const float4*>(a.g)[i];
    float4 m = reinterpret_cast<float4*>(a.m)[i];
    float4 v = reinterpret_cast<float4*>(a.v)[i];
    float* pp = &p.x;
    const float* gg = &g4.x;
    float* mm = &m.x;
    float* vv = &v.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g = gg[j] * scale;
      pp[j] *= decay;
      mm[j] = mm[j] + (1.f - a.beta1) * (g - mm[j]);
      vv[j] = vv[j] * a.beta2 + (1.f - a.beta2) * g * g;
      const float denom = sqrtf(vv[j]) / a.bc2_sqrt + a.eps;
      pp[j] -= step_size * mm[j] / denom;
    }
    reinterpret_cast<float4*>(a.p)[i] = p;
    reinterpret_cast<float4*>(a.m)[i] = m;
    reinterpret_cast<float4*>(a.v)[i] = v;
    if (a.p_bf16 != nullptr) {
      uint2 u;
      u.x = pack_bf16x2(p.x, p.y);
      u.y = pack_bf16x2(p.z, p.w);
      reinterpret_cast<uint2*>(a.p_bf16)[i] = u;
    }
  }
  for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < a.n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float g = a.g[i] * scale;
    float p = a.p[i] * decay;
    const float m = a.m[i] + (1.f - a.beta1) * (g - a.m[i]);
    const float v = a.v[i] * a.beta2 + (1.f - a.beta2) * g * g;
    p -= step_size * m / (sqrtf(v) / a.bc2_sqrt + a.eps);
    a.p[i] = p;
    a.m[i] = m;
    a.v[i] = v;
    if (a.p_bf16 != nullptr) a.p_bf16[i] = __float2bfloat16_rn(p);
  }
}

// Deterministic two-level sum of squares: per-block partials, summed on host side by torch.
template <typename T>
__global__ void sumsq_kernel(const T* __restrict__ x, int64_t n, float* __restrict__ partial) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = static_cast<float>(x[i]);
    s += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) partial[blockIdx.x] = s;
  }
}

// ----------------------------------------------------------- embedding
// Out-of-range ids read as zero rows and set the status word (kBadArgument).
__global__ void embedding_fwd_kernel(const __nv_bfloat16* __restrict__ w, const int64_t* __restrict__ ids,
                                     __nv_bfloat16* __restrict__ out, int64_t T, int H, int64_t V, int* status) {
  const int H8 = H / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < T * H8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / H8;
    const int c = static_cast<int>(i % H8);
    const int64_t id = ids[t];
    if (id < 0 || id >= V) {
      reinterpret_cast<uint4*>(out + t * H)[c] = make_uint4(0u, 0u, 0u, 0u);
      if (c == 0) record_status(status, kBadArgument);
      continue;
    }
    reinterpret_cast<uint4*>(out + t * H)[c] = reinterpret_cast<const uint4*>(w + id * H)[c];
  }
}

__global__ void embedding_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const int64_t* __restrict__ ids,
                                     float* __restrict__ dw, int64_t T, int H, int64_t V) {
  const int H4 = H / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < T * H4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / H4;
    const int c = static_cast<int>(i % H4);
    if (ids[t] < 0 || ids[t] >= V) continue;
    const uint2 u = reinterpret_cast<const uint2*>(dout + t * H)[c];
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    atomicAdd(reinterpret_cast<float4*>(dw + ids[t] * H) + c, make_float4(a.x, a.y, b.x, b.y));
  }
}

inline int grid_for(int64_t n, int threads) {
  const int64_t g = (n + threads - 1) / threads;
  return static_cast<int>(std::min<int64_t>(std::max<int64_t>(g, 1), 148 * 8));
}

}  // namespace
}  // namespace mvp

std::vector<torch::Tensor> ce_fwd(const torch::Tensor& logits, const torch::Tensor& labels) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "ce_fwd: bf16 logits, unit col stride");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "ce_fwd: int64 labels");
  TORCH_CHECK(logits.stride(0) % 8 == 0, "ce_fwd: row stride must be a multiple of 8");
  const int rows = static_cast<int>(logits.size(0));
  const int V = static_cast<int>(logits.size(1));
  const at::cuda::CUDAGuard guard(logits.device());
  auto loss = torch::empty({rows}, logits.options().dtype(at::kFloat));
  auto lse = torch::empty({rows}, logits.options().dtype(at::kFloat));
  if (rows == 0) return {loss, lse};
  mvp::ce_fwd_kernel<512><<<rows, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), V, labels.data_ptr<int64_t>(),
      loss.data_ptr<float>(), lse.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {loss, lse};
}

void ce_bwd_(torch::Tensor& logits, const torch::Tensor& labels, const torch::Tensor& lse, const torch::Tensor& g) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "ce_bwd: bf16 logits");
  TORCH_CHECK(g.scalar_type() == at::kFloat, "ce_bwd: fp32 grad");
  const int rows = static_cast<int>(logits.size(0));
  if (rows == 0) return;
  const at::cuda::CUDAGuard guard(logits.device());
  mvp::ce_bwd_kernel<512><<<rows, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), logits.stride(0), static_cast<int>(logits.size(1)),
      labels.data_ptr<int64_t>(), lse.data_ptr<float>(), g.data_ptr<float>(), g.numel() == 1 ? 0 : g.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw_step_(torch::Tensor& p, const torch::Tensor& g, torch::Tensor& m, torch::Tensor& v,
                 const c10::optional<torch::Tensor>& p_bf16, double lr, double beta1, double beta2, double eps,
                 double wd, int64_t step, double grad_scale, const c10::optional<torch::Tensor>& norm_sq,
                 double max_norm) {
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat &&
                  v.scalar_type() == at::kFloat,
              "adamw: fp32 state");
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  TORCH_CHECK(p.numel() == g.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "adamw: sizes");
  const at::cuda::CUDAGuard guard(p.device());
  mvp::AdamWArgs a;
  a.p = p.data_ptr<float>();
  a.g = g.data_ptr<float>();
  a.m = m.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.p_bf16 = nullptr;
  if (p_bf16.has_value()) {
    TORCH_CHECK(p_bf16->scalar_type() == at::kBFloat16 && p_bf16->numel() == p.numel() && p_bf16->is_contiguous(),
                "adamw: bf16 shadow");
    a.p_bf16 = reinterpret_cast<__nv_bfloat16*>(p_bf16->data_ptr());
  }
  a.n = p.numel();
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.wd = static_cast<float>(wd);
  a.bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  a.bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  a.grad_scale = static_cast<float>(grad_scale);
  a.norm_sq = norm_sq.has_value() ? norm_sq->data_ptr<float>() : nullptr;
  a.max_norm = static_cast<float>(max_norm);
  if (a.n == 0) return;
  mvp::adamw_kernel<<<mvp::grid_for((a.n + 3) / 4, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

torch::Tensor sumsq(const torch::Tensor& x) {
  TORCH_CHECK(x.is_contiguous(), "sumsq: contiguous");
  const at::cuda::CUDAGuard guard(x.device());
  const int blocks = 148 * 4;
  auto partial = torch::zeros({blocks}, x.options().dtype(at::kFloat));
  if (x.numel() > 0) {
    if (x.scalar_type() == at::kFloat)
      mvp::sumsq_kernel<float><<<blocks, 512, 0, at::cuda::getCurrentCUDAStream()>>>(x.data_ptr<float>(), x.numel(),
                                                                                     partial.data_ptr<float>());
    else {
      TORCH_CHECK(x.scalar_type() == at::kBFloat16, "sumsq: fp32 or bf16");
      mvp::sumsq_kernel<__nv_bfloat16><<<blocks, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.numel(), partial.data_ptr<float>());
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return partial.sum();
}

torch::Tensor embedding_fwd(const torch::Tensor& w, const torch::Tensor& ids, int64_t status_ptr) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.is_contiguous(), "embedding: bf16 weight");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "embedding: int64 ids");
  const int H = static_cast<int>(w.size(1));
  TORCH_CHECK(H % 8 == 0, "embedding: H % 8");
  const int64_t T = ids.numel();
  const at::cuda::CUDAGuard guard(w.device());
  auto out = torch::empty({T, H}, w.options());
  if (T > 0) {
    mvp::embedding_fwd_kernel<<<mvp::grid_for(T * H / 8, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), ids.data_ptr<int64_t>(),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, H, w.size(0), reinterpret_cast<int*>(status_ptr));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return out;
}

void embedding_bwd_(torch::Tensor& dw, const torch::Tensor& dout, const torch::Tensor& ids) {
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous(), "embedding_bwd: fp32 grad");
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && dout.is_contiguous(), "embedding_bwd: bf16 dout");
  const int H = static_cast<int>(dw.size(1));
  const int64_t T = ids.numel();
  const at::cuda::CUDAGuard guard(dw.device());
  if (T == 0) return;
  mvp::embedding_bwd_kernel<<<mvp::grid_for(T * H / 4, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), ids.data_ptr<int64_t>(), dw.data_ptr<float>(), T, H,
      dw.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
