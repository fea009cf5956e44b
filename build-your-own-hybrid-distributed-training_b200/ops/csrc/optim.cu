// Fused AdamW over flat fp32 buffers and the weighted gradient sum of squares.
//
// AdamW (decoupled weight decay, bias-corrected moments, PyTorch's update order):
//   p *= 1 - lr * wd
//   m  = lerp(m, g, 1 - beta1);  v = beta2 * v + (1 - beta2) * g^2
//   p -= (lr / (1 - beta1^t)) * m / (sqrt(v) / sqrt(1 - beta2^t) + eps)
// with g = grad * grad_scale.  lr, t, grad_scale and a skip flag come from a device vector so a
// captured CUDA graph replays with the current schedule.  One read and one write per element of
// each buffer, plus the bf16 compute copy of the parameter in the same pass.

#include "common.cuh"

namespace ht {
namespace opt {

__global__ void adamw_kernel(float4* __restrict__ param, const float4* __restrict__ grad, float4* __restrict__ m,
                             float4* __restrict__ v, uint2* __restrict__ copy16, const float* __restrict__ hyper, long long n4,
                             float beta1, float beta2, float eps, float wd) {
  if (hyper[3] != 0.f) return;
  const float lr = hyper[0], t = hyper[1], gs = hyper[2];
  const float bc1 = 1.f - powf(beta1, t);
  const float bc2_sqrt = sqrtf(1.f - powf(beta2, t));
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    if (!HT_IN_BOUNDS(i, n4, 20)) continue;
    float4 p = param[i], g = grad[i], mm = m[i], vv = v[i];
    float* pp = reinterpret_cast<float*>(&p);
    const float* gg = reinterpret_cast<const float*>(&g);
    float* ma = reinterpret_cast<float*>(&mm);
    float* va = reinterpret_cast<float*>(&vv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = gg[j] * gs;
      ma[j] = ma[j] + (1.f - beta1) * (gj - ma[j]);
      va[j] = beta2 * va[j] + (1.f - beta2) * gj * gj;
      const float denom = sqrtf(va[j]) / bc2_sqrt + eps;
      pp[j] = pp[j] * decay - step * ma[j] / denom;
    }
    param[i] = p;
    m[i] = mm;
    v[i] = vv;
    if (copy16 != nullptr) {
      __align__(8) __nv_bfloat16 b[4] = {f2bf(pp[0]), f2bf(pp[1]), f2bf(pp[2]), f2bf(pp[3])};
      copy16[i] = *reinterpret_cast<uint2*>(b);
    }
  }
}

// The same update in a small footprint, for slices updated while the backward pass runs: one block
// of 128 threads per SM (at most 80 registers each, no shared memory) fits next to a resident
// persistent GEMM CTA, so the update streams through memory without waiting for the GEMM to end.
// Each thread keeps two 16-byte vectors of each buffer in flight.
constexpr int RESIDENT_THREADS = 128;

__global__ void __launch_bounds__(RESIDENT_THREADS, 6)
    adamw_resident_kernel(float4* __restrict__ param, const float4* __restrict__ grad, float4* __restrict__ m,
                          float4* __restrict__ v, uint2* __restrict__ copy16, const float* __restrict__ hyper, long long n4,
                          float beta1, float beta2, float eps, float wd) {
  if (hyper[3] != 0.f) return;
  const float lr = hyper[0], t = hyper[1], gs = hyper[2];
  const float bc1 = 1.f - powf(beta1, t);
  const float bc2_sqrt = sqrtf(1.f - powf(beta2, t));
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  constexpr int U = 2;
  const long long stride = (long long)gridDim.x * RESIDENT_THREADS;
  for (long long i0 = blockIdx.x * (long long)RESIDENT_THREADS + threadIdx.x; i0 < n4; i0 += stride * U) {
    float4 p[U], g[U], mm[U], vv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * stride;
      if (i < n4 && HT_IN_BOUNDS(i, n4, 21)) {
        p[u] = param[i];
        g[u] = grad[i];
        mm[u] = m[i];
        vv[u] = v[i];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * stride;
      if (i >= n4) continue;
      float* pp = reinterpret_cast<float*>(&p[u]);
      const float* gg = reinterpret_cast<const float*>(&g[u]);
      float* ma = reinterpret_cast<float*>(&mm[u]);
      float* va = reinterpret_cast<float*>(&vv[u]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gj = gg[j] * gs;
        ma[j] = ma[j] + (1.f - beta1) * (gj - ma[j]);
        va[j] = beta2 * va[j] + (1.f - beta2) * gj * gj;
        const float denom = sqrtf(va[j]) / bc2_sqrt + eps;
        pp[j] = pp[j] * decay - step * ma[j] / denom;
      }
      param[i] = p[u];
      m[i] = mm[u];
      v[i] = vv[u];
      if (copy16 != nullptr) {
        __align__(8) __nv_bfloat16 b[4] = {f2bf(pp[0]), f2bf(pp[1]), f2bf(pp[2]), f2bf(pp[3])};
        copy16[i] = *reinterpret_cast<uint2*>(b);
      }
    }
  }
}

__global__ void sumsq_kernel(const float* __restrict__ g, const float* __restrict__ w, float* __restrict__ out, long long n,
                             float scale) {
  __shared__ float scratch[32];
  float s = 0.f;
  int bad = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float x = g[i];
    bad |= !isfinite(x);
    s += (w != nullptr ? w[i] : 1.f) * x * x;
  }
  s = block_sum(s, scratch);
  const int any_bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    atomicAdd(out, s * scale);
    if (any_bad) out[1] = 1.f;
  }
}

}  // namespace opt

void adamw_flat(at::Tensor param, at::Tensor grad, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> copy, at::Tensor hyper,
                double beta1, double beta2, double eps, double wd, bool resident) {
  const c10::cuda::CUDAGuard guard(param.device());
  for (const at::Tensor* t : {&param, &grad, &m, &v})
    HT_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == param.numel(), "adamw buffers: fp32, same size");
  HT_CHECK(param.numel() % 4 == 0, "flat buffers must hold a multiple of 4 elements");
  uint2* c16 = nullptr;
  if (copy.has_value() && copy->defined()) {
    HT_CHECK(copy->scalar_type() == at::kBFloat16 && copy->numel() == param.numel() && copy->is_contiguous(), "bf16 copy size");
    c16 = reinterpret_cast<uint2*>(copy->data_ptr());
  }
  const long long n4 = param.numel() / 4;
  if (n4 == 0) return;
  for (const at::Tensor* t : {&param, &grad, &m, &v})
    HT_CHECK((reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0, "adamw buffers must start on a 16-byte boundary");
  if (resident) {
    static bool configured = false;
    if (!configured) {
      HT_CUDA_CHECK(cudaFuncSetAttribute(opt::adamw_resident_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         cudaSharedmemCarveoutMaxShared));
      configured = true;
    }
    const int grid = (int)std::max<long long>(1, std::min<long long>((n4 + opt::RESIDENT_THREADS * 2 - 1) /
                                                                         (opt::RESIDENT_THREADS * 2), num_sms()));
    opt::adamw_resident_kernel<<<grid, opt::RESIDENT_THREADS, 0, stream()>>>(
        reinterpret_cast<float4*>(param.data_ptr()), reinterpret_cast<const float4*>(grad.data_ptr()),
        reinterpret_cast<float4*>(m.data_ptr()), reinterpret_cast<float4*>(v.data_ptr()), c16, hyper.data_ptr<float>(), n4,
        (float)beta1, (float)beta2, (float)eps, (float)wd);
    HT_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int threads = 256;
  const int grid = (int)std::min<long long>((n4 + threads - 1) / threads, (long long)num_sms() * 8);
  opt::adamw_kernel<<<grid, threads, 0, stream()>>>(reinterpret_cast<float4*>(param.data_ptr()),
                                                    reinterpret_cast<const float4*>(grad.data_ptr()),
                                                    reinterpret_cast<float4*>(m.data_ptr()), reinterpret_cast<float4*>(v.data_ptr()),
                                                    c16, hyper.data_ptr<float>(), n4, (float)beta1, (float)beta2, (float)eps, (float)wd);
  HT_CUDA_CHECK(cudaGetLastError());
}

void grad_sumsq(at::Tensor g, c10::optional<at::Tensor> w, at::Tensor out, double scale) {
  const c10::cuda::CUDAGuard guard(g.device());
  HT_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && out.scalar_type() == at::kFloat && out.numel() >= 2, "sumsq args");
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    HT_CHECK(w->scalar_type() == at::kFloat && w->numel() == g.numel(), "weights must match the gradient");
    wp = w->data_ptr<float>();
  }
  const long long n = g.numel();
  if (n == 0) return;
  const int threads = 512;
  const int grid = (int)std::min<long long>((n + threads - 1) / threads, (long long)num_sms() * 4);
  opt::sumsq_kernel<<<grid, threads, 0, stream()>>>(g.data_ptr<float>(), wp, out.data_ptr<float>(), n, (float)scale);
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
