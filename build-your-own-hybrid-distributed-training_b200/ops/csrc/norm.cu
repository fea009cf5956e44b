// Fused residual-add + LayerNorm / RMSNorm, forward and backward.
//
// Forward (one CTA per row, 8 contiguous elements per thread held in registers):
//   r = residual + delta (fp32, written back as the new residual stream)
//   y = (r - mean) * rstd * w + b        (LayerNorm; two-pass mean / variance over registers)
//   y = r * rstd * w                     (RMSNorm)
// Backward (a grid of CTAs strides over rows; each keeps its columns' dw/db partial sums in
// registers and writes one partial row per CTA, reduced by sum_rows):
//   xhat = (r - mean) * rstd, g = dy * w
//   dr_total = rstd * (g - mean(g) - xhat * mean(g * xhat)) + dr_in      (LayerNorm)
//   dr_total = rstd * (g - xhat * mean(g * xhat)) + dr_in                 (RMSNorm)

#include "common.cuh"

namespace ht {
namespace norm {

constexpr int VPT = 8;  // elements per thread

template <typename T>
__device__ __forceinline__ float ld(const T* p, long long i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, long long i) { return p[i]; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, long long i) { return bf2f(p[i]); }

template <typename T>
__device__ __forceinline__ void st(T* p, long long i, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, long long i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, long long i, float v) { p[i] = f2bf(v); }

template <bool RMS, typename DeltaT, typename WT, typename OutT>
__global__ void norm_forward_kernel(const float* __restrict__ res, const DeltaT* __restrict__ delta, const WT* __restrict__ w,
                                    const WT* __restrict__ b, float* __restrict__ r_out, OutT* __restrict__ y,
                                    float* __restrict__ mean_out, float* __restrict__ rstd_out, int d, float eps) {
  __shared__ float scratch[32];
  const long long row = blockIdx.x;
  const long long base = row * d;
  const int c0 = threadIdx.x * VPT;
  float x[VPT];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = c0 + i;
    float v = 0.f;
    if (c < d) {
      v = res[base + c];
      if (delta != nullptr) v += ld(delta, base + c);
      r_out[base + c] = v;
    }
    x[i] = v;
    s += v;
  }
  float mean = 0.f;
  if (!RMS) mean = block_sum(s, scratch) / d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const float t = (c0 + i < d) ? x[i] - mean : 0.f;
    q += t * t;
  }
  const float var = block_sum(q, scratch) / d;
  const float rstd = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = c0 + i;
    if (c < d) {
      float o = (x[i] - mean) * rstd * ld(w, c);
      if (!RMS && b != nullptr) o += ld(b, c);
      st(y, base + c, o);
    }
  }
  if (threadIdx.x == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

template <bool RMS, typename DyT, typename WT, typename DdT>
__global__ void norm_backward_kernel(const DyT* __restrict__ dy, const float* __restrict__ dr_in, const float* __restrict__ r,
                                     const WT* __restrict__ w, const float* __restrict__ mean, const float* __restrict__ rstd,
                                     float* __restrict__ dres, DdT* __restrict__ ddelta, float* __restrict__ part_w,
                                     float* __restrict__ part_b, int rows, int d) {
  __shared__ float scratch[32];
  const int c0 = threadIdx.x * VPT;
  float aw[VPT], ab[VPT], wv[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    aw[i] = ab[i] = 0.f;
    wv[i] = (c0 + i < d) ? ld(w, c0 + i) : 0.f;
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = (long long)row * d;
    const float mu = mean[row], rs = rstd[row];
    float xh[VPT], g[VPT];
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = c0 + i;
      float gy = 0.f, xhat = 0.f;
      if (c < d) {
        xhat = (r[base + c] - mu) * rs;
        gy = dy != nullptr ? ld(dy, base + c) : 0.f;
      }
      xh[i] = xhat;
      g[i] = gy * wv[i];
      aw[i] += gy * xhat;
      ab[i] += gy;
      sg += g[i];
      sgx += g[i] * xhat;
    }
    const float mg = RMS ? 0.f : block_sum(sg, scratch) / d;
    const float mgx = block_sum(sgx, scratch) / d;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = c0 + i;
      if (c < d) {
        float v = rs * (g[i] - mg - xh[i] * mgx);
        if (dr_in != nullptr) v += dr_in[base + c];
        dres[base + c] = v;
        if (ddelta != nullptr) st(ddelta, base + c, v);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = c0 + i;
    if (c < d) {
      part_w[(long long)blockIdx.x * d + c] = aw[i];
      if (part_b != nullptr) part_b[(long long)blockIdx.x * d + c] = ab[i];
    }
  }
}

// out[c] = sum_b part[b, c] + beta * out[c]
__global__ void sum_rows_kernel(const float* __restrict__ part, float* __restrict__ out, int nrows, int d, float beta) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float s = 0.f;
  for (int r = 0; r < nrows; ++r) s += part[(long long)r * d + c];
  out[c] = s + (beta != 0.f ? beta * out[c] : 0.f);
}

inline int threads_for(int d) {
  const int t = ((d + VPT - 1) / VPT + 31) / 32 * 32;
  return t < 32 ? 32 : t;
}

}  // namespace norm

int64_t norm_backward_blocks(int64_t rows) { return std::max<int64_t>(1, std::min<int64_t>(rows, 2 * num_sms())); }

#define HT_DISPATCH_W(WT_TENSOR, ...)                                                   \
  if ((WT_TENSOR).scalar_type() == at::kFloat) {                                        \
    using WT = float;                                                                   \
    __VA_ARGS__                                                                         \
  } else {                                                                              \
    TORCH_CHECK((WT_TENSOR).scalar_type() == at::kBFloat16, "norm weight must be fp32 or bf16"); \
    using WT = __nv_bfloat16;                                                           \
    __VA_ARGS__                                                                         \
  }

void norm_forward(at::Tensor res, c10::optional<at::Tensor> delta, at::Tensor w, c10::optional<at::Tensor> b, at::Tensor r_out,
                  at::Tensor y, at::Tensor mean, at::Tensor rstd, double eps, bool rms) {
  const c10::cuda::CUDAGuard guard(res.device());
  HT_CHECK(res.scalar_type() == at::kFloat && res.is_contiguous(), "residual must be contiguous fp32");
  const int rows = res.size(0), d = res.size(1);
  HT_CHECK(d <= 1024 * norm::VPT, "hidden size too large for the norm kernel");
  HT_CHECK(w.is_contiguous() && w.numel() == d, "norm weight must be [d]");
  const bool has_delta = delta.has_value() && delta->defined();
  if (has_delta) HT_CHECK(delta->is_contiguous() && delta->size(0) == rows && delta->size(1) == d, "delta shape mismatch");
  const bool has_b = b.has_value() && b->defined();
  if (rows == 0) return;
  const int threads = norm::threads_for(d);
  cudaStream_t s = stream();
  auto launch = [&](auto rms_tag, auto* delta_ptr, auto* w_ptr, auto* y_ptr) {
    using DeltaT = std::remove_const_t<std::remove_pointer_t<decltype(delta_ptr)>>;
    using WT = std::remove_const_t<std::remove_pointer_t<decltype(w_ptr)>>;
    using OutT = std::remove_pointer_t<decltype(y_ptr)>;
    constexpr bool RMS = decltype(rms_tag)::value;
    const WT* bp = has_b ? reinterpret_cast<const WT*>(b->data_ptr()) : nullptr;
    norm::norm_forward_kernel<RMS, DeltaT, WT, OutT><<<rows, threads, 0, s>>>(
        res.data_ptr<float>(), delta_ptr, w_ptr, bp, r_out.data_ptr<float>(), y_ptr, mean.data_ptr<float>(),
        rstd.data_ptr<float>(), d, static_cast<float>(eps));
  };
  auto with_y = [&](auto rms_tag, auto* delta_ptr, auto* w_ptr) {
    if (y.scalar_type() == at::kBFloat16) launch(rms_tag, delta_ptr, w_ptr, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
    else launch(rms_tag, delta_ptr, w_ptr, y.data_ptr<float>());
  };
  auto with_w = [&](auto rms_tag, auto* delta_ptr) {
    if (w.scalar_type() == at::kFloat) with_y(rms_tag, delta_ptr, w.data_ptr<float>());
    else with_y(rms_tag, delta_ptr, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()));
  };
  auto with_delta = [&](auto rms_tag) {
    if (!has_delta) with_w(rms_tag, static_cast<const __nv_bfloat16*>(nullptr));
    else if (delta->scalar_type() == at::kBFloat16) with_w(rms_tag, reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr()));
    else with_w(rms_tag, delta->data_ptr<float>());
  };
  if (rms) with_delta(std::true_type{});
  else with_delta(std::false_type{});
  HT_CUDA_CHECK(cudaGetLastError());
}

void norm_backward(c10::optional<at::Tensor> dy, c10::optional<at::Tensor> dr, at::Tensor r, at::Tensor w, at::Tensor mean,
                   at::Tensor rstd, at::Tensor dres, c10::optional<at::Tensor> ddelta, at::Tensor part_w,
                   c10::optional<at::Tensor> part_b, bool rms) {
  const c10::cuda::CUDAGuard guard(r.device());
  const int rows = r.size(0), d = r.size(1);
  const int blocks = part_w.size(0);
  if (rows == 0) return;
  const int threads = norm::threads_for(d);
  cudaStream_t s = stream();
  const bool has_dy = dy.has_value() && dy->defined();
  const float* drp = (dr.has_value() && dr->defined()) ? dr->data_ptr<float>() : nullptr;
  float* pbp = (part_b.has_value() && part_b->defined()) ? part_b->data_ptr<float>() : nullptr;
  const bool has_dd = ddelta.has_value() && ddelta->defined();
  auto launch = [&](auto rms_tag, auto* dy_ptr, auto* w_ptr, auto* dd_ptr) {
    using DyT = std::remove_const_t<std::remove_pointer_t<decltype(dy_ptr)>>;
    using WT = std::remove_const_t<std::remove_pointer_t<decltype(w_ptr)>>;
    using DdT = std::remove_pointer_t<decltype(dd_ptr)>;
    constexpr bool RMS = decltype(rms_tag)::value;
    norm::norm_backward_kernel<RMS, DyT, WT, DdT><<<blocks, threads, 0, s>>>(
        dy_ptr, drp, r.data_ptr<float>(), w_ptr, mean.data_ptr<float>(), rstd.data_ptr<float>(), dres.data_ptr<float>(),
        dd_ptr, part_w.data_ptr<float>(), pbp, rows, d);
  };
  auto with_dd = [&](auto rms_tag, auto* dy_ptr, auto* w_ptr) {
    if (!has_dd) launch(rms_tag, dy_ptr, w_ptr, static_cast<__nv_bfloat16*>(nullptr));
    else if (ddelta->scalar_type() == at::kBFloat16) launch(rms_tag, dy_ptr, w_ptr, reinterpret_cast<__nv_bfloat16*>(ddelta->data_ptr()));
    else launch(rms_tag, dy_ptr, w_ptr, ddelta->data_ptr<float>());
  };
  auto with_w = [&](auto rms_tag, auto* dy_ptr) {
    if (w.scalar_type() == at::kFloat) with_dd(rms_tag, dy_ptr, w.data_ptr<float>());
    else with_dd(rms_tag, dy_ptr, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()));
  };
  auto with_dy = [&](auto rms_tag) {
    if (!has_dy) with_w(rms_tag, static_cast<const __nv_bfloat16*>(nullptr));
    else if (dy->scalar_type() == at::kBFloat16) with_w(rms_tag, reinterpret_cast<const __nv_bfloat16*>(dy->data_ptr()));
    else with_w(rms_tag, dy->data_ptr<float>());
  };
  if (rms) with_dy(std::true_type{});
  else with_dy(std::false_type{});
  HT_CUDA_CHECK(cudaGetLastError());
}

void sum_rows(at::Tensor part, at::Tensor out, double beta) {
  const c10::cuda::CUDAGuard guard(part.device());
  HT_CHECK(part.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat && out.is_contiguous(), "sum_rows takes fp32");
  const int nrows = part.size(0), d = part.size(1);
  HT_CHECK(out.numel() == d, "sum_rows output size mismatch");
  norm::sum_rows_kernel<<<(d + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), out.data_ptr<float>(), nrows, d,
                                                               static_cast<float>(beta));
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
