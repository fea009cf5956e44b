// Fused residual-add + LayerNorm / RMSNorm, forward and backward.
//
// Forward (one CTA per row, 8 contiguous elements per thread held in registers):
//   r = residual + delta (fp32, written back as the new residual stream)
//   y = (r - mean) * rstd * w + b        (LayerNorm; two-pass mean / variance over registers)
//   y = r * rstd * w                     (RMSNorm)
// Backward (a grid of CTAs strides over rows; each keeps its columns' dw/db partial sums in
// registers and writes one partial row per CTA, reduced by sum_rows):
//
// Two implementations: for the common case (hidden size a multiple of 4 and at most 1024, fp32
// weight, bf16 branch tensors) one warp owns a row, loads and stores 16-byte (fp32) or 8-byte
// (bf16) vectors and reduces with shuffles only; every other case uses a CTA per row with eight
// scalar elements per thread.
//   xhat = (r - mean) * rstd, g = dy * w
//   dr_total = rstd * (g - mean(g) - xhat * mean(g * xhat)) + dr_in      (LayerNorm)
//   dr_total = rstd * (g - xhat * mean(g * xhat)) + dr_in                 (RMSNorm)

#include "common.cuh"

namespace ht {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

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

// The CTA-per-row kernels launch up to 1024 threads (8192 columns at 8 per thread); the bound keeps
// the compiler at 64 registers per thread so that the widest row fits one SM's register file.
template <bool RMS, typename DeltaT, typename WT, typename OutT>
__global__ void __launch_bounds__(1024) norm_forward_kernel(const float* __restrict__ res, const DeltaT* __restrict__ delta, const WT* __restrict__ w,
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
    if (c < d && HT_IN_BOUNDS(base + c, (long long)gridDim.x * d, 30)) {
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
__global__ void __launch_bounds__(1024) norm_backward_kernel(const DyT* __restrict__ dy, const float* __restrict__ dr_in, const float* __restrict__ r,
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

// ---------------------------------------------------------------------------------------------
// Warp-per-row kernels (hidden size d % 4 == 0, d <= 32 * 4 * NV).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void ld4(const float* p, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float* v) {
  const uint2 a = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
  v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
}
__device__ __forceinline__ void st4(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, const float* v) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
  uint2 a;
  a.x = *reinterpret_cast<uint32_t*>(&lo);
  a.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = a;
}

constexpr int WARP_ROWS_THREADS = 256;

// Lane `l` owns the 4-element vectors l, l + 32, ..., l + 32 * (NV - 1) of every row it visits.
template <bool RMS, bool HAS_DELTA, int NV>
__global__ void __launch_bounds__(WARP_ROWS_THREADS)
    norm_forward_warp_kernel(const float* __restrict__ res, const __nv_bfloat16* __restrict__ delta, const float* __restrict__ w,
                             const float* __restrict__ b, float* __restrict__ r_out, __nv_bfloat16* __restrict__ y,
                             float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int d, float eps) {
  const int lane = threadIdx.x & 31;
  const int nvec = d >> 2;
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  float wv[NV][4], bv[NV][4];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int v = lane + 32 * j;
#pragma unroll
    for (int e = 0; e < 4; ++e) wv[j][e] = bv[j][e] = 0.f;
    if (v < nvec) {
      ld4(w + 4 * v, wv[j]);
      if (!RMS && b != nullptr) ld4(b + 4 * v, bv[j]);
    }
  }
  for (int row = warp_global; row < rows; row += warps) {
    const long long base = (long long)row * d;
    float x[NV][4];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = lane + 32 * j;
#pragma unroll
      for (int e = 0; e < 4; ++e) x[j][e] = 0.f;
      if (v < nvec) {
        ld4(res + base + 4 * v, x[j]);
        if (HAS_DELTA) {
          float t[4];
          ld4(delta + base + 4 * v, t);
#pragma unroll
          for (int e = 0; e < 4; ++e) x[j][e] += t[e];
        }
        st4(r_out + base + 4 * v, x[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) s += x[j][e];
      }
    }
    const float mean = RMS ? 0.f : warp_sum(s) / d;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      if (lane + 32 * j < nvec) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float t = x[j][e] - mean;
          q += t * t;
        }
      }
    }
    const float rstd = rsqrtf(warp_sum(q) / d + eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) {
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = (x[j][e] - mean) * rstd * wv[j][e] + bv[j][e];
        st4(y + base + 4 * v, o);
      }
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

// Every CTA writes one full partial row of dw (and db): zeros for columns it never touched.
// Each warp accumulates its rows' dw/db contributions in its own slice of shared memory rather
// than in registers, which keeps the kernel at 64 registers and four CTAs (32 warps) per SM:
// profiled at two CTAs per SM it was latency bound (long-scoreboard stalls, 22 % warps active,
// 24 % of DRAM peak).  The second pass re-reads the row's r and dy (cache hits: the same warp
// read them moments before).  Per-warp sums and the final fixed-order CTA reduction keep the
// result deterministic.
template <bool RMS, bool HAS_DY, bool HAS_DR, int NV>
__global__ void __launch_bounds__(WARP_ROWS_THREADS, 4)
    norm_backward_warp_kernel(const __nv_bfloat16* __restrict__ dy, const float* __restrict__ dr_in, const float* __restrict__ r,
                              const float* __restrict__ w, const float* __restrict__ mean, const float* __restrict__ rstd,
                              float* __restrict__ dres, __nv_bfloat16* __restrict__ ddelta, float* __restrict__ part_w,
                              float* __restrict__ part_b, int rows, int d) {
  constexpr int WARPS = WARP_ROWS_THREADS / 32;
  extern __shared__ float red[];  // dw accumulators [WARPS][d], then db accumulators [WARPS][d] when part_b is given
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = d >> 2;
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const bool with_b = part_b != nullptr;
  float* acc_w = red + warp * d;
  float* acc_b = red + (WARPS + warp) * d;
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int v = lane + 32 * j;
    if (v < nvec) {
      st4(acc_w + 4 * v, zero);
      if (with_b) st4(acc_b + 4 * v, zero);
    }
  }
  for (int row = warp_global; row < rows; row += warps) {
    const long long base = (long long)row * d;
    const float mu = RMS ? 0.f : mean[row], rs = rstd[row];
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) {
        float rv[4], gy[4] = {0.f, 0.f, 0.f, 0.f}, wv[4], aw[4], ab[4];
        ld4(r + base + 4 * v, rv);
        if (HAS_DY) ld4(dy + base + 4 * v, gy);
        ld4(w + 4 * v, wv);
        ld4(acc_w + 4 * v, aw);
        if (with_b) ld4(acc_b + 4 * v, ab);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float xhat = (rv[e] - mu) * rs;
          const float g = gy[e] * wv[e];
          aw[e] += gy[e] * xhat;
          ab[e] += gy[e];
          sg += g;
          sgx += g * xhat;
        }
        st4(acc_w + 4 * v, aw);
        if (with_b) st4(acc_b + 4 * v, ab);
      }
    }
    const float mg = RMS ? 0.f : warp_sum(sg) / d;
    const float mgx = warp_sum(sgx) / d;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = lane + 32 * j;
      if (v < nvec) {
        float rv[4], gy[4] = {0.f, 0.f, 0.f, 0.f}, wv[4], o[4], din[4] = {0.f, 0.f, 0.f, 0.f};
        ld4(r + base + 4 * v, rv);
        if (HAS_DY) ld4(dy + base + 4 * v, gy);
        ld4(w + 4 * v, wv);
        if (HAS_DR) ld4(dr_in + base + 4 * v, din);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float xhat = (rv[e] - mu) * rs;
          o[e] = rs * (gy[e] * wv[e] - mg - xhat * mgx) + din[e];
        }
        st4(dres + base + 4 * v, o);
        if (ddelta != nullptr) st4(ddelta + base + 4 * v, o);
      }
    }
  }
  // CTA reduction of the per-warp partial sums, in a fixed order.
  __syncthreads();
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < WARPS; ++k) t += red[k * d + c];
    part_w[(long long)blockIdx.x * d + c] = t;
    if (with_b) {
      float tb = 0.f;
#pragma unroll
      for (int k = 0; k < WARPS; ++k) tb += red[(WARPS + k) * d + c];
      part_b[(long long)blockIdx.x * d + c] = tb;
    }
  }
}

// out[c] = sum_r part[r, c] (+ beta * out[c]).  A block owns 32 columns (128-byte row segments);
// its 32 warps take interleaved rows, four independent loads in flight per thread, and the 32
// per-warp sums are added in a fixed order, so the result is deterministic.  The partial-row
// counts here are small (a few hundred rows), so the kernel is bound by load latency: more warps
// per column strip shorten each thread's dependent chain.
constexpr int SR_WARPS = 32;

__global__ void __launch_bounds__(SR_WARPS * 32) sum_rows_kernel(const float* __restrict__ part, float* __restrict__ out, int nrows,
                                                                  int d, float beta) {
  __shared__ float red[SR_WARPS][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (c < d) {
    int r = ty;
    for (; r + 3 * SR_WARPS < nrows; r += 4 * SR_WARPS) {
      s0 += part[(long long)r * d + c];
      s1 += part[(long long)(r + SR_WARPS) * d + c];
      s2 += part[(long long)(r + 2 * SR_WARPS) * d + c];
      s3 += part[(long long)(r + 3 * SR_WARPS) * d + c];
    }
    for (; r < nrows; r += SR_WARPS) s0 += part[(long long)r * d + c];
  }
  red[ty][tx] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (ty == 0 && c < d && HT_IN_BOUNDS(c, d, 31)) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < SR_WARPS; ++k) t += red[k][tx];
    out[c] = t + (beta != 0.f ? beta * out[c] : 0.f);
  }
}

// Two independent column reductions in one launch (the weight and bias gradients of a norm):
// blocks [0, strips) reduce `part_a` into `out_a`, the rest `part_b` into `out_b`, each exactly as
// sum_rows_kernel does (same order, same result).
__global__ void __launch_bounds__(SR_WARPS * 32) sum_rows_pair_kernel(const float* __restrict__ part_a, float* __restrict__ out_a,
                                                                       float beta_a, const float* __restrict__ part_b,
                                                                       float* __restrict__ out_b, float beta_b, int nrows, int d,
                                                                       int strips) {
  __shared__ float red[SR_WARPS][33];
  const bool second = (int)blockIdx.x >= strips;
  const float* part = second ? part_b : part_a;
  float* out = second ? out_b : out_a;
  const float beta = second ? beta_b : beta_a;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = (second ? blockIdx.x - strips : blockIdx.x) * 32 + tx;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (c < d) {
    int r = ty;
    for (; r + 3 * SR_WARPS < nrows; r += 4 * SR_WARPS) {
      s0 += part[(long long)r * d + c];
      s1 += part[(long long)(r + SR_WARPS) * d + c];
      s2 += part[(long long)(r + 2 * SR_WARPS) * d + c];
      s3 += part[(long long)(r + 3 * SR_WARPS) * d + c];
    }
    for (; r < nrows; r += SR_WARPS) s0 += part[(long long)r * d + c];
  }
  red[ty][tx] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (ty == 0 && c < d) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < SR_WARPS; ++k) t += red[k][tx];
    out[c] = t + (beta != 0.f ? beta * out[c] : 0.f);
  }
}

// Vectors of 4 per lane for the warp-per-row kernels (2, 4, 6 or 8), or 0 when d does not fit.
inline int warp_vectors(int d) {
  if (d % 4 != 0 || d > 32 * 4 * 8) return 0;
  const int nv = (d / 4 + 31) / 32;
  return nv <= 2 ? 2 : (nv + 1) / 2 * 2;
}

inline int threads_for(int d) {
  const int t = ((d + VPT - 1) / VPT + 31) / 32 * 32;
  return t < 32 ? 32 : t;
}

}  // namespace norm

int64_t norm_backward_blocks(int64_t rows) { return std::max<int64_t>(1, std::min<int64_t>(rows, 4 * num_sms())); }

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
  const bool delta_ok = !has_delta || (delta->scalar_type() == at::kBFloat16 && aligned16(delta->data_ptr()));
  const int nv = norm::warp_vectors(d);
  if (nv > 0 && delta_ok && w.scalar_type() == at::kFloat && (!has_b || b->scalar_type() == at::kFloat) &&
      y.scalar_type() == at::kBFloat16 && y.is_contiguous() && r_out.is_contiguous() && aligned16(res.data_ptr()) &&
      aligned16(r_out.data_ptr()) && aligned16(y.data_ptr()) && aligned16(w.data_ptr()) &&
      (!has_b || aligned16(b->data_ptr()))) {
    const int blocks = (int)std::min<int64_t>((rows + 7) / 8, 16LL * num_sms());
    auto go = [&](auto rms_tag, auto delta_tag, auto nv_tag) {
      norm::norm_forward_warp_kernel<decltype(rms_tag)::value, decltype(delta_tag)::value, decltype(nv_tag)::value>
          <<<blocks, norm::WARP_ROWS_THREADS, 0, s>>>(
              res.data_ptr<float>(), has_delta ? reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr()) : nullptr,
              w.data_ptr<float>(), has_b ? b->data_ptr<float>() : nullptr, r_out.data_ptr<float>(),
              reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, d,
              static_cast<float>(eps));
    };
    auto with_nv = [&](auto rms_tag, auto delta_tag) {
      switch (nv) {
        case 2: go(rms_tag, delta_tag, std::integral_constant<int, 2>{}); break;
        case 4: go(rms_tag, delta_tag, std::integral_constant<int, 4>{}); break;
        case 6: go(rms_tag, delta_tag, std::integral_constant<int, 6>{}); break;
        default: go(rms_tag, delta_tag, std::integral_constant<int, 8>{}); break;
      }
    };
    auto with_delta = [&](auto rms_tag) {
      if (has_delta) with_nv(rms_tag, std::true_type{});
      else with_nv(rms_tag, std::false_type{});
    };
    if (rms) with_delta(std::true_type{});
    else with_delta(std::false_type{});
    HT_CUDA_CHECK(cudaGetLastError());
    return;
  }
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
  const int nv = norm::warp_vectors(d);
  if (nv > 0 && (!has_dy || (dy->scalar_type() == at::kBFloat16 && aligned16(dy->data_ptr()))) &&
      (!has_dd || (ddelta->scalar_type() == at::kBFloat16 && aligned16(ddelta->data_ptr()))) &&
      (drp == nullptr || aligned16(drp)) && w.scalar_type() == at::kFloat && aligned16(w.data_ptr()) &&
      aligned16(r.data_ptr()) && aligned16(dres.data_ptr())) {
    const size_t smem = (size_t)(pbp != nullptr ? 2 : 1) * (norm::WARP_ROWS_THREADS / 32) * d * sizeof(float);
    auto go = [&](auto rms_tag, auto dy_tag, auto dr_tag, auto nv_tag) {
      auto kernel = norm::norm_backward_warp_kernel<decltype(rms_tag)::value, decltype(dy_tag)::value,
                                                    decltype(dr_tag)::value, decltype(nv_tag)::value>;
      if (smem > 48 * 1024) HT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      kernel<<<blocks, norm::WARP_ROWS_THREADS, smem, s>>>(
          has_dy ? reinterpret_cast<const __nv_bfloat16*>(dy->data_ptr()) : nullptr, drp, r.data_ptr<float>(),
          w.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), dres.data_ptr<float>(),
          has_dd ? reinterpret_cast<__nv_bfloat16*>(ddelta->data_ptr()) : nullptr, part_w.data_ptr<float>(), pbp, rows, d);
    };
    auto with_nv = [&](auto rms_tag, auto dy_tag, auto dr_tag) {
      switch (nv) {
        case 2: go(rms_tag, dy_tag, dr_tag, std::integral_constant<int, 2>{}); break;
        case 4: go(rms_tag, dy_tag, dr_tag, std::integral_constant<int, 4>{}); break;
        case 6: go(rms_tag, dy_tag, dr_tag, std::integral_constant<int, 6>{}); break;
        default: go(rms_tag, dy_tag, dr_tag, std::integral_constant<int, 8>{}); break;
      }
    };
    auto with_dr = [&](auto rms_tag, auto dy_tag) {
      if (drp != nullptr) with_nv(rms_tag, dy_tag, std::true_type{});
      else with_nv(rms_tag, dy_tag, std::false_type{});
    };
    auto with_dy = [&](auto rms_tag) {
      if (has_dy) with_dr(rms_tag, std::true_type{});
      else with_dr(rms_tag, std::false_type{});
    };
    if (rms) with_dy(std::true_type{});
    else with_dy(std::false_type{});
    HT_CUDA_CHECK(cudaGetLastError());
    return;
  }
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

void sum_rows_pair(at::Tensor part_a, at::Tensor out_a, double beta_a, at::Tensor part_b, at::Tensor out_b, double beta_b) {
  const c10::cuda::CUDAGuard guard(part_a.device());
  for (const at::Tensor* t : {&part_a, &out_a, &part_b, &out_b})
    HT_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous(), "sum_rows_pair takes contiguous fp32 tensors");
  HT_CHECK(part_a.dim() == 2 && part_b.sizes() == part_a.sizes(), "sum_rows_pair: the two partial blocks must have one shape");
  const int nrows = part_a.size(0), d = part_a.size(1);
  HT_CHECK(out_a.numel() == d && out_b.numel() == d, "sum_rows_pair output size mismatch");
  if (d == 0) return;
  const int strips = (d + 31) / 32;
  norm::sum_rows_pair_kernel<<<2 * strips, norm::SR_WARPS * 32, 0, stream()>>>(
      part_a.data_ptr<float>(), out_a.data_ptr<float>(), (float)beta_a, part_b.data_ptr<float>(), out_b.data_ptr<float>(),
      (float)beta_b, nrows, d, strips);
  HT_CUDA_CHECK(cudaGetLastError());
}

void sum_rows(at::Tensor part, at::Tensor out, double beta) {
  const c10::cuda::CUDAGuard guard(part.device());
  HT_CHECK(part.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat && out.is_contiguous(), "sum_rows takes fp32");
  const int nrows = part.size(0), d = part.size(1);
  HT_CHECK(out.numel() == d, "sum_rows output size mismatch");
  HT_CHECK(part.is_contiguous() && part.dim() == 2, "sum_rows takes a contiguous [rows, d] tensor");
  norm::sum_rows_kernel<<<(d + 31) / 32, norm::SR_WARPS * 32, 0, stream()>>>(part.data_ptr<float>(), out.data_ptr<float>(), nrows,
                                                                              d, static_cast<float>(beta));
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
