// Cross-entropy over (vocab-parallel) logits, producing the loss and the logit gradient.
//
// One CTA per token row.  Pass 1 streams the row once with 16-byte loads and keeps an online
// (max, sum of exponentials) pair per thread, merged across the block; pass 2 re-reads the row
// (an L2 hit: the CTA touched it microseconds earlier) and writes
//     dlogit = (exp(x - lse) - [c == target]) * scale
// in place.  With the vocabulary split over ranks, pass 1 emits (max, sumexp, target logit)
// per row, the ranks exchange those three floats, `combine` forms the global log-sum-exp and
// the loss, and pass 2 runs with the global log-sum-exp.

#include "common.cuh"

namespace ht {
namespace ce {

constexpr int THREADS = 512;

struct MS {
  float m, s;
};
__device__ __forceinline__ MS merge(MS a, MS b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

__device__ __forceinline__ MS block_merge(MS v, float* sm, float* ss) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o)};
    v = merge(v, other);
  }
  __syncthreads();
  if (lane == 0) {
    sm[warp] = v.m;
    ss[warp] = v.s;
  }
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = lane < nw ? MS{sm[lane], ss[lane]} : MS{-INFINITY, 0.f};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o)};
    v = merge(v, other);
  }
  return v;
}

__device__ __forceinline__ MS row_stats(const __nv_bfloat16* __restrict__ row, int V) {
  // Online (max, sum) per thread: the running sum is rescaled only when a vector raises the
  // running maximum, so the common case costs one exponential per element.
  MS acc{-INFINITY, 0.f};
  const int nv = V / 8;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const uint4 raw = reinterpret_cast<const uint4*>(row)[i];
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(&raw);
    float x[8];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] = bf2f(p[j]);
      m = fmaxf(m, x[j]);
    }
    if (m > acc.m) {
      acc.s = acc.m == -INFINITY ? 0.f : acc.s * __expf(acc.m - m);
      acc.m = m;
    }
    if (acc.m == -INFINITY) continue;  // every logit so far is -inf: nothing to add
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += __expf(x[j] - acc.m);
    acc.s += s;
  }
  for (int c = nv * 8 + threadIdx.x; c < V; c += blockDim.x) acc = merge(acc, MS{bf2f(row[c]), 1.f});
  return acc;
}

__device__ __forceinline__ void row_grad(const __nv_bfloat16* row, __nv_bfloat16* grow, int V, int target, float lse, float scale) {
  const int nv = V / 8;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const uint4 raw = reinterpret_cast<const uint4*>(row)[i];
    const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(&raw);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = i * 8 + j;
      o[j] = f2bf((__expf(bf2f(p[j]) - lse) - (c == target ? 1.f : 0.f)) * scale);
    }
    reinterpret_cast<uint4*>(grow)[i] = *reinterpret_cast<uint4*>(o);
  }
  for (int c = nv * 8 + threadIdx.x; c < V; c += blockDim.x)
    grow[c] = f2bf((__expf(bf2f(row[c]) - lse) - (c == target ? 1.f : 0.f)) * scale);
}

__global__ void __launch_bounds__(THREADS) fused_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                        const int64_t* __restrict__ targets, __nv_bfloat16* __restrict__ grad,
                                                        long long ldg, float* __restrict__ loss, int rows, int V, int vocab_start,
                                                        float scale) {
  __shared__ float sm[32], ss[32];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* row = logits + (long long)r * ld;
    const MS st = block_merge(row_stats(row, V), sm, ss);
    const float lse = st.m + __logf(st.s);
    const int target = (int)(targets[r] - vocab_start);
    if (threadIdx.x == 0) {
      const float xt = (target >= 0 && target < V) ? bf2f(row[target]) : 0.f;
      atomicAdd(loss, (lse - xt) * scale);
    }
    __syncthreads();  // the target logit is read before any thread overwrites the row
    row_grad(row, grad + (long long)r * ldg, V, target, lse, scale);
    __syncthreads();
  }
}

__global__ void __launch_bounds__(THREADS) stats_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                        const int64_t* __restrict__ targets, float* __restrict__ stats,
                                                        int rows, int V, int vocab_start) {
  __shared__ float sm[32], ss[32];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* row = logits + (long long)r * ld;
    const MS st = block_merge(row_stats(row, V), sm, ss);
    if (threadIdx.x == 0) {
      const int target = (int)(targets[r] - vocab_start);
      stats[3 * r] = st.m;
      stats[3 * r + 1] = st.s;
      stats[3 * r + 2] = (target >= 0 && target < V) ? bf2f(row[target]) : 0.f;
    }
  }
}

// gathered: [world * rows, 3] in rank order -> lse[rows], loss += mean contribution
__global__ void combine_kernel(const float* __restrict__ gathered, float* __restrict__ lse, float* __restrict__ loss, int rows,
                               int world, float scale) {
  float local = 0.f;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    MS acc{-INFINITY, 0.f};
    float target = 0.f;
    for (int w = 0; w < world; ++w) {
      const float* g = gathered + 3 * ((long long)w * rows + r);
      acc = merge(acc, MS{g[0], g[1]});
      target += g[2];
    }
    const float l = acc.m + __logf(acc.s);
    lse[r] = l;
    local += (l - target) * scale;
  }
  local = warp_sum(local);
  if ((threadIdx.x & 31) == 0) atomicAdd(loss, local);
}

__global__ void __launch_bounds__(THREADS) grad_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                       const int64_t* __restrict__ targets, const float* __restrict__ lse,
                                                       __nv_bfloat16* __restrict__ grad, long long ldg, int rows, int V,
                                                       int vocab_start, float scale) {
  for (int r = blockIdx.x; r < rows; r += gridDim.x)
    row_grad(logits + (long long)r * ld, grad + (long long)r * ldg, V, (int)(targets[r] - vocab_start), lse[r], scale);
}

}  // namespace ce

static void ce_check(const at::Tensor& logits, const at::Tensor& targets) {
  HT_CHECK(logits.scalar_type() == at::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1, "logits must be bf16 [rows, V]");
  HT_CHECK((logits.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0,
           "logit rows must be 16-byte aligned");
  HT_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous() && targets.numel() == logits.size(0), "targets int64 [rows]");
}

void cross_entropy_fused(at::Tensor logits, at::Tensor targets, at::Tensor grad, at::Tensor loss, int64_t vocab_start, double scale) {
  const c10::cuda::CUDAGuard guard(logits.device());
  ce_check(logits, targets);
  const int rows = logits.size(0), V = logits.size(1);
  if (rows == 0) return;
  const int grid = std::min(rows, num_sms() * 4);
  ce::fused_kernel<<<grid, ce::THREADS, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), targets.data_ptr<int64_t>(),
      reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()), grad.stride(0), loss.data_ptr<float>(), rows, V, (int)vocab_start,
      (float)scale);
  HT_CUDA_CHECK(cudaGetLastError());
}

void cross_entropy_stats(at::Tensor logits, at::Tensor targets, at::Tensor stats, int64_t vocab_start) {
  const c10::cuda::CUDAGuard guard(logits.device());
  ce_check(logits, targets);
  const int rows = logits.size(0), V = logits.size(1);
  if (rows == 0) return;
  ce::stats_kernel<<<std::min(rows, num_sms() * 4), ce::THREADS, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), targets.data_ptr<int64_t>(),
      stats.data_ptr<float>(), rows, V, (int)vocab_start);
  HT_CUDA_CHECK(cudaGetLastError());
}

void cross_entropy_combine(at::Tensor gathered, at::Tensor lse, at::Tensor loss, int64_t world, double scale) {
  const c10::cuda::CUDAGuard guard(gathered.device());
  const int rows = lse.numel();
  if (rows == 0) return;
  ce::combine_kernel<<<std::max(1, std::min((rows + 255) / 256, num_sms() * 2)), 256, 0, stream()>>>(
      gathered.data_ptr<float>(), lse.data_ptr<float>(), loss.data_ptr<float>(), rows, (int)world, (float)scale);
  HT_CUDA_CHECK(cudaGetLastError());
}

void cross_entropy_grad(at::Tensor logits, at::Tensor targets, at::Tensor lse, at::Tensor grad, int64_t vocab_start, double scale) {
  const c10::cuda::CUDAGuard guard(logits.device());
  ce_check(logits, targets);
  const int rows = logits.size(0), V = logits.size(1);
  if (rows == 0) return;
  ce::grad_kernel<<<std::min(rows, num_sms() * 4), ce::THREADS, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), targets.data_ptr<int64_t>(),
      lse.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(grad.data_ptr()), grad.stride(0), rows, V, (int)vocab_start,
      (float)scale);
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
