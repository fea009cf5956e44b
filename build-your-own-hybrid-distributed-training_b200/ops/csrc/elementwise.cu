// Memory-bound kernels: activation backward, SwiGLU, column sums (bias gradients),
// (vocab-parallel) embedding gather/scatter, position-gradient reduction and rotary embeddings.
// All use 16-byte vector accesses where the layout allows and grid-stride loops sized to the SM count.

#include "common.cuh"

namespace ht {
namespace ew {

__global__ void gelu_backward_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ pre,
                                     __nv_bfloat16* __restrict__ out, long long n8) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    if (!HT_IN_BOUNDS(i, n8, 1)) continue;
    uint4 gv = reinterpret_cast<const uint4*>(g)[i];
    uint4 pv = reinterpret_cast<const uint4*>(pre)[i];
    const __nv_bfloat16* ga = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* pa = reinterpret_cast<const __nv_bfloat16*>(&pv);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = f2bf(bf2f(ga[j]) * gelu_tanh_grad(bf2f(pa[j])));
    reinterpret_cast<uint4*>(out)[i] = *reinterpret_cast<uint4*>(o);
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

// h = [gate | up] per row (width 2f) -> out = silu(gate) * up (width f)
__global__ void swiglu_forward_kernel(const __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ out, long long rows, int f) {
  const long long total = rows * f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / f;
    const int c = i - r * f;
    if (!HT_IN_BOUNDS(r * 2 * f + f + c, total * 2, 2)) continue;
    const float gt = bf2f(h[r * 2 * f + c]);
    const float up = bf2f(h[r * 2 * f + f + c]);
    out[i] = f2bf(silu(gt) * up);
  }
}

__global__ void swiglu_backward_kernel(const __nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ g,
                                       __nv_bfloat16* __restrict__ dh, long long rows, int f) {
  const long long total = rows * f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / f;
    const int c = i - r * f;
    if (!HT_IN_BOUNDS(r * 2 * f + f + c, total * 2, 3)) continue;
    const float gt = bf2f(h[r * 2 * f + c]);
    const float up = bf2f(h[r * 2 * f + f + c]);
    const float go = bf2f(g[i]);
    const float sig = 1.f / (1.f + __expf(-gt));
    const float s = gt * sig;
    dh[r * 2 * f + c] = f2bf(go * up * sig * (1.f + gt * (1.f - sig)));
    dh[r * 2 * f + f + c] = f2bf(go * s);
  }
}

// Column sums of a row block: CTA (strip of 32 * VEC columns) x (block of rows); warp w adds
// rows w, w + 8, ... with VEC contiguous columns per lane, then the eight warps are summed in a
// fixed order.  part[blockIdx.y, c] receives the block's sums (deterministic: no atomics).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) column_partial_kernel(const T* __restrict__ x, float* __restrict__ part, long long rows,
                                                             int cols, int rows_per_block) {
  __shared__ float red[8][32 * VEC];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int strip0 = blockIdx.x * 32 * VEC;
  const int c0 = strip0 + lane * VEC;
  const long long r0 = (long long)blockIdx.y * rows_per_block;
  const long long r1 = min(rows, r0 + rows_per_block);
  float acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) acc[e] = 0.f;
  if (c0 < cols) {
#pragma unroll 8
    for (long long r = r0 + warp; r < r1; r += 8) {
      const T* p = x + r * cols + c0;
      if constexpr (VEC == 8 && std::is_same<T, __nv_bfloat16>::value) {
        const uint4 raw = *reinterpret_cast<const uint4*>(p);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          acc[2 * q] += f.x;
          acc[2 * q + 1] += f.y;
        }
      } else if constexpr (VEC == 4 && std::is_same<T, float>::value) {
        const float4 f = *reinterpret_cast<const float4*>(p);
        acc[0] += f.x;
        acc[1] += f.y;
        acc[2] += f.z;
        acc[3] += f.w;
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          if (c0 + e < cols) {
            if constexpr (std::is_same<T, float>::value) acc[e] += p[e];
            else acc[e] += bf2f(p[e]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) red[warp][lane * VEC + e] = acc[e];
  __syncthreads();
  for (int i = threadIdx.x; i < 32 * VEC; i += blockDim.x) {
    const int c = strip0 + i;
    if (c < cols) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) t += red[k][i];
      if (HT_IN_BOUNDS((long long)blockIdx.y * cols + c, (long long)gridDim.y * cols, 8)) part[(long long)blockIdx.y * cols + c] = t;
    }
  }
}

// out[b, s, :] = (ids in shard ? table[ids - start] : 0) + pos[s]   (fp32 out)
template <typename WT>
__global__ void embedding_forward_kernel(const int* __restrict__ ids, const WT* __restrict__ table, const WT* __restrict__ pos,
                                         float* __restrict__ out, long long tokens, int seq, int d, int vocab_start, int rows) {
  for (long long t = blockIdx.x; t < tokens; t += gridDim.x) {
    const int id = ids[t] - vocab_start;
    const bool own = id >= 0 && id < rows;
    const int s = t % seq;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
      float v = 0.f;
      if (own && HT_IN_BOUNDS((long long)id * d + c, (long long)rows * d, 4)) {
        if constexpr (std::is_same<WT, float>::value) v = table[(long long)id * d + c];
        else v = bf2f(table[(long long)id * d + c]);
      }
      if (pos != nullptr) {
        if constexpr (std::is_same<WT, float>::value) v += pos[(long long)s * d + c];
        else v += bf2f(pos[(long long)s * d + c]);
      }
      if (HT_IN_BOUNDS(t * d + c, tokens * d, 5)) out[t * d + c] = v;
    }
  }
}

// dtable[ids - start] += grad (atomics; duplicates in a batch accumulate)
__global__ void embedding_backward_kernel(const int* __restrict__ ids, const float* __restrict__ grad, float* __restrict__ dtable,
                                          long long tokens, int d, int vocab_start, int rows) {
  for (long long t = blockIdx.x; t < tokens; t += gridDim.x) {
    const int id = ids[t] - vocab_start;
    if (id < 0 || id >= rows) continue;
    for (int c = threadIdx.x; c < d; c += blockDim.x)
      if (HT_IN_BOUNDS((long long)id * d + c, (long long)rows * d, 6)) atomicAdd(dtable + (long long)id * d + c, grad[t * d + c]);
  }
}

// out[s, c] = sum_b grad[b, s, c] + beta * out[s, c]
__global__ void sum_batch_kernel(const float* __restrict__ grad, float* __restrict__ out, int batch, long long sd, float beta) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < sd; i += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int b = 0; b < batch; ++b) s += grad[b * sd + i];
    out[i] = s + (beta != 0.f ? beta * out[i] : 0.f);
  }
}

// In-place rotate-half RoPE on the first `heads` heads of each token row of a packed tensor.
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, const float* __restrict__ cosv, const float* __restrict__ sinv,
                            long long tokens, int seq, int row_width, int heads, int hd, int inverse) {
  const int half = hd / 2;
  const long long total = tokens * heads * half;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int j = i % half;
    const long long th = i / half;
    const int h = th % heads;
    const long long t = th / heads;
    const int s = t % seq;
    if (!HT_IN_BOUNDS(t * row_width + (long long)h * hd + j + half, tokens * row_width, 7)) continue;
    const float c = cosv[s * half + j];
    const float sn = inverse ? -sinv[s * half + j] : sinv[s * half + j];
    __nv_bfloat16* p = x + t * row_width + (long long)h * hd;
    const float a = bf2f(p[j]), b = bf2f(p[j + half]);
    p[j] = f2bf(a * c - b * sn);
    p[j + half] = f2bf(b * c + a * sn);
  }
}

inline int grid_for(long long n, int threads) {
  const long long want = (n + threads - 1) / threads;
  return (int)std::max<long long>(1, std::min<long long>(want, (long long)num_sms() * 8));
}

}  // namespace ew

void gelu_backward(at::Tensor g, at::Tensor pre, at::Tensor out) {
  const c10::cuda::CUDAGuard guard(g.device());
  HT_CHECK(g.scalar_type() == at::kBFloat16 && pre.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
           "gelu_backward takes bf16");
  HT_CHECK(g.is_contiguous() && pre.is_contiguous() && out.is_contiguous() && g.numel() % 8 == 0, "contiguous, numel % 8");
  const long long n8 = g.numel() / 8;
  if (n8 == 0) return;
  ew::gelu_backward_kernel<<<ew::grid_for(n8, 256), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), n8);
  HT_CUDA_CHECK(cudaGetLastError());
}

void swiglu_forward(at::Tensor h, at::Tensor out) {
  const c10::cuda::CUDAGuard guard(h.device());
  HT_CHECK(h.scalar_type() == at::kBFloat16 && h.is_contiguous() && out.is_contiguous(), "swiglu takes contiguous bf16");
  const int f = out.size(-1);
  const long long rows = out.numel() / f;
  if (rows == 0) return;
  ew::swiglu_forward_kernel<<<ew::grid_for(rows * f, 256), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rows, f);
  HT_CUDA_CHECK(cudaGetLastError());
}

void swiglu_backward(at::Tensor h, at::Tensor g, at::Tensor dh) {
  const c10::cuda::CUDAGuard guard(h.device());
  const int f = g.size(-1);
  const long long rows = g.numel() / f;
  if (rows == 0) return;
  ew::swiglu_backward_kernel<<<ew::grid_for(rows * f, 256), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dh.data_ptr()), rows, f);
  HT_CUDA_CHECK(cudaGetLastError());
}

namespace ew {
__global__ void exp2_eval_kernel(const float* __restrict__ x, float* __restrict__ poly, float* __restrict__ mufu, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    poly[i] = exp2_poly(x[i]);
    mufu[i] = exp2f(x[i]);
  }
}
}  // namespace ew

// Evaluates the FMA-pipe 2^x used by the attention softmax and CUDA's exp2f on the same inputs (tests).
void exp2_poly_eval(at::Tensor x, at::Tensor poly, at::Tensor mufu) {
  const c10::cuda::CUDAGuard guard(x.device());
  for (const at::Tensor* t : {&x, &poly, &mufu})
    HT_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == x.numel(), "fp32 args");
  const long long n = x.numel();
  if (n == 0) return;
  const int blocks = (int)std::min<long long>((n + 255) / 256, 4LL * num_sms());
  ew::exp2_eval_kernel<<<blocks, 256, 0, stream()>>>(x.data_ptr<float>(), poly.data_ptr<float>(), mufu.data_ptr<float>(), n);
  HT_CUDA_CHECK(cudaGetLastError());
}

void sum_rows(at::Tensor part, at::Tensor out, double beta);

// out = column sums of x + beta * out (deterministic): per-row-block partial sums, then sum_rows.
void column_sum(at::Tensor x, at::Tensor out, double beta) {
  const c10::cuda::CUDAGuard guard(x.device());
  HT_CHECK(x.dim() == 2 && x.is_contiguous() && out.scalar_type() == at::kFloat && out.numel() == x.size(1), "column_sum shapes");
  const long long rows = x.size(0);
  const int cols = x.size(1);
  if (cols == 0) return;
  if (rows == 0) {
    if (beta == 0.0) out.zero_();
    else out.mul_(beta);
    return;
  }
  const bool bf16 = x.scalar_type() == at::kBFloat16;
  HT_CHECK(bf16 || x.scalar_type() == at::kFloat, "column_sum takes bf16 or fp32");
  const bool vec_ok = (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 && cols % (bf16 ? 8 : 4) == 0;
  const int vec = vec_ok ? (bf16 ? 8 : 4) : 1;
  const int strips = (cols + 32 * vec - 1) / (32 * vec);
  int row_blocks = (int)std::max<long long>(1, std::min<long long>((rows + 63) / 64, (4LL * num_sms() + strips - 1) / strips));
  const int rpb = (int)((rows + row_blocks - 1) / row_blocks);
  row_blocks = (int)((rows + rpb - 1) / rpb);
  at::Tensor part = at::empty({row_blocks, cols}, out.options());
  const dim3 grid(strips, row_blocks);
  cudaStream_t s = stream();
  if (bf16) {
    const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
    if (vec == 8) ew::column_partial_kernel<__nv_bfloat16, 8><<<grid, 256, 0, s>>>(xp, part.data_ptr<float>(), rows, cols, rpb);
    else ew::column_partial_kernel<__nv_bfloat16, 1><<<grid, 256, 0, s>>>(xp, part.data_ptr<float>(), rows, cols, rpb);
  } else {
    if (vec == 4) ew::column_partial_kernel<float, 4><<<grid, 256, 0, s>>>(x.data_ptr<float>(), part.data_ptr<float>(), rows, cols, rpb);
    else ew::column_partial_kernel<float, 1><<<grid, 256, 0, s>>>(x.data_ptr<float>(), part.data_ptr<float>(), rows, cols, rpb);
  }
  HT_CUDA_CHECK(cudaGetLastError());
  sum_rows(part, out, beta);
}

void embedding_forward(at::Tensor ids, at::Tensor table, c10::optional<at::Tensor> pos, at::Tensor out, int64_t vocab_start) {
  const c10::cuda::CUDAGuard guard(table.device());
  HT_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && table.is_contiguous() && out.is_contiguous(), "embedding args");
  const long long tokens = ids.numel();
  const int seq = ids.size(-1), d = table.size(1), rows = table.size(0);
  const bool has_pos = pos.has_value() && pos->defined();
  if (tokens == 0) return;
  const int grid = (int)std::min<long long>(tokens, num_sms() * 16);
  const int threads = std::min(1024, std::max(32, (d + 31) / 32 * 32));
  if (table.scalar_type() == at::kFloat) {
    ew::embedding_forward_kernel<float><<<grid, threads, 0, stream()>>>(ids.data_ptr<int>(), table.data_ptr<float>(),
                                                                        has_pos ? pos->data_ptr<float>() : nullptr,
                                                                        out.data_ptr<float>(), tokens, seq, d, (int)vocab_start, rows);
  } else {
    ew::embedding_forward_kernel<__nv_bfloat16><<<grid, threads, 0, stream()>>>(
        ids.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
        has_pos ? reinterpret_cast<const __nv_bfloat16*>(pos->data_ptr()) : nullptr, out.data_ptr<float>(), tokens, seq, d,
        (int)vocab_start, rows);
  }
  HT_CUDA_CHECK(cudaGetLastError());
}

void embedding_backward(at::Tensor ids, at::Tensor grad, at::Tensor dtable, int64_t vocab_start) {
  const c10::cuda::CUDAGuard guard(grad.device());
  HT_CHECK(grad.scalar_type() == at::kFloat && dtable.scalar_type() == at::kFloat && dtable.is_contiguous(), "fp32 grads");
  const long long tokens = ids.numel();
  const int d = dtable.size(1), rows = dtable.size(0);
  if (tokens == 0) return;
  const int grid = (int)std::min<long long>(tokens, num_sms() * 16);
  const int threads = std::min(1024, std::max(32, (d + 31) / 32 * 32));
  ew::embedding_backward_kernel<<<grid, threads, 0, stream()>>>(ids.data_ptr<int>(), grad.data_ptr<float>(),
                                                                dtable.data_ptr<float>(), tokens, d, (int)vocab_start, rows);
  HT_CUDA_CHECK(cudaGetLastError());
}

void sum_batch_into(at::Tensor grad, at::Tensor out, double beta) {
  const c10::cuda::CUDAGuard guard(grad.device());
  HT_CHECK(grad.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat && grad.is_contiguous() && out.is_contiguous(),
           "sum_batch_into takes contiguous fp32");
  const int batch = grad.size(0);
  const long long sd = grad.numel() / batch;
  HT_CHECK(out.numel() == sd, "sum_batch_into size mismatch");
  ew::sum_batch_kernel<<<ew::grid_for(sd, 256), 256, 0, stream()>>>(grad.data_ptr<float>(), out.data_ptr<float>(), batch, sd,
                                                                    static_cast<float>(beta));
  HT_CUDA_CHECK(cudaGetLastError());
}

void rope_(at::Tensor x, at::Tensor cosv, at::Tensor sinv, int64_t heads, int64_t hd, bool inverse) {
  const c10::cuda::CUDAGuard guard(x.device());
  HT_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 3, "rope takes contiguous bf16 [B, S, W]");
  const long long tokens = x.size(0) * x.size(1);
  const int seq = x.size(1), width = x.size(2);
  const long long total = tokens * heads * (hd / 2);
  if (total == 0) return;
  ew::rope_kernel<<<ew::grid_for(total, 256), 256, 0, stream()>>>(reinterpret_cast<__nv_bfloat16*>(x.data_ptr()),
                                                                  cosv.data_ptr<float>(), sinv.data_ptr<float>(), tokens, seq,
                                                                  width, (int)heads, (int)hd, inverse ? 1 : 0);
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
