// Allocation-free entry point for the fused residual-add + LayerNorm / RMSNorm backward.
//
// This entry point has no counterpart in the reference implementation.  It exists for callers that
// cannot allocate device memory: code running inside an environment that owns the allocator (a
// runtime that pre-plans every buffer in a fixed memory pool, or a host process that forbids
// cudaMalloc once start-up is over) can call it with only its own inputs and outputs.  The
// per-block partial sums of the weight and bias gradients, which the regular entry point
// (`norm_backward` followed by `sum_rows`, called from Python) receives as caller-allocated
// scratch, live here in one file-scope device array instead:
//
//   * capacity: NORM_NOALLOC_MAX_BLOCKS (128) x NORM_NOALLOC_MAX_COLS (8192) x 2 floats = 8 MiB,
//     held on every GPU that loads this library until the process exits;
//   * hidden sizes above 8192 are rejected with return code 2 (there is no fallback);
//   * the array is shared by every call and keeps the last call's contents.  Calls that overlap
//     on the GPU (different streams, or different host threads) race on it and must be serialised
//     by the caller.  Each call overwrites every partial row that it later reads, so nothing has
//     to be cleared between calls;
//   * the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it.  Make that first call before
//     any stream capture begins;
//   * the entry point calls no cudaMalloc, cudaFree or allocating library routine;
//   * `mean` is read for LayerNorm only: RMSNorm callers may pass null or any buffer there.
//
// Results equal the regular path: dres = d(residual) + norm-backward(dy), ddelta = the same values
// in the branch dtype, dw = sum over rows of dy * xhat, db = sum over rows of dy (LayerNorm only),
// all fp32 except ddelta.

#include "norm_noalloc.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace {

constexpr int NORM_NOALLOC_MAX_BLOCKS = 128;
constexpr int NORM_NOALLOC_MAX_COLS = HT_NORM_NOALLOC_MAX_COLS;
constexpr int VPT = 8;  // columns per thread
constexpr int MAX_THREADS = NORM_NOALLOC_MAX_COLS / VPT;  // 1024: one block row covers the widest hidden size

// Partial weight-gradient rows, then partial bias-gradient rows.
static __device__ __align__(256) float g_norm_partials[2 * NORM_NOALLOC_MAX_BLOCKS * NORM_NOALLOC_MAX_COLS];

__device__ __forceinline__ float load(const void* p, long long i, int is_bf16) {
  return is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  v = lane < nw ? scratch[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Bounded to 1024 threads so that the compiler keeps every thread within 64 registers: the widest
// hidden size (8192 columns, 8 per thread) launches 1024 threads and must fit in one SM's registers.
__global__ void __launch_bounds__(MAX_THREADS) backward_kernel(const void* __restrict__ dy, int dy_bf16, const float* __restrict__ dr,
                                const float* __restrict__ r, const void* __restrict__ w, int w_bf16,
                                const float* __restrict__ mean, const float* __restrict__ rstd, float* __restrict__ dres,
                                void* __restrict__ ddelta, int ddelta_bf16, float* __restrict__ partials, int rows, int d,
                                int rms) {
  __shared__ float scratch[32];
  const int c0 = threadIdx.x * VPT;
  float aw[VPT], ab[VPT], wv[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    aw[i] = ab[i] = 0.f;
    wv[i] = (c0 + i < d) ? load(w, c0 + i, w_bf16) : 0.f;
  }
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const long long base = (long long)row * d;
    const float mu = rms ? 0.f : mean[row];  // RMSNorm normalises by the root mean square only
    const float rs = rstd[row];
    float xh[VPT], g[VPT];
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = c0 + i;
      float gy = 0.f, xhat = 0.f;
      if (c < d) {
        xhat = (r[base + c] - mu) * rs;
        gy = dy != nullptr ? load(dy, base + c, dy_bf16) : 0.f;
      }
      xh[i] = xhat;
      g[i] = gy * wv[i];
      aw[i] += gy * xhat;
      ab[i] += gy;
      sg += g[i];
      sgx += g[i] * xhat;
    }
    const float mg = rms ? 0.f : block_sum(sg, scratch) / d;
    const float mgx = block_sum(sgx, scratch) / d;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = c0 + i;
      if (c < d) {
        float v = rs * (g[i] - mg - xh[i] * mgx);
        if (dr != nullptr) v += dr[base + c];
        dres[base + c] = v;
        if (ddelta != nullptr) {
          if (ddelta_bf16) reinterpret_cast<__nv_bfloat16*>(ddelta)[base + c] = __float2bfloat16_rn(v);
          else reinterpret_cast<float*>(ddelta)[base + c] = v;
        }
      }
    }
  }
  // Every block writes its whole partial row (zeros when it saw no rows), so contents left in the
  // shared array by an earlier call never reach this call's sums.
  float* pw = partials + (long long)blockIdx.x * d;
  float* pb = partials + (long long)NORM_NOALLOC_MAX_BLOCKS * NORM_NOALLOC_MAX_COLS + (long long)blockIdx.x * d;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = c0 + i;
    if (c < d) {
      pw[c] = aw[i];
      pb[c] = ab[i];
    }
  }
}

__global__ void reduce_kernel(const float* __restrict__ partials, float* __restrict__ dw, float* __restrict__ db, int blocks,
                              int d) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  float sw = 0.f, sb = 0.f;
  const float* pb = partials + (long long)NORM_NOALLOC_MAX_BLOCKS * NORM_NOALLOC_MAX_COLS;
  for (int b = 0; b < blocks; ++b) {
    sw += partials[(long long)b * d + c];
    sb += pb[(long long)b * d + c];
  }
  dw[c] = sw;
  if (db != nullptr) db[c] = sb;
}

constexpr int kMaxDevices = 64;
float* g_partials_addr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

// Device address of the static array on the current device, looked up once per device.  The
// array's name in host code is only a host-side handle, so kernels must be given this address.
cudaError_t partials_for_current_device(int dev, float** out) {
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_partials_addr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_norm_partials);
    if (err != cudaSuccess) return err;
    g_partials_addr[dev] = static_cast<float*>(ptr);
  }
  *out = g_partials_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" {

// Fused residual-add + LayerNorm (rms = 0) or RMSNorm (rms = 1) backward without any allocation.
// The arguments, limits and return codes are documented with the declaration in norm_noalloc.h.
__attribute__((visibility("default"))) int ht_norm_backward_noalloc(
    const void* dy, int dy_is_bf16, const float* dr, const float* r, const void* w, int w_is_bf16, const float* mean,
    const float* rstd, float* dres, void* ddelta, int ddelta_is_bf16, float* dw, float* db, int rows, int d, int rms,
    cudaStream_t stream) {
  if (rows < 0 || d <= 0 || r == nullptr || w == nullptr || (!rms && mean == nullptr) || rstd == nullptr ||
      dres == nullptr || dw == nullptr || (!rms && db == nullptr))
    return 1;
  if (d > NORM_NOALLOC_MAX_COLS) return 2;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return 1000 + (int)err;
  float* partials = nullptr;
  err = partials_for_current_device(dev, &partials);
  if (err != cudaSuccess) return 1000 + (int)err;
  int sms = 0;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return 1000 + (int)err;
  int blocks = rows < 2 * sms ? rows : 2 * sms;
  if (blocks > NORM_NOALLOC_MAX_BLOCKS) blocks = NORM_NOALLOC_MAX_BLOCKS;
  if (blocks < 1) blocks = 1;
  int threads = ((d + VPT - 1) / VPT + 31) / 32 * 32;
  if (threads < 32) threads = 32;
  backward_kernel<<<blocks, threads, 0, stream>>>(dy, dy_is_bf16, dr, r, w, w_is_bf16, mean, rstd, dres, ddelta,
                                                  ddelta_is_bf16, partials, rows, d, rms);
  err = cudaGetLastError();
  if (err != cudaSuccess) return 1000 + (int)err;
  reduce_kernel<<<(d + 255) / 256, 256, 0, stream>>>(partials, dw, rms ? nullptr : db, blocks, d);
  err = cudaGetLastError();
  return err == cudaSuccess ? 0 : 1000 + (int)err;
}

}  // extern "C"
