// In-kernel collectives over NVLink peer memory (one process per GPU, buffers mapped into every
// peer's address space by the symmetric-memory runtime).
//
// bucket_allreduce: averaged all-reduce of one DDP gradient bucket, in one kernel:
//   1. per-block barrier with the same block on every peer (the peers' buckets are complete);
//   2. reduce-scatter: rank r sums chunk r of the bucket over all peers with 16-byte P2P loads,
//      multiplies by the scale (1/G for AVG) and writes it into its own buffer;
//   3. barrier;  4. all-gather: rank r copies every peer's reduced chunk into its own buffer;
//   5. barrier (no peer may overwrite a chunk that another rank is still reading).
// With an NVLink-switch multicast address, steps 2-4 collapse into one
// multimem.ld_reduce (the switch sums the G copies) + multimem.st (the switch writes all G).
//
// Barriers use per-(block, peer) flags in the peers' signal pads: a release fence then a 0->1
// compare-and-swap on the peer's slot, and an acquire wait that swaps our own slot 1->0.  Every
// wait is bounded by a %globaltimer deadline; on expiry the kernel records the stage in `status`
// and returns, so a missing peer produces an error on the host instead of a hung GPU.

#include "common.cuh"

namespace ht {
namespace comm {

constexpr int MAX_RANKS = 8;
constexpr int THREADS = 512;

struct Peers {
  float* buf[MAX_RANKS];
  uint32_t* pad[MAX_RANKS];
};

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Block-level barrier with block `b` of every peer.  Returns false on timeout (status recorded).
__device__ bool block_barrier(const Peers& pp, int rank, int world, int slot_base, int* status, int stage,
                              unsigned long long timeout_ns) {
  __shared__ int failed;
  __syncthreads();
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  const int p = threadIdx.x;
  if (p < world && p != rank) {
    const unsigned long long deadline = now_ns() + timeout_ns;
    bool ok = true;
    __threadfence_system();
    uint32_t* put = pp.pad[p] + slot_base + blockIdx.x * world + rank;
    while (atomicCAS_system(put, 0u, 1u) != 0u) {
      if (now_ns() > deadline || *((volatile int*)status) != 0) {
        ok = false;
        break;
      }
    }
    uint32_t* mine = pp.pad[rank] + slot_base + blockIdx.x * world + p;
    while (ok && atomicCAS_system(mine, 1u, 0u) != 1u) {
      if (now_ns() > deadline || *((volatile int*)status) != 0) {
        ok = false;
        break;
      }
    }
    __threadfence_system();
    if (!ok) failed = 1;
  }
  __syncthreads();
  if (failed) {
    if (threadIdx.x == 0) {
      atomicCAS(status, 0, 1);
      atomicCAS(status + 1, 0, stage);
    }
    return false;
  }
  return true;
}

__global__ void __launch_bounds__(THREADS) bucket_allreduce_kernel(Peers pp, float* mc, long long start, long long n, float scale,
                                                                   int rank, int world, int slot_base, int* status,
                                                                   unsigned long long timeout_ns) {
  // chunk per rank (multiple of 4 floats), sub-range per block
  const long long chunk = ((n + world - 1) / world + 3) / 4 * 4;
  const long long per_block = ((chunk + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
  auto range = [&](int owner, long long& lo, long long& hi) {
    const long long c0 = (long long)owner * chunk;
    lo = c0 + (long long)blockIdx.x * per_block;
    hi = min(min(lo + per_block, c0 + chunk), n);
  };
  if (!block_barrier(pp, rank, world, slot_base, status, 1, timeout_ns)) return;
  long long lo, hi;
  range(rank, lo, hi);
  if (mc != nullptr) {
    for (long long i = lo + threadIdx.x * 4; i < hi; i += THREADS * 4) {
      float* addr = mc + start + i;
      if (i + 3 < hi) {
        float a, b, c, d;
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                     : "=f"(a), "=f"(b), "=f"(c), "=f"(d)
                     : "l"(addr)
                     : "memory");
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(addr), "f"(a * scale), "f"(b * scale),
                     "f"(c * scale), "f"(d * scale)
                     : "memory");
      } else {
        for (long long j = i; j < hi; ++j) {
          float a;
          float* aj = mc + start + j;
          asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(a) : "l"(aj) : "memory");
          asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(aj), "f"(a * scale) : "memory");
        }
      }
    }
    block_barrier(pp, rank, world, slot_base, status, 2, timeout_ns);
    return;
  }
  // two-shot: reduce-scatter my chunk.  Each thread keeps UNROLL independent 16-byte vectors
  // (UNROLL x world peer loads) in flight: the loop is bound by NVLink latency otherwise.
  constexpr int UNROLL = 4;
  constexpr long long STEP = (long long)THREADS * 4 * UNROLL;
  for (long long i0 = lo + threadIdx.x * 4; i0 < hi; i0 += STEP) {
    float4 acc[UNROLL];
    bool vec[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const long long i = i0 + (long long)u * THREADS * 4;
      vec[u] = i + 3 < hi;
      acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int p = 0; p < MAX_RANKS; ++p) {
      if (p >= world) break;
      float4 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
        if (vec[u]) v[u] = *reinterpret_cast<const float4*>(pp.buf[p] + start + i0 + (long long)u * THREADS * 4);
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (vec[u]) {
          acc[u].x += v[u].x;
          acc[u].y += v[u].y;
          acc[u].z += v[u].z;
          acc[u].w += v[u].w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const long long i = i0 + (long long)u * THREADS * 4;
      if (vec[u]) {
        acc[u].x *= scale;
        acc[u].y *= scale;
        acc[u].z *= scale;
        acc[u].w *= scale;
        *reinterpret_cast<float4*>(pp.buf[rank] + start + i) = acc[u];
      } else {
        for (long long j = i; j < hi; ++j) {  // ragged tail of the range
          float sum = 0.f;
          for (int p = 0; p < world; ++p) sum += pp.buf[p][start + j];
          pp.buf[rank][start + j] = sum * scale;
        }
      }
    }
  }
  if (!block_barrier(pp, rank, world, slot_base, status, 2, timeout_ns)) return;
  // all-gather the other ranks' reduced chunks
  for (int q = 1; q < world; ++q) {
    const int p = (rank + q) % world;
    range(p, lo, hi);
    for (long long i0 = lo + threadIdx.x * 4; i0 < hi; i0 += STEP) {
      float4 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = i0 + (long long)u * THREADS * 4;
        if (i + 3 < hi) v[u] = *reinterpret_cast<const float4*>(pp.buf[p] + start + i);
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = i0 + (long long)u * THREADS * 4;
        if (i + 3 < hi) *reinterpret_cast<float4*>(pp.buf[rank] + start + i) = v[u];
        else
          for (long long j = i; j < hi; ++j) pp.buf[rank][start + j] = pp.buf[p][start + j];
      }
    }
  }
  block_barrier(pp, rank, world, slot_base, status, 3, timeout_ns);
}

}  // namespace comm

void bucket_all_reduce(at::Tensor flat, std::vector<int64_t> buffer_ptrs, std::vector<int64_t> pad_ptrs, int64_t multicast_ptr,
                       int64_t start, int64_t numel, double scale, int64_t rank, int64_t slot_base, int64_t max_blocks,
                       at::Tensor status, double timeout_s) {
  const c10::cuda::CUDAGuard guard(flat.device());
  const int world = (int)buffer_ptrs.size();
  HT_CHECK(world >= 2 && world <= comm::MAX_RANKS, "bucket_all_reduce supports 2..8 ranks");
  HT_CHECK((int)pad_ptrs.size() == world, "one signal pad per rank expected");
  HT_CHECK(flat.scalar_type() == at::kFloat && status.scalar_type() == at::kInt, "fp32 buffer and int32 status expected");
  HT_CHECK(start % 4 == 0, "bucket start must be 16-byte aligned");
  if (numel == 0) return;
  comm::Peers pp{};
  for (int p = 0; p < world; ++p) {
    pp.buf[p] = reinterpret_cast<float*>(buffer_ptrs[p]);
    pp.pad[p] = reinterpret_cast<uint32_t*>(pad_ptrs[p]);
  }
  const long long chunk = (numel + world - 1) / world;
  const int blocks =
      (int)std::max<long long>(1, std::min<long long>(max_blocks, (chunk + comm::THREADS * 8 - 1) / (comm::THREADS * 8)));
  comm::bucket_allreduce_kernel<<<blocks, comm::THREADS, 0, stream()>>>(
      pp, reinterpret_cast<float*>(multicast_ptr), start, numel, (float)scale, (int)rank, world, (int)slot_base,
      status.data_ptr<int>(), (unsigned long long)(timeout_s * 1e9));
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
