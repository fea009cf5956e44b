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

// Two shapes of the same kernel:
//
// * narrow (buckets reduced while the backward pass still runs): it runs next to the persistent
//   tcgen05 GEMM instead of waiting for it.  The GEMM keeps one 320-thread CTA per SM with 168
//   registers per thread (53,760 of the SM's 65,536) and 226 KB of the SM's 228 KB of shared
//   memory, so what is left on every SM fits one block of 128 threads with at most 88 registers
//   each and only static shared memory.  The grid is one such block per SM, so the all-reduce
//   proceeds during the backward pass rather than in the gaps between GEMMs;
// * wide (the last bucket, reduced when the backward pass has finished and the GPU is otherwise
//   idle): 512 threads per block, four times the loads in flight, for NVLink bandwidth.
//
// Every thread issues all of its peer loads (peers x vectors, 8 vectors of 16 bytes) before it
// uses any: the loop is bound by NVLink latency (a few microseconds), so bytes in flight decide
// the rate.
constexpr int AR_THREADS = 128;       // narrow
constexpr int AR_MIN_BLOCKS = 6;      // 65,536 / (128 x 6) -> the compiler stays at or below 85 registers
constexpr int AR_WIDE_THREADS = 512;  // wide

template <int MAXW, int AR_THREADS_, int MINB>
__global__ void __launch_bounds__(AR_THREADS_, MINB)
    bucket_allreduce_kernel(Peers pp, float* mc, long long start, long long n, float scale, int rank, int world, int slot_base,
                            int* status, unsigned long long timeout_ns) {
  constexpr int AR_THREADS = AR_THREADS_;
  // chunk per owner rank (multiple of 4 floats), sub-range per block
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
    // NVLink-switch reduction: the switch sums the G copies (ld_reduce) and writes the result to
    // every rank (st); each rank handles its own chunk.  Eight vectors per thread in flight.  The
    // gradients were written through the unicast address and are read through the multicast one,
    // two virtual aliases of the same memory: the alias fence orders the two views.
    asm volatile("fence.proxy.alias;" ::: "memory");
    constexpr int U = 8;
    constexpr long long STEP = (long long)AR_THREADS * 4 * U;
    for (long long i0 = lo + threadIdx.x * 4; i0 < hi; i0 += STEP) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long i = i0 + (long long)u * AR_THREADS * 4;
        if (i + 3 < hi)
          asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                       : "=f"(v[u].x), "=f"(v[u].y), "=f"(v[u].z), "=f"(v[u].w)
                       : "l"(mc + start + i)
                       : "memory");
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long i = i0 + (long long)u * AR_THREADS * 4;
        if (i + 3 < hi) {
          asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + start + i), "f"(v[u].x * scale),
                       "f"(v[u].y * scale), "f"(v[u].z * scale), "f"(v[u].w * scale)
                       : "memory");
        } else {
          for (long long j = i; j < hi; ++j) {  // ragged tail of the range
            float a;
            asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(a) : "l"(mc + start + j) : "memory");
            asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc + start + j), "f"(a * scale) : "memory");
          }
        }
      }
    }
    asm volatile("fence.proxy.alias;" ::: "memory");
    block_barrier(pp, rank, world, slot_base, status, 2, timeout_ns);
    return;
  }
  // Two-shot over P2P loads.  Reduce-scatter: this rank sums its chunk over all peers (fixed rank
  // order, so every rank's copy of the result is bitwise identical) and scales it.
  constexpr int U = 8 / MAXW > 0 ? 8 / MAXW : 1;  // vectors per peer in flight
  constexpr long long STEP = (long long)AR_THREADS * 4 * U;
  for (long long i0 = lo + threadIdx.x * 4; i0 < hi; i0 += STEP) {
    float4 acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 v[MAXW][U];
#pragma unroll
    for (int p = 0; p < MAXW; ++p)
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long i = i0 + (long long)u * AR_THREADS * 4;
        if (p < world && i + 3 < hi) v[p][u] = *reinterpret_cast<const float4*>(pp.buf[p] + start + i);
      }
#pragma unroll
    for (int p = 0; p < MAXW; ++p)
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (p < world) {
          acc[u].x += v[p][u].x;
          acc[u].y += v[p][u].y;
          acc[u].z += v[p][u].z;
          acc[u].w += v[p][u].w;
        }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + (long long)u * AR_THREADS * 4;
      if (i + 3 < hi) {
        *reinterpret_cast<float4*>(pp.buf[rank] + start + i) =
            make_float4(acc[u].x * scale, acc[u].y * scale, acc[u].z * scale, acc[u].w * scale);
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
  // All-gather: copy every peer's reduced chunk (8 vectors in flight per thread).
  constexpr int UG = 8;
  constexpr long long STEPG = (long long)AR_THREADS * 4 * UG;
  for (int q = 1; q < world; ++q) {
    const int p = (rank + q) % world;
    range(p, lo, hi);
    for (long long i0 = lo + threadIdx.x * 4; i0 < hi; i0 += STEPG) {
      float4 v[UG];
#pragma unroll
      for (int u = 0; u < UG; ++u) {
        const long long i = i0 + (long long)u * AR_THREADS * 4;
        if (i + 3 < hi) v[u] = *reinterpret_cast<const float4*>(pp.buf[p] + start + i);
      }
#pragma unroll
      for (int u = 0; u < UG; ++u) {
        const long long i = i0 + (long long)u * AR_THREADS * 4;
        if (i + 3 < hi) *reinterpret_cast<float4*>(pp.buf[rank] + start + i) = v[u];
        else
          for (long long j = i; j < hi; ++j) pp.buf[rank][start + j] = pp.buf[p][start + j];
      }
    }
  }
  block_barrier(pp, rank, world, slot_base, status, 3, timeout_ns);
}


// ---------------------------------------------------------------------------------------------------
// FSDP: the reduce-scatter of one unit's gradient fused with the cast and the sharded AdamW update,
// and the all-gather of the unit's bf16 parameter shards, both over NVLink peer memory.
//
// fsdp_rs_adamw_kernel: every rank has copied its full (padded) gradient of the unit into its
// peer-mapped staging buffer.  Rank r owns elements [r*shard, (r+1)*shard) of the flat parameter.
// After a barrier with every peer, each block sums its sub-range of the owned shard over the G
// staging buffers in rank order (fp32 accumulation), multiplies by `scale` (1/G for an average),
// zeroes the padding tail (local index >= valid), and applies AdamW to the fp32 master shard and
// its moments in the same pass.  The bf16 copy of the updated shard goes to this rank's
// peer-mapped parameter buffer, which the next all-gather reads.  A closing barrier keeps every
// peer from overwriting its staging buffer while another rank still reads it; once the whole
// kernel has finished on a rank, every peer has finished writing its parameter shard too, so the
// next all-gather (stream-ordered after this kernel) reads updated shards.
//
// fsdp_all_gather_kernel: copies every peer's bf16 shard into the local full buffer with 16-byte
// P2P loads.  It needs no barrier of its own: the reduce-scatter kernels' barriers order every
// write of a shard buffer against every read (see above), and the first all-gather follows a
// stream-ordered barrier after the buffers were initialised.

struct ShardPeers {
  const void* buf[MAX_RANKS];
  uint32_t* pad[MAX_RANKS];
};

template <typename T>
struct Vec8;  // eight consecutive gradient elements

template <>
struct Vec8<__nv_bfloat16> {
  uint4 raw;
  __device__ __forceinline__ void load(const void* base, long long i) {
    raw = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + i);
  }
  __device__ __forceinline__ void add_to(float* acc) const {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      acc[2 * j] += f.x;
      acc[2 * j + 1] += f.y;
    }
  }
  static __device__ __forceinline__ float scalar(const void* base, long long i) {
    return bf2f(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  }
};

template <>
struct Vec8<float> {
  float4 lo, hi;
  __device__ __forceinline__ void load(const void* base, long long i) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    lo = p[0];
    hi = p[1];
  }
  __device__ __forceinline__ void add_to(float* acc) const {
    acc[0] += lo.x; acc[1] += lo.y; acc[2] += lo.z; acc[3] += lo.w;
    acc[4] += hi.x; acc[5] += hi.y; acc[6] += hi.z; acc[7] += hi.w;
  }
  static __device__ __forceinline__ float scalar(const void* base, long long i) {
    return reinterpret_cast<const float*>(base)[i];
  }
};

struct AdamParams {
  float beta1, beta2, eps, wd;
  float lr, gs, step, decay, bc2_sqrt;
  bool skip;
};

__device__ __forceinline__ void adam_one(float g, float& p, float& m, float& v, const AdamParams& a) {
  const float gj = g * a.gs;
  m = m + (1.f - a.beta1) * (gj - m);
  v = a.beta2 * v + (1.f - a.beta2) * gj * gj;
  const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
  p = p * a.decay - a.step * m / denom;
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(THREADS) fsdp_rs_adamw_kernel(ShardPeers sp, long long shard, long long valid, float scale,
                                                                float* __restrict__ param, float* __restrict__ mom1,
                                                                float* __restrict__ mom2, __nv_bfloat16* __restrict__ out16,
                                                                float* __restrict__ grad_out, const float* __restrict__ hyper,
                                                                float beta1, float beta2, float eps, float wd, int rank, int world,
                                                                int slot_base, int* status, unsigned long long timeout_ns,
                                                                int slice) {
  Peers pp{};
#pragma unroll
  for (int p = 0; p < MAX_RANKS; ++p) pp.pad[p] = sp.pad[p];
  if (!block_barrier(pp, rank, world, slot_base, status, 11, timeout_ns)) return;
  AdamParams a;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.wd = wd;
  a.lr = hyper[0];
  a.gs = hyper[2];
  a.skip = hyper[3] != 0.f;
  const float t = hyper[1];
  a.step = a.lr / (1.f - powf(beta1, t));
  a.bc2_sqrt = sqrtf(1.f - powf(beta2, t));
  a.decay = 1.f - a.lr * wd;
  // This rank's shard inside every staging buffer: slice `slice` (its index in the shard group;
  // under hybrid sharding the peers are every rank of the data-parallel x shard group, and the
  // replicas of a shard sum the same slice of each other's buffers).
  const long long base = (long long)slice * shard;
  const long long per_block = ((shard + gridDim.x - 1) / gridDim.x + 7) / 8 * 8;
  const long long lo = (long long)blockIdx.x * per_block;
  const long long hi = min(lo + per_block, shard);
  if (VEC) {
    for (long long i = lo + threadIdx.x * 8; i < hi; i += (long long)THREADS * 8) {
      // all peers' vectors in flight before any is used
      Vec8<T> in[MAX_RANKS];
#pragma unroll
      for (int p = 0; p < MAX_RANKS; ++p)
        if (p < world) in[p].load(sp.buf[p], base + i);
      float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < MAX_RANKS; ++p)
        if (p < world) in[p].add_to(g);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[j] = (i + j < valid) ? g[j] * scale : 0.f;
      if (grad_out != nullptr) {
        float4* go = reinterpret_cast<float4*>(grad_out + i);
        go[0] = make_float4(g[0], g[1], g[2], g[3]);
        go[1] = make_float4(g[4], g[5], g[6], g[7]);
      }
      if (a.skip) continue;
      float4* pp4 = reinterpret_cast<float4*>(param + i);
      float4* m4 = reinterpret_cast<float4*>(mom1 + i);
      float4* v4 = reinterpret_cast<float4*>(mom2 + i);
      float4 pv[2] = {pp4[0], pp4[1]}, mv[2] = {m4[0], m4[1]}, vv[2] = {v4[0], v4[1]};
      float* pf = reinterpret_cast<float*>(pv);
      float* mf = reinterpret_cast<float*>(mv);
      float* vf = reinterpret_cast<float*>(vv);
#pragma unroll
      for (int j = 0; j < 8; ++j) adam_one(g[j], pf[j], mf[j], vf[j], a);
      pp4[0] = pv[0];
      pp4[1] = pv[1];
      m4[0] = mv[0];
      m4[1] = mv[1];
      v4[0] = vv[0];
      v4[1] = vv[1];
      __align__(16) __nv_bfloat16 b[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = f2bf(pf[j]);
      *reinterpret_cast<uint4*>(out16 + i) = *reinterpret_cast<const uint4*>(b);
    }
  } else {
    for (long long i = lo + threadIdx.x; i < hi; i += THREADS) {
      float g = 0.f;
      for (int p = 0; p < world; ++p) g += Vec8<T>::scalar(sp.buf[p], base + i);
      g = i < valid ? g * scale : 0.f;
      if (grad_out != nullptr) grad_out[i] = g;
      if (a.skip) continue;
      float pv = param[i], mv = mom1[i], vv = mom2[i];
      adam_one(g, pv, mv, vv, a);
      param[i] = pv;
      mom1[i] = mv;
      mom2[i] = vv;
      out16[i] = f2bf(pv);
    }
  }
  block_barrier(pp, rank, world, slot_base, status, 12, timeout_ns);
}

template <bool VEC>
__global__ void __launch_bounds__(THREADS) fsdp_all_gather_kernel(ShardPeers sp, __nv_bfloat16* __restrict__ out, long long shard,
                                                                  int rank, int world) {
  const long long stride = (long long)gridDim.x * THREADS;
  if (VEC) {
    constexpr int UNROLL = 4;
    const long long n8 = shard / 8;
    const long long total = n8 * world;
    uint4* dst = reinterpret_cast<uint4*>(out);
    for (long long i0 = blockIdx.x * (long long)THREADS + threadIdx.x; i0 < total; i0 += stride * UNROLL) {
      uint4 v[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = i0 + u * stride;
        if (i < total) {
          const int q = (int)(i / n8);
          const int p = (rank + q) % world;  // the local shard first, then the peers in rotation
          v[u] = reinterpret_cast<const uint4*>(sp.buf[p])[i - (long long)q * n8];
        }
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const long long i = i0 + u * stride;
        if (i < total) {
          const int q = (int)(i / n8);
          const int p = (rank + q) % world;
          dst[(long long)p * n8 + (i - (long long)q * n8)] = v[u];
        }
      }
    }
  } else {
    const long long total = shard * world;
    for (long long i = blockIdx.x * (long long)THREADS + threadIdx.x; i < total; i += stride) {
      const int p = (int)(i / shard);
      out[i] = reinterpret_cast<const __nv_bfloat16*>(sp.buf[p])[i - (long long)p * shard];
    }
  }
}


// One block running the peer barrier of rank 0 in a group of two, with both "signal pads" in local
// memory.  Used by the tests to exercise the bounded wait: with nothing setting this rank's slot
// the wait runs out and the status word records the stage; with the slot pre-set (a peer that
// already arrived) the barrier completes at once.
__global__ void __launch_bounds__(THREADS) barrier_probe_kernel(uint32_t* pad0, uint32_t* pad1, int* status,
                                                                 unsigned long long timeout_ns) {
  Peers pp{};
  pp.pad[0] = pad0;
  pp.pad[1] = pad1;
  block_barrier(pp, 0, 2, 0, status, 99, timeout_ns);
}

}  // namespace comm

void bucket_all_reduce(at::Tensor flat, std::vector<int64_t> buffer_ptrs, std::vector<int64_t> pad_ptrs, int64_t multicast_ptr,
                       int64_t start, int64_t numel, double scale, int64_t rank, int64_t slot_base, int64_t max_blocks,
                       at::Tensor status, double timeout_s, bool wide, int64_t min_peer_slots) {
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
  // One block per SM (the blocks co-reside with a running GEMM, see bucket_allreduce_kernel), fewer
  // when the bucket is small.  Every block waits on its peers, and all of them fit on the GPU at once.
  const long long chunk = (numel + world - 1) / world;
  const int blocks = (int)std::max<long long>(
      1, std::min<long long>(std::min<long long>(max_blocks, num_sms()),
                             (chunk + (wide ? comm::AR_WIDE_THREADS : comm::AR_THREADS) * 32 - 1) /
                                 ((wide ? comm::AR_WIDE_THREADS : comm::AR_THREADS) * 32)));
  auto launch = [&](auto kernel, int threads) {
    static bool configured = false;  // per instantiation: prefer the shared-memory carveout of the GEMM it runs beside
    if (!configured) {
      HT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared));
      configured = true;
    }
    kernel<<<blocks, threads, 0, stream()>>>(pp, reinterpret_cast<float*>(multicast_ptr), start, numel, (float)scale, (int)rank,
                                             world, (int)slot_base, status.data_ptr<int>(), (unsigned long long)(timeout_s * 1e9));
  };
  constexpr int NT = comm::AR_THREADS, WT = comm::AR_WIDE_THREADS, NB = comm::AR_MIN_BLOCKS;
  // The instantiation for up to `slots` peers (2, 4 or 8); `min_peer_slots` can ask for a wider one
  // than the group needs (tests run the 8-peer code on two GPUs that way).
  const int slots = std::max<int>(world, (int)min_peer_slots);
  if (wide) {
    if (slots <= 2) launch(comm::bucket_allreduce_kernel<2, WT, 1>, WT);
    else if (slots <= 4) launch(comm::bucket_allreduce_kernel<4, WT, 1>, WT);
    else launch(comm::bucket_allreduce_kernel<8, WT, 1>, WT);
  } else {
    if (slots <= 2) launch(comm::bucket_allreduce_kernel<2, NT, NB>, NT);
    else if (slots <= 4) launch(comm::bucket_allreduce_kernel<4, NT, NB>, NT);
    else launch(comm::bucket_allreduce_kernel<8, NT, NB>, NT);
  }
  HT_CUDA_CHECK(cudaGetLastError());
}


namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

void fsdp_reduce_scatter_adamw(at::Tensor staging, std::vector<int64_t> grad_ptrs, std::vector<int64_t> pad_ptrs, int64_t rank,
                               int64_t shard, int64_t valid, double scale, at::Tensor param, at::Tensor exp_avg,
                               at::Tensor exp_avg_sq, at::Tensor shard16, c10::optional<at::Tensor> grad_out, at::Tensor hyper,
                               double beta1, double beta2, double eps, double wd, int64_t slot_base, int64_t max_blocks,
                               at::Tensor status, double timeout_s, int64_t slice) {
  const c10::cuda::CUDAGuard guard(param.device());
  const int world = (int)grad_ptrs.size();
  HT_CHECK(world >= 2 && world <= comm::MAX_RANKS, "fsdp_reduce_scatter_adamw supports 2..8 ranks");
  HT_CHECK((int)pad_ptrs.size() == world, "one signal pad per rank expected");
  HT_CHECK(rank >= 0 && rank < world, "rank out of range");
  if (slice < 0) slice = rank;
  HT_CHECK(slice < world, "shard slice out of range");
  HT_CHECK(staging.scalar_type() == at::kBFloat16 || staging.scalar_type() == at::kFloat, "bf16 or fp32 gradient staging expected");
  HT_CHECK(staging.numel() >= shard * (slice + 1), "the staging buffer must hold the unit's padded gradient");
  HT_CHECK(valid >= 0 && valid <= shard, "valid must lie in [0, shard]");
  for (const at::Tensor* t : {&param, &exp_avg, &exp_avg_sq})
    HT_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == shard, "fp32 shard, moments of the shard size");
  HT_CHECK(shard16.scalar_type() == at::kBFloat16 && shard16.is_contiguous() && shard16.numel() == shard, "bf16 shard buffer size");
  HT_CHECK(hyper.scalar_type() == at::kFloat && hyper.numel() >= 4 && hyper.is_cuda(), "device hyper-parameter vector expected");
  HT_CHECK(status.scalar_type() == at::kInt, "int32 status expected");
  float* gout = nullptr;
  if (grad_out.has_value() && grad_out->defined()) {
    HT_CHECK(grad_out->scalar_type() == at::kFloat && grad_out->is_contiguous() && grad_out->numel() == shard, "grad_out size");
    gout = grad_out->data_ptr<float>();
  }
  if (shard == 0) return;
  comm::ShardPeers sp{};
  bool vec = shard % 8 == 0;
  for (int p = 0; p < world; ++p) {
    sp.buf[p] = reinterpret_cast<const void*>(grad_ptrs[p]);
    sp.pad[p] = reinterpret_cast<uint32_t*>(pad_ptrs[p]);
    vec = vec && aligned16(sp.buf[p]);
  }
  vec = vec && aligned16(param.data_ptr()) && aligned16(exp_avg.data_ptr()) && aligned16(exp_avg_sq.data_ptr()) &&
        aligned16(shard16.data_ptr()) && (gout == nullptr || aligned16(gout));
  // At most one block per SM: every block waits at the barriers for the same block index on the
  // peers, so the whole grid must be resident at once (one 512-thread block per SM fits).
  const int blocks = (int)std::max<long long>(
      1, std::min<long long>(std::min<long long>(max_blocks, num_sms()), (shard + comm::THREADS * 8 - 1) / (comm::THREADS * 8)));
  const unsigned long long tns = (unsigned long long)(timeout_s * 1e9);
  auto* out16 = reinterpret_cast<__nv_bfloat16*>(shard16.data_ptr());
#define HT_FSDP_RS(T, V)                                                                                                   \
  comm::fsdp_rs_adamw_kernel<T, V><<<blocks, comm::THREADS, 0, stream()>>>(                                                \
      sp, shard, valid, (float)scale, param.data_ptr<float>(), exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(), out16, \
      gout, hyper.data_ptr<float>(), (float)beta1, (float)beta2, (float)eps, (float)wd, (int)rank, world, (int)slot_base,      \
      status.data_ptr<int>(), tns, (int)slice)
  if (staging.scalar_type() == at::kBFloat16) {
    if (vec) HT_FSDP_RS(__nv_bfloat16, true); else HT_FSDP_RS(__nv_bfloat16, false);
  } else {
    if (vec) HT_FSDP_RS(float, true); else HT_FSDP_RS(float, false);
  }
#undef HT_FSDP_RS
  HT_CUDA_CHECK(cudaGetLastError());
}

void fsdp_all_gather(std::vector<int64_t> shard_ptrs, at::Tensor out, int64_t shard, int64_t rank) {
  const c10::cuda::CUDAGuard guard(out.device());
  const int world = (int)shard_ptrs.size();
  HT_CHECK(world >= 2 && world <= comm::MAX_RANKS, "fsdp_all_gather supports 2..8 ranks");
  HT_CHECK(rank >= 0 && rank < world, "rank out of range");
  HT_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == shard * world,
           "bf16 output of world x shard elements expected");
  if (shard == 0) return;
  comm::ShardPeers sp{};
  bool vec = shard % 8 == 0 && aligned16(out.data_ptr());
  for (int p = 0; p < world; ++p) {
    sp.buf[p] = reinterpret_cast<const void*>(shard_ptrs[p]);
    vec = vec && aligned16(sp.buf[p]);
  }
  const long long work = vec ? shard / 8 * world : shard * world;
  const int blocks = (int)std::max<long long>(
      1, std::min<long long>((long long)num_sms() * 4, (work + comm::THREADS * 4 - 1) / (comm::THREADS * 4)));
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (vec)
    comm::fsdp_all_gather_kernel<true><<<blocks, comm::THREADS, 0, stream()>>>(sp, o, shard, (int)rank, world);
  else
    comm::fsdp_all_gather_kernel<false><<<blocks, comm::THREADS, 0, stream()>>>(sp, o, shard, (int)rank, world);
  HT_CUDA_CHECK(cudaGetLastError());
}


// All-gather of bf16 shards by the copy engines: one cudaMemcpyAsync per peer (the local shard first,
// then the peers in rotation).  Uses no SMs, so it overlaps a compute kernel that occupies all of them.
void fsdp_all_gather_copy_engine(std::vector<int64_t> shard_ptrs, at::Tensor out, int64_t shard, int64_t rank) {
  const c10::cuda::CUDAGuard guard(out.device());
  const int world = (int)shard_ptrs.size();
  HT_CHECK(world >= 1 && world <= comm::MAX_RANKS, "fsdp_all_gather_copy_engine supports 1..8 ranks");
  HT_CHECK(rank >= 0 && rank < world, "rank out of range");
  HT_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == shard * world,
           "bf16 output of world x shard elements expected");
  const size_t bytes = (size_t)shard * sizeof(__nv_bfloat16);
  char* dst = reinterpret_cast<char*>(out.data_ptr());
  for (int q = 0; q < world; ++q) {
    const int p = (int)((rank + q) % world);
    HT_CUDA_CHECK(cudaMemcpyAsync(dst + (size_t)p * bytes, reinterpret_cast<const void*>(shard_ptrs[p]), bytes,
                                  cudaMemcpyDeviceToDevice, stream()));
  }
}


void barrier_probe(at::Tensor pads, at::Tensor status, double timeout_s) {
  const c10::cuda::CUDAGuard guard(pads.device());
  HT_CHECK(pads.is_cuda() && pads.scalar_type() == at::kInt && pads.dim() == 2 && pads.size(0) == 2 && pads.size(1) >= 2 &&
               pads.is_contiguous(), "pads: int32 [2, >=2] on the device");
  HT_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 2, "status: int32 [>=2] on the device");
  HT_CHECK(timeout_s > 0 && timeout_s <= 10, "the probe's timeout must lie in (0, 10] seconds");
  auto* base = reinterpret_cast<uint32_t*>(pads.data_ptr());
  comm::barrier_probe_kernel<<<1, comm::THREADS, 0, stream()>>>(base, base + pads.size(1), status.data_ptr<int>(),
                                                                  (unsigned long long)(timeout_s * 1e9));
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
