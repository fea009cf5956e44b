// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[M,N] = epilogue(alpha * A . B^T + bias) (+ beta * D)
//
// Data path: TMA (cp.async.bulk.tensor, 128-byte swizzle) moves A/B tiles into a 4-stage
// shared-memory ring; one thread issues tcgen05.mma (M=128, N=256, K=16) into a
// double-buffered fp32 accumulator in tensor memory; eight epilogue warps read it back with
// tcgen05.ld, apply the fused epilogue in registers, stage 32-row x 128-byte pieces in swizzled
// shared memory and write them with TMA bulk-tensor stores (or TMA fp32 reduce-add for the
// `beta = 1` gradient accumulation), while the tensor cores already work on the next tile.
// Outputs whose rows are not 16-byte aligned fall back to per-thread stores.  One CTA per SM
// loops over output tiles (grouped along M for L2 reuse).
//
// Operands may be K-major or MN-major (the instruction descriptor's transpose bits), which
// covers the forward (A=X, B=W), data-gradient (B=W read MN-major) and weight-gradient (both
// MN-major) products of a linear layer without any transpose in memory.
//
// Warp roles (320 threads): warp 0 = TMA producer, warp 1 = MMA issuer and TMEM owner,
// warps 2..9 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31, i.e. tile rows; warps 2..5 take
// the even 128-byte column chunks of the tile and warps 6..9 the odd ones).
// Every wait is bounded; on timeout an error code is written to `err` and the CTA unwinds,
// still freeing its tensor memory.

#include "common.cuh"

#include <cstring>

namespace ht {
namespace tcg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KiB
constexpr int B_BYTES = BN * BK * 2;   // 32 KiB
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 2 * BN;      // double-buffered accumulator (512 columns)
constexpr int GROUP_M = 8;
constexpr int EPI_STAGE_BYTES = 32 * 128;  // one 32-row x 128-byte output piece per epilogue warp
constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + EPI_WARPS * EPI_STAGE_BYTES + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget of one sm_100 CTA exceeded");

enum Epilogue : int { kPlain = 0, kGelu = 1, kGeluBwd = 2, kSwiGLU = 3, kSwiGLUBwd = 4 };

// Compile-time epilogue kind of a kernel instance.  Each instance carries only its own epilogue
// code, which keeps the kernel small enough that the epilogue warps do not evict the MMA
// issue loop from the instruction cache.  kKindGeneric decides everything at run time (the
// fallback for unaligned outputs and the collective kernels).
enum EpiKind : int { kKindGeneric = 0, kKindBf16 = 1, kKindF32 = 2, kKindGelu = 3, kKindGeluBwd = 4, kKindSwiGLU = 5,
                     kKindSwiGLUBwd = 6 };

struct EpiParams {
  void* d;
  long long ldd;
  int d_fp32;
  const float* bias_f32;
  const __nv_bfloat16* bias_bf16;
  __nv_bfloat16* aux;
  long long ldaux;
  const float* alpha;
  float beta;
  int epi;
  int vec_ok;      // D (and aux) rows are 16-byte aligned: vector stores allowed
  int tma_d;       // write D through the output tensor map
  int tma_aux;     // write the GELU pre-activation through the aux tensor map
  int reduce_add;  // D (fp32) += result through TMA reduce-add (beta == 1)
  int splits;      // split-K factor: work unit u covers tile u / splits, K-range u % splits
  int split_rows;  // rows per split slice of the fp32 workspace (split-K only)
  int half_n;      // SwiGLU kinds: F, the column of the first `up` feature in the [gate | up] tensors
};

// ------------------------------------------------------------------------------------------------
// Collective mode (tensor / sequence parallelism over NVLink peer memory).
//
// Operand rows that are sequence positions may live on another GPU: every rank holds a shard of
// `rows_per_rank` positions of each of the `batch` sequences in a peer-mapped buffer, and the
// logical operand is the concatenation of the shards.  The producer warp then loads each tile
// straight from the owner's shard with a (non-multicast) TMA load through that peer's tensor
// map, after the owner has published the shard (a device-side epoch written into this rank's
// flag word).  In reduce-scatter mode the epilogue stores every output tile into the receive
// slot of the rank that owns its rows; the last CTA to finish publishes the epoch to all peers.
// Epochs live in device memory, so the same launch can be replayed from a CUDA graph.
// ------------------------------------------------------------------------------------------------
constexpr int MAX_PEERS = 8;

struct CollParams {
  CUtensorMap a[MAX_PEERS];    // per-owner A shard maps (a_mode != 0)
  CUtensorMap b[MAX_PEERS];    // per-owner B shard maps (b_mode != 0)
  CUtensorMap out[MAX_PEERS];  // per-owner receive maps [world * batch][rows_per_rank][N] (rs)
  uint32_t* flags_local;       // this rank's flag words [site][MAX_PEERS], written by the peers
  uint32_t* flags_peer[MAX_PEERS];
  uint32_t* epoch;             // this call site's epoch counter (local memory)
  int* done;                   // this call site's completion counter (local memory)
  int site;
  int advance;                 // 1: a new collective call (epoch + 1, publish); 0: reuse the epoch
  int a_mode;                  // 0 local; 1 owner by M block (K-major A); 2 owner by K block (MN-major A)
  int b_mode;                  // 0 local; 2 owner by K block (MN-major B)
  int rs;                      // epilogue writes rows into their owner's receive slot
  int rank, world, batch, seq, rows_per_rank;
  unsigned long long timeout_ns;
  // a_mode 1 (all-gather of a K-major A): every remote 128-row block crosses NVLink once.  The
  // copy warp of each CTA pulls blocks from the owners' shards (a_src) into the local gathered
  // buffer and flags them (block_flags, indexed by physical M block); tiles of remote blocks are
  // then loaded from the gathered buffer through `gathered_map`.  The gathered buffer also
  // serves the backward pass.
  CUtensorMap gathered_map;
  const __nv_bfloat16* a_src[MAX_PEERS];
  __nv_bfloat16* gathered;
  uint32_t* block_flags;
  int k_dim;
};

constexpr int COLL_THREADS = THREADS + 32;  // + one copy warp

// a_mode 1 schedules M blocks by owner, starting with this rank's own shard: logical block L
// -> physical block.  Both the producer and the epilogue use it.
__device__ __forceinline__ int coll_phys_mblock(const CollParams& c, int L) {
  const int per_batch = c.rows_per_rank / BM;
  const int per_owner = c.batch * per_batch;
  const int q = L / per_owner;
  const int rem = L - q * per_owner;
  const int bidx = rem / per_batch;
  const int j = rem - bidx * per_batch;
  const int owner = (c.rank + q) % c.world;
  return (bidx * c.seq + owner * c.rows_per_rank) / BM + j;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Owner rank, local row and sequence index of logical sequence row `g`.
__device__ __forceinline__ void seq_owner(const CollParams& c, int g, int& owner, int& local_row, int& bidx) {
  bidx = g / c.seq;
  const int s = g - bidx * c.seq;
  owner = s / c.rows_per_rank;
  local_row = s - owner * c.rows_per_rank;
}

// Bounded wait until `owner` has published epoch `epoch` for this call site.
__device__ __forceinline__ bool wait_published(const CollParams& c, int owner, uint32_t epoch, int* err) {
  const uint32_t* f = c.flags_local + c.site * MAX_PEERS + owner;
  const unsigned long long deadline = globaltimer_ns() + c.timeout_ns;
  while ((int)(ld_acquire_sys(f) - epoch) < 0) {
    if (globaltimer_ns() > deadline || *((volatile int*)err) != 0) {
      atomicCAS(err, 0, 40);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void publish_epoch(const CollParams& c, uint32_t epoch) {
  __threadfence_system();
  for (int q = 0; q < c.world; ++q)
    if (q != c.rank) st_release_sys(c.flags_peer[q] + c.site * MAX_PEERS + c.rank, epoch);
}

// K-blocks [kb0, kb1) of work unit `split` when the K loop is split `splits` ways.
__device__ __forceinline__ void split_range(int kblocks, int splits, int split, int& kb0, int& kb1) {
  const int per = (kblocks + splits - 1) / splits;
  kb0 = split * per;
  kb1 = min(kblocks, kb0 + per);
}

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = GROUP_M * num_n;
  const int group = tile / per_group;
  const int first_m = group * GROUP_M;
  const int gm = min(GROUP_M, num_m - first_m);
  const int r = tile - group * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

__device__ __forceinline__ void store_chunk(const EpiParams& ep, int row, int col0, int N, float alpha, float* v) {
  const bool full = col0 + 32 <= N;
  const bool vec = full && ep.vec_ok;
  // bias + alpha
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float x = v[i] * alpha;
    const int c = col0 + i;
    if (ep.bias_f32 != nullptr && (full || c < N)) x += ep.bias_f32[c];
    if (ep.bias_bf16 != nullptr && (full || c < N)) x += bf2f(ep.bias_bf16[c]);
    v[i] = x;
  }
  if (ep.epi == kGelu) {
    __nv_bfloat16* aux = ep.aux + (long long)row * ep.ldaux + col0;
    if (vec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __align__(16) __nv_bfloat16 pk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) pk[j] = f2bf(v[q * 8 + j]);
        *reinterpret_cast<uint4*>(aux + q * 8) = *reinterpret_cast<uint4*>(pk);
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) aux[i] = f2bf(v[i]);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
  } else if (ep.epi == kGeluBwd) {
    const __nv_bfloat16* aux = ep.aux + (long long)row * ep.ldaux + col0;
    if (vec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 raw = *reinterpret_cast<const uint4*>(aux + q * 8);
        const __nv_bfloat16* pk = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[q * 8 + j] *= gelu_tanh_grad(bf2f(pk[j]));
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) v[i] *= gelu_tanh_grad(bf2f(aux[i]));
    }
  }
  if (ep.d_fp32) {
    float* d = reinterpret_cast<float*>(ep.d) + (long long)row * ep.ldd + col0;
    if (vec) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 o = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
        if (ep.beta != 0.f) {
          const float4 old = *reinterpret_cast<const float4*>(d + q * 4);
          o.x += ep.beta * old.x;
          o.y += ep.beta * old.y;
          o.z += ep.beta * old.z;
          o.w += ep.beta * old.w;
        }
        *reinterpret_cast<float4*>(d + q * 4) = o;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) d[i] = v[i] + (ep.beta != 0.f ? ep.beta * d[i] : 0.f);
    }
  } else {
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(ep.d) + (long long)row * ep.ldd + col0;
    if (vec) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __align__(16) __nv_bfloat16 pk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) pk[j] = f2bf(v[q * 8 + j] + (ep.beta != 0.f ? ep.beta * bf2f(d[q * 8 + j]) : 0.f));
        *reinterpret_cast<uint4*>(d + q * 8) = *reinterpret_cast<uint4*>(pk);
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) d[i] = f2bf(v[i] + (ep.beta != 0.f ? ep.beta * bf2f(d[i]) : 0.f));
    }
  }
}

// Writes one thread's row of a 128-byte output piece into a 32-row staging tile laid out with the
// 128-byte swizzle the output tensor map expects (16-byte unit j of row r sits at unit j ^ (r % 8)).
__device__ __forceinline__ void stage_row(uint8_t* tile, int r, const uint4* units) {
  uint8_t* row = tile + r * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) << 4)) = units[j];
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void pack_bf16x64(const float* v, uint4* units) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    __align__(16) __nv_bfloat162 h[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(v[j * 8 + 2 * q], v[j * 8 + 2 * q + 1]);
    units[j] = *reinterpret_cast<const uint4*>(h);
  }
}

// Epilogue of one 128-byte column piece (CW = 64 bf16 or 32 fp32 output columns) of one row,
// through the staging tile and a TMA store.  `v` holds the raw accumulator values.
template <int CW, int KIND>
__device__ __forceinline__ void epilogue_piece_tma(const EpiParams& ep, const CUtensorMap* map_d, const CUtensorMap* map_aux,
                                                   uint8_t* tile, int lane, int row, int M, int col0, int N, int tile_row0,
                                                   float alpha, float* v, int z = -1) {
  const bool full = col0 + CW <= N;
#pragma unroll
  for (int i = 0; i < CW; ++i) v[i] *= alpha;
  if (ep.bias_f32 != nullptr) {
    const float* bp = ep.bias_f32 + col0;
    if (full && (reinterpret_cast<uintptr_t>(bp) & 15) == 0) {  // the same 16-byte vectors for every lane
#pragma unroll
      for (int q = 0; q < CW / 4; ++q) {
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(bp) + q);
        v[4 * q] += b4.x;
        v[4 * q + 1] += b4.y;
        v[4 * q + 2] += b4.z;
        v[4 * q + 3] += b4.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < CW; ++i)
        if (col0 + i < N) v[i] += __ldg(bp + i);
    }
  } else if (ep.bias_bf16 != nullptr) {
#pragma unroll
    for (int i = 0; i < CW; ++i)
      if (col0 + i < N) v[i] += bf2f(ep.bias_bf16[col0 + i]);
  }
  uint4 units[8];
  constexpr bool GENERIC = KIND == kKindGeneric;
  if (KIND == kKindGeluBwd || (GENERIC && ep.epi == kGeluBwd)) {
    const __nv_bfloat16* aux = ep.aux + (long long)row * ep.ldaux + col0;
    if (row < M && full) {
#pragma unroll
      for (int q = 0; q < CW / 8; ++q) {
        const uint4 raw = *reinterpret_cast<const uint4*>(aux + q * 8);
        const __nv_bfloat16* pk = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[q * 8 + j] *= gelu_tanh_grad(bf2f(pk[j]));
      }
    } else if (row < M) {
#pragma unroll
      for (int i = 0; i < CW; ++i) v[i] *= (col0 + i < N) ? gelu_tanh_grad(bf2f(aux[i])) : 0.f;
    }
  }
  if (KIND == kKindGelu || (GENERIC && ep.tma_aux)) {  // GELU forward: store the pre-activation first (bf16, CW == 64)
    if (CW == 64) {
      pack_bf16x64(v, units);
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
      stage_row(tile, lane, units);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(map_aux, tile, col0, tile_row0);
        bulk_commit();
      }
    }
  }
  if (KIND == kKindGelu || (GENERIC && ep.epi == kGelu)) {
#pragma unroll
    for (int i = 0; i < CW; ++i) v[i] = gelu_tanh(v[i]);
  }
  if (CW == 64) {
    pack_bf16x64(v, units);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) units[j] = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                                     __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
  }
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
  stage_row(tile, lane, units);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (GENERIC && z >= 0) tma_store_3d(map_d, tile, col0, tile_row0, z);
    else if ((KIND == kKindF32 || GENERIC) && ep.reduce_add) tma_reduce_add_2d(map_d, tile, col0, tile_row0);
    else tma_store_2d(map_d, tile, col0, tile_row0);
    bulk_commit();
  }
}

// All output tiles of one epilogue warp.  CW = output columns per 128-byte piece; TN = tile width.
// PAIR: a CTA of a pair kernel (tiles of 256 rows, this CTA's 128 rows in its own TMEM; the
// accumulator-free signal goes to the pair's first CTA, which issues the MMAs).
template <int CW, int KIND, int TN = BN, bool PAIR = false>
__device__ __forceinline__ void epilogue_loop(const EpiParams& ep, const CUtensorMap* map_d, const CUtensorMap* map_aux,
                                              uint8_t* tile, uint32_t tmem_base, uint64_t* tfull_bar, uint64_t* tempty_bar,
                                              int M, int N, int num_m, int num_n, int num_tiles, int warp, int lane, int* err,
                                              const CollParams* coll = nullptr) {
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const int row_in_tile = quarter * 32 + lane;
  const float alpha = ep.alpha != nullptr ? *ep.alpha : 1.f;
  constexpr int PIECES = TN / CW;
  int acc = 0;
  uint32_t acc_phase = 0;
  const int num_units = num_tiles * ep.splits;
  const int first = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int stride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int crank = PAIR ? (int)cluster_ctarank() : 0;
  for (int unit = first; unit < num_units; unit += stride) {
    int mb, nb;
    tile_coords(unit / ep.splits, num_m, num_n, mb, nb);
    if (PAIR) mb = mb * 2 + crank;  // this CTA's 128-row half of the pair tile
    if (coll != nullptr && coll->a_mode == 1) mb = coll_phys_mblock(*coll, mb);
    int out_row0 = (unit % ep.splits) * ep.split_rows + mb * BM + quarter * 32;
    const CUtensorMap* dmap = map_d;
    int z = -1;
    if (coll != nullptr && coll->rs) {  // rows go to their owner's receive slot for this rank
      int owner, lrow, bidx;
      seq_owner(*coll, mb * BM, owner, lrow, bidx);
      dmap = &coll->out[owner];
      out_row0 = lrow + quarter * 32;
      z = coll->rank * coll->batch + bidx;
    }
    if (!(PAIR ? mbar_wait_cluster(&tfull_bar[acc], acc_phase, err, 4) : mbar_wait(&tfull_bar[acc], acc_phase, err, 4))) break;
    tc_fence_after();
    const int row = mb * BM + row_in_tile;
#pragma unroll 1
    for (int c = half; c < PIECES; c += 2) {
      const int col0 = nb * TN + c * CW;
      if (col0 >= N) break;
      float v[CW];
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + c * CW;
#pragma unroll
      for (int s = 0; s < CW / 32; ++s) tmem_ld_32x32b_x32(taddr + 32 * s, v + 32 * s);
      if (KIND != kKindGeneric || ep.tma_d) {
        epilogue_piece_tma<CW, KIND>(ep, dmap, map_aux, tile, lane, row, M, col0, N, out_row0, alpha, v, z);
      } else if (row < M) {
#pragma unroll
        for (int s = 0; s < CW / 32; ++s)
          if (col0 + 32 * s < N) store_chunk(ep, row, col0 + 32 * s, N, alpha, v + 32 * s);
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (PAIR) mbar_arrive_cluster(smem_in_cta(&tempty_bar[acc], 0));
      else mbar_arrive(&tempty_bar[acc]);
    }
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1u;
    }
  }
  if (lane == 0) {
    bulk_wait_all();
    if (coll != nullptr && coll->rs) {
      // The stores went to peers' memory: order them before this CTA's completion signal at
      // system scope (the publishing thread is another warp).
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence_system();
    }
  }
  __syncwarp();
}

// ---------------- SwiGLU epilogues ----------------
// Output pieces here are 32 bf16 columns (64 bytes): the staging tile of each epilogue warp holds
// two 32-row x 64-byte slots used alternately, written with the 64-byte swizzle their tensor maps
// expect (16-byte unit j of row r at unit j ^ ((r / 2) % 4)).  Before a slot is rewritten, every
// bulk store but the most recent one (which read the other slot) must have read its source.
__device__ __forceinline__ void bulk_wait_read_allbut1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

__device__ __forceinline__ void pack_bf16x32(const float* v, uint4* units) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    units[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                          pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}

// Stages one 32-column piece of this lane's row in `slot` and stores it at (col, row0) of `map`.
__device__ __forceinline__ void store_piece64(const CUtensorMap* map, uint8_t* slot, int lane, const float* v, int col, int row0) {
  uint4 units[4];
  pack_bf16x32(v, units);
  if (lane == 0) bulk_wait_read_allbut1();
  __syncwarp();
  uint8_t* row = slot + lane * 64;
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(row + ((j ^ ((lane >> 1) & 3)) << 4)) = units[j];
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, slot, col, row0);
    bulk_commit();
  }
}

__device__ __forceinline__ float swiglu_bias(const EpiParams& ep, int c) {
  if (ep.bias_f32 != nullptr) return __ldg(ep.bias_f32 + c);
  if (ep.bias_bf16 != nullptr) return bf2f(ep.bias_bf16[c]);
  return 0.f;
}

// BWD = false (forward, tiles of TN/2 output columns): h[:, n] = gate + bias, h[:, F + n] = up +
//   bias through `map_aux`, and D[:, n] = silu(gate) * up through `map_d`.
// BWD = true (the down projection's data gradient, tiles of TN columns of dA): with gate and up
//   read back from h (`ep.aux`), D[:, n] = dA * up * silu'(gate) and D[:, F + n] = dA * silu(gate).
template <bool BWD, int TN>
__device__ __forceinline__ void epilogue_loop_swiglu(const EpiParams& ep, const CUtensorMap* map_d, const CUtensorMap* map_aux,
                                                     uint8_t* tile, uint32_t tmem_base, uint64_t* tfull_bar,
                                                     uint64_t* tempty_bar, int M, int N, int num_m, int num_n, int num_tiles,
                                                     int warp, int lane, int* err) {
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const float alpha = ep.alpha != nullptr ? *ep.alpha : 1.f;
  constexpr int TN_OUT = BWD ? TN : TN / 2;
  int acc = 0, slot = 0;
  uint32_t acc_phase = 0;
  for (int unit = blockIdx.x; unit < num_tiles; unit += gridDim.x) {
    int mb, nb;
    tile_coords(unit, num_m, num_n, mb, nb);
    const int row0 = mb * BM + quarter * 32;
    const int row = row0 + lane;
    if (!mbar_wait(&tfull_bar[acc], acc_phase, err, 4)) break;
    tc_fence_after();
    const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
    // The two warpgroups take alternate 32-column pieces of the tile's output columns.
#pragma unroll 1
    for (int c = half * 32; c < TN_OUT; c += 64) {
      const int col = nb * TN_OUT + c;
      if (col >= N) break;
      float x[32], y[32];
      tmem_ld_32x32b_x32(tbase + c, x);
      if constexpr (!BWD) {
        tmem_ld_32x32b_x32(tbase + TN / 2 + c, y);  // up features sit TN / 2 accumulator columns further on
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = x[i] * alpha + swiglu_bias(ep, col + i);
          y[i] = y[i] * alpha + swiglu_bias(ep, ep.half_n + col + i);
        }
        store_piece64(map_aux, tile + slot * 2048, lane, x, col, row0);
        slot ^= 1;
        store_piece64(map_aux, tile + slot * 2048, lane, y, ep.half_n + col, row0);
        slot ^= 1;
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = x[i] / (1.f + __expf(-x[i])) * y[i];
        store_piece64(map_d, tile + slot * 2048, lane, x, col, row0);
        slot ^= 1;
      } else {
        float g[32];
        if (row < M) {
          const __nv_bfloat16* hp = ep.aux + (long long)row * ep.ldaux + col;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 gr = *reinterpret_cast<const uint4*>(hp + q * 8);
            const uint4 ur = *reinterpret_cast<const uint4*>(hp + ep.half_n + q * 8);
            const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(&gr);
            const __nv_bfloat16* up = reinterpret_cast<const __nv_bfloat16*>(&ur);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              g[q * 8 + j] = bf2f(gp[j]);
              y[q * 8 + j] = bf2f(up[j]);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) g[i] = y[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float da = x[i] * alpha;
          const float sig = 1.f / (1.f + __expf(-g[i]));
          const float sl = g[i] * sig;
          x[i] = da * y[i] * sig * (1.f + g[i] * (1.f - sig));  // d gate
          y[i] = da * sl;                                         // d up
        }
        store_piece64(map_d, tile + slot * 2048, lane, x, col, row0);
        slot ^= 1;
        store_piece64(map_d, tile + slot * 2048, lane, y, ep.half_n + col, row0);
        slot ^= 1;
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1u;
    }
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Copies A slices of 128 rows x 64 columns (16 KB) from the owners' shards into the gathered
// buffer: remote owners rank+1, rank+2, ... first in the order the GEMM consumes them, this
// rank's own shard last (it is only needed by the backward pass).  The slices are spread over
// the copy warps of every CTA so that enough bytes are in flight to fill NVLink; each slice is
// flagged (per 128-row block and 64-column block) once its bytes are visible to TMA loads.
__device__ __noinline__ void coll_copy_warp(const CollParams& c, uint32_t epoch, int lane, int* err) {
  const int per_batch = c.rows_per_rank / BM;
  const int per_owner = c.batch * per_batch;
  const int kbs = c.k_dim / BK;
  const int total = c.world * per_owner * kbs;
  uint32_t ready = 0;
  for (int ci = blockIdx.x; ci < total; ci += gridDim.x) {
    const int blk = ci / kbs;
    const int kb = ci - blk * kbs;
    const int q = (blk / per_owner + 1) % c.world;  // remote owners first, own shard last
    const int rem = blk % per_owner;
    const int bidx = rem / per_batch;
    const int j = rem - bidx * per_batch;
    const int owner = (c.rank + q) % c.world;
    if (owner != c.rank && !(ready >> owner & 1u)) {
      bool ok = true;
      if (lane == 0) ok = wait_published(c, owner, epoch, err);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return;
      ready |= 1u << owner;
    }
    const __nv_bfloat16* src = c.a_src[owner] + ((long long)bidx * c.rows_per_rank + j * BM) * c.k_dim + kb * BK;
    const int row0 = bidx * c.seq + owner * c.rows_per_rank + j * BM;
    __nv_bfloat16* dst = c.gathered + (long long)row0 * c.k_dim + kb * BK;
    // 128 rows x 8 vectors of 16 bytes: 32 per lane, in two waves of 16 loads in flight.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint4 buf[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int v = (half * 16 + u) * 32 + lane;
        buf[u] = *reinterpret_cast<const uint4*>(src + (long long)(v >> 3) * c.k_dim + (v & 7) * 8);
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int v = (half * 16 + u) * 32 + lane;
        *reinterpret_cast<uint4*>(dst + (long long)(v >> 3) * c.k_dim + (v & 7) * 8) = buf[u];
      }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence();
    __syncwarp();
    if (lane == 0 && owner != c.rank) {
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(c.block_flags + (row0 / BM) * kbs + kb), "r"(epoch)
                   : "memory");
    }
  }
}

template <bool A_MN, bool B_MN, bool COLL, int KIND, int TN = BN>
__device__ __forceinline__ void gemm_body(const CUtensorMap& tma_a, const CUtensorMap& tma_b, const CUtensorMap& tma_d,
                                          const CUtensorMap& tma_aux, int M, int N, int K, const EpiParams& ep, int* err,
                                          const CollParams* coll) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  constexpr int TB_BYTES = TN * BK * 2;  // one stage of the B tile
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sEpi = smem + STAGES * (A_BYTES + TB_BYTES);  // 1024-byte aligned staging tiles

  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_slot;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // SwiGLU forward: a tile's TN accumulator columns are TN / 2 gate features and the same TN / 2
  // up features, so it covers TN / 2 output columns.
  constexpr bool SWI = KIND == kKindSwiGLU;
  constexpr int TN_OUT = SWI ? TN / 2 : TN;
  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + TN_OUT - 1) / TN_OUT;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles * ep.splits;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], EPI_WARPS);
    }
    fence_barrier_init();
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
    if (ep.tma_d) prefetch_tensormap(&tma_d);
    if (ep.tma_aux) prefetch_tensormap(&tma_aux);
  }
  uint32_t epoch = 0;
  if constexpr (COLL) {
    epoch = *((volatile uint32_t*)coll->epoch) + (uint32_t)coll->advance;
    // Gather-side publication: this rank's shard (written by earlier work on this stream) is
    // ready for the peers' loads.
    if (blockIdx.x == 0 && threadIdx.x == 0 && coll->advance && !coll->rs && (coll->a_mode || coll->b_mode))
      publish_epoch(*coll, epoch);
  }
  if (warp == 1) tmem_alloc(&tmem_base_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    uint32_t ready_mask = 0;
    (void)ready_mask;
    // Collective-mode constants, read from the parameter block once.
    const int c_rank = COLL ? coll->rank : 0;
    const int c_amode = COLL ? coll->a_mode : 0;
    const int c_bmode = COLL ? coll->b_mode : 0;
    const CUtensorMap* own_map = COLL ? &coll->a[c_rank] : nullptr;
    const CUtensorMap* gathered_map = COLL ? &coll->gathered_map : nullptr;
    for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x) {
      int mb, nb, kb0, kb1;
      tile_coords(unit / ep.splits, num_m, num_n, mb, nb);
      if (COLL && coll->a_mode == 1) mb = coll_phys_mblock(*coll, mb);
      split_range(kblocks, ep.splits, unit % ep.splits, kb0, kb1);
      const int m0 = mb * BM, n0 = nb * TN_OUT;
      int tile_src = 0, tile_lrow = 0, tile_b = 0;  // A source of this tile: 0 local map, 1 own shard, 2 gathered copy
      if (COLL && c_amode == 1) {
        // A tile of a remote block: the whole warp polls the block's slice flags in parallel
        // until every slice is in the gathered copy (one round trip per tile, not per slice).
        int owner;
        seq_owner(*coll, m0, owner, tile_lrow, tile_b);
        tile_src = owner == c_rank ? 1 : 2;
        if (owner != c_rank) {
          const int kbs = coll->k_dim / BK;
          const uint32_t* f = coll->block_flags + mb * kbs;
          const unsigned long long deadline = globaltimer_ns() + coll->timeout_ns;
          while (true) {
            bool mine = true;
            for (int i = lane; i < kbs; i += 32) mine = mine && (int)(ld_acquire_gpu(f + i) - epoch) >= 0;
            if (__all_sync(0xffffffffu, mine)) break;
            if (globaltimer_ns() > deadline || *((volatile int*)err) != 0) {
              if (lane == 0) atomicCAS(err, 0, 42);
              ok = false;
              break;
            }
          }
          __syncwarp();
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, 1)) {
          ok = false;
          break;
        }
        if (COLL && lane == 0) {
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * TB_BYTES;
          const int k0 = kb * BK;
          int b_owner = c_rank, b_row = 0, b_b = 0, a_owner2 = c_rank, a_row2 = 0, a_b2 = 0;
          if (c_amode == 2) seq_owner(*coll, k0, a_owner2, a_row2, a_b2);
          if (c_bmode == 2) seq_owner(*coll, k0, b_owner, b_row, b_b);
          if (c_amode == 2 && a_owner2 != c_rank && !(ready_mask >> a_owner2 & 1u)) {
            ok = wait_published(*coll, a_owner2, epoch, err);
            ready_mask |= 1u << a_owner2;
          }
          if (ok && c_bmode == 2 && b_owner != c_rank && !(ready_mask >> b_owner & 1u)) {
            ok = wait_published(*coll, b_owner, epoch, err);
            ready_mask |= 1u << b_owner;
          }
          mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + TB_BYTES);
          if (tile_src == 1) {
            tma_load_3d(a_dst, own_map, &full_bar[stage], k0, tile_lrow, tile_b);
          } else if (tile_src == 2) {
            tma_load_2d(a_dst, gathered_map, &full_bar[stage], k0, m0);
          } else if (c_amode == 2) {
            tma_load_3d(a_dst, &coll->a[a_owner2], &full_bar[stage], m0, a_row2, a_b2);
            tma_load_3d(a_dst + BK * 128, &coll->a[a_owner2], &full_bar[stage], m0 + 64, a_row2, a_b2);
          } else if (A_MN) {
            tma_load_2d(a_dst, &tma_a, &full_bar[stage], m0, k0);
            tma_load_2d(a_dst + BK * 128, &tma_a, &full_bar[stage], m0 + 64, k0);
          } else {
            tma_load_2d(a_dst, &tma_a, &full_bar[stage], k0, m0);
          }
          if (c_bmode == 2) {
#pragma unroll
            for (int j = 0; j < TN / 64; ++j)
              tma_load_3d(b_dst + j * BK * 128, &coll->b[b_owner], &full_bar[stage], n0 + 64 * j, b_row, b_b);
          } else if (B_MN) {
#pragma unroll
            for (int j = 0; j < TN / 64; ++j) tma_load_2d(b_dst + j * BK * 128, &tma_b, &full_bar[stage], n0 + 64 * j, k0);
          } else {
            tma_load_2d(b_dst, &tma_b, &full_bar[stage], k0, n0);
          }
        } else if (lane == 0) {
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * TB_BYTES;
          const int k0 = kb * BK;
          mbar_arrive_expect_tx(&full_bar[stage], A_BYTES + TB_BYTES);
          if (A_MN) {
            tma_load_2d(a_dst, &tma_a, &full_bar[stage], m0, k0);
            tma_load_2d(a_dst + BK * 128, &tma_a, &full_bar[stage], m0 + 64, k0);
          } else {
            tma_load_2d(a_dst, &tma_a, &full_bar[stage], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < TN / 64; ++j) tma_load_2d(b_dst + j * BK * 128, &tma_b, &full_bar[stage], n0 + 64 * j, k0);
          } else if (SWI) {  // gate rows n0.., then up rows F + n0.. (two boxes of TN / 2 rows)
            tma_load_2d(b_dst, &tma_b, &full_bar[stage], k0, n0);
            tma_load_2d(b_dst + (TN / 2) * 128, &tma_b, &full_bar[stage], k0, ep.half_n + n0);
          } else {
            tma_load_2d(b_dst, &tma_b, &full_bar[stage], k0, n0);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_bf16(BM, TN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x) {
      int kb0, kb1;
      split_range(kblocks, ep.splits, unit % ep.splits, kb0, kb1);
      if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, err, 2)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;  // accumulator buffers 256 columns apart for every tile width
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, err, 3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * TB_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? umma_desc_sw128(a_addr + k * 2048, BK * 128, 1024)
                                        : umma_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? umma_desc_sw128(b_addr + k * 2048, BK * 128, 1024)
                                        : umma_desc_sw128(b_addr + k * 32, 16, 1024);
            tc_mma_f16(d_tmem, adesc, bdesc, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) tc_commit(&tfull_bar[acc]);
      __syncwarp();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  } else if (COLL && warp == 2 + EPI_WARPS) {
    // ---------------- copy warp (a_mode 1) ----------------
    if (coll->a_mode == 1) coll_copy_warp(*coll, epoch, lane, err);
  } else {
    // ---------------- epilogue ----------------
    uint8_t* tile = sEpi + (warp - 2) * EPI_STAGE_BYTES;
    if constexpr (KIND == kKindGeneric) {
      if (ep.d_fp32)
        epilogue_loop<32, KIND, TN>(ep, &tma_d, &tma_aux, tile, tmem_base, tfull_bar, tempty_bar, M, N, num_m, num_n, num_tiles, warp,
                                lane, err, COLL ? coll : nullptr);
      else
        epilogue_loop<64, KIND, TN>(ep, &tma_d, &tma_aux, tile, tmem_base, tfull_bar, tempty_bar, M, N, num_m, num_n, num_tiles, warp,
                                lane, err, COLL ? coll : nullptr);
    } else if constexpr (KIND == kKindSwiGLU || KIND == kKindSwiGLUBwd) {
      epilogue_loop_swiglu<KIND == kKindSwiGLUBwd, TN>(ep, &tma_d, &tma_aux, tile, tmem_base, tfull_bar, tempty_bar, M, N, num_m,
                                                       num_n, num_tiles, warp, lane, err);
    } else {
      epilogue_loop<KIND == kKindF32 ? 32 : 64, KIND, TN>(ep, &tma_d, &tma_aux, tile, tmem_base, tfull_bar, tempty_bar, M, N, num_m,
                                                      num_n, num_tiles, warp, lane, err, nullptr);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
  if constexpr (COLL) {
    // Completion: the last CTA advances the call site's epoch and, in reduce-scatter mode,
    // tells every peer that this rank's slots in their receive buffers are written.
    if (threadIdx.x == 0 && coll->advance) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence_system();
      if (atomicAdd(coll->done, 1) == (int)gridDim.x - 1) {
        __threadfence_system();
        if (coll->rs) publish_epoch(*coll, epoch);
        *((volatile uint32_t*)coll->epoch) = epoch;
        *((volatile int*)coll->done) = 0;
        __threadfence();
      }
    }
  }
}

template <bool A_MN, bool B_MN, int KIND, int TN = BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_d, const __grid_constant__ CUtensorMap tma_aux, int M, int N, int K,
                EpiParams ep, int* err) {
  gemm_body<A_MN, B_MN, false, KIND, TN>(tma_a, tma_b, tma_d, tma_aux, M, N, K, ep, err, nullptr);
}

// ------------------------------------------------------------------------------------------------
// CTA-pair GEMM (cluster of two CTAs, tcgen05.mma.cta_group::2): 256 x TN output tiles.  Each CTA
// loads its own 128 rows of A and its half (TN / 2 rows or columns) of B into its own shared
// memory, so a stage holds 16 KB + TN * 64 bytes per CTA instead of 16 KB + TN * 128: six stages
// fit where the single-CTA kernel holds four, and every CTA reads a third fewer operand bytes per
// multiply-add from L2.  CTA 0 issues the MMAs for the pair (rows 0-127 accumulate in its TMEM,
// rows 128-255 in CTA 1's) and its commits arrive on both CTAs' barriers.  Every TMA load
// completes on a barrier of the CTA that issued it; CTA 1's MMA warp relays "stage full" to CTA 0
// with a cluster-scope arrive, so no asynchronous copy ever targets the other CTA's memory and no
// CTA can leave while its partner still uses its shared memory (a cluster barrier closes the
// kernel, after every issued MMA has completed).  No load is multicast.
// ------------------------------------------------------------------------------------------------
constexpr int PAIR_STAGES = 6;

template <int TN>
struct PairCfg {
  static constexpr int TB_BYTES = (TN / 2) * BK * 2;  // this CTA's half of a B stage
  static constexpr int STAGE_BYTES = A_BYTES + TB_BYTES;
  static constexpr int SMEM = PAIR_STAGES * STAGE_BYTES + EPI_WARPS * EPI_STAGE_BYTES + 1024;
  static_assert(SMEM <= 232448, "shared memory budget of one sm_100 CTA exceeded");
};

__device__ __forceinline__ void tc_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <bool A_MN, bool B_MN, int KIND, int TN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_d, const __grid_constant__ CUtensorMap tma_aux, int M, int N, int K,
                     EpiParams ep, int* err) {
  using P = PairCfg<TN>;
  static_assert(!B_MN || (TN / 2) % 64 == 0, "an MN-major B half is loaded in 64-column boxes");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + PAIR_STAGES * A_BYTES;
  uint8_t* sEpi = smem + PAIR_STAGES * P::STAGE_BYTES;

  __shared__ __align__(8) uint64_t full_bar[PAIR_STAGES];   // this CTA's stage landed (its own loads)
  __shared__ __align__(8) uint64_t peer_full[PAIR_STAGES];  // CTA 0 only: CTA 1's stage landed (relayed)
  __shared__ __align__(8) uint64_t empty_bar[PAIR_STAGES];  // the pair's MMAs have read the stage
  __shared__ __align__(8) uint64_t tfull_bar[2], tempty_bar[2], mma_done;
  __shared__ uint32_t tmem_base_slot;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
  const int num_m = (M + 2 * BM - 1) / (2 * BM);
  const int num_n = (N + TN - 1) / TN;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles * ep.splits;
  const int kblocks = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&peer_full[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * EPI_WARPS);  // every epilogue warp of both CTAs (used in CTA 0)
    }
    mbar_init(&mma_done, 1);
    fence_barrier_init();
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
    if (ep.tma_d) prefetch_tensormap(&tma_d);
    if (ep.tma_aux) prefetch_tensormap(&tma_aux);
  }
  if (warp == 1) tmem_alloc_pair(&tmem_base_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any arrive crosses the pair
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs): this CTA's A rows and B half ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = pair; unit < num_units && ok; unit += npairs) {
        int mb, nb, kb0, kb1;
        tile_coords(unit / ep.splits, num_m, num_n, mb, nb);
        split_range(kblocks, ep.splits, unit % ep.splits, kb0, kb1);
        const int m0 = mb * 2 * BM + (int)crank * BM;
        const int nh = nb * TN + (int)crank * (TN / 2);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_cluster(&empty_bar[stage], phase ^ 1u, err, 61)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * P::TB_BYTES;
          const int k0 = kb * BK;
          mbar_arrive_expect_tx(&full_bar[stage], P::STAGE_BYTES);
          if (A_MN) {
            tma_load_2d(a_dst, &tma_a, &full_bar[stage], m0, k0);
            tma_load_2d(a_dst + BK * 128, &tma_a, &full_bar[stage], m0 + 64, k0);
          } else {
            tma_load_2d(a_dst, &tma_a, &full_bar[stage], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < TN / 128; ++j) tma_load_2d(b_dst + j * BK * 128, &tma_b, &full_bar[stage], nh + 64 * j, k0);
          } else {
            tma_load_2d(b_dst, &tma_b, &full_bar[stage], k0, nh);
          }
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every filled stage has been read by the pair's MMAs (all their commits have
      // arrived here) before this CTA may reach the closing cluster barrier.
      for (int i = 0; i < PAIR_STAGES; ++i) {
        if (!mbar_wait_cluster(&empty_bar[stage], phase ^ 1u, err, 62)) break;
        if (++stage == PAIR_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1 && crank == 1) {
    // ---------------- relay (CTA 1): "my half of the stage landed" -> CTA 0 ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = pair; unit < num_units && ok; unit += npairs) {
        int kb0, kb1;
        split_range(kblocks, ep.splits, unit % ep.splits, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err, 63)) {
            ok = false;
            break;
          }
          mbar_arrive_cluster(smem_in_cta(&peer_full[stage], 0));
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (CTA 0) for the pair ----------------
    constexpr uint32_t idesc = umma_idesc_bf16(2 * BM, TN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int unit = pair; unit < num_units && ok; unit += npairs) {
      int kb0, kb1;
      split_range(kblocks, ep.splits, unit % ep.splits, kb0, kb1);
      if (!mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1u, err, 64)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, err, 65) || !mbar_wait_cluster(&peer_full[stage], phase, err, 66)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * P::TB_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = A_MN ? umma_desc_sw128(a_addr + k * 2048, BK * 128, 1024)
                                        : umma_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? umma_desc_sw128(b_addr + k * 2048, BK * 128, 1024)
                                        : umma_desc_sw128(b_addr + k * 32, 16, 1024);
            tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          tc_commit_pair(&empty_bar[stage]);
        }
        __syncwarp();
        if (++stage == PAIR_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) tc_commit_pair(&tfull_bar[acc]);
      __syncwarp();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Every MMA issued above has completed (it reads both CTAs' shared memory and writes both
    // TMEMs) before the pair may leave.
    if (lane == 0) tc_commit_pair_local(&mma_done);
    __syncwarp();
    mbar_wait(&mma_done, 0, err, 67);
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows ----------------
    uint8_t* tile = sEpi + (warp - 2) * EPI_STAGE_BYTES;
    epilogue_loop<KIND == kKindF32 ? 32 : 64, KIND, TN, true>(ep, &tma_d, &tma_aux, tile, tmem_base, tfull_bar, tempty_bar, M, N,
                                                              num_m, num_n, num_tiles, warp, lane, err, nullptr);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(COLL_THREADS, 1)
    gemm_coll_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_d, const __grid_constant__ CUtensorMap tma_aux, int M, int N, int K,
                     EpiParams ep, int* err, const __grid_constant__ CollParams coll) {
  gemm_body<A_MN, B_MN, true, kKindGeneric>(tma_a, tma_b, tma_d, tma_aux, M, N, K, ep, err, &coll);
}

// out[b, r, n] = sum over ranks p (in order) of recv[p][b, r, n], after every peer has published
// its slots for this call site's current epoch.  bf16 in/out, fp32 accumulation.
__global__ void __launch_bounds__(256) rs_sum_kernel(const __nv_bfloat16* __restrict__ recv, __nv_bfloat16* __restrict__ out,
                                                     long long slot_elems, int world, int rank, const uint32_t* flags_row,
                                                     const uint32_t* epoch_ptr, unsigned long long timeout_ns, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const uint32_t epoch = *((volatile const uint32_t*)epoch_ptr);
    const unsigned long long deadline = globaltimer_ns() + timeout_ns;
    int good = 1;
    for (int p = 0; p < world && good; ++p) {
      if (p == rank) continue;
      while ((int)(ld_acquire_sys(flags_row + p) - epoch) < 0) {
        if (globaltimer_ns() > deadline || *((volatile int*)err) != 0) {
          atomicCAS(err, 0, 41);
          good = 0;
          break;
        }
      }
    }
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const long long vecs = slot_elems / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < vecs; i += (long long)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < world; ++p) {
      const uint4 raw = *reinterpret_cast<const uint4*>(recv + p * slot_elems + i * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + i * 8) = o;
  }
}

// D = beta * D + sum over s of W[s] (fixed order), W: fp32 [splits, split_rows, ldw].  Four
// independent partial loads are in flight per thread; when D's rows allow it (`vec_d`: 16-byte
// aligned fp32 or 8-byte aligned bf16 rows) a full group of four outputs is read and written as
// one vector.
template <typename DT>
__global__ void split_reduce_kernel(const float* __restrict__ w, DT* __restrict__ d, int M, int N, long long ldd, int ldw,
                                    int splits, long long split_stride, float beta, int vec_d) {
  const long long n4 = (N + 3) / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)M * n4; i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / n4);
    const int c = (int)(i - (long long)m * n4) * 4;
    const float* src = w + (long long)m * ldw + c;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int sidx = 0;
    for (; sidx + 3 < splits; sidx += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = *reinterpret_cast<const float4*>(src + (sidx + u) * split_stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // still added in split order
        acc[0] += v[u].x;
        acc[1] += v[u].y;
        acc[2] += v[u].z;
        acc[3] += v[u].w;
      }
    }
    for (; sidx < splits; ++sidx) {
      const float4 v = *reinterpret_cast<const float4*>(src + sidx * split_stride);
      acc[0] += v.x;
      acc[1] += v.y;
      acc[2] += v.z;
      acc[3] += v.w;
    }
    DT* p = d + (long long)m * ldd + c;
    if (vec_d && c + 3 < N) {
      if constexpr (std::is_same<DT, float>::value) {
        float4 o = make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (beta != 0.f) {
          const float4 old = *reinterpret_cast<const float4*>(p);
          o.x += beta * old.x;
          o.y += beta * old.y;
          o.z += beta * old.z;
          o.w += beta * old.w;
        }
        *reinterpret_cast<float4*>(p) = o;
      } else {
        __align__(8) __nv_bfloat16 o[4];
        __align__(8) __nv_bfloat16 old[4];
        if (beta != 0.f) *reinterpret_cast<uint2*>(old) = *reinterpret_cast<const uint2*>(p);
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = f2bf(acc[e] + (beta != 0.f ? beta * bf2f(old[e]) : 0.f));
        *reinterpret_cast<uint2*>(p) = *reinterpret_cast<const uint2*>(o);
      }
      continue;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (c + e < N) {
        float o = acc[e];
        if constexpr (std::is_same<DT, float>::value) {
          if (beta != 0.f) o += beta * p[e];
          p[e] = o;
        } else {
          if (beta != 0.f) o += beta * bf2f(p[e]);
          p[e] = f2bf(o);
        }
      }
    }
  }
}

// Split factor for a GEMM with `tiles` output tiles: the factor (<= 16, >= 4 K-blocks each) that
// fills the most SMs in its last wave; 1 when the tiles already fill the GPU.  GEMMs with enough
// tiles but a long K (>= 128 K-blocks, e.g. the LM head's input gradient: 192 tiles, K = 50257)
// are split too when their last wave is mostly idle: there the fp32 partial tiles (one extra
// write and read of the output per split) cost far less than an idle half wave.
static int choose_splits(int tiles, int kblocks, int sms) {
  if (kblocks < 8) return 1;
  const bool long_k = kblocks >= 128;
  if (tiles * 2 > sms && !long_k) return 1;
  int best = 1;
  double best_eff = (double)tiles / (double)(((tiles + sms - 1) / sms) * sms);
  const int max_split = tiles * 2 > sms ? 4 : 16;
  const double margin = tiles * 2 > sms ? 0.10 : 0.02;
  for (int sp = 2; sp <= max_split; ++sp) {
    const int per = (kblocks + sp - 1) / sp;
    if (per < 4 || (sp - 1) * per >= kblocks) break;
    const int units = tiles * sp;
    const double eff = (double)units / (double)(((units + sms - 1) / sms) * sms);
    if (eff > best_eff + margin) {
      best = sp;
      best_eff = eff;
    }
  }
  return best;
}

// ------------------------------------------------------------------------------------------------
// Host side: tensor maps and launch.
// ------------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    HT_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    HT_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 map over a row-major matrix with `rows` rows of `cols` elements (row stride `ld`).
static CUtensorMap make_map(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r, " (rows=", rows, " cols=", cols,
           " ld=", ld, ")");
  return map;
}

// 2-D map over a row-major output (bf16 or fp32) for the epilogue's 32-row x 128-byte stores.
static CUtensorMap make_out_map(void* base, int64_t rows, int64_t cols, int64_t ld, bool fp32) {
  CUtensorMap map;
  const int esize = fp32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / esize), 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output) failed with code ", (int)r, " (rows=", rows,
           " cols=", cols, " ld=", ld, ")");
  return map;
}

// bf16 [rows][cols] map with 32-column x 32-row boxes and the 64-byte swizzle (SwiGLU epilogues).
static CUtensorMap make_out_map64(void* base, int64_t rows, int64_t cols, int64_t ld) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (SwiGLU output) failed with code ", (int)r);
  return map;
}

int* error_word(const at::Device& dev) {
  // Intentionally leaked: a static tensor destroyed after the CUDA context would fault at exit.
  static at::Tensor* words = new at::Tensor[64];
  const int idx = dev.index();
  if (!words[idx].defined()) words[idx] = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(dev));
  return words[idx].data_ptr<int>();
}

static void check_operand(const at::Tensor& t, const char* name) {
  HT_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be a CUDA bf16 tensor");
  HT_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with unit inner stride");
  HT_CHECK((t.stride(0) * 2) % 16 == 0, name, " row stride must be a multiple of 16 bytes");
  HT_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

template <bool A_MN, bool B_MN, int KIND, int TN = BN>
static void launch_kind(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& maux, int M,
                        int N, int K, const EpiParams& ep, int* err, cudaStream_t s) {
  auto kernel = gemm_kernel<A_MN, B_MN, KIND, TN>;
  constexpr int smem = STAGES * (A_BYTES + TN * BK * 2) + EPI_WARPS * EPI_STAGE_BYTES + 1024;
  static bool configured = false;
  if (!configured) {
    HT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  constexpr int TN_OUT = KIND == kKindSwiGLU ? TN / 2 : TN;
  const int units = ((M + BM - 1) / BM) * ((N + TN_OUT - 1) / TN_OUT) * ep.splits;
  const int grid = std::min(units, num_sms());
  kernel<<<grid, THREADS, smem, s>>>(ma, mb, md, maux, M, N, K, ep, err);
  HT_CUDA_CHECK(cudaGetLastError());
}

// Output-tile width: 256 columns, or 192 when it packs the tiles into fewer full waves over the
// SMs (N = 768: 192 tiles of 128 x 256 fill 148 SMs 1.3 times, 256 tiles of 128 x 192 fill them
// 1.7 times, so the last wave idles less).  Cost model: waves x tile width (per-tile time grows
// with its width); the narrow tile must win by 10 % to be used.
static constexpr int NARROW_TN = 192;

static int choose_tile_n(int64_t M, int64_t N, int splits) {
  if (splits > 1 || N % 64 != 0) return BN;
  const int sms = num_sms();
  auto cost = [&](int tn) {
    const long long tiles = ((M + BM - 1) / BM) * ((N + tn - 1) / tn);
    return (double)((tiles + sms - 1) / sms) * tn;
  };
  return cost(NARROW_TN) < 0.9 * cost(BN) ? NARROW_TN : BN;
}

// The epilogue kind that covers `ep` with the least code.
static int epilogue_kind(const EpiParams& ep) {
  if (!ep.tma_d || ep.tma_aux != (ep.epi == kGelu)) return kKindGeneric;
  if (ep.d_fp32) return ep.epi == kPlain ? kKindF32 : kKindGeneric;
  if (ep.reduce_add) return kKindGeneric;
  if (ep.epi == kGelu) return kKindGelu;
  if (ep.epi == kGeluBwd) return kKindGeluBwd;
  return kKindBf16;
}

template <bool A_MN, bool B_MN>
static void launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& maux, int M,
                   int N, int K, const EpiParams& ep, int* err, cudaStream_t s, int tn = BN) {
  if constexpr (!A_MN) {  // the narrow tile exists for the forward and data-gradient products (A K-major)
    if (tn == NARROW_TN) {
      switch (epilogue_kind(ep)) {
        case kKindBf16: launch_kind<A_MN, B_MN, kKindBf16, NARROW_TN>(ma, mb, md, maux, M, N, K, ep, err, s); return;
        case kKindGelu: launch_kind<A_MN, B_MN, kKindGelu, NARROW_TN>(ma, mb, md, maux, M, N, K, ep, err, s); return;
        case kKindGeluBwd: launch_kind<A_MN, B_MN, kKindGeluBwd, NARROW_TN>(ma, mb, md, maux, M, N, K, ep, err, s); return;
        default: break;
      }
    }
  }
  switch (epilogue_kind(ep)) {
    case kKindBf16: launch_kind<A_MN, B_MN, kKindBf16>(ma, mb, md, maux, M, N, K, ep, err, s); break;
    case kKindF32: launch_kind<A_MN, B_MN, kKindF32>(ma, mb, md, maux, M, N, K, ep, err, s); break;
    case kKindGelu: launch_kind<A_MN, B_MN, kKindGelu>(ma, mb, md, maux, M, N, K, ep, err, s); break;
    case kKindGeluBwd: launch_kind<A_MN, B_MN, kKindGeluBwd>(ma, mb, md, maux, M, N, K, ep, err, s); break;
    default: launch_kind<A_MN, B_MN, kKindGeneric>(ma, mb, md, maux, M, N, K, ep, err, s); break;
  }
}

// CTA-pair launch (256-row tiles, 74 pairs); returns false when this combination has no pair instance.
template <bool A_MN, bool B_MN, int KIND>
static void launch_pair_kind(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& maux, int M,
                             int N, int K, const EpiParams& ep, int* err, cudaStream_t s) {
  auto kernel = gemm_pair_kernel<A_MN, B_MN, KIND, BN>;
  constexpr int smem = PairCfg<BN>::SMEM;
  static bool configured = false;
  if (!configured) {
    HT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  const int units = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN) * ep.splits;
  const int pairs = std::min(units, num_sms() / 2);
  kernel<<<2 * pairs, THREADS, smem, s>>>(ma, mb, md, maux, M, N, K, ep, err);
  HT_CUDA_CHECK(cudaGetLastError());
}

template <bool A_MN, bool B_MN>
static bool launch_pair(int kind, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& maux,
                        int M, int N, int K, const EpiParams& ep, int* err, cudaStream_t s) {
  if constexpr (!A_MN && !B_MN) {  // forward
    if (kind == kKindBf16) return launch_pair_kind<false, false, kKindBf16>(ma, mb, md, maux, M, N, K, ep, err, s), true;
    if (kind == kKindGelu) return launch_pair_kind<false, false, kKindGelu>(ma, mb, md, maux, M, N, K, ep, err, s), true;
    if (kind == kKindF32) return launch_pair_kind<false, false, kKindF32>(ma, mb, md, maux, M, N, K, ep, err, s), true;
  } else if constexpr (!A_MN && B_MN) {  // data gradient
    if (kind == kKindBf16) return launch_pair_kind<false, true, kKindBf16>(ma, mb, md, maux, M, N, K, ep, err, s), true;
    if (kind == kKindGeluBwd) return launch_pair_kind<false, true, kKindGeluBwd>(ma, mb, md, maux, M, N, K, ep, err, s), true;
    if (kind == kKindF32) return launch_pair_kind<false, true, kKindF32>(ma, mb, md, maux, M, N, K, ep, err, s), true;
  } else if constexpr (A_MN && B_MN) {  // weight gradient
    if (kind == kKindF32) return launch_pair_kind<true, true, kKindF32>(ma, mb, md, maux, M, N, K, ep, err, s), true;
    if (kind == kKindBf16) return launch_pair_kind<true, true, kKindBf16>(ma, mb, md, maux, M, N, K, ep, err, s), true;
  }
  return false;
}

// CTA pairs for every eligible GEMM (1), or never (0, the default); HT_GEMM_PAIR=1 in the
// environment sets 1.
static int g_pair_mode = -1;

static bool pair_enabled() {
  if (g_pair_mode < 0) {
    const char* e = std::getenv("HT_GEMM_PAIR");
    g_pair_mode = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return g_pair_mode == 1;
}

}  // namespace tcg

void set_gemm_pair(int64_t mode) { tcg::g_pair_mode = mode ? 1 : 0; }

// Split-K GEMMs with an fp32 output either sum their partial tiles in a fixed order (a workspace
// and a reduction pass: bitwise reproducible), or, when reproducibility is switched off, add every
// partial tile straight into D with TMA fp32 reduce-adds (D zeroed first for beta = 0): no
// workspace and no extra pass, but the order of the partial sums varies from run to run.
static bool g_ordered_split_k = true;

void set_deterministic_reductions(bool on) { g_ordered_split_k = on; }

bool deterministic_reductions() { return g_ordered_split_k; }

void gemm(at::Tensor a, at::Tensor b, at::Tensor d, c10::optional<at::Tensor> bias, c10::optional<at::Tensor> aux,
          c10::optional<at::Tensor> alpha, bool a_mn_major, bool b_mn_major, int64_t epilogue, double beta) {
  using namespace tcg;
  check_operand(a, "A");
  check_operand(b, "B");
  const c10::cuda::CUDAGuard guard(a.device());
  bind_context(a.device().index());
  const int64_t M = a_mn_major ? a.size(1) : a.size(0);
  const int64_t K = a_mn_major ? a.size(0) : a.size(1);
  const int64_t N = b_mn_major ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn_major ? b.size(0) : b.size(1);
  HT_CHECK(K == Kb, "GEMM reduction sizes differ: ", K, " vs ", Kb);
  HT_CHECK(d.dim() == 2 && d.size(0) == M && d.size(1) == N && d.stride(1) == 1, "D must be [M, N] with unit inner stride");
  HT_CHECK(d.scalar_type() == at::kBFloat16 || d.scalar_type() == at::kFloat, "D must be bf16 or fp32");
  const bool d32 = d.scalar_type() == at::kFloat;
  if (M == 0 || N == 0) return;
  EpiParams ep{};
  ep.d = d.data_ptr();
  ep.ldd = d.stride(0);
  ep.d_fp32 = d32 ? 1 : 0;
  ep.beta = static_cast<float>(beta);
  ep.epi = static_cast<int>(epilogue);
  ep.vec_ok = ((d.stride(0) * d.element_size()) % 16 == 0 && reinterpret_cast<uintptr_t>(d.data_ptr()) % 16 == 0) ? 1 : 0;
  if (bias.has_value() && bias->defined()) {
    HT_CHECK(bias->is_contiguous() && bias->numel() == N, "bias must be a contiguous [N] tensor");
    if (bias->scalar_type() == at::kFloat) ep.bias_f32 = bias->data_ptr<float>();
    else if (bias->scalar_type() == at::kBFloat16) ep.bias_bf16 = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
    else HT_CHECK(false, "bias must be fp32 or bf16");
  }
  if (epilogue != kPlain) {
    HT_CHECK(aux.has_value() && aux->defined() && aux->scalar_type() == at::kBFloat16 && aux->size(0) == M &&
                 aux->size(1) == N && aux->stride(1) == 1,
             "GELU epilogues need a bf16 [M, N] aux tensor");
    ep.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
    ep.ldaux = aux->stride(0);
    if ((aux->stride(0) * 2) % 16 != 0 || reinterpret_cast<uintptr_t>(aux->data_ptr()) % 16 != 0) ep.vec_ok = 0;
  }
  if (alpha.has_value() && alpha->defined()) {
    HT_CHECK(alpha->scalar_type() == at::kFloat && alpha->numel() == 1 && alpha->is_cuda(), "alpha must be one fp32 device value");
    ep.alpha = alpha->data_ptr<float>();
  }
  if (K == 0) {
    HT_CHECK(false, "GEMM with K == 0 is not supported");
  }
  const CUtensorMap ma = a_mn_major ? make_map(a.data_ptr(), K, M, a.stride(0), 64, 64)
                                    : make_map(a.data_ptr(), M, K, a.stride(0), 64, BM);
  // TMA output path: aligned rows, and a store or an fp32 accumulate (beta = 1); the GELU
  // pre-activation is written through its own map when D is bf16.  GEMMs with too few output
  // tiles to fill the GPU (weight gradients: small M x N, long K) split K over several CTAs
  // that store fp32 partial tiles into a workspace, summed in a fixed order afterwards.
  CUtensorMap md{}, maux{};
  ep.splits = 1;
  // CTA pairs (256-row tiles) for the epilogues they carry; the kind is confirmed below.
  const bool pair_shape = pair_enabled() && M > BM && (epilogue == kPlain || epilogue == kGelu || epilogue == kGeluBwd) &&
                          !(a_mn_major && !b_mn_major);
  const int tile_rows = pair_shape ? 2 * BM : BM;
  const int tiles = (int)(((M + tile_rows - 1) / tile_rows) * ((N + BN - 1) / BN));
  const int kblocks = (int)((K + BK - 1) / BK);
  const int splits = (epilogue == kPlain && ep.bias_f32 == nullptr && ep.bias_bf16 == nullptr)
                         ? choose_splits(tiles, kblocks, pair_shape ? num_sms() / 2 : num_sms())
                         : 1;
  at::Tensor workspace;
  const int64_t split_rows = (M + tile_rows - 1) / tile_rows * tile_rows, ldw = (N + 3) / 4 * 4;
  const bool split_reduce_add = splits > 1 && !g_ordered_split_k && d32 && ep.vec_ok && (beta == 0.0 || beta == 1.0);
  if (split_reduce_add) {
    if (beta == 0.0)
      HT_CUDA_CHECK(cudaMemset2DAsync(d.data_ptr(), (size_t)d.stride(0) * 4, 0, (size_t)N * 4, (size_t)M, stream()));
    md = make_out_map(d.data_ptr(), M, N, d.stride(0), true);
    ep.splits = splits;
    ep.split_rows = 0;  // every split adds into the same rows of D
    ep.tma_d = 1;
    ep.reduce_add = 1;
    ep.beta = 0.f;
  } else if (splits > 1) {
    workspace = at::empty({splits * split_rows, ldw}, a.options().dtype(at::kFloat));
    md = make_out_map(workspace.data_ptr(), splits * split_rows, N, ldw, true);
    ep.splits = splits;
    ep.split_rows = (int)split_rows;
    ep.tma_d = 1;
    ep.reduce_add = 0;
    ep.d_fp32 = 1;
    ep.beta = 0.f;
  } else if (ep.vec_ok && (beta == 0.0 || (beta == 1.0 && d32)) && !(epilogue == kGelu && d32)) {
    md = make_out_map(d.data_ptr(), M, N, d.stride(0), d32);
    if (epilogue == kGelu) maux = make_out_map(aux->data_ptr(), M, N, aux->stride(0), false);
    ep.tma_d = 1;
    ep.tma_aux = epilogue == kGelu ? 1 : 0;
    ep.reduce_add = beta == 1.0 ? 1 : 0;
  }
  // The narrow tile is compiled for A K-major products with the bf16 / GELU / GELU' epilogues; the
  // K-major B map's box must match the tile width the kernel expects.
  const int kind = epilogue_kind(ep);
  int* err = error_word(a.device());
  cudaStream_t s = stream();
  const bool pair = pair_shape && (kind == kKindBf16 || kind == kKindF32 || kind == kKindGelu || kind == kKindGeluBwd);
  if (pair) {
    // Each CTA of a pair loads half of the B tile: K-major boxes of BN / 2 rows.
    const CUtensorMap mbp = b_mn_major ? make_map(b.data_ptr(), K, N, b.stride(0), 64, 64)
                                       : make_map(b.data_ptr(), N, K, b.stride(0), 64, BN / 2);
    bool done = false;
    if (!a_mn_major && !b_mn_major) done = launch_pair<false, false>(kind, ma, mbp, md, maux, M, N, K, ep, err, s);
    else if (!a_mn_major && b_mn_major) done = launch_pair<false, true>(kind, ma, mbp, md, maux, M, N, K, ep, err, s);
    else if (a_mn_major && b_mn_major) done = launch_pair<true, true>(kind, ma, mbp, md, maux, M, N, K, ep, err, s);
    HT_CHECK(done, "no CTA-pair GEMM instance for this operand layout and epilogue");
  }
  const bool narrow_ok = !a_mn_major && (kind == kKindBf16 || kind == kKindGelu || kind == kKindGeluBwd);
  const int tn = narrow_ok ? choose_tile_n(M, N, ep.splits) : BN;
  const CUtensorMap mb = b_mn_major ? make_map(b.data_ptr(), K, N, b.stride(0), 64, 64)
                                    : make_map(b.data_ptr(), N, K, b.stride(0), 64, tn);
  if (pair) {
    // launched above
  } else if (!a_mn_major && !b_mn_major) launch<false, false>(ma, mb, md, maux, M, N, K, ep, err, s, tn);
  else if (!a_mn_major && b_mn_major) launch<false, true>(ma, mb, md, maux, M, N, K, ep, err, s, tn);
  else if (a_mn_major && b_mn_major) launch<true, true>(ma, mb, md, maux, M, N, K, ep, err, s);
  else launch<true, false>(ma, mb, md, maux, M, N, K, ep, err, s);
  if (splits > 1 && !split_reduce_add) {
    const long long work = M * ((N + 3) / 4);
    const int blocks = (int)std::min<long long>((work + 255) / 256, 8LL * num_sms());
    const uintptr_t dp = reinterpret_cast<uintptr_t>(d.data_ptr());
    const int vec_d = d32 ? (dp % 16 == 0 && d.stride(0) % 4 == 0) : (dp % 8 == 0 && d.stride(0) % 4 == 0);
    if (d32)
      split_reduce_kernel<float><<<blocks, 256, 0, s>>>(workspace.data_ptr<float>(), d.data_ptr<float>(), (int)M, (int)N, d.stride(0),
                                                        (int)ldw, splits, split_rows * ldw, (float)beta, vec_d);
    else
      split_reduce_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(workspace.data_ptr<float>(),
                                                                reinterpret_cast<__nv_bfloat16*>(d.data_ptr()), (int)M, (int)N,
                                                                d.stride(0), (int)ldw, splits, split_rows * ldw, (float)beta, vec_d);
    HT_CUDA_CHECK(cudaGetLastError());
  }
}

// SwiGLU fused into GEMM epilogues (see epilogue_loop_swiglu).
//   backward == false: a = X [M, K], b = W [2F, K] (F gate rows, then F up rows), bias [2F] or none;
//     writes h = X W^T + bias as [M, 2F] (gate | up) and out = silu(gate) * up as [M, F].
//   backward == true: a = dY [M, K], b = W2 [K, F] (the down projection's weight, read MN-major),
//     h from the forward; writes out = dH [M, 2F] = (dA * up * silu'(gate) | dA * silu(gate)) with
//     dA = dY W2, so neither dA nor a separate element-wise pass is needed.
// F must be a multiple of 128 (a forward tile holds 128 gate and 128 up features).
void gemm_swiglu(at::Tensor a, at::Tensor b, at::Tensor h, at::Tensor out, c10::optional<at::Tensor> bias, bool backward) {
  using namespace tcg;
  check_operand(a, "A");
  check_operand(b, "B");
  check_operand(h, "h");
  check_operand(out, "out");
  const c10::cuda::CUDAGuard guard(a.device());
  bind_context(a.device().index());
  const int64_t M = a.size(0), K = a.size(1);
  const int64_t F = backward ? b.size(1) : b.size(0) / 2;
  HT_CHECK(F > 0 && F % 128 == 0, "SwiGLU GEMM: the feature count F must be a positive multiple of 128, got ", F);
  HT_CHECK((backward ? b.size(0) : b.size(1)) == K, "SwiGLU GEMM: reduction sizes differ");
  HT_CHECK(backward || b.size(0) == 2 * F, "SwiGLU GEMM: W must have 2F rows");
  HT_CHECK(h.size(0) == M && h.size(1) == 2 * F, "SwiGLU GEMM: h must be [M, 2F]");
  HT_CHECK(out.size(0) == M && out.size(1) == (backward ? 2 * F : F), "SwiGLU GEMM: out must be [M, ", backward ? "2F" : "F",
           "]");
  if (M == 0) return;
  EpiParams ep{};
  ep.d = out.data_ptr();
  ep.ldd = out.stride(0);
  ep.beta = 0.f;
  ep.epi = backward ? kSwiGLUBwd : kSwiGLU;
  ep.vec_ok = 1;
  ep.tma_d = 1;
  ep.splits = 1;
  ep.half_n = (int)F;
  ep.aux = reinterpret_cast<__nv_bfloat16*>(h.data_ptr());
  ep.ldaux = h.stride(0);
  if (!backward && bias.has_value() && bias->defined()) {
    HT_CHECK(bias->is_contiguous() && bias->numel() == 2 * F, "SwiGLU GEMM: bias must be a contiguous [2F] tensor");
    if (bias->scalar_type() == at::kFloat) ep.bias_f32 = bias->data_ptr<float>();
    else if (bias->scalar_type() == at::kBFloat16) ep.bias_bf16 = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
    else HT_CHECK(false, "bias must be fp32 or bf16");
  }
  const CUtensorMap ma = make_map(a.data_ptr(), M, K, a.stride(0), 64, BM);
  const CUtensorMap md = make_out_map64(out.data_ptr(), M, out.size(1), out.stride(0));
  int* err = error_word(a.device());
  cudaStream_t s = stream();
  if (!backward) {
    const CUtensorMap mb = make_map(b.data_ptr(), 2 * F, K, b.stride(0), 64, BN / 2);
    const CUtensorMap maux = make_out_map64(h.data_ptr(), M, 2 * F, h.stride(0));
    ep.tma_aux = 1;
    launch_kind<false, false, kKindSwiGLU>(ma, mb, md, maux, (int)M, (int)F, (int)K, ep, err, s);
  } else {
    const CUtensorMap mb = make_map(b.data_ptr(), K, F, b.stride(0), 64, 64);
    launch_kind<false, true, kKindSwiGLUBwd>(ma, mb, md, md, (int)M, (int)F, (int)K, ep, err, s);
  }
}

namespace tcg {

// bf16 [d2][d1][d0] map (d0 innermost, contiguous) with box {box0, box1, 1} and the 128-byte swizzle.
static CUtensorMap make_map3(int64_t base, int64_t d0, int64_t d1, int64_t d2, int box0, int box1) {
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)(d0 * 2), (cuuint64_t)(d0 * d1 * 2)};
  cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  HT_CHECK(base % 16 == 0 && (d0 * 2) % 16 == 0, "peer shard must be 16-byte aligned with 16-byte rows");
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, reinterpret_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HT_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (peer shard) failed with code ", (int)r);
  return map;
}

template <bool A_MN, bool B_MN>
static void launch_coll(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& maux, int M,
                        int N, int K, const EpiParams& ep, int* err, const CollParams& coll, cudaStream_t s) {
  auto kernel = gemm_coll_kernel<A_MN, B_MN>;
  static bool configured = false;
  if (!configured) {
    HT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, num_sms());
  // CTAs wait for blocks that other CTAs' copy warps bring in: a cooperative launch guarantees
  // that every CTA of the grid is resident.
  int m = M, n = N, k = K;
  const EpiParams e = ep;
  int* w = err;
  const CollParams c = coll;
  void* args[] = {const_cast<CUtensorMap*>(&ma), const_cast<CUtensorMap*>(&mb), const_cast<CUtensorMap*>(&md),
                  const_cast<CUtensorMap*>(&maux), &m, &n, &k, const_cast<EpiParams*>(&e), &w, const_cast<CollParams*>(&c)};
  HT_CUDA_CHECK(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(kernel), dim3(grid), dim3(COLL_THREADS), args,
                                            (size_t)SMEM_BYTES, s));
}

}  // namespace tcg

// GEMM with operands gathered from, or results scattered to, the peers of a tensor-parallel group
// (see CollParams).  a_mode 1: `a` is this rank's [B, R, K] shard of A (K-major, rows = sequence);
// a_mode 2: `a` is the [B, R, M] shard of an MN-major A whose K dimension is the sequence;
// b_mode 2: `b` is the [B, R, N] shard of an MN-major B whose K dimension is the sequence;
// rs: `d` is this rank's receive buffer [world, B, R, N] and every output row goes to the slot
// `rank` of its owner's buffer; otherwise `d` is a local [M, N] output as in `gemm`.
void gemm_collective(at::Tensor a, at::Tensor b, at::Tensor d, c10::optional<at::Tensor> bias, c10::optional<at::Tensor> aux,
                     bool a_mn_major, bool b_mn_major, int64_t epilogue, double beta, int64_t a_mode, std::vector<int64_t> a_ptrs,
                     int64_t b_mode, std::vector<int64_t> b_ptrs, int64_t rs, std::vector<int64_t> out_ptrs, at::Tensor flags_local,
                     std::vector<int64_t> flag_ptrs, at::Tensor counters, int64_t site, int64_t advance, int64_t rank,
                     double timeout_s, c10::optional<at::Tensor> gathered, c10::optional<at::Tensor> block_flags) {
  using namespace tcg;
  const c10::cuda::CUDAGuard guard(a.device());
  bind_context(a.device().index());
  const int world = (int)flag_ptrs.size();
  HT_CHECK(world >= 2 && world <= MAX_PEERS, "gemm_collective supports 2..8 ranks");
  HT_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_collective takes bf16 operands");
  HT_CHECK(a_mode == 0 || a_mode == 1 || a_mode == 2, "bad a_mode");
  HT_CHECK(b_mode == 0 || b_mode == 2, "bad b_mode");
  HT_CHECK((a_mode == 2) == (a_mode == 2 && a_mn_major) && (a_mode != 1 || !a_mn_major), "a_mode and A majorness disagree");
  HT_CHECK(b_mode != 2 || b_mn_major, "b_mode 2 needs an MN-major B");
  int64_t batch = 0, rows = 0, M = 0, N = 0, K = 0;
  const at::Tensor& sharded = a_mode ? a : (b_mode ? b : d);
  if (a_mode || b_mode) {
    HT_CHECK(sharded.dim() == 3 && sharded.is_contiguous(), "a peer-sharded operand must be a contiguous [B, R, C] shard");
    batch = sharded.size(0);
    rows = sharded.size(1);
  } else {
    HT_CHECK(rs && d.dim() == 4, "a local-only collective GEMM must reduce-scatter");
    batch = d.size(1);
    rows = d.size(2);
  }
  const int64_t total = batch * rows * world;
  if (a_mode == 1) { M = total; K = a.size(2); }
  else if (a_mode == 2) { K = total; M = a.size(2); }
  else {
    check_operand(a, "A");
    M = a_mn_major ? a.size(1) : a.size(0);
    K = a_mn_major ? a.size(0) : a.size(1);
  }
  if (b_mode == 2) {
    N = b.size(2);
    HT_CHECK(K == total, "peer-sharded B must share the sequence K dimension");
  } else {
    check_operand(b, "B");
    N = b_mn_major ? b.size(1) : b.size(0);
    HT_CHECK((b_mn_major ? b.size(0) : b.size(1)) == K, "GEMM reduction sizes differ");
  }
  if (a_mode == 1 || rs) HT_CHECK(rows % BM == 0, "sequence rows per rank must be a multiple of 128 for this mode");
  if (a_mode == 2 || b_mode == 2) HT_CHECK(rows % BK == 0, "sequence rows per rank must be a multiple of 64");
  HT_CHECK((int)a_ptrs.size() == (a_mode ? world : 0) && (int)b_ptrs.size() == (b_mode ? world : 0) &&
               (int)out_ptrs.size() == (rs ? world : 0), "one peer pointer per rank expected");

  CollParams coll;
  std::memset(&coll, 0, sizeof(coll));
  for (int p = 0; p < world; ++p) {
    if (a_mode == 1) coll.a[p] = make_map3(a_ptrs[p], K, rows, batch, 64, BM);
    if (a_mode == 2) coll.a[p] = make_map3(a_ptrs[p], M, rows, batch, 64, BK);
    if (b_mode == 2) coll.b[p] = make_map3(b_ptrs[p], N, rows, batch, 64, BK);
    if (rs) coll.out[p] = make_map3(out_ptrs[p], N, rows, (int64_t)world * batch, 64, 32);
    coll.flags_peer[p] = reinterpret_cast<uint32_t*>(flag_ptrs[p]);
  }
  HT_CHECK(flags_local.scalar_type() == at::kInt && counters.scalar_type() == at::kInt && counters.is_cuda(), "int32 flags expected");
  HT_CHECK(site >= 0 && (site + 1) * MAX_PEERS <= flags_local.numel() && (site + 1) * 2 <= counters.numel(), "call site out of range");
  coll.flags_local = reinterpret_cast<uint32_t*>(flags_local.data_ptr<int>());
  coll.epoch = reinterpret_cast<uint32_t*>(counters.data_ptr<int>() + 2 * site);
  coll.done = counters.data_ptr<int>() + 2 * site + 1;
  coll.site = (int)site;
  coll.advance = advance ? 1 : 0;
  coll.a_mode = (int)a_mode;
  coll.b_mode = (int)b_mode;
  coll.rs = rs ? 1 : 0;
  coll.rank = (int)rank;
  coll.world = world;
  coll.batch = (int)batch;
  coll.rows_per_rank = (int)rows;
  coll.seq = (int)(rows * world);
  coll.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  if (a_mode == 1) {
    HT_CHECK(gathered.has_value() && gathered->defined() && block_flags.has_value() && block_flags->defined(),
             "the all-gather mode needs a gathered buffer and block flags");
    HT_CHECK(gathered->scalar_type() == at::kBFloat16 && gathered->is_contiguous() && gathered->numel() == M * K,
             "gathered buffer must be a contiguous bf16 [B, S, K]");
    HT_CHECK(K % BK == 0, "K must be a multiple of 64 for the all-gather mode");
    HT_CHECK(block_flags->scalar_type() == at::kInt && block_flags->numel() >= (M / BM) * (K / BK),
             "one int32 flag per 128-row x 64-column slice");
    coll.gathered_map = make_map(gathered->data_ptr(), M, K, K, 64, BM);
    coll.gathered = reinterpret_cast<__nv_bfloat16*>(gathered->data_ptr());
    coll.block_flags = reinterpret_cast<uint32_t*>(block_flags->data_ptr<int>());
    coll.k_dim = (int)K;
    HT_CHECK(K % 8 == 0, "K must be a multiple of 8");
    for (int p = 0; p < world; ++p) coll.a_src[p] = reinterpret_cast<const __nv_bfloat16*>(a_ptrs[p]);
  }

  EpiParams ep{};
  ep.splits = 1;
  CUtensorMap ma{}, mb{}, md{}, maux{};
  if (a_mode == 0) ma = a_mn_major ? make_map(a.data_ptr(), K, M, a.stride(0), 64, 64) : make_map(a.data_ptr(), M, K, a.stride(0), 64, BM);
  if (b_mode == 0) mb = b_mn_major ? make_map(b.data_ptr(), K, N, b.stride(0), 64, 64) : make_map(b.data_ptr(), N, K, b.stride(0), 64, BN);
  if (rs) {
    HT_CHECK(d.scalar_type() == at::kBFloat16 && d.is_contiguous() && d.size(0) == world && d.size(3) == N,
             "receive buffer must be a contiguous bf16 [world, B, R, N]");
    HT_CHECK(epilogue == kPlain && !(bias.has_value() && bias->defined()), "reduce-scatter GEMMs take a plain epilogue");
    ep.d = d.data_ptr();
    ep.ldd = N;
    ep.tma_d = 1;
    ep.vec_ok = 1;
  } else {
    HT_CHECK(d.dim() == 2 && d.size(0) == M && d.size(1) == N && d.stride(1) == 1, "D must be [M, N] with unit inner stride");
    const bool d32 = d.scalar_type() == at::kFloat;
    ep.d = d.data_ptr();
    ep.ldd = d.stride(0);
    ep.d_fp32 = d32 ? 1 : 0;
    ep.beta = (float)beta;
    ep.epi = (int)epilogue;
    ep.vec_ok = ((d.stride(0) * d.element_size()) % 16 == 0 && reinterpret_cast<uintptr_t>(d.data_ptr()) % 16 == 0) ? 1 : 0;
    if (bias.has_value() && bias->defined()) {
      HT_CHECK(bias->is_contiguous() && bias->numel() == N, "bias must be a contiguous [N] tensor");
      if (bias->scalar_type() == at::kFloat) ep.bias_f32 = bias->data_ptr<float>();
      else ep.bias_bf16 = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
    }
    if (epilogue != kPlain) {
      HT_CHECK(aux.has_value() && aux->defined() && aux->scalar_type() == at::kBFloat16 && aux->size(0) == M && aux->size(1) == N,
               "GELU epilogues need a bf16 [M, N] aux tensor");
      ep.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
      ep.ldaux = aux->stride(0);
      if ((aux->stride(0) * 2) % 16 != 0 || reinterpret_cast<uintptr_t>(aux->data_ptr()) % 16 != 0) ep.vec_ok = 0;
    }
    HT_CHECK(ep.vec_ok && (beta == 0.0 || (beta == 1.0 && d32)) && !(epilogue == kGelu && d32),
             "collective GEMM outputs need 16-byte aligned rows and beta 0 (or 1 into fp32)");
    md = make_out_map(d.data_ptr(), M, N, d.stride(0), d32);
    if (epilogue == kGelu) maux = make_out_map(aux->data_ptr(), M, N, aux->stride(0), false);
    ep.tma_d = 1;
    ep.tma_aux = epilogue == kGelu ? 1 : 0;
    ep.reduce_add = beta == 1.0 ? 1 : 0;
  }
  int* err = error_word(a.device());
  cudaStream_t s = stream();
  const bool amn = a_mode == 2 || (a_mode == 0 && a_mn_major);
  if (!amn && !b_mn_major) launch_coll<false, false>(ma, mb, md, maux, (int)M, (int)N, (int)K, ep, err, coll, s);
  else if (!amn && b_mn_major) launch_coll<false, true>(ma, mb, md, maux, (int)M, (int)N, (int)K, ep, err, coll, s);
  else if (amn && b_mn_major) launch_coll<true, true>(ma, mb, md, maux, (int)M, (int)N, (int)K, ep, err, coll, s);
  else launch_coll<true, false>(ma, mb, md, maux, (int)M, (int)N, (int)K, ep, err, coll, s);
}

// out = sum over ranks of this rank's receive slots, once every peer has published them.
void reduce_scatter_sum(at::Tensor recv, at::Tensor out, at::Tensor flags_local, at::Tensor counters, int64_t site, int64_t rank,
                        double timeout_s) {
  const c10::cuda::CUDAGuard guard(recv.device());
  HT_CHECK(recv.dim() == 4 && recv.is_contiguous() && recv.scalar_type() == at::kBFloat16, "receive buffer must be bf16 [world, B, R, N]");
  const int world = (int)recv.size(0);
  const long long slot = recv.numel() / world;
  HT_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() == slot, "output must be a contiguous bf16 slot");
  HT_CHECK(slot % 8 == 0, "slot size must be a multiple of 8 elements");
  const int blocks = (int)std::min<long long>((slot / 8 + 255) / 256, 4LL * num_sms());
  tcg::rs_sum_kernel<<<std::max(blocks, 1), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(recv.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), slot, world,
      (int)rank, reinterpret_cast<const uint32_t*>(flags_local.data_ptr<int>()) + site * tcg::MAX_PEERS,
      reinterpret_cast<const uint32_t*>(counters.data_ptr<int>() + 2 * site), (unsigned long long)(timeout_s * 1e9),
      tcg::error_word(recv.device()));
  HT_CUDA_CHECK(cudaGetLastError());
}

at::Tensor gemm_error_word(at::Tensor like) { return at::from_blob(tcg::error_word(like.device()), {4}, like.options().dtype(at::kInt)); }

}  // namespace ht
