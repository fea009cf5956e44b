// Flash-attention backward on the 5th-generation tensor cores (sm_100a), deterministic (no
// atomics), packed QKV [B, S, (H + 2*Hkv) * D] (D = 64 or 128), GQA, causal or full.
//
// Given lse (natural log, from the forward) and delta = rowsum(dO * O) (pre-pass), with
// P = exp(S * scale - lse) and dS = P * (dP - delta):
//
// dq_kernel    one CTA per (128-query tile, head, batch), two per SM.  For each tile of 64 keys:
//              S = Q K^T and dP = dO V^T into TMEM (M=128, N=64), softmax threads (one per
//              query row) turn them into dS (bf16, written back over S), then
//              dQ += dS K with dS read from TMEM and K as an MN-major operand.
//              dQ * scale is stored (bf16) into the Q slot of dqkv.
// dkdv_kernel  one CTA per (128-key tile, kv head, batch).  For each query head of the group
//              and each 64-query tile at or after the key tile: S^T = K Q^T and dP^T = V dO^T
//              into TMEM (M=128 keys, N=64 queries), threads (one per key row) form P^T and
//              dS^T (bf16, written back over S^T / dP^T), then dV += P^T dO and dK += dS^T Q
//              with the A operands read from TMEM.  dK * scale and dV are stored into dqkv.
//
// The MMA thread waits for the previous step's A-from-TMEM MMAs before it overwrites the
// aliased columns.  Warp roles as in the forward: warp 0 TMA producer, warp 1 MMA issuer and
// TMEM owner, warps 2..5 element-wise work and the epilogue.  Every wait is bounded.

#include "common.cuh"

namespace ht {
namespace attn_bwd {

constexpr int THREADS = 192;
constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ------------------------------------------------------------------------------------------------
// dQ
// ------------------------------------------------------------------------------------------------
template <int D>
struct DqCfg {
  static constexpr int BQ = 128, BKV = 64;
  static constexpr int Q_BYTES = BQ * D * 2;    // Q and dO tiles
  static constexpr int KV_BYTES = BKV * D * 2;  // K and V tiles
  static constexpr int STAGES = D == 64 ? 2 : 1;
  static constexpr int SMEM = 2 * Q_BYTES + STAGES * 2 * KV_BYTES + 1024;
  static constexpr uint32_t S_COL = 0, DP_COL = 64, DQ_COL = 128, TMEM_COLS = 256;
};

template <int D>
__global__ void __launch_bounds__(THREADS, 2)
    dq_kernel(const __grid_constant__ CUtensorMap map_q128, const __grid_constant__ CUtensorMap map_kv64,
              const __grid_constant__ CUtensorMap map_do128, const __grid_constant__ CUtensorMap map_dqkv128,
              const float* __restrict__ lse, const float* __restrict__ delta, int S, int H, int HKV, int causal, float scale,
              int* err) {
  using C = DqCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sDO = smem + C::Q_BYTES;
  uint8_t* sK = smem + 2 * C::Q_BYTES;
  uint8_t* sV = sK + C::STAGES * C::KV_BYTES;

  __shared__ __align__(8) uint64_t q_full, s_full, p_full, o_full;
  __shared__ __align__(8) uint64_t kv_full[C::STAGES], kv_empty[C::STAGES];
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (S + C::BQ - 1) / C::BQ;
  const int qt = nqt - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (H / HKV);
  const int q0 = qt * C::BQ;
  const int nkt = (S + C::BKV - 1) / C::BKV;
  const int n_kv = causal ? min((q0 + C::BQ + C::BKV - 1) / C::BKV, nkt) : nkt;
  const float scale_log2 = scale * LOG2E;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&s_full, 1);
    mbar_init(&p_full, 4);
    mbar_init(&o_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&q_full, 2 * C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(sQ + c * (C::BQ * 128), &map_q128, &q_full, h * D + c * 64, q0, b);
        tma_load_3d(sDO + c * (C::BQ * 128), &map_do128, &q_full, h * D + c * 64, q0, b);
      }
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % C::STAGES;
        if (!mbar_wait(&kv_empty[st], ((j / C::STAGES) & 1) ^ 1u, err, 21)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sK + st * C::KV_BYTES + c * (C::BKV * 128), &map_kv64, &kv_full[st], (H + hk) * D + c * 64, j * C::BKV, b);
          tma_load_3d(sV + st * C::KV_BYTES + c * (C::BKV * 128), &map_kv64, &kv_full[st], (H + HKV + hk) * D + c * 64,
                      j * C::BKV, b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, C::BKV, false, false);
    constexpr uint32_t idesc_q = umma_idesc_bf16(128, D, false, true);
    bool ok = mbar_wait(&q_full, 0, err, 22);
    for (int j = 0; j < n_kv && ok; ++j) {
      const int st = j % C::STAGES;
      if (!mbar_wait(&kv_full[st], (j / C::STAGES) & 1, err, 23)) break;
      if (j > 0 && !mbar_wait(&o_full, (j - 1) & 1, err, 24)) break;  // dS (aliased on S) consumed
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(sQ), da = smem_u32(sDO);
        const uint32_t ka = smem_u32(sK + st * C::KV_BYTES), va = smem_u32(sV + st * C::KV_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t aoff = (k / 4) * (C::BQ * 128) + (k % 4) * 32;
          const uint32_t boff = (k / 4) * (C::BKV * 128) + (k % 4) * 32;
          tc_mma_f16(tmem + C::S_COL, umma_desc_sw128(qa + aoff, 16, 1024), umma_desc_sw128(ka + boff, 16, 1024), idesc_s,
                     k != 0 ? 1u : 0u);
          tc_mma_f16(tmem + C::DP_COL, umma_desc_sw128(da + aoff, 16, 1024), umma_desc_sw128(va + boff, 16, 1024), idesc_s,
                     k != 0 ? 1u : 0u);
        }
        tc_commit(&s_full);
      }
      __syncwarp();
      if (!mbar_wait(&p_full, j & 1, err, 25)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t ka = smem_u32(sK + st * C::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BKV / 16; ++kk)
          tc_mma_f16_ts(tmem + C::DQ_COL, tmem + C::S_COL + kk * 8, umma_desc_sw128(ka + kk * 2048, C::BKV * 128, 1024), idesc_q,
                        (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&kv_empty[st]);
        tc_commit(&o_full);
      }
      __syncwarp();
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int q = q0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const long long row_idx = ((long long)b * H + h) * S + (q < S ? q : S - 1);
    const float lse2 = lse[row_idx] * LOG2E;
    const float dl = delta[row_idx];
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait(&s_full, j & 1, err, 26)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kv0 = j * C::BKV;
      const bool edge = (kv0 + C::BKV > S) || (causal && kv0 + C::BKV - 1 > q0);
      const int limit = causal ? min(S - 1, q) : S - 1;
#pragma unroll 1
      for (int c = 0; c < C::BKV / 32; ++c) {
        float sv[32], dp[32];
        tmem_ld_32x32b_x32(tmem + lane_off + C::S_COL + c * 32, sv);
        tmem_ld_32x32b_x32(tmem + lane_off + C::DP_COL + c * 32, dp);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p0 = fast_exp2(fmaf(sv[e], scale_log2, -lse2)), p1 = fast_exp2(fmaf(sv[e + 1], scale_log2, -lse2));
          if (edge) {
            if (kv0 + c * 32 + e > limit) p0 = 0.f;
            if (kv0 + c * 32 + e + 1 > limit) p1 = 0.f;
          }
          pk[e / 2] = pack2(p0 * (dp[e] - dl), p1 * (dp[e + 1] - dl));
        }
        tmem_st_32x32b_x16(tmem + lane_off + C::S_COL + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
    }
    if (ok && mbar_wait(&o_full, (n_kv - 1) & 1, err, 27)) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + lane_off + C::DQ_COL + c * 32, v);
        uint8_t* row = sQ + (c / 2) * (C::BQ * 128) + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 pkd;
          pkd.x = pack2(v[u * 8 + 0] * scale, v[u * 8 + 1] * scale);
          pkd.y = pack2(v[u * 8 + 2] * scale, v[u * 8 + 3] * scale);
          pkd.z = pack2(v[u * 8 + 4] * scale, v[u * 8 + 5] * scale);
          pkd.w = pack2(v[u * 8 + 6] * scale, v[u * 8 + 7] * scale);
          const int unit = (c % 2) * 4 + u;
          *reinterpret_cast<uint4*>(row + ((unit ^ (r & 7)) << 4)) = pkd;
        }
      }
      fence_proxy_async_smem();
      named_barrier_sync(1, 128);
      if (threadIdx.x == 64) {
#pragma unroll
        for (int c = 0; c < D / 64; ++c) tma_store_3d(&map_dqkv128, sQ + c * (C::BQ * 128), h * D + c * 64, q0, b);
        bulk_commit();
        bulk_wait_all();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------
// dK, dV
// ------------------------------------------------------------------------------------------------
template <int D>
struct DkvCfg {
  static constexpr int BKV = 128, BQ = 64;
  static constexpr int KV_BYTES = BKV * D * 2;  // K and V tiles (resident)
  static constexpr int Q_BYTES = BQ * D * 2;    // Q and dO tiles (streamed)
  static constexpr int STAGES = 2;
  static constexpr int SMEM = 2 * KV_BYTES + STAGES * 2 * Q_BYTES + 1024;
  static constexpr uint32_t ST_COL = 0, DPT_COL = 64, DV_COL = 128, DK_COL = 128 + D;
  static constexpr uint32_t TMEM_COLS = D == 64 ? 256 : 512;
  static constexpr int MIN_BLOCKS = D == 64 ? 2 : 1;
};

template <int D>
__global__ void __launch_bounds__(THREADS, DkvCfg<D>::MIN_BLOCKS)
    dkdv_kernel(const __grid_constant__ CUtensorMap map_kv128, const __grid_constant__ CUtensorMap map_q64,
                const __grid_constant__ CUtensorMap map_do64, const __grid_constant__ CUtensorMap map_dqkv128,
                const float* __restrict__ lse, const float* __restrict__ delta, int S, int H, int HKV, int causal, float scale,
                int* err) {
  using C = DkvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sK = smem;
  uint8_t* sV = smem + C::KV_BYTES;
  uint8_t* sQ = smem + 2 * C::KV_BYTES;
  uint8_t* sDO = sQ + C::STAGES * C::Q_BYTES;

  __shared__ __align__(8) uint64_t kv_ready, s_full, p_full, o_full;
  __shared__ __align__(8) uint64_t q_full[C::STAGES], q_empty[C::STAGES];
  __shared__ uint32_t tmem_slot;
  __shared__ __align__(16) float s_lse2[2][C::BQ];   // lse * log2(e) of the step's queries (double-buffered)
  __shared__ __align__(16) float s_delta[2][C::BQ];  // delta of the step's queries

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = (S + C::BKV - 1) / C::BKV;
  const int kt = nkt - 1 - (int)blockIdx.x;  // causal: early key tiles see the most queries
  const int hk = blockIdx.y, b = blockIdx.z;
  const int group = H / HKV;
  const int kv0 = kt * C::BKV;
  const int nqt = (S + C::BQ - 1) / C::BQ;
  const int first_qt = causal ? kv0 / C::BQ : 0;
  const int per_head = nqt - first_qt;
  const int n_steps = per_head * group;
  const float scale_log2 = scale * LOG2E;

  if (threadIdx.x == 0) {
    mbar_init(&kv_ready, 1);
    mbar_init(&s_full, 1);
    mbar_init(&p_full, 4);
    mbar_init(&o_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&kv_ready, 2 * C::KV_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(sK + c * (C::BKV * 128), &map_kv128, &kv_ready, (H + hk) * D + c * 64, kv0, b);
        tma_load_3d(sV + c * (C::BKV * 128), &map_kv128, &kv_ready, (H + HKV + hk) * D + c * 64, kv0, b);
      }
      for (int t = 0; t < n_steps; ++t) {
        const int st = t % C::STAGES;
        const int h = hk * group + t / per_head;
        const int qt = first_qt + t % per_head;
        if (!mbar_wait(&q_empty[st], ((t / C::STAGES) & 1) ^ 1u, err, 31)) break;
        mbar_arrive_expect_tx(&q_full[st], 2 * C::Q_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sQ + st * C::Q_BYTES + c * (C::BQ * 128), &map_q64, &q_full[st], h * D + c * 64, qt * C::BQ, b);
          tma_load_3d(sDO + st * C::Q_BYTES + c * (C::BQ * 128), &map_do64, &q_full[st], h * D + c * 64, qt * C::BQ, b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, C::BQ, false, false);
    constexpr uint32_t idesc_acc = umma_idesc_bf16(128, D, false, true);
    bool ok = mbar_wait(&kv_ready, 0, err, 32);
    for (int t = 0; t < n_steps && ok; ++t) {
      const int st = t % C::STAGES;
      if (!mbar_wait(&q_full[st], (t / C::STAGES) & 1, err, 33)) break;
      if (t > 0 && !mbar_wait(&o_full, (t - 1) & 1, err, 34)) break;  // P^T / dS^T (aliased) consumed
      tc_fence_after();
      if (lane == 0) {
        const uint32_t ka = smem_u32(sK), va = smem_u32(sV);
        const uint32_t qa = smem_u32(sQ + st * C::Q_BYTES), da = smem_u32(sDO + st * C::Q_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t aoff = (k / 4) * (C::BKV * 128) + (k % 4) * 32;
          const uint32_t boff = (k / 4) * (C::BQ * 128) + (k % 4) * 32;
          tc_mma_f16(tmem + C::ST_COL, umma_desc_sw128(ka + aoff, 16, 1024), umma_desc_sw128(qa + boff, 16, 1024), idesc_s,
                     k != 0 ? 1u : 0u);
          tc_mma_f16(tmem + C::DPT_COL, umma_desc_sw128(va + aoff, 16, 1024), umma_desc_sw128(da + boff, 16, 1024), idesc_s,
                     k != 0 ? 1u : 0u);
        }
        tc_commit(&s_full);
      }
      __syncwarp();
      if (!mbar_wait(&p_full, t & 1, err, 35)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(sQ + st * C::Q_BYTES), da = smem_u32(sDO + st * C::Q_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BQ / 16; ++kk) {
          tc_mma_f16_ts(tmem + C::DV_COL, tmem + C::ST_COL + kk * 8, umma_desc_sw128(da + kk * 2048, C::BQ * 128, 1024),
                        idesc_acc, (t > 0 || kk > 0) ? 1u : 0u);
          tc_mma_f16_ts(tmem + C::DK_COL, tmem + C::DPT_COL + kk * 8, umma_desc_sw128(qa + kk * 2048, C::BQ * 128, 1024),
                        idesc_acc, (t > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&q_empty[st]);
        tc_commit(&o_full);
      }
      __syncwarp();
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row within the tile
    const int kv = kv0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    const int tid = threadIdx.x - 64;  // 0..127 across the four element-wise warps
    for (int t = 0; t < n_steps; ++t) {
      const int h = hk * group + t / per_head;
      const int qt = first_qt + t % per_head;
      const int qb = qt * C::BQ;
      // Stage the per-query statistics of this step once (each thread loads one value); the
      // barrier also orders the previous step's reads of this buffer before the overwrite.
      {
        const int qi = min(qb + (tid & (C::BQ - 1)), S - 1);
        const long long idx = ((long long)b * H + h) * S + qi;
        if (tid < C::BQ) s_lse2[t & 1][tid] = lse[idx] * LOG2E;
        else s_delta[t & 1][tid - C::BQ] = delta[idx];
      }
      named_barrier_sync(1, 128);
      const float* sl = s_lse2[t & 1];
      const float* sd = s_delta[t & 1];
      if (!mbar_wait(&s_full, t & 1, err, 36)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool edge = (qb + C::BQ > S) || (causal && qb < kv0 + C::BKV);
#pragma unroll 1
      for (int c = 0; c < C::BQ / 32; ++c) {
        float sv[32], dp[32];
        tmem_ld_32x32b_x32(tmem + lane_off + C::ST_COL + c * 32, sv);
        tmem_ld_32x32b_x32(tmem + lane_off + C::DPT_COL + c * 32, dp);
        uint32_t pp[16], pd[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 l2 = *reinterpret_cast<const float2*>(sl + c * 32 + e);
          const float2 d2 = *reinterpret_cast<const float2*>(sd + c * 32 + e);
          float p0 = fast_exp2(fmaf(sv[e], scale_log2, -l2.x));
          float p1 = fast_exp2(fmaf(sv[e + 1], scale_log2, -l2.y));
          if (edge) {
            const int qa = qb + c * 32 + e;
            if (qa >= S || (causal && qa < kv)) p0 = 0.f;
            if (qa + 1 >= S || (causal && qa + 1 < kv)) p1 = 0.f;
          }
          pp[e / 2] = pack2(p0, p1);
          pd[e / 2] = pack2(p0 * (dp[e] - d2.x), p1 * (dp[e + 1] - d2.y));
        }
        tmem_st_32x32b_x16(tmem + lane_off + C::ST_COL + c * 16, pp);
        tmem_st_32x32b_x16(tmem + lane_off + C::DPT_COL + c * 16, pd);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
    }
    if (ok && (n_steps == 0 || mbar_wait(&o_full, (n_steps - 1) & 1, err, 37))) {
      tc_fence_after();
      // dV (unscaled) into the V buffer, dK * scale into the K buffer (both no longer read).
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        uint8_t* buf = which == 0 ? sV : sK;
        const uint32_t col = which == 0 ? C::DV_COL : C::DK_COL;
        const float f = which == 0 ? 1.f : scale;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          if (n_steps > 0) {
            tmem_ld_32x32b_x32(tmem + lane_off + col + c * 32, v);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = 0.f;
          }
          uint8_t* row = buf + (c / 2) * (C::BKV * 128) + r * 128;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 pkd;
            pkd.x = pack2(v[u * 8 + 0] * f, v[u * 8 + 1] * f);
            pkd.y = pack2(v[u * 8 + 2] * f, v[u * 8 + 3] * f);
            pkd.z = pack2(v[u * 8 + 4] * f, v[u * 8 + 5] * f);
            pkd.w = pack2(v[u * 8 + 6] * f, v[u * 8 + 7] * f);
            const int unit = (c % 2) * 4 + u;
            *reinterpret_cast<uint4*>(row + ((unit ^ (r & 7)) << 4)) = pkd;
          }
        }
      }
      fence_proxy_async_smem();
      named_barrier_sync(1, 128);
      if (threadIdx.x == 64) {
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_store_3d(&map_dqkv128, sK + c * (C::BKV * 128), (H + hk) * D + c * 64, kv0, b);
          tma_store_3d(&map_dqkv128, sV + c * (C::BKV * 128), (H + HKV + hk) * D + c * 64, kv0, b);
        }
        bulk_commit();
        bulk_wait_all();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    HT_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr));
    HT_CHECK(qr == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// bf16 [batch][rows][width] map with 64-column x `box_rows` boxes and the 128-byte swizzle.
static CUtensorMap make_map(const void* base, int64_t batch, int64_t rows, int64_t width, int box_rows) {
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(width * 2), (cuuint64_t)(rows * width * 2)};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult res = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HT_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled (attention backward) failed with code ", (int)res);
  return map;
}

template <typename K>
static void set_smem(K kernel, int bytes) {
  HT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

template <int D>
static void launch(const at::Tensor& qkv, const at::Tensor& dout, const at::Tensor& lse, const at::Tensor& delta,
                   at::Tensor& dqkv, int H, int HKV, bool causal, float scale, int* err, cudaStream_t s) {
  const int64_t B = qkv.size(0), S = qkv.size(1), W = qkv.size(2);
  const CUtensorMap q128 = make_map(qkv.data_ptr(), B, S, W, 128);
  const CUtensorMap q64 = make_map(qkv.data_ptr(), B, S, W, 64);
  const CUtensorMap do128 = make_map(dout.data_ptr(), B, S, (int64_t)H * D, 128);
  const CUtensorMap do64 = make_map(dout.data_ptr(), B, S, (int64_t)H * D, 64);
  const CUtensorMap dqkv128 = make_map(dqkv.data_ptr(), B, S, W, 128);
  static bool once = [] {
    set_smem(dq_kernel<D>, DqCfg<D>::SMEM);
    set_smem(dkdv_kernel<D>, DkvCfg<D>::SMEM);
    return true;
  }();
  (void)once;
  const dim3 gq((unsigned)((S + 127) / 128), (unsigned)H, (unsigned)B);
  const dim3 gk((unsigned)((S + 127) / 128), (unsigned)HKV, (unsigned)B);
  dkdv_kernel<D><<<gk, THREADS, DkvCfg<D>::SMEM, s>>>(q128, q64, do64, dqkv128, lse.data_ptr<float>(), delta.data_ptr<float>(),
                                                       (int)S, H, HKV, causal ? 1 : 0, scale, err);
  dq_kernel<D><<<gq, THREADS, DqCfg<D>::SMEM, s>>>(q128, q64, do128, dqkv128, lse.data_ptr<float>(), delta.data_ptr<float>(),
                                                   (int)S, H, HKV, causal ? 1 : 0, scale, err);
}

}  // namespace attn_bwd

int* attention_error_word(const at::Device& dev);

// Runs both backward kernels after the caller has filled `delta`; returns false (nothing
// launched) when the tensor-core path does not apply.
bool attention_backward_tcgen05(at::Tensor qkv, at::Tensor dout, at::Tensor lse, at::Tensor delta, at::Tensor dqkv, int64_t H,
                                int64_t HKV, int64_t D, bool causal, double scale) {
  if (!(D == 64 || D == 128) || !qkv.is_contiguous() || !dout.is_contiguous() || !dqkv.is_contiguous()) return false;
  for (const at::Tensor* t : {&qkv, &dout, &dqkv})
    if (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) return false;
  bind_context(qkv.device().index());
  int* err = attention_error_word(qkv.device());
  cudaStream_t s = stream();
  if (D == 64) attn_bwd::launch<64>(qkv, dout, lse, delta, dqkv, (int)H, (int)HKV, causal, (float)scale, err, s);
  else attn_bwd::launch<128>(qkv, dout, lse, delta, dqkv, (int)H, (int)HKV, causal, (float)scale, err, s);
  HT_CUDA_CHECK(cudaGetLastError());
  return true;
}

}  // namespace ht
