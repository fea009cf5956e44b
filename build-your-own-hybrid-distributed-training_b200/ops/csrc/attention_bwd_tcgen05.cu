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
              int qt0, int nqt_w, int* err) {
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
  int qt, h, b;  // query tiles qt0 .. qt0 + nqt_w - 1
  tile_major_block(nqt_w, H, qt, h, b);
  qt = qt0 + nqt_w - 1 - qt;  // causal: the last query tiles see the most keys; they start first
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
  static constexpr int BKV = 128, BQ = 64;  // BQ divides 128 (query windows are given in 128-row tiles)
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
                int qt0, int nqt_w, int* err) {
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
  int kt, hk, b;  // causal: key tile kt sees nqt - kt query tiles, so tile 0 is the heaviest
  tile_major_block(nkt, HKV, kt, hk, b);
  const int group = H / HKV;
  const int kv0 = kt * C::BKV;
  const int nqt = (S + C::BQ - 1) / C::BQ;
  // Query tiles (of BQ rows) that can see this key tile, inside the window of 128-row tiles
  // qt0 .. qt0 + nqt_w - 1.
  const int win_lo = qt0 * 128 / C::BQ, win_hi = (qt0 + nqt_w) * 128 / C::BQ;
  const int first_qt = max(causal ? kv0 / C::BQ : 0, win_lo);
  const int per_head = max(0, min(nqt, win_hi) - first_qt);
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
    // With no query step (a key tile outside a query window) the K / V loads may still be in
    // flight: wait for them before the zeros below overwrite the same buffers.
    if (ok && (n_steps == 0 ? mbar_wait(&kv_ready, 0, err, 38) : mbar_wait(&o_full, (n_steps - 1) & 1, err, 37))) {
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

// ------------------------------------------------------------------------------------------------
// Fused dK, dV and dQ for D = 64 (used when bitwise reproducibility is not required).
//
// One CTA per (128-key tile, kv head, batch), 14 warps, one CTA per SM.  For each query head of
// the group and each 128-query tile at or after the key tile:
//   S^T = K Q^T and dP^T = V dO^T into TMEM (M = 128 keys, N = 128 queries);
//   eight element-wise warps (two per TMEM lane quarter, 64 queries each) form P^T and
//   dS^T = P^T (dP^T - delta) and write them as bf16 into shared memory, 128-byte swizzled;
//   dV += P^T dO and dK += dS^T Q read them there as K-major A operands, and dQ_tile = dS K reads
//   the same dS^T bytes as an MN-major A operand;
//   four epilogue warps add dQ_tile (fp32, double-buffered in TMEM) into a global fp32 dQ
//   accumulator with TMA reduce-adds, whose order across key tiles is not fixed.
// The MMA of the next tile's S^T / dP^T starts as soon as the element-wise warps have read the
// current one, so the tensor cores and the exponentials overlap.  S and dP are computed once per
// (key tile, query tile), against twice in the reproducible two-kernel path.
// TMEM columns: S^T [0,128), dP^T [128,256), dV [256,320), dK [320,384), dQ [384,448) and [448,512).
// ------------------------------------------------------------------------------------------------
struct FusedCfg {
  static constexpr int D = 64, BKV = 128, BQ = 128;
  static constexpr int TILE = 128 * 64 * 2;  // one 128-row x 64-column bf16 tile (16 KB)
  static constexpr int STAGES = 2;
  static constexpr int OFF_K = 0, OFF_V = TILE, OFF_Q = 2 * TILE;  // stage s: Q at OFF_Q + 2 s TILE, dO next to it
  static constexpr int OFF_P = OFF_Q + STAGES * 2 * TILE;          // P^T: two 64-query chunks of 128 key rows
  static constexpr int OFF_DS = OFF_P + 2 * TILE;                  // dS^T: same layout
  static constexpr int OFF_DQ = OFF_DS + 2 * TILE;                 // dQ staging: 4 warps x 2 pieces x 4 KB
  static constexpr int PIECE = 32 * 128;
  static constexpr int SMEM = OFF_DQ + 4 * 2 * PIECE + 1024;
  static constexpr uint32_t ST_COL = 0, DPT_COL = 128, DV_COL = 256, DK_COL = 320, DQ_COL = 384;
  static constexpr int THREADS = 448;  // warp 0 TMA, warp 1 MMA, warps 2..9 element-wise, warps 10..13 dQ
};

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(FusedCfg::THREADS, 1)
    fused_bwd_kernel(const __grid_constant__ CUtensorMap map_qkv128, const __grid_constant__ CUtensorMap map_do128,
                     const __grid_constant__ CUtensorMap map_dqkv128, const __grid_constant__ CUtensorMap map_dq_acc,
                     const float* __restrict__ lse, const float* __restrict__ delta, int S, int H, int HKV, int causal,
                     float scale, int qt0, int nqt_w, int* err) {
  using C = FusedCfg;
  constexpr int D = C::D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sP = smem + C::OFF_P;
  uint8_t* sDS = smem + C::OFF_DS;

  __shared__ __align__(8) uint64_t kv_ready, s_full, st_free, p_ready, pd_free, acc_full, kv_staged;
  __shared__ __align__(8) uint64_t q_full[C::STAGES], q_empty[C::STAGES], dq_full[2], dq_free[2];
  __shared__ uint32_t tmem_slot;
  // Per stage: lse and delta of the step's 128 queries, bulk-copied with the Q / dO tiles.
  __shared__ __align__(16) float s_stats[C::STAGES][2][C::BQ];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = (S + C::BKV - 1) / C::BKV;
  int kt, hk, b;  // causal: key tile kt sees nqt - kt query tiles, so tile 0 is the heaviest
  tile_major_block(nkt, HKV, kt, hk, b);
  const int group = H / HKV;
  const int kv0 = kt * C::BKV;
  const int nqt = (S + C::BQ - 1) / C::BQ;
  // Query tiles (of BQ rows) that can see this key tile, inside the window of 128-row tiles
  // qt0 .. qt0 + nqt_w - 1.
  const int win_lo = qt0 * 128 / C::BQ, win_hi = (qt0 + nqt_w) * 128 / C::BQ;
  const int first_qt = max(causal ? kv0 / C::BQ : 0, win_lo);
  const int per_head = max(0, min(nqt, win_hi) - first_qt);
  const int n_steps = per_head * group;
  const float scale_log2 = scale * LOG2E;

  if (threadIdx.x == 0) {
    mbar_init(&kv_ready, 1);
    mbar_init(&s_full, 1);
    mbar_init(&st_free, 8);
    mbar_init(&p_ready, 8);
    mbar_init(&pd_free, 1);
    mbar_init(&acc_full, 1);
    mbar_init(&kv_staged, 256);
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  auto step_head = [&](int t) { return hk * group + t / per_head; };
  auto step_q0 = [&](int t) { return (first_qt + t % per_head) * C::BQ; };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&kv_ready, 2 * C::TILE);
      tma_load_3d(sK, &map_qkv128, &kv_ready, (H + hk) * D, kv0, b);
      tma_load_3d(sV, &map_qkv128, &kv_ready, (H + HKV + hk) * D, kv0, b);
      for (int t = 0; t < n_steps; ++t) {
        const int st = t % C::STAGES;
        if (!mbar_wait(&q_empty[st], ((t / C::STAGES) & 1) ^ 1u, err, 51)) break;
        // The statistics of queries qb .. qb + n - 1 (n rounded down to a multiple of 4 floats; the
        // element-wise warps read the ragged tail from global memory).
        const int qb = step_q0(t);
        const int nstat = (min(C::BQ, S - qb) / 4) * 4;
        const long long row0 = ((long long)b * H + step_head(t)) * S + qb;
        mbar_arrive_expect_tx(&q_full[st], 2 * C::TILE + 2 * nstat * 4);
        uint8_t* q_dst = smem + C::OFF_Q + st * 2 * C::TILE;
        tma_load_3d(q_dst, &map_qkv128, &q_full[st], step_head(t) * D, qb, b);
        tma_load_3d(q_dst + C::TILE, &map_do128, &q_full[st], step_head(t) * D, qb, b);
        if (nstat > 0) {
          bulk_load(s_stats[st][0], lse + row0, nstat * 4, &q_full[st]);
          bulk_load(s_stats[st][1], delta + row0, nstat * 4, &q_full[st]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);   // S^T, dP^T
    constexpr uint32_t idesc_kv = umma_idesc_bf16(128, D, false, true);    // dV, dK: A K-major (smem), B MN-major
    constexpr uint32_t idesc_q = umma_idesc_bf16(128, D, true, true);      // dQ: A = dS MN-major, B = K MN-major
    const uint32_t ka = smem_u32(sK), va = smem_u32(sV), pa = smem_u32(sP), dsa = smem_u32(sDS);
    bool ok = mbar_wait(&kv_ready, 0, err, 52);
    for (int j = 0; j <= n_steps && ok; ++j) {
      if (j < n_steps) {
        const int st = j % C::STAGES;
        if (!mbar_wait(&q_full[st], (j / C::STAGES) & 1, err, 53)) break;
        if (j > 0 && !mbar_wait(&st_free, (j - 1) & 1, err, 54)) break;  // S^T / dP^T of step j-1 read
        tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = smem_u32(smem + C::OFF_Q + st * 2 * C::TILE), da = qa + C::TILE;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            tc_mma_f16(tmem + C::ST_COL, umma_desc_sw128(ka + k * 32, 16, 1024), umma_desc_sw128(qa + k * 32, 16, 1024),
                       idesc_s, k != 0 ? 1u : 0u);
            tc_mma_f16(tmem + C::DPT_COL, umma_desc_sw128(va + k * 32, 16, 1024), umma_desc_sw128(da + k * 32, 16, 1024),
                       idesc_s, k != 0 ? 1u : 0u);
          }
          tc_commit(&s_full);
        }
        __syncwarp();
      }
      if (j > 0) {
        const int i = j - 1, sti = i % C::STAGES, buf = i & 1;
        if (!mbar_wait(&p_ready, i & 1, err, 55)) break;              // P^T / dS^T of step i in shared memory
        if (i >= 2 && !mbar_wait(&dq_free[buf], ((i >> 1) - 1) & 1, err, 56)) break;  // dQ buffer drained
        tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = smem_u32(smem + C::OFF_Q + sti * 2 * C::TILE), da = qa + C::TILE;
#pragma unroll
          for (int kk = 0; kk < C::BQ / 16; ++kk) {
            const uint32_t aoff = (kk >> 2) * C::TILE + (kk & 3) * 32;
            tc_mma_f16(tmem + C::DV_COL, umma_desc_sw128(pa + aoff, 16, 1024), umma_desc_sw128(da + kk * 2048, C::TILE, 1024),
                       idesc_kv, (i > 0 || kk > 0) ? 1u : 0u);
            tc_mma_f16(tmem + C::DK_COL, umma_desc_sw128(dsa + aoff, 16, 1024), umma_desc_sw128(qa + kk * 2048, C::TILE, 1024),
                       idesc_kv, (i > 0 || kk > 0) ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < C::BKV / 16; ++kk)
            tc_mma_f16(tmem + C::DQ_COL + buf * D, umma_desc_sw128(dsa + kk * 2048, C::TILE, 1024),
                       umma_desc_sw128(ka + kk * 2048, C::TILE, 1024), idesc_q, kk > 0 ? 1u : 0u);
          tc_commit(&pd_free);
          tc_commit(&q_empty[sti]);
          tc_commit(&dq_full[buf]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) tc_commit(&acc_full);
    __syncwarp();
  } else if (warp < 10) {
    // ---------------- element-wise: P^T and dS^T ----------------
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // key row within the tile
    const int kv = kv0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int t = 0; t < n_steps; ++t) {
      const int h = step_head(t), qb = step_q0(t);
      // Per-query statistics: in shared memory, bulk-copied with this step's Q / dO tiles (the
      // q_full phase of the stage covers them); the ragged tail beyond a multiple of 4 comes from
      // global memory.
      const long long row0 = ((long long)b * H + h) * S;
      const int qh = qb + half * 64;  // first query of this thread's 64
      const int st = t % C::STAGES;
      const int nstat = (min(C::BQ, S - qb) / 4) * 4;
      if (!mbar_wait(&q_full[st], (t / C::STAGES) & 1, err, 62)) {
        ok = false;
        break;
      }
      const float* sl = s_stats[st][0] + half * 64;
      const float* sd = s_stats[st][1] + half * 64;
      if (!mbar_wait(&s_full, t & 1, err, 57)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool edge = (qb + C::BQ > S) || (causal && qb < kv0 + C::BKV);
      uint8_t* prow = sP + half * C::TILE + r * 128;
      uint8_t* drow = sDS + half * C::TILE + r * 128;
      // One chunk of 16 queries at a time, written to shared memory as soon as it is computed: a
      // rolled loop keeps the instruction footprint and the live registers small.
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float ls[16], dl[16];
        const int qc = qh + c * 16;
        if (qc + 16 - qb <= nstat) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float4 l4 = reinterpret_cast<const float4*>(sl + c * 16)[u];
            const float4 d4 = reinterpret_cast<const float4*>(sd + c * 16)[u];
            ls[4 * u] = l4.x; ls[4 * u + 1] = l4.y; ls[4 * u + 2] = l4.z; ls[4 * u + 3] = l4.w;
            dl[4 * u] = d4.x; dl[4 * u + 1] = d4.y; dl[4 * u + 2] = d4.z; dl[4 * u + 3] = d4.w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int q = min(qc + e, S - 1);  // queries past the end reuse the last one's (finite) statistics
            const int k = q - qb;
            ls[e] = k < nstat ? s_stats[st][0][k] : __ldg(lse + row0 + q);
            dl[e] = k < nstat ? s_stats[st][1][k] : __ldg(delta + row0 + q);
          }
        }
        float sv[16], dp[16];
        tmem_ld_32x32b_x16(tmem + lane_off + C::ST_COL + half * 64 + c * 16, sv);
        tmem_ld_32x32b_x16(tmem + lane_off + C::DPT_COL + half * 64 + c * 16, dp);
        if (c == 3) {  // last TMEM read of this tile: S^T / dP^T may be overwritten by the next one
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&st_free);
        }
        uint32_t pp[8], pd[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float2 l2 = make_float2(ls[e] * LOG2E, ls[e + 1] * LOG2E);
          const float2 d2 = make_float2(dl[e], dl[e + 1]);
          float p0 = fast_exp2(fmaf(sv[e], scale_log2, -l2.x));
          float p1 = fast_exp2(fmaf(sv[e + 1], scale_log2, -l2.y));
          if (edge) {
            const int qa = qc + e;
            if (qa >= S || (causal && qa < kv)) p0 = 0.f;
            if (qa + 1 >= S || (causal && qa + 1 < kv)) p1 = 0.f;
          }
          pp[e / 2] = pack2(p0, p1);
          pd[e / 2] = pack2(p0 * (dp[e] - d2.x), p1 * (dp[e + 1] - d2.y));
        }
        // The previous step's dV / dK MMAs read sP / sDS: wait for them before the first store.
        if (c == 0 && t > 0 && !mbar_wait(&pd_free, (t - 1) & 1, err, 58)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int off = ((2 * c + j) ^ (r & 7)) << 4;
          *reinterpret_cast<uint4*>(prow + off) = make_uint4(pp[4 * j], pp[4 * j + 1], pp[4 * j + 2], pp[4 * j + 3]);
          *reinterpret_cast<uint4*>(drow + off) = make_uint4(pd[4 * j], pd[4 * j + 1], pd[4 * j + 2], pd[4 * j + 3]);
        }
      }
      if (!ok) break;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready);
    }
    // ---------------- dV / dK epilogue ----------------
    if (ok && mbar_wait(&acc_full, 0, err, 59)) {
      tc_fence_after();
      uint8_t* buf = half == 0 ? sV : sK;  // no MMA reads K or V any more
      const uint32_t col = half == 0 ? C::DV_COL : C::DK_COL;
      const float f = half == 0 ? 1.f : scale;
      uint8_t* row = buf + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        if (n_steps > 0) {
          tmem_ld_32x32b_x32(tmem + lane_off + col + c * 32, v);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0.f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 pkd;
          pkd.x = pack2(v[u * 8 + 0] * f, v[u * 8 + 1] * f);
          pkd.y = pack2(v[u * 8 + 2] * f, v[u * 8 + 3] * f);
          pkd.z = pack2(v[u * 8 + 4] * f, v[u * 8 + 5] * f);
          pkd.w = pack2(v[u * 8 + 6] * f, v[u * 8 + 7] * f);
          const int unit = c * 4 + u;
          *reinterpret_cast<uint4*>(row + ((unit ^ (r & 7)) << 4)) = pkd;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&kv_staged);  // every element-wise thread; the storing thread waits (bounded)
      if (threadIdx.x == 64 && mbar_wait(&kv_staged, 0, err, 61)) {
        tma_store_3d(&map_dqkv128, sK, (H + hk) * D, kv0, b);
        tma_store_3d(&map_dqkv128, sV, (H + HKV + hk) * D, kv0, b);
        bulk_commit();
        bulk_wait_all();
      }
    }
  } else {
    // ---------------- dQ: TMEM -> fp32 reduce-add into the global accumulator ----------------
    const int quarter = warp & 3;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* stage = smem + C::OFF_DQ + (warp - 10) * 2 * C::PIECE;
    for (int i = 0; i < n_steps; ++i) {
      const int buf = i & 1;
      if (!mbar_wait(&dq_full[buf], (i >> 1) & 1, err, 60)) break;
      tc_fence_after();
      const int h = step_head(i), qb = step_q0(i);
#pragma unroll
      for (int piece = 0; piece < 2; ++piece) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + lane_off + C::DQ_COL + buf * D + piece * 32, v);
        uint4 units[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          units[j] = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]), __float_as_uint(v[4 * j + 2]),
                                __float_as_uint(v[4 * j + 3]));
        uint8_t* tile = stage + piece * C::PIECE;
        if (lane == 0) bulk_wait_read_all();  // the previous reduce-add from this staging tile has read it
        __syncwarp();
        uint8_t* row = tile + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(row + ((j ^ (lane & 7)) << 4)) = units[j];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&map_dq_acc, tile, h * D + piece * 32, b * S + qb + quarter * 32);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[buf]);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// dqkv[b, s, h*D + d] = bf16(scale * acc[(b*S + s), h*D + d]) for the query columns of dqkv.
__global__ void __launch_bounds__(256) dq_finish_kernel(const float4* __restrict__ acc, __nv_bfloat16* __restrict__ dqkv,
                                                        long long rows, int hd4, long long row_stride, float scale) {
  const long long n = rows * hd4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / hd4;
    const int c = (int)(i - row * hd4);
    const float4 v = acc[i];
    __align__(8) __nv_bfloat16 o[4] = {f2bf(v.x * scale), f2bf(v.y * scale), f2bf(v.z * scale), f2bf(v.w * scale)};
    *reinterpret_cast<uint2*>(dqkv + row * row_stride + 4 * c) = *reinterpret_cast<const uint2*>(o);
  }
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
                   at::Tensor& dqkv, int H, int HKV, bool causal, float scale, int qt0, int nqt_w, int* err, cudaStream_t s) {
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
  const dim3 gq((unsigned)(nqt_w * H * B));
  const dim3 gk((unsigned)(((S + 127) / 128) * HKV * B));
  dkdv_kernel<D><<<gk, THREADS, DkvCfg<D>::SMEM, s>>>(q128, q64, do64, dqkv128, lse.data_ptr<float>(), delta.data_ptr<float>(),
                                                       (int)S, H, HKV, causal ? 1 : 0, scale, qt0, nqt_w, err);
  dq_kernel<D><<<gq, THREADS, DqCfg<D>::SMEM, s>>>(q128, q64, do128, dqkv128, lse.data_ptr<float>(), delta.data_ptr<float>(),
                                                   (int)S, H, HKV, causal ? 1 : 0, scale, qt0, nqt_w, err);
}

// fp32 [rows][cols] map with 32-column x 32-row boxes and the 128-byte swizzle (dQ accumulator).
static CUtensorMap make_acc_map(void* base, int64_t rows, int64_t cols) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 4)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult res = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HT_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dQ accumulator) failed with code ", (int)res);
  return map;
}

static void launch_fused(const at::Tensor& qkv, const at::Tensor& dout, const at::Tensor& lse, const at::Tensor& delta,
                         at::Tensor& dqkv, int H, int HKV, bool causal, float scale, int qt0, int nqt_w, int* err,
                         cudaStream_t s) {
  constexpr int D = FusedCfg::D;
  const int64_t B = qkv.size(0), S = qkv.size(1), W = qkv.size(2);
  at::Tensor acc = at::zeros({B * S, (int64_t)H * D}, qkv.options().dtype(at::kFloat));
  const CUtensorMap q128 = make_map(qkv.data_ptr(), B, S, W, 128);
  const CUtensorMap do128 = make_map(dout.data_ptr(), B, S, (int64_t)H * D, 128);
  const CUtensorMap dqkv128 = make_map(dqkv.data_ptr(), B, S, W, 128);
  const CUtensorMap macc = make_acc_map(acc.data_ptr(), B * S, (int64_t)H * D);
  static bool once = [] {
    set_smem(fused_bwd_kernel, FusedCfg::SMEM);
    return true;
  }();
  (void)once;
  const dim3 grid((unsigned)(((S + 127) / 128) * HKV * B));
  fused_bwd_kernel<<<grid, FusedCfg::THREADS, FusedCfg::SMEM, s>>>(q128, do128, dqkv128, macc, lse.data_ptr<float>(),
                                                                   delta.data_ptr<float>(), (int)S, H, HKV, causal ? 1 : 0,
                                                                   scale, qt0, nqt_w, err);
  HT_CUDA_CHECK(cudaGetLastError());
  const long long rows = B * S;
  const int hd4 = H * D / 4;
  const int blocks = (int)std::min<long long>((rows * hd4 + 255) / 256, 8LL * num_sms());
  dq_finish_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(acc.data_ptr<float>()),
                                          reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), rows, hd4, W, scale);
}

}  // namespace attn_bwd

int* attention_error_word(const at::Device& dev);
bool deterministic_reductions();

// Runs both backward kernels after the caller has filled `delta`; returns false (nothing
// launched) when the tensor-core path does not apply.
// Queries [q_begin, q_begin + q_len) only (q_len < 0: all): dQ rows of that window, and dK / dV
// summed over those queries (rows of dQ outside the window are not written).
bool attention_backward_tcgen05(at::Tensor qkv, at::Tensor dout, at::Tensor lse, at::Tensor delta, at::Tensor dqkv, int64_t H,
                                int64_t HKV, int64_t D, bool causal, double scale, int64_t q_begin, int64_t q_len) {
  if (!(D == 64 || D == 128) || !qkv.is_contiguous() || !dout.is_contiguous() || !dqkv.is_contiguous()) return false;
  const int64_t S = qkv.size(1);
  if (q_len < 0) q_begin = 0, q_len = S;
  HT_CHECK(q_begin % 128 == 0 && q_begin >= 0 && q_len > 0 && q_begin + q_len <= S,
           "attention query window must start at a multiple of 128 inside the sequence");
  const int qt0 = (int)(q_begin / 128), nqt_w = (int)((q_len + 127) / 128);
  for (const at::Tensor* t : {&qkv, &dout, &dqkv})
    if (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) return false;
  bind_context(qkv.device().index());
  int* err = attention_error_word(qkv.device());
  cudaStream_t s = stream();
  // D = 64 without the reproducibility requirement: one fused kernel (dQ summed by reduce-adds).
  if (D == 64 && !deterministic_reductions() && (H * D) % 32 == 0)
    attn_bwd::launch_fused(qkv, dout, lse, delta, dqkv, (int)H, (int)HKV, causal, (float)scale, qt0, nqt_w, err, s);
  else if (D == 64) attn_bwd::launch<64>(qkv, dout, lse, delta, dqkv, (int)H, (int)HKV, causal, (float)scale, qt0, nqt_w, err, s);
  else attn_bwd::launch<128>(qkv, dout, lse, delta, dqkv, (int)H, (int)HKV, causal, (float)scale, qt0, nqt_w, err, s);
  HT_CUDA_CHECK(cudaGetLastError());
  return true;
}

}  // namespace ht
