// Flash-attention forward on the 5th-generation tensor cores (sm_100a), packed QKV input
// [B, S, (H + 2*Hkv) * D] (D = 64 or 128), grouped-query attention, causal or full.
//
// One CTA per (128-query tile, head, batch), two CTAs per SM:
//   warp 0      TMA producer: the Q tile once, then K/V tiles of 128 keys through a ring;
//   warp 1      MMA issuer and TMEM owner: S = Q K^T into TMEM (M=128, N=128, K=D), then
//               O += P V with P read straight from TMEM (the `.kind::f16` A-from-TMEM form) and
//               V from shared memory as an MN-major operand;
//   warps 2..5  softmax, one thread per query row: read the S row from TMEM, online max / sum in
//               the exp2 domain, write P (bf16 pairs) back to TMEM, rescale the O row in TMEM
//               when the running max moved, and finally normalise O, stage it in swizzled
//               shared memory (the Q buffer, no longer needed) and TMA-store it.
// TMEM columns: S [0,128); P [128,192) for D = 64, or aliased onto S [0,64) for D = 128 (the
// MMA thread then waits for P V to finish before the next S overwrites it); O after that.
// The per-row log-sum-exp (natural log) is written for the backward pass, in the same format
// as the mma.sync kernels in attention.cu.  Every wait is bounded and reports through `err`.

#include "common.cuh"

namespace ht {
namespace attn_tc {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int THREADS = 192;
constexpr float LN2 = 0.6931471805599453f;

template <int D>
struct Cfg {
  static constexpr int CHUNKS = D / 64;                  // 64-column (128-byte) boxes per row
  static constexpr int TILE_BYTES = 128 * D * 2;         // one 128-row tile of Q, K, V or O
  static constexpr int STAGES = D == 64 ? 2 : 1;         // K/V ring depth
  static constexpr int SMEM = TILE_BYTES * (1 + 2 * STAGES) + 1024;
  static constexpr uint32_t S_COL = 0;
  static constexpr uint32_t P_COL = D == 64 ? 128 : 0;  // aliased onto S for D = 128
  static constexpr uint32_t O_COL = D == 64 ? 192 : 128;
  static constexpr uint32_t TMEM_COLS = 256;
};

// Scores of keys that a query may not see (beyond the sequence, or after the query when causal)
// become -inf; only the last key tile of a row can contain such keys.
__device__ __forceinline__ void mask_chunk(float* v, int kv0, int q, int S, int causal) {
  const int limit = causal ? min(S - 1, q) : S - 1;
#pragma unroll
  for (int e = 0; e < 32; ++e)
    if (kv0 + e > limit) v[e] = -INFINITY;
}

template <int D>
__global__ void __launch_bounds__(THREADS, 2)
    fwd_kernel(const __grid_constant__ CUtensorMap map_qkv, const __grid_constant__ CUtensorMap map_out, float* __restrict__ lse,
               int S, int H, int HKV, int causal, float scale_log2, int qt0, int nqt_w, int* err) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::TILE_BYTES;
  uint8_t* sV = sK + C::STAGES * C::TILE_BYTES;

  __shared__ __align__(8) uint64_t q_full, s_full, p_full, o_full;
  __shared__ __align__(8) uint64_t kv_full[C::STAGES], kv_empty[C::STAGES];
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Query tiles qt0 .. qt0 + nqt_w - 1 (the whole sequence, or one rank's window of it under
  // context parallelism); keys always cover the whole sequence.
  int qt, h, b;
  tile_major_block(nqt_w, H, qt, h, b);
  qt = qt0 + nqt_w - 1 - qt;  // causal: the last query tiles see the most keys; they start first
  const int hk = h / (H / HKV);
  const int q0 = qt * BQ;
  const int nkt = (S + BKV - 1) / BKV;
  const int n_kv = causal ? min(qt + 1, nkt) : nkt;

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
    prefetch_tensormap(&map_qkv);
    prefetch_tensormap(&map_out);
  }
  if (warp == 1) tmem_alloc(&tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(&q_full, C::TILE_BYTES);
#pragma unroll
      for (int c = 0; c < C::CHUNKS; ++c) tma_load_3d(sQ + c * 16384, &map_qkv, &q_full, h * D + c * 64, q0, b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % C::STAGES;
        if (!mbar_wait(&kv_empty[st], ((j / C::STAGES) & 1) ^ 1u, err, 11)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) {
          tma_load_3d(sK + st * C::TILE_BYTES + c * 16384, &map_qkv, &kv_full[st], (H + hk) * D + c * 64, j * BKV, b);
          tma_load_3d(sV + st * C::TILE_BYTES + c * 16384, &map_qkv, &kv_full[st], (H + HKV + hk) * D + c * 64, j * BKV, b);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, 128, false, false);
    constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, false, true);
    bool ok = mbar_wait(&q_full, 0, err, 12);
    for (int j = 0; j < n_kv && ok; ++j) {
      const int st = j % C::STAGES;
      if (!mbar_wait(&kv_full[st], (j / C::STAGES) & 1, err, 13)) break;
      if (D == 128 && j > 0 && !mbar_wait(&o_full, (j - 1) & 1, err, 14)) break;  // P (aliased on S) consumed
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK + st * C::TILE_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k / 4) * 16384 + (k % 4) * 32;
          tc_mma_f16(tmem + C::S_COL, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(ka + off, 16, 1024), idesc_s,
                     k != 0 ? 1u : 0u);
        }
        tc_commit(&s_full);
      }
      __syncwarp();
      if (!mbar_wait(&p_full, j & 1, err, 15)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t va = smem_u32(sV + st * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          tc_mma_f16_ts(tmem + C::O_COL, tmem + C::P_COL + kk * 8, umma_desc_sw128(va + kk * 2048, 16384, 1024), idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&kv_empty[st]);
        tc_commit(&o_full);
      }
      __syncwarp();
    }
  } else {
    // ---------------- softmax / correction / epilogue ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int q = q0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait(&s_full, j & 1, err, 16)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool edge = (j == n_kv - 1);  // the only tile that can hold masked keys
      const int kv0 = j * BKV;
      // Pass 1: row max of the raw scores (the scale is positive, so it is applied once after).
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + lane_off + C::S_COL + c * 32, v);
        if (edge) mask_chunk(v, kv0 + c * 32, q, S, causal);
#pragma unroll
        for (int e = 0; e < 32; ++e) mx = fmaxf(mx, v[e]);
      }
      // Lazy rescaling: the running maximum moves only when the tile's maximum exceeds it by more
      // than 8 (a factor of 256 in the exponentials, harmless in fp32 sums and bf16 probabilities),
      // so the O rows are rarely rescaled after the first tiles.
      const float m_cand = fmaxf(m, mx * scale_log2);
      const float m_new = (m_cand > m + 8.f) ? m_cand : m;
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = m_new == m ? 1.f : fast_exp2(m - m_use);
      // Pass 2: p = 2^(s * scale - m), row sum, P as bf16 pairs into TMEM.
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + lane_off + C::S_COL + c * 32, v);
        if (edge) mask_chunk(v, kv0 + c * 32, q, S, causal);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          // Half of the exponentials on the MUFU unit, half on the FMA pipe (exp2_poly).
          const float p0 = fast_exp2(fmaf(v[e], scale_log2, -m_use)), p1 = exp2_poly(fmaf(v[e + 1], scale_log2, -m_use));
          rs += p0 + p1;
          __nv_bfloat162 pr = __floats2bfloat162_rn(p0, p1);
          pk[e / 2] = *reinterpret_cast<uint32_t*>(&pr);
        }
        tmem_st_32x32b_x16(tmem + lane_off + C::P_COL + c * 16, pk);
      }
      l = l * alpha + rs;
      m = m_new;
      if (j > 0) {
        if (!mbar_wait(&o_full, (j - 1) & 1, err, 17)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float v[32];
            tmem_ld_32x32b_x32(tmem + lane_off + C::O_COL + c * 32, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= alpha;
            tmem_st_32x32b_x32(tmem + lane_off + C::O_COL + c * 32, v);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
    }
    if (ok && mbar_wait(&o_full, (n_kv - 1) & 1, err, 18)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      // O row -> bf16 -> swizzled staging in the Q buffer (every S MMA has completed).
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + lane_off + C::O_COL + c * 32, v);
        uint8_t* row = sQ + (c / 2) * 16384 + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          __align__(16) __nv_bfloat162 pr[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) pr[e] = __floats2bfloat162_rn(v[u * 8 + 2 * e] * inv, v[u * 8 + 2 * e + 1] * inv);
          const int unit = (c % 2) * 4 + u;
          *reinterpret_cast<uint4*>(row + ((unit ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4*>(pr);
        }
      }
      fence_proxy_async_smem();
      named_barrier_sync(1, 128);
      if (threadIdx.x == 64) {
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c) tma_store_3d(&map_out, sQ + c * 16384, h * D + c * 64, q0, b);
        bulk_commit();
        bulk_wait_all();
      }
      if (q < S) lse[((long long)b * H + h) * S + q] = l > 0.f ? (m + __log2f(l)) * LN2 : -INFINITY;
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

// bf16 [batch][rows][width] map with 64-column x 128-row boxes and the 128-byte swizzle.
static CUtensorMap make_map_3d(const void* base, int64_t batch, int64_t rows, int64_t width) {
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)width, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(width * 2), (cuuint64_t)(rows * width * 2)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult res = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  HT_CHECK(res == CUDA_SUCCESS, "cuTensorMapEncodeTiled (attention) failed with code ", (int)res);
  return map;
}

}  // namespace attn_tc

int* attention_error_word(const at::Device& dev) {
  // Intentionally leaked: a static tensor destroyed after the CUDA context would fault at exit.
  static at::Tensor* words = new at::Tensor[64];
  const int idx = dev.index();
  if (!words[idx].defined()) words[idx] = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(dev));
  return words[idx].data_ptr<int>();
}

// Returns false (nothing launched) when the tensor-core path does not apply to these tensors.
// Queries [q_begin, q_begin + q_len) only (q_len < 0: all); q_begin a multiple of 128.
bool attention_forward_tcgen05(at::Tensor qkv, at::Tensor out, at::Tensor lse, int64_t H, int64_t HKV, int64_t D, bool causal,
                               double scale, int64_t q_begin, int64_t q_len) {
  const int64_t B = qkv.size(0), S = qkv.size(1), W = qkv.size(2);
  if (q_len < 0) q_begin = 0, q_len = S;
  HT_CHECK(q_begin % attn_tc::BQ == 0 && q_begin >= 0 && q_len > 0 && q_begin + q_len <= S,
           "attention query window must start at a multiple of 128 inside the sequence");
  const int qt0 = (int)(q_begin / attn_tc::BQ), nqt_w = (int)((q_len + attn_tc::BQ - 1) / attn_tc::BQ);
  if (!(D == 64 || D == 128) || !qkv.is_contiguous() || !out.is_contiguous() || out.size(2) != H * D) return false;
  if ((reinterpret_cast<uintptr_t>(qkv.data_ptr()) & 15) || (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15)) return false;
  bind_context(qkv.device().index());
  const CUtensorMap mq = attn_tc::make_map_3d(qkv.data_ptr(), B, S, W);
  const CUtensorMap mo = attn_tc::make_map_3d(out.data_ptr(), B, S, H * D);
  int* err = attention_error_word(qkv.device());
  const float sl2 = (float)(scale * 1.4426950408889634);
  const dim3 grid((unsigned)(nqt_w * H * B));
  cudaStream_t s = stream();
  if (D == 64) {
    constexpr int smem = attn_tc::Cfg<64>::SMEM;
    static bool once = [] {
      HT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc::fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      return true;
    }();
    (void)once;
    attn_tc::fwd_kernel<64><<<grid, attn_tc::THREADS, smem, s>>>(mq, mo, lse.data_ptr<float>(), (int)S, (int)H, (int)HKV,
                                                                 causal ? 1 : 0, sl2, qt0, nqt_w, err);
  } else {
    constexpr int smem = attn_tc::Cfg<128>::SMEM;
    static bool once = [] {
      HT_CUDA_CHECK(cudaFuncSetAttribute(attn_tc::fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      return true;
    }();
    (void)once;
    attn_tc::fwd_kernel<128><<<grid, attn_tc::THREADS, smem, s>>>(mq, mo, lse.data_ptr<float>(), (int)S, (int)H, (int)HKV,
                                                                  causal ? 1 : 0, sl2, qt0, nqt_w, err);
  }
  HT_CUDA_CHECK(cudaGetLastError());
  return true;
}

at::Tensor attention_error_word_tensor(at::Tensor like) {
  return at::from_blob(attention_error_word(like.device()), {4}, like.options().dtype(at::kInt));
}

}  // namespace ht
