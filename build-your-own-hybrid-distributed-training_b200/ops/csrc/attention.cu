// Causal flash attention on a packed QKV tensor [B, S, (H + 2*Hkv) * D] (D = 64 or 128), with
// grouped-query attention, bf16 in/out and fp32 softmax statistics.
//
// Forward: one CTA per (64-query tile, head, batch); 4 warps x 16 query rows.  K/V tiles of 64
// keys stream through a double-buffered, XOR-swizzled shared-memory ring (cp.async); S = Q K^T
// and O += P V run on m16n8k16 bf16 tensor-core MMAs with fp32 accumulation; the softmax is
// online (running max / running sum, exp2 domain) so the S x S matrix never exists.  The
// per-row log-sum-exp is kept for the backward pass.
//
// Backward (no atomics): `dq` kernel -- per query tile, recompute P, dP = dO V^T,
// dS = P (dP - delta), dQ = scale * dS K; `dkdv` kernel -- per key tile and KV head, loop over
// the query heads of the group and the query tiles at or after the key tile, recompute
// P^T and dP^T and accumulate dV = P^T dO and dK = scale * dS^T Q in registers.
// delta = rowsum(dO * O) comes from a small pre-pass.

#include "common.cuh"

#include <cstdlib>

namespace ht {
namespace attn {

constexpr int BQ = 64;   // query rows per tile
constexpr int BKV = 64;  // key rows per tile
constexpr int THREADS = 128;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int bytes = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Byte offset of element (row, col) in a swizzled tile with D columns (16-byte chunks XOR row%8).
template <int D>
__device__ __forceinline__ uint32_t sw(int row, int col) {
  constexpr int CH = D / 8;
  return (uint32_t)((row * CH + ((col >> 3) ^ (row & 7))) * 16 + (col & 7) * 2);
}

// Load `ROWS` rows starting at sequence row `row0` (rows >= S are zero-filled).
template <int D, int ROWS>
__device__ __forceinline__ void load_tile(uint32_t base, const __nv_bfloat16* g, long long ld, int row0, int S) {
  constexpr int CH = D / 8;
  for (int idx = threadIdx.x; idx < ROWS * CH; idx += THREADS) {
    const int r = idx / CH, c = idx % CH;
    const bool ok = row0 + r < S;
    const __nv_bfloat16* src = g + (long long)(ok ? row0 + r : 0) * ld + c * 8;
    cp_async16(base + (uint32_t)((r * CH + (c ^ (r & 7))) * 16), src, ok);
  }
}

// A fragment (16 rows x 16 cols at (r0, c0)) of a row-major swizzled tile.
template <int D>
__device__ __forceinline__ void load_a(uint32_t* a, uint32_t base, int r0, int c0) {
  const int lane = threadIdx.x & 31;
  ldsm4(a, base + sw<D>(r0 + (lane & 15), c0 + (lane >> 4) * 8));
}
// B fragments for two n8 blocks (rows n0..n0+15 of the tile are the N index, cols c0..c0+15 the K index).
template <int D>
__device__ __forceinline__ void load_b_rows(uint32_t* b, uint32_t base, int n0, int c0) {
  const int lane = threadIdx.x & 31;
  ldsm4(b, base + sw<D>(n0 + (lane & 7) + ((lane >> 4) << 3), c0 + ((lane >> 3) & 1) * 8));
}
// B fragments for two n8 blocks where the tile's rows are the K index (k0..k0+15) and cols n0..n0+15 the N index.
template <int D>
__device__ __forceinline__ void load_b_cols(uint32_t* b, uint32_t base, int k0, int n0) {
  const int lane = threadIdx.x & 31;
  ldsm4_t(b, base + sw<D>(k0 + (lane & 15), n0 + (lane >> 4) * 8));
}

// ------------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(THREADS) fwd_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out,
                                                      float* __restrict__ lse, int S, int H, int HKV, int causal, float scale_log2) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (H / HKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const long long W = (long long)(H + 2 * HKV) * D;
  const __nv_bfloat16* qp = qkv + (long long)b * S * W + (long long)h * D;
  const __nv_bfloat16* kp = qkv + (long long)b * S * W + (long long)(H + kvh) * D;
  const __nv_bfloat16* vp = qkv + (long long)b * S * W + (long long)(H + HKV + kvh) * D;
  constexpr int TILE = BQ * D * 2;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK[2] = {sQ + TILE, sQ + 2 * TILE};
  const uint32_t sV[2] = {sQ + 3 * TILE, sQ + 4 * TILE};
  const int q0 = qt * BQ;
  const int nkv = (S + BKV - 1) / BKV;
  const int ntiles = causal ? min(qt + 1, nkv) : nkv;

  load_tile<D, BQ>(sQ, qp, W, q0, S);
  load_tile<D, BKV>(sK[0], kp, W, 0, S);
  load_tile<D, BKV>(sV[0], vp, W, 0, S);
  cp_commit();
  cp_wait_all();
  __syncthreads();

  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) load_a<D>(qf[kk], sQ, warp * 16, kk * 16);

  float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) {
      load_tile<D, BKV>(sK[buf ^ 1], kp, W, (j + 1) * BKV, S);
      load_tile<D, BKV>(sV[buf ^ 1], vp, W, (j + 1) * BKV, S);
    }
    cp_commit();
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bf[4];
        load_b_rows<D>(bf, sK[buf], np * 16, kk * 16);
        mma16816(s[2 * np], qf[kk], bf[0], bf[1]);
        mma16816(s[2 * np + 1], qf[kk], bf[2], bf[3]);
      }
    }
    // scale, mask, online softmax
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = q0 + warp * 16 + g + r * 8;
      float mx = -INFINITY;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = j * BKV + nb * 8 + t * 2 + e;
          float v = s[nb][2 * r + e] * scale_log2;
          if (key >= S || (causal && key > row)) v = -INFINITY;
          s[nb][2 * r + e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_i[r], mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m_i[r] - m_use);
      float rs = 0.f;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p = exp2f(s[nb][2 * r + e] - m_use);
          s[nb][2 * r + e] = p;
          rs += p;
        }
      }
      l_i[r] = l_i[r] * alpha + rs;
      m_i[r] = m_new;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        acc[i][2 * r] *= alpha;
        acc[i][2 * r + 1] *= alpha;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      uint32_t a[4] = {pack_bf16(s[2 * kk][0], s[2 * kk][1]), pack_bf16(s[2 * kk][2], s[2 * kk][3]),
                       pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bf[4];
        load_b_cols<D>(bf, sV[buf], kk * 16, dp * 16);
        mma16816(acc[2 * dp], a, bf[0], bf[1]);
        mma16816(acc[2 * dp + 1], a, bf[2], bf[3]);
      }
    }
    cp_wait_all();
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_i[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int row = q0 + warp * 16 + g + r * 8;
    if (row < S) {
      __nv_bfloat16* op = out + ((long long)b * S + row) * ((long long)H * D) + (long long)h * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<uint32_t*>(op + i * 8 + t * 2) = pack_bf16(acc[i][2 * r] * inv, acc[i][2 * r + 1] * inv);
      if (t == 0) lse[((long long)b * H + h) * S + row] = l > 0.f ? (m_i[r] + log2f(l)) * LN2 : -INFINITY;
    }
  }
}

// delta[b, h, s] = sum_d dO * O
template <int D>
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ dout, float* __restrict__ delta,
                             int S, int H, long long rows) {
  const long long wid = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= rows) return;
  const long long bs = wid / H;  // b * S + s
  const int h = wid % H;
  const __nv_bfloat16* o = out + bs * H * D + (long long)h * D;
  const __nv_bfloat16* d = dout + bs * H * D + (long long)h * D;
  float acc = 0.f;
  for (int i = lane; i < D; i += 32) acc += bf2f(o[i]) * bf2f(d[i]);
  acc = warp_sum(acc);
  if (lane == 0) {
    const long long b = bs / S, s = bs % S;
    delta[(b * H + h) * S + s] = acc;
  }
}

// delta with 16-byte loads: D / 8 lanes per (token, head) row, 8 products per lane, the row's lanes
// reduced with shuffles inside their aligned group (both tensors contiguous and 16-byte aligned).
template <int D>
__global__ void __launch_bounds__(256) delta_vec_kernel(const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ dout,
                                                        float* __restrict__ delta, int S, int H, long long rows) {
  constexpr int LPR = D / 8;
  static_assert(32 % LPR == 0, "a row's lanes must be an aligned group inside one warp");
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long row = t / LPR;
  const int sub = (int)(t % LPR);
  float acc = 0.f;
  if (row < rows) {
    const long long off = row * D + sub * 8;  // [B*S, H, D] contiguous: row = (b*S + s)*H + h
    const uint4 a = *reinterpret_cast<const uint4*>(out + off);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + off);
    const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 x = __bfloat1622float2(ah[q]), y = __bfloat1622float2(gh[q]);
      acc += x.x * y.x + x.y * y.y;
    }
  }
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (row < rows && sub == 0) {
    const long long bs = row / H, h = row % H;
    const long long b = bs / S, s = bs % S;
    delta[(b * H + h) * S + s] = acc;
  }
}

// dQ for one query tile of one head.
template <int D>
__global__ void __launch_bounds__(THREADS) dq_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ dout,
                                                     const float* __restrict__ lse, const float* __restrict__ delta,
                                                     __nv_bfloat16* __restrict__ dqkv, int S, int H, int HKV, int causal,
                                                     float scale, float scale_log2) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (H / HKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const long long W = (long long)(H + 2 * HKV) * D;
  const long long OW = (long long)H * D;
  const __nv_bfloat16* qp = qkv + (long long)b * S * W + (long long)h * D;
  const __nv_bfloat16* kp = qkv + (long long)b * S * W + (long long)(H + kvh) * D;
  const __nv_bfloat16* vp = qkv + (long long)b * S * W + (long long)(H + HKV + kvh) * D;
  const __nv_bfloat16* dop = dout + (long long)b * S * OW + (long long)h * D;
  constexpr int TILE = BQ * D * 2;
  const uint32_t sQ = smem_u32(smem), sDO = sQ + TILE;
  const uint32_t sK[2] = {sQ + 2 * TILE, sQ + 3 * TILE};
  const uint32_t sV[2] = {sQ + 4 * TILE, sQ + 5 * TILE};
  const int q0 = qt * BQ;
  const int nkv = (S + BKV - 1) / BKV;
  const int ntiles = causal ? min(qt + 1, nkv) : nkv;

  load_tile<D, BQ>(sQ, qp, W, q0, S);
  load_tile<D, BQ>(sDO, dop, OW, q0, S);
  load_tile<D, BKV>(sK[0], kp, W, 0, S);
  load_tile<D, BKV>(sV[0], vp, W, 0, S);
  cp_commit();
  cp_wait_all();
  __syncthreads();

  uint32_t qf[D / 16][4], df[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    load_a<D>(qf[kk], sQ, warp * 16, kk * 16);
    load_a<D>(df[kk], sDO, warp * 16, kk * 16);
  }
  float lse2[2], dl[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = q0 + warp * 16 + g + r * 8;
    const long long idx = ((long long)b * H + h) * S + min(row, S - 1);
    lse2[r] = lse[idx] * LOG2E;
    dl[r] = delta[idx];
  }
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) {
      load_tile<D, BKV>(sK[buf ^ 1], kp, W, (j + 1) * BKV, S);
      load_tile<D, BKV>(sV[buf ^ 1], vp, W, (j + 1) * BKV, S);
    }
    cp_commit();
    float s[8][4], dp[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nb][e] = dp[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bf[4];
        load_b_rows<D>(bf, sK[buf], np * 16, kk * 16);
        mma16816(s[2 * np], qf[kk], bf[0], bf[1]);
        mma16816(s[2 * np + 1], qf[kk], bf[2], bf[3]);
        load_b_rows<D>(bf, sV[buf], np * 16, kk * 16);
        mma16816(dp[2 * np], df[kk], bf[0], bf[1]);
        mma16816(dp[2 * np + 1], df[kk], bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const int row = q0 + warp * 16 + g + r * 8;
        const int key = j * BKV + nb * 8 + t * 2 + (e & 1);
        const bool masked = key >= S || (causal && key > row);
        const float p = masked ? 0.f : exp2f(s[nb][e] * scale_log2 - lse2[r]);
        s[nb][e] = p * (dp[nb][e] - dl[r]);  // dS
      }
    }
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      uint32_t a[4] = {pack_bf16(s[2 * kk][0], s[2 * kk][1]), pack_bf16(s[2 * kk][2], s[2 * kk][3]),
                       pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
      for (int dpair = 0; dpair < D / 16; ++dpair) {
        uint32_t bf[4];
        load_b_cols<D>(bf, sK[buf], kk * 16, dpair * 16);
        mma16816(dq[2 * dpair], a, bf[0], bf[1]);
        mma16816(dq[2 * dpair + 1], a, bf[2], bf[3]);
      }
    }
    cp_wait_all();
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = q0 + warp * 16 + g + r * 8;
    if (row < S) {
      __nv_bfloat16* o = dqkv + ((long long)b * S + row) * W + (long long)h * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<uint32_t*>(o + i * 8 + t * 2) = pack_bf16(dq[i][2 * r] * scale, dq[i][2 * r + 1] * scale);
    }
  }
}

// dK, dV for one key tile of one KV head (summed over the query heads that share it).
template <int D>
__global__ void __launch_bounds__(THREADS) dkdv_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ dout,
                                                       const float* __restrict__ lse, const float* __restrict__ delta,
                                                       __nv_bfloat16* __restrict__ dqkv, int S, int H, int HKV, int causal,
                                                       float scale, float scale_log2) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int kt = blockIdx.x;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int group = H / HKV;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const long long W = (long long)(H + 2 * HKV) * D;
  const long long OW = (long long)H * D;
  const __nv_bfloat16* kp = qkv + (long long)b * S * W + (long long)(H + kvh) * D;
  const __nv_bfloat16* vp = qkv + (long long)b * S * W + (long long)(H + HKV + kvh) * D;
  constexpr int TILE = BQ * D * 2;
  const uint32_t sK = smem_u32(smem), sV = sK + TILE;
  const uint32_t sQ[2] = {sK + 2 * TILE, sK + 3 * TILE};
  const uint32_t sDO[2] = {sK + 4 * TILE, sK + 5 * TILE};
  float* sL = reinterpret_cast<float*>(smem + 6 * TILE);  // [2][BQ] lse * log2e
  float* sD = sL + 2 * BQ;                                // [2][BQ] delta
  const int k0 = kt * BKV;
  const int nq = (S + BQ - 1) / BQ;
  const int first_q = causal ? kt : 0;
  const int per_head = nq - first_q;
  const int total = per_head * group;

  load_tile<D, BKV>(sK, kp, W, k0, S);
  load_tile<D, BKV>(sV, vp, W, k0, S);
  auto stage = [&](int it, int buf) {
    const int hq = kvh * group + it / per_head;
    const int qt = first_q + it % per_head;
    const __nv_bfloat16* qp = qkv + (long long)b * S * W + (long long)hq * D;
    const __nv_bfloat16* dop = dout + (long long)b * S * OW + (long long)hq * D;
    load_tile<D, BQ>(sQ[buf], qp, W, qt * BQ, S);
    load_tile<D, BQ>(sDO[buf], dop, OW, qt * BQ, S);
    if (threadIdx.x < BQ) {
      const int row = min(qt * BQ + (int)threadIdx.x, S - 1);
      const long long idx = ((long long)b * H + hq) * S + row;
      sL[buf * BQ + threadIdx.x] = lse[idx] * LOG2E;
      sD[buf * BQ + threadIdx.x] = delta[idx];
    }
  };
  if (total > 0) stage(0, 0);
  cp_commit();
  cp_wait_all();
  __syncthreads();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    if (it + 1 < total) stage(it + 1, buf ^ 1);
    cp_commit();
    const int qt = first_q + it % per_head;
    const int q0 = qt * BQ;
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[nb][e] = dpt[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t ka[4], va[4];
      load_a<D>(ka, sK, warp * 16, kk * 16);
      load_a<D>(va, sV, warp * 16, kk * 16);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t bf[4];
        load_b_rows<D>(bf, sQ[buf], np * 16, kk * 16);
        mma16816(st[2 * np], ka, bf[0], bf[1]);
        mma16816(st[2 * np + 1], ka, bf[2], bf[3]);
        load_b_rows<D>(bf, sDO[buf], np * 16, kk * 16);
        mma16816(dpt[2 * np], va, bf[0], bf[1]);
        mma16816(dpt[2 * np + 1], va, bf[2], bf[3]);
      }
    }
    // P^T and dS^T (rows = keys, cols = queries)
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + warp * 16 + g + (e >> 1) * 8;
        const int qi = nb * 8 + t * 2 + (e & 1);
        const int query = q0 + qi;
        const bool masked = query >= S || key >= S || (causal && key > query);
        const float p = masked ? 0.f : exp2f(st[nb][e] * scale_log2 - sL[buf * BQ + qi]);
        st[nb][e] = p;
        dpt[nb][e] = p * (dpt[nb][e] - sD[buf * BQ + qi]);
      }
    }
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      uint32_t pa[4] = {pack_bf16(st[2 * kk][0], st[2 * kk][1]), pack_bf16(st[2 * kk][2], st[2 * kk][3]),
                        pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]), pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3])};
      uint32_t sa[4] = {pack_bf16(dpt[2 * kk][0], dpt[2 * kk][1]), pack_bf16(dpt[2 * kk][2], dpt[2 * kk][3]),
                        pack_bf16(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]), pack_bf16(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3])};
#pragma unroll
      for (int dpair = 0; dpair < D / 16; ++dpair) {
        uint32_t bf[4];
        load_b_cols<D>(bf, sDO[buf], kk * 16, dpair * 16);
        mma16816(dv[2 * dpair], pa, bf[0], bf[1]);
        mma16816(dv[2 * dpair + 1], pa, bf[2], bf[3]);
        load_b_cols<D>(bf, sQ[buf], kk * 16, dpair * 16);
        mma16816(dk[2 * dpair], sa, bf[0], bf[1]);
        mma16816(dk[2 * dpair + 1], sa, bf[2], bf[3]);
      }
    }
    cp_wait_all();
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = k0 + warp * 16 + g + r * 8;
    if (key < S) {
      __nv_bfloat16* ko = dqkv + ((long long)b * S + key) * W + (long long)(H + kvh) * D;
      __nv_bfloat16* vo = dqkv + ((long long)b * S + key) * W + (long long)(H + HKV + kvh) * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        *reinterpret_cast<uint32_t*>(ko + i * 8 + t * 2) = pack_bf16(dk[i][2 * r] * scale, dk[i][2 * r + 1] * scale);
        *reinterpret_cast<uint32_t*>(vo + i * 8 + t * 2) = pack_bf16(dv[i][2 * r], dv[i][2 * r + 1]);
      }
    }
  }
}

template <typename K>
static void set_smem(K kernel, int bytes) {
  HT_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

}  // namespace attn

static void attn_check(const at::Tensor& qkv, int64_t H, int64_t HKV, int64_t D) {
  HT_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() && qkv.dim() == 3,
           "attention expects a contiguous bf16 [B, S, (H + 2*Hkv) * D] tensor");
  HT_CHECK(D == 64 || D == 128, "attention supports head_dim 64 or 128, got ", D);
  HT_CHECK(HKV > 0 && H % HKV == 0, "num_heads must be a multiple of num_kv_heads");
  HT_CHECK(qkv.size(2) == (H + 2 * HKV) * D, "packed width mismatch");
}

bool attention_forward_tcgen05(at::Tensor qkv, at::Tensor out, at::Tensor lse, int64_t H, int64_t HKV, int64_t D, bool causal,
                               double scale, int64_t q_begin, int64_t q_len);

// `q_begin` / `q_len` (q_len < 0: every query) restrict the queries to one window of the sequence
// (context parallelism: a rank's own positions against the gathered keys); windows run on the
// tcgen05 kernels only.
void attention_forward(at::Tensor qkv, at::Tensor out, at::Tensor lse, int64_t H, int64_t HKV, int64_t D, bool causal, double scale,
                       int64_t q_begin, int64_t q_len) {
  attn_check(qkv, H, HKV, D);
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int B = qkv.size(0), S = qkv.size(1);
  if (B == 0 || S == 0) return;
  const bool window = q_len >= 0 && !(q_begin == 0 && q_len == S);
  // The tcgen05 kernel (attention_tcgen05.cu) covers contiguous, 16-byte aligned tensors; the
  // mma.sync kernel below remains for any other layout.
  if ((window || std::getenv("HT_ATTN_MMA_SYNC") == nullptr) &&
      attention_forward_tcgen05(qkv, out, lse, H, HKV, D, causal, scale, q_begin, q_len))
    return;
  HT_CHECK(!window, "a query window needs contiguous, 16-byte aligned tensors and D of 64 or 128");
  dim3 grid((S + attn::BQ - 1) / attn::BQ, H, B);
  const float sl2 = (float)scale * attn::LOG2E;
  const auto* q = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (D == 64) {
    constexpr int smem = 5 * attn::BQ * 64 * 2;
    static bool once = (attn::set_smem(attn::fwd_kernel<64>, smem), true);
    (void)once;
    attn::fwd_kernel<64><<<grid, attn::THREADS, smem, stream()>>>(q, o, lse.data_ptr<float>(), S, H, HKV, causal, sl2);
  } else {
    constexpr int smem = 5 * attn::BQ * 128 * 2;
    static bool once = (attn::set_smem(attn::fwd_kernel<128>, smem), true);
    (void)once;
    attn::fwd_kernel<128><<<grid, attn::THREADS, smem, stream()>>>(q, o, lse.data_ptr<float>(), S, H, HKV, causal, sl2);
  }
  HT_CUDA_CHECK(cudaGetLastError());
}

bool attention_backward_tcgen05(at::Tensor qkv, at::Tensor dout, at::Tensor lse, at::Tensor delta, at::Tensor dqkv, int64_t H,
                                int64_t HKV, int64_t D, bool causal, double scale, int64_t q_begin, int64_t q_len);

// With a query window the rows of `out` and `dout` outside it must be zero (their delta is then
// zero and they contribute nothing to dK / dV).
void attention_backward(at::Tensor qkv, at::Tensor out, at::Tensor dout, at::Tensor lse, at::Tensor delta, at::Tensor dqkv,
                        int64_t H, int64_t HKV, int64_t D, bool causal, double scale, int64_t q_begin, int64_t q_len) {
  attn_check(qkv, H, HKV, D);
  const c10::cuda::CUDAGuard guard(qkv.device());
  HT_CHECK(dout.is_contiguous() && dqkv.is_contiguous() && dqkv.sizes() == qkv.sizes(), "attention backward buffers");
  const int B = qkv.size(0), S = qkv.size(1);
  if (B == 0 || S == 0) return;
  const auto* q = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  const auto* o = reinterpret_cast<const __nv_bfloat16*>(out.data_ptr());
  const auto* d = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  auto* dq = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  cudaStream_t s = stream();
  const long long rows = (long long)B * S * H;
  const int dthreads = 256;
  const int dgrid = (int)((rows * 32 + dthreads - 1) / dthreads);
  const float sl2 = (float)scale * attn::LOG2E;
  dim3 gq((S + attn::BQ - 1) / attn::BQ, H, B), gk((S + attn::BKV - 1) / attn::BKV, HKV, B);
  const bool vec = out.is_contiguous() && (reinterpret_cast<uintptr_t>(o) & 15) == 0 && (reinterpret_cast<uintptr_t>(d) & 15) == 0;
  if (vec) {
    const long long threads_total = rows * (D / 8);
    const int vgrid = (int)((threads_total + dthreads - 1) / dthreads);
    if (D == 64) attn::delta_vec_kernel<64><<<vgrid, dthreads, 0, s>>>(o, d, delta.data_ptr<float>(), S, H, rows);
    else attn::delta_vec_kernel<128><<<vgrid, dthreads, 0, s>>>(o, d, delta.data_ptr<float>(), S, H, rows);
  } else if (D == 64) {
    attn::delta_kernel<64><<<dgrid, dthreads, 0, s>>>(o, d, delta.data_ptr<float>(), S, H, rows);
  } else {
    attn::delta_kernel<128><<<dgrid, dthreads, 0, s>>>(o, d, delta.data_ptr<float>(), S, H, rows);
  }
  // The tcgen05 kernels (attention_bwd_tcgen05.cu) cover contiguous, 16-byte aligned tensors.
  const bool window = q_len >= 0 && !(q_begin == 0 && q_len == S);
  if ((window || std::getenv("HT_ATTN_MMA_SYNC") == nullptr) &&
      attention_backward_tcgen05(qkv, dout, lse, delta, dqkv, H, HKV, D, causal, scale, q_begin, q_len)) {
    HT_CUDA_CHECK(cudaGetLastError());
    return;
  }
  HT_CHECK(!window, "a query window needs contiguous, 16-byte aligned tensors and D of 64 or 128");
  if (D == 64) {
    constexpr int smem_q = 6 * attn::BQ * 64 * 2;
    constexpr int smem_k = 6 * attn::BQ * 64 * 2 + 4 * attn::BQ * 4;
    static bool once = (attn::set_smem(attn::dq_kernel<64>, smem_q), attn::set_smem(attn::dkdv_kernel<64>, smem_k), true);
    (void)once;
    attn::dq_kernel<64><<<gq, attn::THREADS, smem_q, s>>>(q, d, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, S, H, HKV,
                                                          causal, (float)scale, sl2);
    attn::dkdv_kernel<64><<<gk, attn::THREADS, smem_k, s>>>(q, d, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, S, H, HKV,
                                                            causal, (float)scale, sl2);
  } else {
    constexpr int smem_q = 6 * attn::BQ * 128 * 2;
    constexpr int smem_k = 6 * attn::BQ * 128 * 2 + 4 * attn::BQ * 4;
    static bool once = (attn::set_smem(attn::dq_kernel<128>, smem_q), attn::set_smem(attn::dkdv_kernel<128>, smem_k), true);
    (void)once;
    attn::dq_kernel<128><<<gq, attn::THREADS, smem_q, s>>>(q, d, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, S, H, HKV,
                                                           causal, (float)scale, sl2);
    attn::dkdv_kernel<128><<<gk, attn::THREADS, smem_k, s>>>(q, d, lse.data_ptr<float>(), delta.data_ptr<float>(), dq, S, H, HKV,
                                                             causal, (float)scale, sl2);
  }
  HT_CUDA_CHECK(cudaGetLastError());
}

}  // namespace ht
