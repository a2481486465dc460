// Fused flash-style attention for the ChessDecoder backbone, head_dim 64.
//
// Replaces torchtune MultiHeadAttention's scaled_dot_product_attention call as
// the reference model drives it (chessdecoder/models/model.py:158-171):
//   pass 1: is_causal=True                                 -> allowed(i,j) = j <= i
//   pass 2: bool mask tril | block_id[i] == block_id[j]    -> allowed(i,j) = j <= i || bid[i] == bid[j]
// The [B,S,S] mask is never materialised: each CTA reads the block ids of its
// rows/columns and the per-tile bounds computed once per step by
// cdk_attn_prefix_meta, which also lets it skip key tiles that no row of the
// query tile may see.
//
// Layout: qkv bf16 [nseq*S, 3E] (token rows, [q | k | v], head h at columns
// h*64), out bf16 [nseq*S, E], lse f32 [nseq, H, S] (base-2 log-sum-exp of the
// scaled scores).  Tiles are 64 tokens; each of the 4 warps owns 16 rows and
// computes with mma.sync m16n8k16 (bf16 in, fp32 accumulate).
#include "../../include/cdk.h"
#include "cdk_common.cuh"

#include <cstdlib>

namespace cdk {

constexpr int kHd = 64;
constexpr int kTile = 64;
constexpr float kLog2e = 1.4426950408889634f;

// byte offset of element (r, c) in a 64x64 bf16 tile with 16-byte chunk XOR swizzle
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + ((c & 7) << 1));
}

// Async copy of a 64-row x 64-col bf16 tile (rows [row0, row0+64) of a matrix
// with pitch ld, starting at column col0); rows >= nrows are zero-filled.
__device__ __forceinline__ void load_tile_async(uint32_t s_tile, const __nv_bfloat16* g, long long ld, int row0,
                                                int nrows, int col0) {
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + 128 * j;
    const int r = i >> 3, ch = i & 7;
    const bool ok = row0 + r < nrows;
    const __nv_bfloat16* src = g + (long long)(ok ? row0 + r : 0) * ld + col0 + ch * 8;
    cp_async_16_zfill(s_tile + swz(r, ch * 8), src, ok);
  }
}

// Write a 64x64 bf16 tile from shared memory to global rows [row0, row0+64) (rows < nrows).
__device__ __forceinline__ void store_tile(const uint8_t* s_tile, __nv_bfloat16* g, long long ld, int row0, int nrows,
                                           int col0) {
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + 128 * j;
    const int r = i >> 3, ch = i & 7;
    if (row0 + r < nrows)
      *reinterpret_cast<uint4*>(g + (long long)(row0 + r) * ld + col0 + ch * 8) =
          *reinterpret_cast<const uint4*>(s_tile + swz(r, ch * 8));
  }
}

// A-operand fragments of a warp's 16 rows (r0..r0+15) x 64 columns.
__device__ __forceinline__ void load_a_frags(uint32_t s_tile, int r0, uint32_t (&a)[4][4]) {
  const int lane = threadIdx.x & 31;
  #pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int r = r0 + (lane & 15);
    const int c = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(s_tile + swz(r, c), a[kk][0], a[kk][1], a[kk][2], a[kk][3]);
  }
}

// acc[16 rows x 64 cols] += A(16 x 64, fragments) * T^T where T is a 64x64 tile
// stored [n][k] (n = output column, k = reduction index): "non-transposed" B.
__device__ __forceinline__ void mma_a_bt(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t s_tile) {
  const int lane = threadIdx.x & 31;
  const int m = lane >> 3;
  #pragma unroll
  for (int np = 0; np < 4; ++np) {
    #pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int n = np * 16 + (m >> 1) * 8 + (lane & 7);
      const int k = kk * 16 + (m & 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(s_tile + swz(n, k), b0, b1, b2, b3);
      mma_bf16_16816(acc[2 * np], a[kk], b0, b1);
      mma_bf16_16816(acc[2 * np + 1], a[kk], b2, b3);
    }
  }
}

// acc[16 x 64] += A(16 x 64) * T where T is a 64x64 tile stored [k][n]: transposed B.
__device__ __forceinline__ void mma_a_b(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t s_tile) {
  const int lane = threadIdx.x & 31;
  const int m = lane >> 3;
  #pragma unroll
  for (int dp = 0; dp < 4; ++dp) {
    #pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int k = kk * 16 + (m & 1) * 8 + (lane & 7);
      const int n = dp * 16 + (m >> 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(s_tile + swz(k, n), b0, b1, b2, b3);
      mma_bf16_16816(acc[2 * dp], a[kk], b0, b1);
      mma_bf16_16816(acc[2 * dp + 1], a[kk], b2, b3);
    }
  }
}

// C fragments (16 x 64 fp32) -> bf16 A fragments for the next product.
__device__ __forceinline__ void c_to_a(const float (&c)[8][4], uint32_t (&a)[4][4]) {
  #pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    a[kk][0] = pack_bf16(c[2 * kk][0], c[2 * kk][1]);
    a[kk][1] = pack_bf16(c[2 * kk][2], c[2 * kk][3]);
    a[kk][2] = pack_bf16(c[2 * kk + 1][0], c[2 * kk + 1][1]);
    a[kk][3] = pack_bf16(c[2 * kk + 1][2], c[2 * kk + 1][3]);
  }
}

__device__ __forceinline__ void zero_acc(float (&c)[8][4]) {
  #pragma unroll
  for (int i = 0; i < 8; ++i) c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0.f;
}

// Stage C fragments (rows r0.., 16 x 64) as bf16 into a swizzled tile.
__device__ __forceinline__ void c_to_smem(const float (&c)[8][4], uint8_t* s_tile, int r0) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  #pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int col = n * 8 + 2 * t;
    *reinterpret_cast<uint32_t*>(s_tile + swz(r0 + g, col)) = pack_bf16(c[n][0], c[n][1]);
    *reinterpret_cast<uint32_t*>(s_tile + swz(r0 + g + 8, col)) = pack_bf16(c[n][2], c[n][3]);
  }
}

// Inverse interleaved RoPE on C fragments: rows r0+g / r0+g+8 at sequence positions pos0+...
__device__ __forceinline__ void unrope_c(float (&c)[8][4], const float* rope, int pos_g, int pos_g8) {
  if (rope == nullptr) return;
  const int t = threadIdx.x & 3;
  #pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int pair = n * 4 + t;
    const float2 a = *reinterpret_cast<const float2*>(rope + ((long long)pos_g * 32 + pair) * 2);
    const float2 b = *reinterpret_cast<const float2*>(rope + ((long long)pos_g8 * 32 + pair) * 2);
    float x0 = c[n][0], x1 = c[n][1];
    c[n][0] = x0 * a.x + x1 * a.y;
    c[n][1] = x1 * a.x - x0 * a.y;
    x0 = c[n][2];
    x1 = c[n][3];
    c[n][2] = x0 * b.x + x1 * b.y;
    c[n][3] = x1 * b.x - x0 * b.y;
  }
}

struct AttnArgs {
  const __nv_bfloat16* qkv;
  __nv_bfloat16* out;
  float* lse;
  const __nv_bfloat16* dout;
  float* dsum;
  __nv_bfloat16* dqkv;
  const int32_t* bid;   // [nseq - n_causal, S]
  const int32_t* meta;  // per prefix sequence: kv_hi[nt], q_lo[nt]
  const float* rope;
  int S, H, n_causal, nt, nseq;
};

// Per-sequence prefix-mask metadata, laid out as
//   [nseq][2*nt]  per tile: kv_hi[qt] (exclusive key bound of query tile qt),
//                           q_lo[kt] (lowest query row that may see key tile kt)
//   [nseq][S]     first[i] = lowest  j with bid[j] == bid[i]
//   [nseq][S]     last[i]  = highest j with bid[j] == bid[i]
__global__ void attn_meta_kernel(const int32_t* __restrict__ bid, int S, int nt, int nseq,
                                 int32_t* __restrict__ meta) {
  extern __shared__ int32_t sm_meta[];
  int32_t* sb = sm_meta;           // S block ids
  int32_t* skv = sm_meta + S;      // nt
  int32_t* sql = skv + nt;         // nt
  const int seq = blockIdx.x;
  const int32_t* b = bid + (long long)seq * S;
  int32_t* first_out = meta + (long long)nseq * 2 * nt + (long long)seq * S;
  int32_t* last_out = meta + (long long)nseq * 2 * nt + (long long)nseq * S + (long long)seq * S;
  for (int i = threadIdx.x; i < S; i += blockDim.x) sb[i] = b[i];
  for (int i = threadIdx.x; i < nt; i += blockDim.x) {
    skv[i] = 0;
    sql[i] = S;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    const int my = sb[i];
    int first = i, last = i;
    for (int j = 0; j < S; ++j) {
      if (sb[j] == my) {
        first = min(first, j);
        last = max(last, j);
      }
    }
    first_out[i] = first;
    last_out[i] = last;
    atomicMax(&skv[i / kTile], last + 1);
    atomicMin(&sql[i / kTile], first);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nt; i += blockDim.x) {
    meta[(long long)seq * 2 * nt + i] = skv[i];
    meta[(long long)seq * 2 * nt + nt + i] = sql[i];
  }
}

// ---------------------------------------------------------------------------
// Forward.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) attn_fwd_kernel(const AttnArgs a) {
  __shared__ __align__(1024) uint8_t sQ[kTile * 128];
  __shared__ __align__(1024) uint8_t sK[2][kTile * 128];
  __shared__ __align__(1024) uint8_t sV[2][kTile * 128];
  __shared__ int32_t sbq[kTile];
  __shared__ int32_t sbk[2][kTile];

  const int qt = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int S = a.S, E = a.H * kHd;
  const long long ld = 3ll * E;
  const bool prefix = seq >= a.n_causal;
  const int q0 = qt * kTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const __nv_bfloat16* base = a.qkv + (long long)seq * S * ld;
  const int32_t* bid = prefix ? a.bid + (long long)(seq - a.n_causal) * S : nullptr;

  int kv_end = min(S, q0 + kTile);
  if (prefix) kv_end = max(kv_end, a.meta[(long long)(seq - a.n_causal) * 2 * a.nt + qt]);
  const int n_kv = (kv_end + kTile - 1) / kTile;

  load_tile_async(smem_u32(sQ), base, ld, q0, S, h * kHd);
  load_tile_async(smem_u32(sK[0]), base, ld, 0, S, E + h * kHd);
  load_tile_async(smem_u32(sV[0]), base, ld, 0, S, 2 * E + h * kHd);
  cp_async_commit();
  if (prefix) {
    for (int i = threadIdx.x; i < kTile; i += 128) {
      sbq[i] = q0 + i < S ? bid[q0 + i] : -1;
      sbk[0][i] = i < S ? bid[i] : -2;
    }
  }

  const float sl2 = 0.125f * kLog2e;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float o[8][4];
  zero_acc(o);
  uint32_t qa[4][4];
  const int r_lo = q0 + warp * 16 + g;  // row for c0/c1; c2/c3 at r_lo + 8

  for (int kt = 0; kt < n_kv; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kv) {
      const int nb = buf ^ 1;
      load_tile_async(smem_u32(sK[nb]), base, ld, (kt + 1) * kTile, S, E + h * kHd);
      load_tile_async(smem_u32(sV[nb]), base, ld, (kt + 1) * kTile, S, 2 * E + h * kHd);
      cp_async_commit();
      if (prefix)
        for (int i = threadIdx.x; i < kTile; i += 128) {
          const int j = (kt + 1) * kTile + i;
          sbk[nb][i] = j < S ? bid[j] : -2;
        }
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kt == 0) load_a_frags(smem_u32(sQ), warp * 16, qa);

    float s[8][4];
    zero_acc(s);
    mma_a_bt(s, qa, smem_u32(sK[buf]));

    const int k0 = kt * kTile;
    const bool full_tile = (k0 + kTile <= q0) && (k0 + kTile <= S);
    #pragma unroll
    for (int n = 0; n < 8; ++n) {
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[n][e] * sl2;
        if (!full_tile) {
          const int i = r_lo + (e >> 1) * 8;
          const int jl = n * 8 + 2 * t + (e & 1);
          const int j = k0 + jl;
          bool ok = j < S && j <= i;
          if (!ok && prefix && j < S && i < S) ok = sbq[i - q0] == sbk[buf][jl];
          if (!ok) v = -INFINITY;
        }
        s[n][e] = v;
      }
    }
    // online softmax, rows g (e=0,1) and g+8 (e=2,3)
    #pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
      #pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_r[hr], mx);
      const float corr = m_new == -INFINITY ? 1.f : exp2f(m_r[hr] - m_new);
      float sum = 0.f;
      #pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float p0 = m_new == -INFINITY ? 0.f : exp2f(s[n][2 * hr] - m_new);
        const float p1 = m_new == -INFINITY ? 0.f : exp2f(s[n][2 * hr + 1] - m_new);
        s[n][2 * hr] = p0;
        s[n][2 * hr + 1] = p1;
        sum += p0 + p1;
      }
      l_r[hr] = l_r[hr] * corr + sum;
      m_r[hr] = m_new;
      #pragma unroll
      for (int n = 0; n < 8; ++n) {
        o[n][2 * hr] *= corr;
        o[n][2 * hr + 1] *= corr;
      }
    }
    uint32_t pa[4][4];
    c_to_a(s, pa);
    mma_a_b(o, pa, smem_u32(sV[buf]));
    __syncthreads();
  }

  // finalize: full row sums across the quad
  #pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = l_r[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    #pragma unroll
    for (int n = 0; n < 8; ++n) {
      o[n][2 * hr] *= inv;
      o[n][2 * hr + 1] *= inv;
    }
    const int i = r_lo + hr * 8;
    if (t == 0 && i < S) a.lse[((long long)seq * a.H + h) * S + i] = m_r[hr] + log2f(l);
  }
  c_to_smem(o, sQ, warp * 16);
  __syncthreads();
  store_tile(sQ, a.out + (long long)seq * S * E, E, q0, S, h * kHd);
}

struct DqSmem {
  uint8_t Q[kTile * 128];
  uint8_t dO[kTile * 128];
  uint8_t K[2][kTile * 128];
  uint8_t V[2][kTile * 128];
  int32_t bq[kTile];
  int32_t bk[2][kTile];
  float D[kTile];
  float L[kTile];
};

struct DkvSmem {
  uint8_t K[kTile * 128];
  uint8_t V[kTile * 128];
  uint8_t Q[2][kTile * 128];
  uint8_t dO[2][kTile * 128];
  int32_t bk[kTile];
  int32_t bq[2][kTile];
  float D[2][kTile];
  float L[2][kTile];
};

// ---------------------------------------------------------------------------
// Backward, part 1: dQ (and D = rowsum(dO * O)), one CTA per query tile.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t dsm_dq[];
  DqSmem& sm = *reinterpret_cast<DqSmem*>(dsm_dq);
  auto& sQ = sm.Q;
  auto& sdO = sm.dO;
  auto& sK = sm.K;
  auto& sV = sm.V;
  auto& sbq = sm.bq;
  auto& sbk = sm.bk;
  auto& sD = sm.D;
  auto& sL = sm.L;

  const int qt = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int S = a.S, E = a.H * kHd;
  const long long ld = 3ll * E;
  const bool prefix = seq >= a.n_causal;
  const int q0 = qt * kTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const __nv_bfloat16* base = a.qkv + (long long)seq * S * ld;
  const __nv_bfloat16* obase = a.out + (long long)seq * S * E;
  const __nv_bfloat16* dobase = a.dout + (long long)seq * S * E;
  const int32_t* bid = prefix ? a.bid + (long long)(seq - a.n_causal) * S : nullptr;
  const long long lrow = ((long long)seq * a.H + h) * S;

  int kv_end = min(S, q0 + kTile);
  if (prefix) kv_end = max(kv_end, a.meta[(long long)(seq - a.n_causal) * 2 * a.nt + qt]);
  const int n_kv = (kv_end + kTile - 1) / kTile;

  load_tile_async(smem_u32(sQ), base, ld, q0, S, h * kHd);
  load_tile_async(smem_u32(sdO), dobase, E, q0, S, h * kHd);
  load_tile_async(smem_u32(sK[0]), base, ld, 0, S, E + h * kHd);
  load_tile_async(smem_u32(sV[0]), base, ld, 0, S, 2 * E + h * kHd);
  cp_async_commit();

  // D_i = sum_d dO[i,d] * O[i,d]; two threads per row, 32 dims each.
  {
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    float acc = 0.f;
    if (q0 + r < S) {
      const uint4* po = reinterpret_cast<const uint4*>(obase + (long long)(q0 + r) * E + h * kHd + half * 32);
      const uint4* pd = reinterpret_cast<const uint4*>(dobase + (long long)(q0 + r) * E + h * kHd + half * 32);
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 wo = po[q], wd = pd[q];
        const __nv_bfloat162* ho = reinterpret_cast<const __nv_bfloat162*>(&wo);
        const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&wd);
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 fo = __bfloat1622float2(ho[j]), fd = __bfloat1622float2(hd[j]);
          acc += fo.x * fd.x + fo.y * fd.y;
        }
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (half == 0) {
      sD[r] = acc;
      sL[r] = q0 + r < S ? a.lse[lrow + q0 + r] : 0.f;
      if (q0 + r < S) a.dsum[lrow + q0 + r] = acc;
    }
  }
  if (prefix) {
    for (int i = threadIdx.x; i < kTile; i += 128) {
      sbq[i] = q0 + i < S ? bid[q0 + i] : -1;
      sbk[0][i] = i < S ? bid[i] : -2;
    }
  }

  const float sl2 = 0.125f * kLog2e;
  float dq[8][4];
  zero_acc(dq);
  uint32_t qa[4][4], doa[4][4];
  const int rl = warp * 16 + g;  // local row of c0/c1
  const int r_lo = q0 + rl;

  for (int kt = 0; kt < n_kv; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_kv) {
      const int nb = buf ^ 1;
      load_tile_async(smem_u32(sK[nb]), base, ld, (kt + 1) * kTile, S, E + h * kHd);
      load_tile_async(smem_u32(sV[nb]), base, ld, (kt + 1) * kTile, S, 2 * E + h * kHd);
      cp_async_commit();
      if (prefix)
        for (int i = threadIdx.x; i < kTile; i += 128) {
          const int j = (kt + 1) * kTile + i;
          sbk[nb][i] = j < S ? bid[j] : -2;
        }
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kt == 0) {
      load_a_frags(smem_u32(sQ), warp * 16, qa);
      load_a_frags(smem_u32(sdO), warp * 16, doa);
    }
    float s[8][4], dp[8][4];
    zero_acc(s);
    zero_acc(dp);
    mma_a_bt(s, qa, smem_u32(sK[buf]));
    mma_a_bt(dp, doa, smem_u32(sV[buf]));

    const int k0 = kt * kTile;
    const bool full_tile = (k0 + kTile <= q0) && (k0 + kTile <= S);
    #pragma unroll
    for (int n = 0; n < 8; ++n) {
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int il = rl + (e >> 1) * 8;
        const int i = q0 + il;
        const int jl = n * 8 + 2 * t + (e & 1);
        const int j = k0 + jl;
        bool ok = true;
        if (!full_tile) {
          ok = j < S && i < S && j <= i;
          if (!ok && prefix && j < S && i < S) ok = sbq[il] == sbk[buf][jl];
        }
        const float p = ok ? exp2f(s[n][e] * sl2 - sL[il]) : 0.f;
        s[n][e] = p * (dp[n][e] - sD[il]);  // dS
      }
    }
    uint32_t dsa[4][4];
    c_to_a(s, dsa);
    mma_a_b(dq, dsa, smem_u32(sK[buf]));
    __syncthreads();
  }

  #pragma unroll
  for (int n = 0; n < 8; ++n)
    #pragma unroll
    for (int e = 0; e < 4; ++e) dq[n][e] *= 0.125f;
  unrope_c(dq, a.rope, min(r_lo, S - 1), min(r_lo + 8, S - 1));
  c_to_smem(dq, sQ, warp * 16);
  __syncthreads();
  store_tile(sQ, a.dqkv + (long long)seq * S * ld, ld, q0, S, h * kHd);
}

// ---------------------------------------------------------------------------
// Backward, part 2: dK and dV, one CTA per key tile.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) attn_bwd_dkv_kernel(const AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t dsm_kv[];
  DkvSmem& sm = *reinterpret_cast<DkvSmem*>(dsm_kv);
  auto& sK = sm.K;
  auto& sV = sm.V;
  auto& sQ = sm.Q;
  auto& sdO = sm.dO;
  auto& sbk = sm.bk;
  auto& sbq = sm.bq;
  auto& sD = sm.D;
  auto& sL = sm.L;

  const int kt = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int S = a.S, E = a.H * kHd;
  const long long ld = 3ll * E;
  const bool prefix = seq >= a.n_causal;
  const int k0 = kt * kTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const __nv_bfloat16* base = a.qkv + (long long)seq * S * ld;
  const __nv_bfloat16* dobase = a.dout + (long long)seq * S * E;
  const int32_t* bid = prefix ? a.bid + (long long)(seq - a.n_causal) * S : nullptr;
  const long long lrow = ((long long)seq * a.H + h) * S;
  const int nq = (S + kTile - 1) / kTile;

  int q_lo = k0;
  if (prefix) q_lo = min(q_lo, a.meta[(long long)(seq - a.n_causal) * 2 * a.nt + a.nt + kt]);
  const int qt0 = q_lo / kTile;

  load_tile_async(smem_u32(sK), base, ld, k0, S, E + h * kHd);
  load_tile_async(smem_u32(sV), base, ld, k0, S, 2 * E + h * kHd);
  load_tile_async(smem_u32(sQ[0]), base, ld, qt0 * kTile, S, h * kHd);
  load_tile_async(smem_u32(sdO[0]), dobase, E, qt0 * kTile, S, h * kHd);
  cp_async_commit();
  for (int i = threadIdx.x; i < kTile; i += 128) {
    const int q = qt0 * kTile + i;
    sD[0][i] = q < S ? a.dsum[lrow + q] : 0.f;
    sL[0][i] = q < S ? a.lse[lrow + q] : 0.f;
    if (prefix) {
      sbk[i] = k0 + i < S ? bid[k0 + i] : -2;
      sbq[0][i] = q < S ? bid[q] : -1;
    }
  }

  const float sl2 = 0.125f * kLog2e;
  float dk[8][4], dv[8][4];
  zero_acc(dk);
  zero_acc(dv);
  uint32_t ka[4][4], va[4][4];
  const int jl_lo = warp * 16 + g;  // local key row of c0/c1

  for (int qt = qt0; qt < nq; ++qt) {
    const int buf = (qt - qt0) & 1;
    if (qt + 1 < nq) {
      const int nb = buf ^ 1;
      load_tile_async(smem_u32(sQ[nb]), base, ld, (qt + 1) * kTile, S, h * kHd);
      load_tile_async(smem_u32(sdO[nb]), dobase, E, (qt + 1) * kTile, S, h * kHd);
      cp_async_commit();
      for (int i = threadIdx.x; i < kTile; i += 128) {
        const int q = (qt + 1) * kTile + i;
        sD[nb][i] = q < S ? a.dsum[lrow + q] : 0.f;
        sL[nb][i] = q < S ? a.lse[lrow + q] : 0.f;
        if (prefix) sbq[nb][i] = q < S ? bid[q] : -1;
      }
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (qt == qt0) {
      load_a_frags(smem_u32(sK), warp * 16, ka);
      load_a_frags(smem_u32(sV), warp * 16, va);
    }
    // S^T[key, q] and dP^T[key, q]
    float st[8][4], dpt[8][4];
    zero_acc(st);
    zero_acc(dpt);
    mma_a_bt(st, ka, smem_u32(sQ[buf]));
    mma_a_bt(dpt, va, smem_u32(sdO[buf]));

    const int qb = qt * kTile;
    const bool full_tile = (k0 + kTile <= qb) && (qb + kTile <= S) && (k0 + kTile <= S);
    float pt[8][4];
    #pragma unroll
    for (int n = 0; n < 8; ++n) {
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int jl = jl_lo + (e >> 1) * 8;
        const int j = k0 + jl;
        const int il = n * 8 + 2 * t + (e & 1);
        const int i = qb + il;
        bool ok = true;
        if (!full_tile) {
          ok = j < S && i < S && j <= i;
          if (!ok && prefix && j < S && i < S) ok = sbk[jl] == sbq[buf][il];
        }
        const float p = ok ? exp2f(st[n][e] * sl2 - sL[buf][il]) : 0.f;
        pt[n][e] = p;
        st[n][e] = p * (dpt[n][e] - sD[buf][il]);  // dS^T
      }
    }
    uint32_t pa[4][4], dsa[4][4];
    c_to_a(pt, pa);
    c_to_a(st, dsa);
    mma_a_b(dv, pa, smem_u32(sdO[buf]));
    mma_a_b(dk, dsa, smem_u32(sQ[buf]));
    __syncthreads();
  }

  #pragma unroll
  for (int n = 0; n < 8; ++n)
    #pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] *= 0.125f;
  const int j_lo = k0 + jl_lo;
  unrope_c(dk, a.rope, min(j_lo, S - 1), min(j_lo + 8, S - 1));
  __nv_bfloat16* dbase = a.dqkv + (long long)seq * S * ld;
  c_to_smem(dk, sK, warp * 16);
  c_to_smem(dv, sV, warp * 16);
  __syncthreads();
  store_tile(sK, dbase, ld, k0, S, E + h * kHd);
  store_tile(sV, dbase, ld, k0, S, 2 * E + h * kHd);
}

// ===========================================================================
// Sequence-resident kernels for S <= 256 (the pretraining length): one CTA per
// (head, sequence) holds the whole sequence's Q/K/V (and dO) tiles in shared
// memory, fetched by TMA with one mbarrier per 64-row tile, so each tile is read
// from HBM once per head instead of once per query tile.  Eight warps own
// 16-row slices, paired (w, 15 - w) so that every warp does the same amount of
// causal work.
// ===========================================================================
constexpr int kSeqTiles = 4;
constexpr int kSeqMax = kSeqTiles * kTile;

// acc += A * T^T over output chunks [c0, c1) (16 columns each); T stored [n][k].
__device__ __forceinline__ void mma_a_bt_r(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t s_tile, int c0,
                                           int c1) {
  const int lane = threadIdx.x & 31;
  const int m = lane >> 3;
  #pragma unroll
  for (int np = 0; np < 4; ++np) {
    if (np < c0 || np >= c1) continue;
    #pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int n = np * 16 + (m >> 1) * 8 + (lane & 7);
      const int k = kk * 16 + (m & 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(s_tile + swz(n, k), b0, b1, b2, b3);
      mma_bf16_16816(acc[2 * np], a[kk], b0, b1);
      mma_bf16_16816(acc[2 * np + 1], a[kk], b2, b3);
    }
  }
}

// acc += A * T over reduction chunks [c0, c1) of A's columns; T stored [k][n].
__device__ __forceinline__ void mma_a_b_r(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t s_tile, int c0,
                                          int c1) {
  const int lane = threadIdx.x & 31;
  const int m = lane >> 3;
  #pragma unroll
  for (int dp = 0; dp < 4; ++dp) {
    #pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if (kk < c0 || kk >= c1) continue;
      const int k = kk * 16 + (m & 1) * 8 + (lane & 7);
      const int n = dp * 16 + (m >> 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(s_tile + swz(k, n), b0, b1, b2, b3);
      mma_bf16_16816(acc[2 * dp], a[kk], b0, b1);
      mma_bf16_16816(acc[2 * dp + 1], a[kk], b2, b3);
    }
  }
}

// Store a warp's 16 staged rows (swizzled, 128 B each) to global rows row0.. (rows < nrows).
__device__ __forceinline__ void store_rows16(const uint8_t* stage, __nv_bfloat16* g, long long ld, int row0,
                                             int nrows, int col0) {
  const int lane = threadIdx.x & 31;
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int idx = lane + 32 * j;
    const int r = idx >> 3, ch = idx & 7;
    if (row0 + r < nrows)
      *reinterpret_cast<uint4*>(g + (long long)(row0 + r) * ld + col0 + ch * 8) =
          *reinterpret_cast<const uint4*>(stage + swz(r, ch * 8));
  }
}

struct SeqFwdSmem {
  uint8_t Q[kSeqTiles][kTile * 128];
  uint8_t K[kSeqTiles][kTile * 128];
  uint8_t V[kSeqTiles][kTile * 128];
  uint64_t bar[kSeqTiles];
  int32_t bid[kSeqMax];
  int32_t last[kSeqMax];
  int abort;
};

struct SeqBwdSmem {
  uint8_t Q[kSeqTiles][kTile * 128];
  uint8_t K[kSeqTiles][kTile * 128];
  uint8_t V[kSeqTiles][kTile * 128];
  uint8_t dO[kSeqTiles][kTile * 128];
  uint8_t stage[8][16 * 128];
  uint64_t bar[kSeqTiles];
  float D[kSeqMax];
  float L[kSeqMax];
  int32_t bid[kSeqMax];
  int32_t first[kSeqMax];
  int32_t last[kSeqMax];
  int abort;
};

template <class T>
__device__ __forceinline__ T& align_smem(uint8_t* raw) {
  return *reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// Per-row block bounds of prefix sequence `pseq` inside the metadata buffer.
__device__ __forceinline__ const int32_t* meta_first(const AttnArgs& a, int pseq) {
  const long long np = a.nseq - a.n_causal;
  return a.meta + np * 2 * a.nt + (long long)pseq * a.S;
}
__device__ __forceinline__ const int32_t* meta_last(const AttnArgs& a, int pseq) {
  const long long np = a.nseq - a.n_causal;
  return a.meta + np * 2 * a.nt + np * a.S + (long long)pseq * a.S;
}

__global__ void __launch_bounds__(256, 1)
    attn_fwd_seq_kernel(const __grid_constant__ CUtensorMap tqkv, const AttnArgs a) {
  extern __shared__ uint8_t dsm_raw[];
  SeqFwdSmem& sm = align_smem<SeqFwdSmem>(dsm_raw);
  const int h = blockIdx.x, seq = blockIdx.y;
  const int S = a.S, E = a.H * kHd;
  const int nt = (S + kTile - 1) / kTile;
  const bool prefix = seq >= a.n_causal;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int row_base = seq * S;

  if (threadIdx.x == 0) {
    for (int i = 0; i < nt; ++i) mbar_init(&sm.bar[i], 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    prefetch_tmap(&tqkv);
    for (int i = 0; i < nt; ++i) {
      mbar_arrive_expect_tx(&sm.bar[i], 3 * kTile * 128);
      tma_load_2d(sm.Q[i], &tqkv, &sm.bar[i], h * kHd, row_base + i * kTile);
      tma_load_2d(sm.K[i], &tqkv, &sm.bar[i], E + h * kHd, row_base + i * kTile);
      tma_load_2d(sm.V[i], &tqkv, &sm.bar[i], 2 * E + h * kHd, row_base + i * kTile);
    }
  }
  const int pseq = seq - a.n_causal;
  const int32_t* bidg = prefix ? a.bid + (long long)pseq * S : nullptr;
  const int32_t* lastg = prefix ? meta_last(a, pseq) : nullptr;
  for (int i = threadIdx.x; i < kSeqMax; i += blockDim.x) {
    sm.bid[i] = i < S ? (prefix ? bidg[i] : i) : -1;
    sm.last[i] = i < S ? (prefix ? lastg[i] : i) : i;
  }
  __syncthreads();

  const float sl2 = 0.125f * kLog2e;
  const int nslices = (S + 15) / 16;
  volatile int* abort_flag = &sm.abort;
  for (int which = 0; which < 2; ++which) {
    const int slice = which == 0 ? warp : 15 - warp;
    if (slice >= nslices) continue;
    const int r0 = slice * 16;
    int kv_end = 0;
    {
      int v = 0;
      if (lane < 16 && r0 + lane < S) v = max(r0 + lane + 1, sm.last[r0 + lane] + 1);
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
      kv_end = min(v, S);
    }
    const int qt = r0 / kTile, rl = r0 % kTile;
    mbar_wait(&sm.bar[qt], 0, abort_flag);
    uint32_t qa[4][4];
    load_a_frags(smem_u32(sm.Q[qt]), rl, qa);
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    float o[8][4];
    zero_acc(o);
    const int i_lo = r0 + g;
    const int n_kv = (kv_end + kTile - 1) / kTile;
    for (int kt = 0; kt < n_kv; ++kt) {
      mbar_wait(&sm.bar[kt], 0, abort_flag);
      const int k0 = kt * kTile;
      const int nk = min(4, (kv_end - k0 + 15) / 16);
      float s[8][4];
      zero_acc(s);
      mma_a_bt_r(s, qa, smem_u32(sm.K[kt]), 0, nk);
      const bool full = k0 + kTile <= r0;
      #pragma unroll
      for (int n = 0; n < 8; ++n) {
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = s[n][e] * sl2;
          if (!full) {
            const int i = i_lo + (e >> 1) * 8;
            const int j = k0 + n * 8 + 2 * t + (e & 1);
            const bool ok = (n >> 1) < nk && j < S && i < S && (j <= i || sm.bid[i] == sm.bid[j]);
            if (!ok) v = -INFINITY;
          }
          s[n][e] = v;
        }
      }
      #pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float mx = -INFINITY;
        #pragma unroll
        for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_r[hr], mx);
        const float corr = m_new == -INFINITY ? 1.f : exp2f(m_r[hr] - m_new);
        float sum = 0.f;
        #pragma unroll
        for (int n = 0; n < 8; ++n) {
          const float p0 = m_new == -INFINITY ? 0.f : exp2f(s[n][2 * hr] - m_new);
          const float p1 = m_new == -INFINITY ? 0.f : exp2f(s[n][2 * hr + 1] - m_new);
          s[n][2 * hr] = p0;
          s[n][2 * hr + 1] = p1;
          sum += p0 + p1;
        }
        l_r[hr] = l_r[hr] * corr + sum;
        m_r[hr] = m_new;
        #pragma unroll
        for (int n = 0; n < 8; ++n) {
          o[n][2 * hr] *= corr;
          o[n][2 * hr + 1] *= corr;
        }
      }
      uint32_t pa[4][4];
      c_to_a(s, pa);
      mma_a_b_r(o, pa, smem_u32(sm.V[kt]), 0, nk);
    }
    #pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float l = l_r[hr];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      const float inv = l > 0.f ? 1.f / l : 0.f;
      #pragma unroll
      for (int n = 0; n < 8; ++n) {
        o[n][2 * hr] *= inv;
        o[n][2 * hr + 1] *= inv;
      }
      const int i = i_lo + hr * 8;
      if (t == 0 && i < S) a.lse[((long long)seq * a.H + h) * S + i] = m_r[hr] + log2f(l);
    }
    // the slice's Q rows belong to this warp alone: reuse them as output staging
    __syncwarp();
    c_to_smem(o, sm.Q[qt], rl);
    __syncwarp();
    {
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int idx = lane + 32 * j;
        const int r = idx >> 3, ch = idx & 7;
        if (r0 + r < S)
          *reinterpret_cast<uint4*>(a.out + (long long)(row_base + r0 + r) * E + h * kHd + ch * 8) =
              *reinterpret_cast<const uint4*>(sm.Q[qt] + swz(rl + r, ch * 8));
      }
    }
  }
}

__global__ void __launch_bounds__(256, 1)
    attn_bwd_seq_kernel(const __grid_constant__ CUtensorMap tqkv, const __grid_constant__ CUtensorMap tdo,
                        const AttnArgs a) {
  extern __shared__ uint8_t dsm_raw[];
  SeqBwdSmem& sm = align_smem<SeqBwdSmem>(dsm_raw);
  const int h = blockIdx.x, seq = blockIdx.y;
  const int S = a.S, E = a.H * kHd;
  const long long ld = 3ll * E;
  const int nt = (S + kTile - 1) / kTile;
  const bool prefix = seq >= a.n_causal;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int row_base = seq * S;
  const long long lrow = ((long long)seq * a.H + h) * S;

  if (threadIdx.x == 0) {
    for (int i = 0; i < nt; ++i) mbar_init(&sm.bar[i], 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    prefetch_tmap(&tqkv);
    prefetch_tmap(&tdo);
    for (int i = 0; i < nt; ++i) {
      mbar_arrive_expect_tx(&sm.bar[i], 4 * kTile * 128);
      tma_load_2d(sm.Q[i], &tqkv, &sm.bar[i], h * kHd, row_base + i * kTile);
      tma_load_2d(sm.K[i], &tqkv, &sm.bar[i], E + h * kHd, row_base + i * kTile);
      tma_load_2d(sm.V[i], &tqkv, &sm.bar[i], 2 * E + h * kHd, row_base + i * kTile);
      tma_load_2d(sm.dO[i], &tdo, &sm.bar[i], h * kHd, row_base + i * kTile);
    }
  }
  const int pseq = seq - a.n_causal;
  const int32_t* bidg = prefix ? a.bid + (long long)pseq * S : nullptr;
  const int32_t* firstg = prefix ? meta_first(a, pseq) : nullptr;
  const int32_t* lastg = prefix ? meta_last(a, pseq) : nullptr;
  for (int i = threadIdx.x; i < kSeqMax; i += blockDim.x) {
    sm.bid[i] = i < S ? (prefix ? bidg[i] : i) : -1;
    sm.first[i] = i < S ? (prefix ? firstg[i] : i) : i;
    sm.last[i] = i < S ? (prefix ? lastg[i] : i) : i;
    float d = 0.f, l = 0.f;
    if (i < S) {
      // D_i = sum_d dO[i,d] * O[i,d]
      const uint4* po = reinterpret_cast<const uint4*>(a.out + (long long)(row_base + i) * E + h * kHd);
      const uint4* pd = reinterpret_cast<const uint4*>(a.dout + (long long)(row_base + i) * E + h * kHd);
      #pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint4 wo = po[q], wd = pd[q];
        const __nv_bfloat162* ho = reinterpret_cast<const __nv_bfloat162*>(&wo);
        const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&wd);
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 fo = __bfloat1622float2(ho[j]), fd = __bfloat1622float2(hd[j]);
          d += fo.x * fd.x + fo.y * fd.y;
        }
      }
      l = a.lse[lrow + i];
    }
    sm.D[i] = d;
    sm.L[i] = l;
  }
  __syncthreads();

  const float sl2 = 0.125f * kLog2e;
  const int nslices = (S + 15) / 16;
  volatile int* abort_flag = &sm.abort;
  uint8_t* stage = sm.stage[warp];

  // ---- dQ for this warp's query slices ---------------------------------------
  for (int which = 0; which < 2; ++which) {
    const int slice = which == 0 ? warp : 15 - warp;
    if (slice >= nslices) continue;
    const int r0 = slice * 16;
    int kv_end;
    {
      int v = 0;
      if (lane < 16 && r0 + lane < S) v = max(r0 + lane + 1, sm.last[r0 + lane] + 1);
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
      kv_end = min(v, S);
    }
    const int qt = r0 / kTile, rl = r0 % kTile;
    mbar_wait(&sm.bar[qt], 0, abort_flag);
    uint32_t qa[4][4], doa[4][4];
    load_a_frags(smem_u32(sm.Q[qt]), rl, qa);
    load_a_frags(smem_u32(sm.dO[qt]), rl, doa);
    float dq[8][4];
    zero_acc(dq);
    const int i_lo = r0 + g;
    const int n_kv = (kv_end + kTile - 1) / kTile;
    for (int kt = 0; kt < n_kv; ++kt) {
      mbar_wait(&sm.bar[kt], 0, abort_flag);
      const int k0 = kt * kTile;
      const int nk = min(4, (kv_end - k0 + 15) / 16);
      float s[8][4], dp[8][4];
      zero_acc(s);
      zero_acc(dp);
      mma_a_bt_r(s, qa, smem_u32(sm.K[kt]), 0, nk);
      mma_a_bt_r(dp, doa, smem_u32(sm.V[kt]), 0, nk);
      const bool full = k0 + kTile <= r0;
      #pragma unroll
      for (int n = 0; n < 8; ++n) {
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = i_lo + (e >> 1) * 8;
          bool ok = true;
          if (!full) {
            const int j = k0 + n * 8 + 2 * t + (e & 1);
            ok = (n >> 1) < nk && j < S && i < S && (j <= i || sm.bid[i] == sm.bid[j]);
          }
          const float p = ok ? exp2f(s[n][e] * sl2 - sm.L[i]) : 0.f;
          s[n][e] = p * (dp[n][e] - sm.D[i]);
        }
      }
      uint32_t dsa[4][4];
      c_to_a(s, dsa);
      mma_a_b_r(dq, dsa, smem_u32(sm.K[kt]), 0, nk);
    }
    #pragma unroll
    for (int n = 0; n < 8; ++n)
      #pragma unroll
      for (int e = 0; e < 4; ++e) dq[n][e] *= 0.125f;
    unrope_c(dq, a.rope, min(i_lo, S - 1), min(i_lo + 8, S - 1));
    __syncwarp();
    c_to_smem(dq, stage, 0);
    __syncwarp();
    store_rows16(stage, a.dqkv + (long long)row_base * ld, ld, r0, S, h * kHd);
    __syncwarp();
  }

  // ---- dK, dV for this warp's key slices -------------------------------------
  for (int which = 0; which < 2; ++which) {
    const int slice = which == 0 ? warp : 15 - warp;
    if (slice >= nslices) continue;
    const int k0 = slice * 16;
    int q_lo;
    {
      int v = 1 << 30;
      if (lane < 16 && k0 + lane < S) v = min(k0 + lane, sm.first[k0 + lane]);
      #pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
      q_lo = v;
    }
    const int kt = k0 / kTile, kl = k0 % kTile;
    mbar_wait(&sm.bar[kt], 0, abort_flag);
    uint32_t ka[4][4], va[4][4];
    load_a_frags(smem_u32(sm.K[kt]), kl, ka);
    load_a_frags(smem_u32(sm.V[kt]), kl, va);
    float dk[8][4], dv[8][4];
    zero_acc(dk);
    zero_acc(dv);
    const int j_lo = k0 + g;
    const int qt0 = q_lo / kTile;
    for (int qt = qt0; qt < nt; ++qt) {
      mbar_wait(&sm.bar[qt], 0, abort_flag);
      const int qb = qt * kTile;
      const int c0 = qt == qt0 ? (q_lo - qb) / 16 : 0;
      const int c1 = min(4, (S - qb + 15) / 16);
      float st[8][4], dpt[8][4];
      zero_acc(st);
      zero_acc(dpt);
      mma_a_bt_r(st, ka, smem_u32(sm.Q[qt]), c0, c1);
      mma_a_bt_r(dpt, va, smem_u32(sm.dO[qt]), c0, c1);
      const bool full = (qb >= k0 + 16) && (qb + kTile <= S);
      float pt[8][4];
      #pragma unroll
      for (int n = 0; n < 8; ++n) {
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int il = n * 8 + 2 * t + (e & 1);
          const int i = qb + il;
          bool ok = true;
          if (!full) {
            const int j = j_lo + (e >> 1) * 8;
            const int chunk = n >> 1;
            ok = chunk >= c0 && chunk < c1 && i < S && j < S && (j <= i || sm.bid[i] == sm.bid[j]);
          }
          const float p = ok ? exp2f(st[n][e] * sl2 - sm.L[i]) : 0.f;
          pt[n][e] = p;
          st[n][e] = p * (dpt[n][e] - sm.D[i]);
        }
      }
      uint32_t pa[4][4], dsa[4][4];
      c_to_a(pt, pa);
      c_to_a(st, dsa);
      mma_a_b_r(dv, pa, smem_u32(sm.dO[qt]), c0, c1);
      mma_a_b_r(dk, dsa, smem_u32(sm.Q[qt]), c0, c1);
    }
    #pragma unroll
    for (int n = 0; n < 8; ++n)
      #pragma unroll
      for (int e = 0; e < 4; ++e) dk[n][e] *= 0.125f;
    unrope_c(dk, a.rope, min(j_lo, S - 1), min(j_lo + 8, S - 1));
    __nv_bfloat16* dbase = a.dqkv + (long long)row_base * ld;
    __syncwarp();
    c_to_smem(dk, stage, 0);
    __syncwarp();
    store_rows16(stage, dbase, ld, k0, S, E + h * kHd);
    __syncwarp();
    c_to_smem(dv, stage, 0);
    __syncwarp();
    store_rows16(stage, dbase, ld, k0, S, 2 * E + h * kHd);
    __syncwarp();
  }
}

}  // namespace cdk

using namespace cdk;

extern "C" int64_t cdk_attn_meta_elems(int64_t nseq_prefix, int64_t S) {
  const int64_t nt = (S + kTile - 1) / kTile;
  return nseq_prefix * (2 * nt + 2 * S);
}

extern "C" int cdk_attn_prefix_meta(const int32_t* bid, int64_t nseq_prefix, int64_t S, int32_t* meta,
                                    void* stream) {
  if (nseq_prefix == 0) return 0;
  if (!bid || !meta || S <= 0 || S > 8192 || nseq_prefix < 0) return -1;
  const int nt = (int)((S + kTile - 1) / kTile);
  const size_t smem = (size_t)(S + 2 * nt) * sizeof(int32_t);
  attn_meta_kernel<<<(unsigned)nseq_prefix, 256, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      bid, (int)S, nt, (int)nseq_prefix, meta);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

// Path selection.  S <= 256: the persistent tcgen05 kernels (attention_pst.cu,
// attention_bwd_pst.cu) by default; CDK_ATTN_PATH=tc selects the tcgen05
// kernels with one CTA per (query tile, head, sequence) (attention_tc.cu),
// CDK_ATTN_PATH=seq the mma.sync sequence-resident kernels and
// CDK_ATTN_PATH=tiled the tiled kernels (the tests cover all of them).  S > 256:
// the tcgen05 kernels of attention_long.cu by default (the backward needs the
// caller's fp32 dQ workspace, cdk_attn_bwd_ws), the tiled kernels with
// CDK_ATTN_PATH=tiled or seq or without a workspace.  CDK_ATTN_PATH=long takes
// the attention_long.cu kernels at every S.
static int attn_path() {
  const char* v = getenv("CDK_ATTN_PATH");
  if (v && v[0] == 't' && v[1] == 'i') return 2;  // tiled
  if (v && v[0] == 't' && v[1] == 'c') return 4;  // one CTA per (query tile, head, sequence) tcgen05 kernels
  if (v && v[0] == 'p') return 5;                  // persistent tcgen05 kernels (the default at S <= 256)
  if (v && v[0] == 's') return 1;                  // seq (mma.sync)
  if (v && v[0] == 'l') return 3;                  // tcgen05 long-sequence kernels at any S
  return 0;                                        // tcgen05
}
static bool long_path(int64_t S) { return (S > kSeqMax && (attn_path() == 0 || attn_path() == 5)) || attn_path() == 3; }
static bool seq_path_enabled() { return attn_path() != 2; }

namespace cdk {
int launch_attn_fwd_pst(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S,
                        int64_t H, const int32_t* bid, const int32_t* meta, cudaStream_t stream);
int launch_attn_fwd_tc(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S, int64_t H,
                       const int32_t* bid, const int32_t* meta, cudaStream_t stream);
int launch_attn_fwd_long(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S,
                         int64_t H, const int32_t* bid, const int32_t* meta, cudaStream_t stream);
int launch_attn_bwd_tc(const void* qkv, const void* out, const void* dout, const float* lse, void* dqkv,
                       int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                       const int32_t* meta, const float* rope, cudaStream_t stream);
}  // namespace cdk

static int attn_check(const void* qkv, int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* meta) {
  if (!qkv || nseq <= 0 || S <= 0 || H <= 0 || H > 64) return -1;
  if (n_causal < 0 || n_causal > nseq) return -2;
  if (n_causal < nseq && !meta) return -3;
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) != 0) return -4;
  if (nseq > 65535 || S > 1 << 20) return -5;
  return 0;
}

extern "C" int cdk_attn_fwd(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S,
                            int64_t H, const int32_t* bid, const int32_t* meta, void* stream) {
  int rc = attn_check(qkv, nseq, n_causal, S, H, meta);
  if (rc) return rc;
  if (!out || !lse) return -1;
  if (n_causal < nseq && !bid) return -3;
  AttnArgs a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv);
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  a.bid = bid;
  a.meta = meta;
  a.S = (int)S;
  a.H = (int)H;
  a.n_causal = (int)n_causal;
  a.nt = (int)((S + kTile - 1) / kTile);
  a.nseq = (int)nseq;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (S <= kSeqMax && (attn_path() == 0 || attn_path() == 5)) {
    return launch_attn_fwd_pst(qkv, out, lse, nseq, n_causal, S, H, bid, meta, s);
  }
  if (S <= kSeqMax && attn_path() == 4) {
    return launch_attn_fwd_tc(qkv, out, lse, nseq, n_causal, S, H, bid, meta, s);
  }
  if (long_path(S)) {
    return launch_attn_fwd_long(qkv, out, lse, nseq, n_causal, S, H, bid, meta, s);
  }
  if (S <= kSeqMax && seq_path_enabled()) {
    CUtensorMap tq;
    if (!make_tmap(&tq, qkv, 3 * H * kHd, nseq * S, 3 * H * kHd, 64, 64)) return -10;
    const size_t smem = sizeof(SeqFwdSmem) + 1024;
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_done[dev]) {
      cudaFuncSetAttribute(attn_fwd_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attr_done[dev] = true;
    }
    attn_fwd_seq_kernel<<<dim3((unsigned)H, (unsigned)nseq), 256, smem, s>>>(tq, a);
  } else {
    dim3 grid((unsigned)a.nt, (unsigned)H, (unsigned)nseq);
    attn_fwd_kernel<<<grid, 128, 0, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

namespace cdk {
int launch_attn_bwd_pst(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum,
                        void* dqkv, int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                        const int32_t* meta, const float* rope, cudaStream_t stream, const Q8Out* q8 = nullptr);
int launch_attn_bwd_long(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum,
                         void* dqkv, int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                         const int32_t* meta, const float* rope, void* workspace, cudaStream_t stream);
}  // namespace cdk

extern "C" int64_t cdk_attn_bwd_workspace(int64_t nseq, int64_t S, int64_t H) {
  if (nseq < 0 || S <= 0 || H <= 0) return -1;
  return long_path(S) ? nseq * S * H * kHd * (int64_t)sizeof(float) : 0;
}

extern "C" int cdk_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum,
                            void* dqkv, int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                            const int32_t* meta, const float* rope, void* stream) {
  return cdk_attn_bwd_ws(qkv, out, dout, lse, dsum, dqkv, nseq, n_causal, S, H, bid, meta, rope, nullptr, 0, stream);
}

extern "C" int cdk_attn_bwd_q8(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum,
                               void* dqkv8, int64_t ld8, int fmt, const float* qscale, float* amax, int64_t nseq,
                               int64_t n_causal, int64_t S, int64_t H, const int32_t* bid, const int32_t* meta,
                               const float* rope, void* stream) {
  int rc = attn_check(qkv, nseq, n_causal, S, H, meta);
  if (rc) return rc;
  if (!out || !dout || !lse || !dsum || !dqkv8 || !qscale || (fmt != 0 && fmt != 1)) return -1;
  if (n_causal < nseq && !bid) return -3;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(dout) & 15) ||
      (reinterpret_cast<uintptr_t>(dqkv8) & 15) || (ld8 % 16) || ld8 < 3 * H * kHd)
    return -4;
  // only the persistent S <= 256 kernel writes the 8-bit form
  if (S > kSeqMax || !(attn_path() == 0 || attn_path() == 5)) return -20;
  Q8Out q8;
  q8.q = reinterpret_cast<uint8_t*>(dqkv8);
  q8.ldq = ld8;
  q8.fmt = fmt;
  q8.qscale = qscale;
  q8.amax = amax;
  return launch_attn_bwd_pst(qkv, out, dout, lse, dsum, nullptr, nseq, n_causal, S, H, bid, meta, rope,
                             reinterpret_cast<cudaStream_t>(stream), &q8);
}

extern "C" int cdk_attn_bwd_ws(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum,
                               void* dqkv, int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                               const int32_t* meta, const float* rope, void* workspace, int64_t workspace_bytes,
                               void* stream) {
  int rc = attn_check(qkv, nseq, n_causal, S, H, meta);
  if (rc) return rc;
  if (!out || !dout || !lse || !dsum || !dqkv) return -1;
  if (n_causal < nseq && !bid) return -3;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(dout) & 15) ||
      (reinterpret_cast<uintptr_t>(dqkv) & 15))
    return -4;
  AttnArgs a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv);
  a.out = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(out));
  a.lse = const_cast<float*>(lse);
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout);
  a.dsum = dsum;
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv);
  a.bid = bid;
  a.meta = meta;
  a.rope = rope;
  a.S = (int)S;
  a.H = (int)H;
  a.n_causal = (int)n_causal;
  a.nt = (int)((S + kTile - 1) / kTile);
  a.nseq = (int)nseq;
  dim3 grid((unsigned)a.nt, (unsigned)H, (unsigned)nseq);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (S <= kSeqMax && (attn_path() == 0 || attn_path() == 5))
    return launch_attn_bwd_pst(qkv, out, dout, lse, dsum, dqkv, nseq, n_causal, S, H, bid, meta, rope, s);
  if (S <= kSeqMax && attn_path() == 4)
    return launch_attn_bwd_tc(qkv, out, dout, lse, dqkv, nseq, n_causal, S, H, bid, meta, rope, s);
  if (long_path(S) && workspace != nullptr && S % 4 == 0) {
    if (workspace_bytes < cdk_attn_bwd_workspace(nseq, S, H) || (reinterpret_cast<uintptr_t>(workspace) & 15))
      return -5;
    return launch_attn_bwd_long(qkv, out, dout, lse, dsum, dqkv, nseq, n_causal, S, H, bid, meta, rope, workspace,
                                s);
  }
  if (S <= kSeqMax && seq_path_enabled()) {
    CUtensorMap tq, tdo;
    if (!make_tmap(&tq, qkv, 3 * H * kHd, nseq * S, 3 * H * kHd, 64, 64)) return -10;
    if (!make_tmap(&tdo, dout, H * kHd, nseq * S, H * kHd, 64, 64)) return -11;
    const size_t smem = sizeof(SeqBwdSmem) + 1024;
    static bool seq_attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !seq_attr[dev]) {
      cudaFuncSetAttribute(attn_bwd_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      seq_attr[dev] = true;
    }
    attn_bwd_seq_kernel<<<dim3((unsigned)H, (unsigned)nseq), 256, smem, s>>>(tq, tdo, a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
  }
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DqSmem));
    cudaFuncSetAttribute(attn_bwd_dkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DkvSmem));
    attr_done[dev] = true;
  }
  attn_bwd_dq_kernel<<<grid, 128, sizeof(DqSmem), s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  attn_bwd_dkv_kernel<<<grid, 128, sizeof(DkvSmem), s>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}
