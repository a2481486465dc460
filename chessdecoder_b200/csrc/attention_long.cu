// Tensor-core (tcgen05 + TMEM) attention forward for sequences longer than 256
// tokens (the thinking-variation rows of the MoE variant, S = 4096; masks of
// chessdecoder/models/model.py:158-171).  Flash-style: one CTA per (128-query
// tile, head, sequence) walks the key tiles of 128 that the tile may see with
// an online softmax.
//
//   warp 0 (lane 0)  TMA: the Q tile once, then K_j / V_j into a 4-stage ring
//   warp 1 (lane 0)  MMA: S_j = Q K_j^T into one of two TMEM score buffers, and
//                    O += P_{j-1} V_{j-1} into the TMEM output accumulator
//   warps 2-9        softmax: two threads per query row (warps w and w+4 share
//                    the TMEM lane quadrant and split the 128 keys of a tile);
//                    row max exchanged through shared memory; P_j written as
//                    a 128-byte-swizzled bf16 K-major operand; O rescaled in
//                    TMEM only when the row max grows by more than 2^8
//                    (p stays <= 256 otherwise), after P_{j-1} V_{j-1} retired
//
// Two score buffers let S_{j+1} run on the tensor cores while the softmax of
// tile j runs; the exponentials of tile j are computed before waiting for
// P_{j-1} V_{j-1}.  The two threads of a row meet on a named barrier per lane
// quadrant (ids 2-5, 64 threads), not on all eight warps.  All waits are
// bounded (cdk_common).
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {
namespace tclong {

constexpr int kHd = 64;
constexpr int kBQ = 128;
constexpr int kBK = 128;
constexpr int kTileBytes = 64 * 128;  // one TMA box: 64 rows x 128 B
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.f;       // lazy rescale threshold (log2 units)
constexpr int kFwdThreads = 320;
constexpr int kStages = 4;            // K/V ring depth (L2 latency of a 32 KB tile pair spans several tiles)

struct FwdSmem {
  uint8_t Q[2 * kTileBytes];
  uint8_t K[kStages][2 * kTileBytes];
  uint8_t V[kStages][2 * kTileBytes];
  uint8_t P[2][2][128 * 128];  // [buffer][64-key block][128 rows x 64 keys]
  uint64_t bar_q, bar_full[kStages], bar_empty[kStages], bar_s[2], bar_p[2], bar_o;
  uint32_t tmem_base;
  int abort;
  int n_kt;
  float red_max[2][2][kBQ];  // [iteration parity][half][row]
  float red_sum[2][kBQ];
};
static_assert(offsetof(FwdSmem, K) % 1024 == 0 && offsetof(FwdSmem, V) % 1024 == 0 &&
                  offsetof(FwdSmem, P) % 1024 == 0,
              "TMA / UMMA operands with the 128-byte swizzle need 1024-byte alignment");

struct LongArgs {
  __nv_bfloat16* out;
  float* lse;
  const int32_t* bid;         // [nseq - n_causal, S]
  const int32_t* last;        // [nseq - n_causal, S]
  const int32_t* tile_kv_hi;  // [nseq - n_causal][2 * nt64]
  int S, H, n_causal, nt64;
};

__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2^x on the SFU (ex2.approx.ftz): the arguments here are <= 2^3 (lazy
// rescale) and results below 2^-126 flush to 0, which the softmax tolerates.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_long_kernel(const __grid_constant__ CUtensorMap tqkv, const LongArgs a) {
  extern __shared__ uint8_t raw[];
  FwdSmem& sm = *reinterpret_cast<FwdSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int mt = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int S = a.S, E = a.H * kHd;
  const bool prefix = seq >= a.n_causal;
  const int pseq = seq - a.n_causal;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_base = seq * S;
  volatile int* abort_flag = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int b = 0; b < kStages; ++b) {
      mbar_init(&sm.bar_full[b], 1);
      mbar_init(&sm.bar_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.bar_s[b], 1);
      mbar_init(&sm.bar_p[b], 256);
    }
    mbar_init(&sm.bar_o, 1);
    sm.abort = 0;
    // key bound of this query tile: causal rows see keys <= row; prefix rows also
    // their block's later keys (per-64-row-tile bounds from the metadata)
    int kv = min(S, (mt + 1) * kBQ);
    if (prefix) {
      const int* kvhi = a.tile_kv_hi + (long long)pseq * 2 * a.nt64;
      for (int t = 2 * mt; t < min(2 * mt + 2, a.nt64); ++t) kv = max(kv, kvhi[t]);
    }
    sm.n_kt = (min(kv, S) + kBK - 1) / kBK;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;  // S buffers: columns [0,128), [128,256); O: [256, 320)
  const int n_kt = sm.n_kt;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tqkv);
      mbar_arrive_expect_tx(&sm.bar_q, 2 * kTileBytes);
      for (int t = 0; t < 2; ++t)
        tma_load_2d(sm.Q + t * kTileBytes, &tqkv, &sm.bar_q, h * kHd, row_base + mt * kBQ + t * 64);
      for (int j = 0; j < n_kt; ++j) {
        const int st = j % kStages;
        mbar_wait(&sm.bar_empty[st], ((j / kStages) & 1) ^ 1u, abort_flag);
        mbar_arrive_expect_tx(&sm.bar_full[st], 4 * kTileBytes);
        for (int t = 0; t < 2; ++t) {
          const int r0 = row_base + j * kBK + t * 64;
          tma_load_2d(sm.K[st] + t * kTileBytes, &tqkv, &sm.bar_full[st], E + h * kHd, r0);
          tma_load_2d(sm.V[st] + t * kTileBytes, &tqkv, &sm.bar_full[st], 2 * E + h * kHd, r0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = make_idesc_bf16(kBQ, kBK, false, false);
      const uint32_t id_o = make_idesc_bf16(kBQ, kHd, false, true);
      const uint32_t qa = smem_u32(sm.Q);
      mbar_wait(&sm.bar_q, 0, abort_flag);
      for (int j = 0; j <= n_kt; ++j) {
        if (j < n_kt) {
          const int st = j % kStages, sb = j & 1;
          mbar_wait(&sm.bar_full[st], (j / kStages) & 1, abort_flag);
          tc_fence_after();
          const uint32_t kb = smem_u32(sm.K[st]);
          #pragma unroll
          for (int kk = 0; kk < kHd / 16; ++kk)
            umma_f16(tmem + sb * kBK, make_sdesc(qa + kk * 32, 16, 1024), make_sdesc(kb + kk * 32, 16, 1024), id_s,
                     kk > 0 ? 1u : 0u);
          tc_commit(&sm.bar_s[sb]);
        }
        if (j >= 1) {
          const int pj = j - 1, pbuf = pj & 1, st = pj % kStages;
          mbar_wait(&sm.bar_p[pbuf], (pj >> 1) & 1, abort_flag);
          tc_fence_after();
          const uint32_t pb = smem_u32(sm.P[pbuf][0]);
          const uint32_t vb = smem_u32(sm.V[st]);
          #pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(tmem + 256, make_sdesc(pb + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024),
                     make_sdesc(vb + kk * 16 * 128, 8192, 1024), id_o, (pj > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sm.bar_o);
          tc_commit(&sm.bar_empty[st]);
        }
      }
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sl2 = 0.125f * kLog2e;
    const int i = mt * kBQ + r;
    const bool row_ok = i < S;
    const int32_t* bidrow = prefix ? a.bid + (long long)pseq * S : nullptr;
    const int my_bid = (prefix && row_ok) ? bidrow[i] : -1;
    const int hi = row_ok ? (prefix ? max(i, a.last[(long long)pseq * S + i]) : i) : -1;
    float m_used = -INFINITY;
    float l = 0.f;
    for (int j = 0; j < n_kt; ++j) {
      const int b = j & 1;
      mbar_wait(&sm.bar_s[b], (j >> 1) & 1, abort_flag);
      tc_fence_after();
      uint32_t u0[32], u1[32];
      tmem_ld_x32_nowait(tmem + lane_off + b * kBK + half * 64, u0);
      tmem_ld_x32_nowait(tmem + lane_off + b * kBK + half * 64 + 32, u1);
      tmem_wait_ld();
      const int k0 = j * kBK + half * 64;  // first key of this thread's 64
      // warp-uniform fast path: every key of every row of the warp visible
      const bool full = row_ok && k0 + 63 <= i && k0 + 63 < S;
      const bool full_w = __all_sync(0xffffffffu, full);
      // scaled scores (masked ones -inf) in place, and their max (4 chains)
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (full_w) {
        #pragma unroll
        for (int e = 0; e < 64; ++e) {
          uint32_t& w = e < 32 ? u0[e] : u1[e - 32];
          const float x = __uint_as_float(w) * sl2;
          w = __float_as_uint(x);
          m4[e & 3] = fmaxf(m4[e & 3], x);
        }
      } else {
        #pragma unroll
        for (int e = 0; e < 64; ++e) {
          uint32_t& w = e < 32 ? u0[e] : u1[e - 32];
          const int k = k0 + e;
          bool vis = row_ok && k < S && k <= hi;
          if (vis && k > i) vis = bidrow != nullptr && bidrow[k] == my_bid;  // future key: same block only
          const float x = vis ? __uint_as_float(w) * sl2 : -INFINITY;
          w = __float_as_uint(x);
          m4[e & 3] = fmaxf(m4[e & 3], x);
        }
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      // the two threads of a row (warps w and w+4) exchange their maxima
      sm.red_max[j & 1][half][r] = mx;
      asm volatile("bar.sync %0, 64;" ::"r"(2 + quad) : "memory");
      const float row_max = fmaxf(mx, sm.red_max[j & 1][half ^ 1][r]);
      float m_new = m_used;
      if (row_max > m_used + kRescale || (m_used == -INFINITY && row_max > -INFINITY)) m_new = row_max;
      const float alpha = (m_new == m_used) ? 1.f : (m_used == -INFINITY ? 0.f : ex2_approx(m_used - m_new));
      const float msub = m_new == -INFINITY ? 0.f : m_new;
      uint32_t pk[32];
      float l4[4] = {0.f, 0.f, 0.f, 0.f};
      #pragma unroll
      for (int e = 0; e < 64; e += 2) {
        const float x0 = __uint_as_float(e < 32 ? u0[e] : u1[e - 32]);
        const float x1 = __uint_as_float(e + 1 < 32 ? u0[e + 1] : u1[e + 1 - 32]);
        const float p0 = ex2_approx(x0 - msub), p1 = ex2_approx(x1 - msub);
        l4[(e >> 1) & 3] += p0 + p1;
        pk[e >> 1] = pack_bf16(p0, p1);
      }
      const float ls = (l4[0] + l4[1]) + (l4[2] + l4[3]);
      l = l * alpha + ls;
      // P_{j-1} V_{j-1} must have retired before O is rescaled and before P
      // buffer b (read by P_{j-2} V_{j-2}) is overwritten
      if (j >= 1) mbar_wait(&sm.bar_o, (j - 1) & 1, abort_flag);
      tc_fence_after();
      uint8_t* pblk = sm.P[b][half];
      #pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4*>(pblk + sw128(r, q * 8)) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                                                                       pk[4 * q + 3]);
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
        uint32_t o[32];
        tmem_ld_x32_nowait(tmem + lane_off + 256 + half * 32, o);
        tmem_wait_ld();
        #pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
        tmem_st_x32(tmem + lane_off + 256 + half * 32, o);
        tmem_wait_st();
      }
      m_used = m_new;
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.bar_p[b]);
    }
    // epilogue: O / l (the two halves' partial sums add: both used m_used)
    sm.red_sum[half][r] = l;
    mbar_wait(&sm.bar_o, (n_kt - 1) & 1, abort_flag);
    asm volatile("bar.sync 1, 256;" ::: "memory");
    tc_fence_after();
    const float lt = sm.red_sum[0][r] + sm.red_sum[1][r];
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    uint32_t o[32];
    tmem_ld_x32_nowait(tmem + lane_off + 256 + half * 32, o);
    tmem_wait_ld();
    if (row_ok) {
      uint4* dst = reinterpret_cast<uint4*>(a.out + (long long)(row_base + i) * E + h * kHd + half * 32);
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int c = q * 8;
        dst[q] = make_uint4(pack_bf16(__uint_as_float(o[c]) * inv, __uint_as_float(o[c + 1]) * inv),
                            pack_bf16(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv),
                            pack_bf16(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv),
                            pack_bf16(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv));
      }
      if (half == 0) a.lse[((long long)seq * a.H + h) * S + i] = (m_used == -INFINITY ? 0.f : m_used) + log2f(lt);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tclong

// Host launcher used by cdk_attn_fwd for S > 256.
int launch_attn_fwd_long(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S,
                         int64_t H, const int32_t* bid, const int32_t* meta, cudaStream_t stream) {
  using namespace tclong;
  if (S <= 0) return -20;
  CUtensorMap tq;
  if (!make_tmap(&tq, qkv, 3 * H * kHd, nseq * S, 3 * H * kHd, 64, 64)) return -21;
  LongArgs a;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  const int64_t np = nseq - n_causal;
  const int nt64 = (int)((S + 63) / 64);
  a.bid = bid;
  a.tile_kv_hi = meta;
  a.last = np > 0 ? meta + np * 2 * nt64 + np * S : nullptr;
  a.nt64 = nt64;
  a.S = (int)S;
  a.H = (int)H;
  a.n_causal = (int)n_causal;
  const size_t smem = sizeof(FwdSmem) + 1024;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_fwd_long_kernel, kFwdThreads, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm * 512 > 512) return -22;
    attr_done[dev] = true;
  }
  attn_fwd_long_kernel<<<dim3((unsigned)((S + kBQ - 1) / kBQ), (unsigned)H, (unsigned)nseq), kFwdThreads, smem,
                         stream>>>(tq, a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace cdk
