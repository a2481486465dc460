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
    {  // the whole warp runs the issue loop; one elected lane issues (uniform operands)
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
            umma_f16_w(tmem + sb * kBK, make_sdesc(qa + kk * 32, 16, 1024), make_sdesc(kb + kk * 32, 16, 1024), id_s,
                     kk > 0 ? 1u : 0u);
          tc_commit_w(&sm.bar_s[sb]);
        }
        if (j >= 1) {
          const int pj = j - 1, pbuf = pj & 1, st = pj % kStages;
          mbar_wait(&sm.bar_p[pbuf], (pj >> 1) & 1, abort_flag);
          tc_fence_after();
          const uint32_t pb = smem_u32(sm.P[pbuf][0]);
          const uint32_t vb = smem_u32(sm.V[st]);
          #pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16_w(tmem + 256, make_sdesc(pb + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024),
                     make_sdesc(vb + kk * 16 * 128, 8192, 1024), id_o, (pj > 0 || kk > 0) ? 1u : 0u);
          tc_commit_w(&sm.bar_o);
          tc_commit_w(&sm.bar_empty[st]);
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


// ===========================================================================
// Backward for S > 256.  One CTA per (128-key tile, head, sequence) walks the
// 64-query sub-tiles s that can see the key tile (two per 128-query tile t):
//   MMA-A(s)  S^T = K Q_s^T, dP^T = V dO_s^T            (TMEM, 64 columns each)
//   EW(s)     P^T = exp2(S^T c - L), dS^T = P^T (dP^T - D)  (bf16 operands in smem)
//   MMA-B(s)  dV += P^T dO_s, dK += dS^T Q_s             (TMEM, accumulated;
//             P^T and dS^T are read from TMEM, where EW(s) stores them in bf16)
//   MMA-Q(t)  dQ_t = dS K over both sub-tiles of t       (TMEM; dS read from smem)
// S^T | dP^T are double-buffered, so the tensor core runs A(s+2), B(s) and
// Q(t) while the elementwise warps work on sub-tile s+1: a tcgen05.mma of
// M=128, K=16 costs about the same for N=64 as for N=128, which makes the
// 40 instructions of a 128 x 128 (key, query) tile as long as its elementwise
// work, and only overlapping the two keeps both busy; taking the A operand of
// the dV / dK products from TMEM keeps their shared-memory reads to the B
// tiles.  The elementwise warps
// also move dQ_t from TMEM into shared memory (the tile's dS^T pair, free
// once Q(t) has retired) for a bulk reduce-add (cp.reduce.async.bulk.tensor)
// into an fp32 [tokens, E] accumulator.  Q, dO, L and D arrive per sub-tile
// in a 4-deep ring.  D = rowsum(dO * O) comes from a pass before; a pass after
// scales dQ by 1/8, undoes RoPE and writes it into dqkv.
// TMEM: S^T|dP^T x 2 (256) | dV (64) | dK (64) | dQ (64) | P^T|dS^T bf16 (64) = 512.
// ===========================================================================
constexpr int kQStages = 4;       // sub-tile ring (Q, dO, L, D of 64 queries)
constexpr int kBwdThreads = 576;  // warp 0 TMA, warp 1 MMA, warps 2-17 elementwise

struct BwdSmem {
  uint8_t K[2 * kTileBytes];
  uint8_t V[2 * kTileBytes];
  uint8_t Q[kQStages][kTileBytes];
  uint8_t dO[kQStages][kTileBytes];
  uint8_t dST[2][2][128 * 128];   // [tile parity][sub-tile]: 128 key rows x 64 queries; after Q(t) the pair stages dQ_t
  float Lq[kQStages][64];
  float Dq[kQStages][64];
  uint64_t bar_kv, bar_full[kQStages], bar_empty[kQStages];
  uint64_t bar_sa[2], bar_ew[2], bar_b[2], bar_dq, bar_dqfree;
  uint32_t tmem_base;
  int abort;
  int q_first, n_q;
};
static_assert(offsetof(BwdSmem, V) % 1024 == 0 && offsetof(BwdSmem, Q) % 1024 == 0 &&
                  offsetof(BwdSmem, dO) % 1024 == 0 && offsetof(BwdSmem, dST) % 1024 == 0 && offsetof(BwdSmem, Lq) % 16 == 0 &&
                  offsetof(BwdSmem, Dq) % 16 == 0,
              "TMA / UMMA operands with the 128-byte swizzle need 1024-byte alignment");

struct LongBwdArgs {
  const float* lse;           // [nseq, H, S]
  const float* dsum;          // [nseq, H, S]  D = rowsum(dO * O)
  float* dq;                  // [nseq * S, E] fp32 accumulator (zeroed)
  __nv_bfloat16* dqkv;
  const int32_t* bid;         // [nseq - n_causal, S]
  const int32_t* first;       // [nseq - n_causal, S]
  const int32_t* q_lo;        // [nseq - n_causal][2 * nt64] (+ nt64 within a sequence's slice)
  const float* rope;
  int S, H, n_causal, nt64;
};

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_long_kernel(const __grid_constant__ CUtensorMap tqkv, const __grid_constant__ CUtensorMap tdo,
                         const __grid_constant__ CUtensorMap tdq, const LongBwdArgs a) {
  extern __shared__ uint8_t raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int kt = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int S = a.S, E = a.H * kHd;
  const long long ld = 3ll * E;
  const bool prefix = seq >= a.n_causal;
  const int pseq = seq - a.n_causal;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_base = seq * S;
  const long long lrow = ((long long)seq * a.H + h) * S;
  volatile int* abort_flag = &sm.abort;
  const int nqt = (S + kBQ - 1) / kBQ;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_kv, 1);
    for (int b = 0; b < kQStages; ++b) {
      mbar_init(&sm.bar_full[b], 1);
      mbar_init(&sm.bar_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.bar_sa[b], 1);
      mbar_init(&sm.bar_ew[b], 512);
      mbar_init(&sm.bar_b[b], 1);
    }
    mbar_init(&sm.bar_dq, 1);
    mbar_init(&sm.bar_dqfree, 512);
    sm.abort = 0;
    // first query tile that can see this key tile: causal -> the diagonal one;
    // prefix -> the lowest query row of the key rows' blocks (metadata)
    int q0 = kt * kBQ;
    if (prefix) {
      const int* ql = a.q_lo + (long long)pseq * 2 * a.nt64 + a.nt64;
      for (int t = 2 * kt; t < min(2 * kt + 2, a.nt64); ++t) q0 = min(q0, ql[t]);
    }
    sm.q_first = q0 / kBQ;
    sm.n_q = nqt - q0 / kBQ;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int q_first = sm.q_first, n_q = sm.n_q;
  const int ns = 2 * n_q;  // 64-query sub-tiles

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tqkv);
      prefetch_tmap(&tdo);
      prefetch_tmap(&tdq);
      mbar_arrive_expect_tx(&sm.bar_kv, 4 * kTileBytes);
      for (int t = 0; t < 2; ++t) {
        const int r0 = row_base + kt * kBK + t * 64;
        tma_load_2d(sm.K + t * kTileBytes, &tqkv, &sm.bar_kv, E + h * kHd, r0);
        tma_load_2d(sm.V + t * kTileBytes, &tqkv, &sm.bar_kv, 2 * E + h * kHd, r0);
      }
      for (int s = 0; s < ns; ++s) {
        const int st = s % kQStages;
        const int q64 = 2 * q_first + s;  // 64-query block within the sequence
        // L / D entries of the sub-tile inside the sequence (S % 4 == 0: a multiple of 16 bytes)
        const int nld = max(0, min(64, S - q64 * 64));
        const uint32_t ld_bytes = (uint32_t)nld * 4u;
        mbar_wait(&sm.bar_empty[st], ((s / kQStages) & 1) ^ 1u, abort_flag);
        mbar_arrive_expect_tx(&sm.bar_full[st], 2 * kTileBytes + 2 * ld_bytes);
        tma_load_2d(sm.Q[st], &tqkv, &sm.bar_full[st], h * kHd, row_base + q64 * 64);
        tma_load_2d(sm.dO[st], &tdo, &sm.bar_full[st], h * kHd, row_base + q64 * 64);
        if (nld > 0) {
          bulk_load_1d(sm.Lq[st], a.lse + lrow + q64 * 64, ld_bytes, &sm.bar_full[st]);
          bulk_load_1d(sm.Dq[st], a.dsum + lrow + q64 * 64, ld_bytes, &sm.bar_full[st]);
        }
      }
    }
  } else if (warp == 1) {
    {  // the whole warp runs the issue loop; one elected lane issues (uniform operands)
      const uint32_t kb = smem_u32(sm.K), vb = smem_u32(sm.V);
      const uint32_t id_s = make_idesc_bf16(128, 64, false, false);   // N = 64 queries
      const uint32_t id_kn = make_idesc_bf16(128, kHd, false, true);  // dV, dK: B read MN-major
      const uint32_t id_nn = make_idesc_bf16(128, kHd, true, true);   // dQ: A (dS) and B (K) MN-major
      mbar_wait(&sm.bar_kv, 0, abort_flag);
      auto issue_a = [&](int s) {
        const int st = s % kQStages, b = s & 1;
        mbar_wait(&sm.bar_full[st], (s / kQStages) & 1, abort_flag);
        tc_fence_after();
        const uint32_t qb = smem_u32(sm.Q[st]), ob = smem_u32(sm.dO[st]);
        #pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          umma_f16_w(tmem + b * 128, make_sdesc(kb + kk * 32, 16, 1024), make_sdesc(qb + kk * 32, 16, 1024), id_s,
                   kk > 0 ? 1u : 0u);
          umma_f16_w(tmem + b * 128 + 64, make_sdesc(vb + kk * 32, 16, 1024), make_sdesc(ob + kk * 32, 16, 1024),
                   id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit_w(&sm.bar_sa[b]);
      };
      if (ns > 0) issue_a(0);
      if (ns > 1) issue_a(1);
      for (int s = 0; s < ns; ++s) {
        const int t = s >> 1, hh = s & 1, b = s & 1, st = s % kQStages;
        mbar_wait(&sm.bar_ew[b], (s >> 1) & 1, abort_flag);
        tc_fence_after();
        const uint32_t qb = smem_u32(sm.Q[st]), ob = smem_u32(sm.dO[st]);
        #pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 64 queries: A = P^T / dS^T columns of 16 queries in TMEM
          const uint32_t acc = (s > 0 || kk > 0) ? 1u : 0u;
          umma_f16_ts_w(tmem + 256, tmem + 448 + kk * 8, make_sdesc(ob + kk * 2048, 8192, 1024), id_kn, acc);
          umma_f16_ts_w(tmem + 320, tmem + 480 + kk * 8, make_sdesc(qb + kk * 2048, 8192, 1024), id_kn, acc);
        }
        tc_commit_w(&sm.bar_b[b]);
        tc_commit_w(&sm.bar_empty[st]);
        if (hh == 1) {
          // dQ_t = dS K: A = the tile's dS^T pair read MN-major (queries 0-63 | 64-127)
          if (t >= 1) mbar_wait(&sm.bar_dqfree, (t - 1) & 1, abort_flag);
          tc_fence_after();
          const uint32_t pair = smem_u32(sm.dST[t & 1][0]);
          #pragma unroll
          for (int kk = 0; kk < 8; ++kk)  // 128 keys
            umma_f16_w(tmem + 384, make_sdesc(pair + kk * 2048, 16384, 1024), make_sdesc(kb + kk * 2048, 8192, 1024),
                     id_nn, kk > 0 ? 1u : 0u);
          tc_commit_w(&sm.bar_dq);
        }
        if (s + 2 < ns) issue_a(s + 2);
      }
    }
  } else {
    const int ew = warp - 2;
    const int g = ew >> 2;  // 16-query column group of a sub-tile
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sl2 = 0.125f * kLog2e;
    const int j = kt * kBK + r;  // this thread's key
    const bool jok = j < S;
    const int32_t* bidrow = prefix ? a.bid + (long long)pseq * S : nullptr;
    const int fj = jok ? (prefix ? a.first[(long long)pseq * S + j] : j) : S;
    const int bj = (jok && prefix) ? bidrow[j] : -2;
    const bool leader = threadIdx.x == 64;
    // dQ of query tile t: TMEM (lane = query row) -> the tile's dS^T pair as two
    // swizzled [128 rows x 32 dims] fp32 boxes -> bulk reduce-add (rows past S
    // are 0: their dS columns are masked)
    auto dq_flush = [&](int t) {
      mbar_wait(&sm.bar_dq, t & 1, abort_flag);
      tc_fence_after();
      uint32_t dqv[16];
      tmem_ld_x16_nowait(tmem + lane_off + 384 + g * 16, dqv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&sm.bar_dqfree);
      uint8_t* box = sm.dST[t & 1][g >> 1];
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int chunk = (g & 1) * 4 + q;  // 16-byte chunk of the 128-byte row
        *reinterpret_cast<uint4*>(box + r * 128 + ((chunk ^ (r & 7)) << 4)) =
            make_uint4(dqv[4 * q], dqv[4 * q + 1], dqv[4 * q + 2], dqv[4 * q + 3]);
      }
      fence_proxy_async();
      asm volatile("bar.sync 1, 512;" ::: "memory");
      if (leader) {
        const int y = row_base + (q_first + t) * kBQ;
        tma_reduce_add_2d(&tdq, sm.dST[t & 1][0], h * kHd, y);
        tma_reduce_add_2d(&tdq, sm.dST[t & 1][1], h * kHd + 32, y);
        bulk_commit();
      }
    };
    for (int s = 0; s < ns; ++s) {
      const int t = s >> 1, hh = s & 1, b = s & 1, st = s % kQStages;
      const int qb = (q_first + t) * kBQ + hh * 64 + g * 16;  // this thread's 16 queries
      const bool full = jok && qb >= j && qb + 15 < S;
      const bool none = !jok || qb + 15 < fj || qb >= S;
      const bool none_w = __all_sync(0xffffffffu, none);
      if (hh == 0 && t >= 2) {
        // the dS^T pair of this tile parity staged dQ_{t-2}: its reduce must have read it
        if (leader) bulk_wait_read0();
        asm volatile("bar.sync 1, 512;" ::: "memory");
      }
      mbar_wait(&sm.bar_sa[b], (s >> 1) & 1, abort_flag);
      tc_fence_after();
      uint32_t pk[8], dk[8];
      if (none_w || none) {
        #pragma unroll
        for (int e = 0; e < 8; ++e) pk[e] = dk[e] = 0u;
      }
      if (!none_w) {
        uint32_t su[16], du[16];
        tmem_ld_x16_nowait(tmem + lane_off + b * 128 + g * 16, su);
        tmem_ld_x16_nowait(tmem + lane_off + b * 128 + 64 + g * 16, du);
        tmem_wait_ld();
        if (!none) {
          // L and D of these 16 queries from the staged sub-tile (broadcast reads;
          // entries past S are stale but their elements are masked)
          float Lv[16], Dv[16];
          const float4* L4 = reinterpret_cast<const float4*>(sm.Lq[st] + g * 16);
          const float4* D4 = reinterpret_cast<const float4*>(sm.Dq[st] + g * 16);
          #pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const float4 l4 = L4[e4], d4 = D4[e4];
            Lv[e4 * 4] = l4.x; Lv[e4 * 4 + 1] = l4.y; Lv[e4 * 4 + 2] = l4.z; Lv[e4 * 4 + 3] = l4.w;
            Dv[e4 * 4] = d4.x; Dv[e4 * 4 + 1] = d4.y; Dv[e4 * 4 + 2] = d4.z; Dv[e4 * 4 + 3] = d4.w;
          }
          #pragma unroll
          for (int e = 0; e < 16; e += 2) {
            float pv[2], dsv[2];
            #pragma unroll
            for (int k = 0; k < 2; ++k) {
              const float p = ex2_approx(fmaf(__uint_as_float(su[e + k]), sl2, -Lv[e + k]));
              pv[k] = p;
              dsv[k] = p * (__uint_as_float(du[e + k]) - Dv[e + k]);
              if (!full) {
                const int i = qb + e + k;
                const bool vis = i < S && (i >= j || (i >= fj && bidrow != nullptr && bidrow[i] == bj));
                pv[k] = vis ? pv[k] : 0.f;
                dsv[k] = vis ? dsv[k] : 0.f;
              }
            }
            pk[e >> 1] = pack_bf16(pv[0], pv[1]);
            dk[e >> 1] = pack_bf16(dsv[0], dsv[1]);
          }
        }
      }
      uint8_t* dst = sm.dST[t & 1][hh];
      #pragma unroll
      for (int q = 0; q < 2; ++q)
        *reinterpret_cast<uint4*>(dst + sw128(r, g * 16 + q * 8)) =
            make_uint4(dk[4 * q], dk[4 * q + 1], dk[4 * q + 2], dk[4 * q + 3]);
      // P^T, dS^T (bf16 pairs) into TMEM once B(s-1) has read the previous ones
      if (s >= 1) mbar_wait(&sm.bar_b[(s - 1) & 1], ((s - 1) >> 1) & 1, abort_flag);
      tc_fence_after();
      tmem_st_x8(tmem + lane_off + 448 + g * 8, pk);
      tmem_st_x8(tmem + lane_off + 480 + g * 8, dk);
      tmem_wait_st();
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.bar_ew[b]);
      if (hh == 0 && t >= 1) dq_flush(t - 1);
    }
    if (n_q > 0) {
      dq_flush(n_q - 1);
      mbar_wait(&sm.bar_b[(ns - 1) & 1], ((ns - 1) >> 1) & 1, abort_flag);  // dV, dK complete
      tc_fence_after();
      uint32_t vv[16], kv[16];
      tmem_ld_x16_nowait(tmem + lane_off + 256 + g * 16, vv);
      tmem_ld_x16_nowait(tmem + lane_off + 320 + g * 16, kv);
      tmem_wait_ld();
      if (leader) bulk_wait0();
      if (jok) {
        float dkf[16];
        #pragma unroll
        for (int e = 0; e < 16; ++e) dkf[e] = __uint_as_float(kv[e]) * 0.125f;
        if (a.rope != nullptr) {
          const float4* cs = reinterpret_cast<const float4*>(a.rope + ((long long)j * 32 + g * 8) * 2);
          #pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float4 t = cs[p];
            float x0 = dkf[4 * p], x1 = dkf[4 * p + 1];
            dkf[4 * p] = x0 * t.x + x1 * t.y;
            dkf[4 * p + 1] = x1 * t.x - x0 * t.y;
            x0 = dkf[4 * p + 2];
            x1 = dkf[4 * p + 3];
            dkf[4 * p + 2] = x0 * t.z + x1 * t.w;
            dkf[4 * p + 3] = x1 * t.z - x0 * t.w;
          }
        }
        __nv_bfloat16* rowp = a.dqkv + (long long)(row_base + j) * ld;
        uint4* dkp = reinterpret_cast<uint4*>(rowp + E + h * kHd + g * 16);
        uint4* dvp = reinterpret_cast<uint4*>(rowp + 2 * E + h * kHd + g * 16);
        #pragma unroll
        for (int q = 0; q < 2; ++q) {
          dkp[q] = make_uint4(pack_bf16(dkf[8 * q], dkf[8 * q + 1]), pack_bf16(dkf[8 * q + 2], dkf[8 * q + 3]),
                              pack_bf16(dkf[8 * q + 4], dkf[8 * q + 5]), pack_bf16(dkf[8 * q + 6], dkf[8 * q + 7]));
          dvp[q] = make_uint4(pack_bf16(__uint_as_float(vv[8 * q]), __uint_as_float(vv[8 * q + 1])),
                              pack_bf16(__uint_as_float(vv[8 * q + 2]), __uint_as_float(vv[8 * q + 3])),
                              pack_bf16(__uint_as_float(vv[8 * q + 4]), __uint_as_float(vv[8 * q + 5])),
                              pack_bf16(__uint_as_float(vv[8 * q + 6]), __uint_as_float(vv[8 * q + 7])));
        }
      }
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

// D[seq, h, i] = sum_d O[row, h*64+d] * dO[row, h*64+d]; one warp per row, a
// lane covers half a head (32 dims).
__global__ void attn_dsum_kernel(const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ dout,
                                 float* __restrict__ dsum, long long T, int S, int H) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= T) return;
  const int E = H * kHd;
  for (int c0 = lane * 32; c0 < E; c0 += 32 * 32) {
    const uint4* po = reinterpret_cast<const uint4*>(out + row * E + c0);
    const uint4* pd = reinterpret_cast<const uint4*>(dout + row * E + c0);
    float d = 0.f;
    #pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 wo = po[q], wd = pd[q];
      const __nv_bfloat162* ho = reinterpret_cast<const __nv_bfloat162*>(&wo);
      const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&wd);
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fo = __bfloat1622float2(ho[e]), fd = __bfloat1622float2(hd[e]);
        d = fmaf(fo.x, fd.x, fmaf(fo.y, fd.y, d));
      }
    }
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    if ((lane & 1) == 0) {
      const int hh = c0 / kHd;
      const long long seq = row / S, i = row - seq * S;
      dsum[(seq * H + hh) * S + i] = d;
    }
  }
}

// dqkv[row, h*64 + d] (q part) = unrope(dq[row, ...] / 8), pairs of dims per thread.
__global__ void attn_dq_finish_kernel(const float* __restrict__ dq, __nv_bfloat16* __restrict__ dqkv,
                                      const float* __restrict__ rope, long long T, int S, int E) {
  const long long n = T * (E / 2);
  for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (long long)gridDim.x * blockDim.x) {
    const long long row = p / (E / 2);
    const int c = (int)(p - row * (E / 2)) * 2;
    const float2 v = *reinterpret_cast<const float2*>(dq + row * E + c);
    float x0 = v.x * 0.125f, x1 = v.y * 0.125f;
    if (rope != nullptr) {
      const int pos = (int)(row % S);
      const float2 t = *reinterpret_cast<const float2*>(rope + ((long long)pos * 32 + ((c & 63) >> 1)) * 2);
      const float y0 = x0 * t.x + x1 * t.y, y1 = x1 * t.x - x0 * t.y;
      x0 = y0;
      x1 = y1;
    }
    *reinterpret_cast<uint32_t*>(dqkv + row * 3ll * E + c) = pack_bf16(x0, x1);
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

namespace cdk {
// D[seq, h, i] = rowsum(dO * O) of every query row (the pass before the backward kernels).
int launch_attn_dsum(const void* out, const void* dout, float* dsum, int64_t T, int64_t S, int64_t H,
                     cudaStream_t stream) {
  tclong::attn_dsum_kernel<<<(unsigned)((T + 7) / 8), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(out), reinterpret_cast<const __nv_bfloat16*>(dout), dsum, T, (int)S,
      (int)H);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

// Host launcher used by cdk_attn_bwd for S > 256 (workspace: fp32 [nseq*S, E]).
int launch_attn_bwd_long(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum,
                         void* dqkv, int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                         const int32_t* meta, const float* rope, void* workspace, cudaStream_t stream) {
  using namespace tclong;
  if (S <= 0 || !workspace) return -20;
  const int64_t E = H * kHd, T = nseq * S;
  if (S % 4) return -23;  // the L / D tiles are bulk-copied in 16-byte units
  CUtensorMap tq, tdo, tdq;
  if (!make_tmap(&tq, qkv, 3 * E, T, 3 * E, 64, 64)) return -21;
  if (!make_tmap(&tdo, dout, E, T, E, 64, 64)) return -21;
  if (!make_tmap_f32(&tdq, workspace, E, T, E, 32, 128)) return -21;
  cudaError_t e = cudaMemsetAsync(workspace, 0, (size_t)T * E * sizeof(float), stream);
  if (e != cudaSuccess) return (int)e;
  attn_dsum_kernel<<<(unsigned)((T + 7) / 8), 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(out),
                                                                  reinterpret_cast<const __nv_bfloat16*>(dout),
                                                                  dsum, T, (int)S, (int)H);
  LongBwdArgs a;
  a.lse = lse;
  a.dsum = dsum;
  a.dq = reinterpret_cast<float*>(workspace);
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv);
  const int64_t np = nseq - n_causal;
  const int nt64 = (int)((S + 63) / 64);
  a.bid = bid;
  a.q_lo = meta;
  a.first = np > 0 ? meta + np * 2 * nt64 : nullptr;
  a.rope = rope;
  a.S = (int)S;
  a.H = (int)H;
  a.n_causal = (int)n_causal;
  a.nt64 = nt64;
  const size_t smem = sizeof(BwdSmem) + 1024;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    e = cudaFuncSetAttribute(attn_bwd_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_bwd_long_kernel, kBwdThreads, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm * 512 > 512) return -22;
    attr_done[dev] = true;
  }
  attn_bwd_long_kernel<<<dim3((unsigned)((S + kBK - 1) / kBK), (unsigned)H, (unsigned)nseq), kBwdThreads, smem,
                         stream>>>(tq, tdo, tdq, a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  long long blocks = (T * (E / 2) + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  attn_dq_finish_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a.dq, a.dqkv, rope, T, (int)S, (int)E);
  e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}
}  // namespace cdk
