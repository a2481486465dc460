// Tensor-core (tcgen05 + TMEM) attention for sequences of at most 256 tokens,
// head_dim 64 -- the pretraining shape of the reference model
// (chessdecoder/train/config.yaml: max_seq_len 256; masks of
// chessdecoder/models/model.py:158-171).
//
// One CTA per (128-row query tile, head, sequence); two CTAs share an SM so
// that one's TMA loads overlap the other's softmax.  TMA brings the query
// tile and the key/value tiles it may see (64 rows x 128 B, 128-byte swizzle)
// into shared memory.  Then:
//   1. one thread issues S = Q K^T as tcgen05.mma (M=128, N=keys<=256, K=64)
//      into TMEM;
//   2. four softmax warps (one TMEM lane = one query row per thread) read the
//      whole score row back with tcgen05.ld, apply the causal / block-prefix
//      mask and a single-pass softmax (the full row is resident, so no online
//      rescaling), and write P in bf16 into a 128-byte-swizzled K-major
//      shared-memory operand;
//   3. O = P V is issued as tcgen05.mma (M=128, N=64, K=keys, V read
//      MN-major straight from its TMA tile) into a second TMEM region;
//   4. the same warps scale O by 1/rowsum and store it, plus the base-2
//      log-sum-exp that the backward needs.
// Warp roles (192 threads): thread 0 = barriers + TMA, warp 1 = TMEM
// allocation + MMA issue, warps 2-5 = softmax / epilogue.  All waits are
// bounded (cdk_common).
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {

namespace tcattn {

constexpr int kHd = 64;
constexpr int kTileRows = 64;
constexpr int kMaxS = 256;
constexpr int kTiles = kMaxS / kTileRows;  // 4 TMA tiles per operand
constexpr int kTileBytes = kTileRows * 128;
constexpr float kLog2e = 1.4426950408889634f;

struct Args {
  __nv_bfloat16* out;
  float* lse;
  const int32_t* bid;   // [nseq - n_causal, S]
  const int32_t* last;  // [nseq - n_causal, S] per-row last index of the row's block
  const int32_t* tile_kv_hi;  // [nseq - n_causal][2 * nt64]: exclusive key bound per 64-row query tile
  int S, H, n_causal, nt64;
};

// Shared memory of the forward (one 128-row query tile per CTA, ~97 KB so that
// two CTAs share an SM).  The first 64 KB hold the Q tile (16 KB) and the K
// tiles (up to 32 KB) until S = Q K^T has retired, then P (4 key blocks of
// [128 rows x 64 keys], 128-byte swizzle).
struct FwdSmem {
  uint8_t qkp[4 * 128 * 128];
  uint8_t V[kTiles][kTileBytes];
  uint64_t bar_q, bar_k, bar_v, bar_s, bar_p, bar_o;
  uint32_t tmem_base;
  int abort;
  int n_keys;                      // keys (multiple of 32) this query tile may see
  int32_t bid[kMaxS];
  int32_t hi[kMaxS];               // max(i, last[i]): no key beyond it is visible to row i
};
constexpr int kQOff = 0;
constexpr int kKOff = 16384;

// Byte offset of element (row r, col c) of a [rows x 64] bf16 operand block
// stored with the 128-byte swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Visibility of key j to query row i (i < S), given hi = max(i, last[i]).
__device__ __forceinline__ bool visible(int i, int j, int S, int hi, int my_bid, const int32_t* bid) {
  return j < S && (j <= i || (j <= hi && bid[j] == my_bid));
}

constexpr int kFwdThreads = 192;  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 softmax / epilogue

__global__ void __launch_bounds__(kFwdThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tqkv, const Args a) {
  extern __shared__ uint8_t raw[];
  FwdSmem& sm = *reinterpret_cast<FwdSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int mt = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int S = a.S, E = a.H * kHd;
  const int nt = (S + kTileRows - 1) / kTileRows;
  const bool prefix = seq >= a.n_causal;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_base = seq * S;
  const int pseq = seq - a.n_causal;
  volatile int* abort_flag = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_q, 1);
    mbar_init(&sm.bar_k, 1);
    mbar_init(&sm.bar_v, 1);
    mbar_init(&sm.bar_s, 1);
    mbar_init(&sm.bar_p, 128);
    mbar_init(&sm.bar_o, 1);
    sm.abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tqkv);
    // Q rows [128 mt, 128 mt + 128): one or two 64-row tiles
    const int qt0 = 2 * mt, nq = min(2, nt - qt0);
    mbar_arrive_expect_tx(&sm.bar_q, nq * kTileBytes);
    for (int t = 0; t < nq; ++t)
      tma_load_2d(sm.qkp + kQOff + t * kTileBytes, &tqkv, &sm.bar_q, h * kHd, row_base + (qt0 + t) * kTileRows);
    // keys this tile may see: per-64-row-tile bounds from the metadata
    int kv = min(S, (mt + 1) * 128);
    if (prefix) {
      const int* kvhi = a.tile_kv_hi + (long long)pseq * 2 * a.nt64;
      for (int t = qt0; t < qt0 + nq; ++t) kv = max(kv, kvhi[t]);
    }
    const int nk = min(kMaxS, (min(kv, S) + 31) / 32 * 32);
    sm.n_keys = nk;
    const int kt = (nk + kTileRows - 1) / kTileRows;
    mbar_arrive_expect_tx(&sm.bar_k, kt * kTileBytes);
    for (int t = 0; t < kt; ++t)
      tma_load_2d(sm.qkp + kKOff + t * kTileBytes, &tqkv, &sm.bar_k, E + h * kHd, row_base + t * kTileRows);
    mbar_arrive_expect_tx(&sm.bar_v, kt * kTileBytes);
    for (int t = 0; t < kt; ++t)
      tma_load_2d(sm.V[t], &tqkv, &sm.bar_v, 2 * E + h * kHd, row_base + t * kTileRows);
  }
  for (int i = threadIdx.x; i < kMaxS; i += blockDim.x) {
    sm.bid[i] = i < S ? (prefix ? a.bid[(long long)pseq * S + i] : i) : -1;
    sm.hi[i] = i < S ? max(i, prefix ? a.last[(long long)pseq * S + i] : i) : -1;
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;  // S in columns [0, nk); O reuses [0, 64) once P is out
  const int nk = sm.n_keys;

  if (warp == 1) {
    if (lane == 0) {
      mbar_wait(&sm.bar_q, 0, abort_flag);
      mbar_wait(&sm.bar_k, 0, abort_flag);
      tc_fence_after();
      const uint32_t idesc_s = make_idesc_bf16(128, nk, false, false);
      const uint32_t qa = smem_u32(sm.qkp + kQOff);
      const uint32_t kb = smem_u32(sm.qkp + kKOff);
      #pragma unroll
      for (int kk = 0; kk < kHd / 16; ++kk)
        umma_f16(tmem, make_sdesc(qa + kk * 32, 16, 1024), make_sdesc(kb + kk * 32, 16, 1024), idesc_s,
                 kk > 0 ? 1u : 0u);
      tc_commit(&sm.bar_s);
      mbar_wait(&sm.bar_p, 0, abort_flag);
      mbar_wait(&sm.bar_v, 0, abort_flag);
      tc_fence_after();
      const uint32_t idesc_o = make_idesc_bf16(128, kHd, false, true);
      const uint32_t pb = smem_u32(sm.qkp);
      const uint32_t vb = smem_u32(sm.V[0]);
      for (int kk = 0; kk < nk / 16; ++kk) {
        const uint64_t ad = make_sdesc(pb + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = make_sdesc(vb + kk * 16 * 128, 8192, 1024);
        umma_f16(tmem, ad, bd, idesc_o, kk > 0 ? 1u : 0u);
      }
      tc_commit(&sm.bar_o);
    }
  } else if (warp >= 2) {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float sl2 = 0.125f * kLog2e;
    const int i = mt * 128 + r;
    const bool row_ok = i < S;
    const int my_bid = row_ok ? sm.bid[i] : -2;
    const int hi = row_ok ? sm.hi[i] : -1;
    const int i_eff = row_ok ? i : -1;
    const int nch = nk / 32;
    // tcgen05.ld is warp-collective (.sync.aligned): every load decision below
    // uses the warp-uniform bound hi_w; per-row bounds only steer arithmetic.
    int hi_w = hi;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) hi_w = max(hi_w, __shfl_xor_sync(0xffffffffu, hi_w, o));
    mbar_wait(&sm.bar_s, 0, abort_flag);
    tc_fence_after();
    // pass 1: max of the raw scores of keys [0, hi] (exact for contiguous
    // blocks, an upper bound otherwise -- either keeps exp2 <= 1)
    float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int c = 0; c < nch; c += 2) {
      if (c * 32 > hi_w) break;
      uint32_t u0[32], u1[32];
      tmem_ld_x32_nowait(trow + c * 32, u0);
      if (c + 1 < nch) tmem_ld_x32_nowait(trow + (c + 1) * 32, u1);
      tmem_wait_ld();
      #pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int base = (c + half) * 32;
        if (c + half >= nch || base > hi) break;
        const uint32_t* u = half ? u1 : u0;
        if (base + 31 <= hi) {
          #pragma unroll
          for (int e = 0; e < 32; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(u[e]));
        } else {
          #pragma unroll
          for (int e = 0; e < 32; ++e)
            if (base + e <= hi) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(u[e]));
        }
      }
    }
    const float ms = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
    // pass 2: probabilities -> bf16 P operand (overwrites Q/K), row sum
    float l4[4] = {0.f, 0.f, 0.f, 0.f};
    uint8_t* P = sm.qkp;
    for (int c = 0; c < nch; c += 2) {
      uint32_t u0[32], u1[32];
      const bool any0 = c * 32 <= hi_w;                      // warp-uniform
      const bool any1 = c + 1 < nch && (c + 1) * 32 <= hi_w;  // warp-uniform
      if (any0) tmem_ld_x32_nowait(trow + c * 32, u0);
      if (any1) tmem_ld_x32_nowait(trow + (c + 1) * 32, u1);
      tmem_wait_ld();
      #pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int cc = c + half;
        if (cc >= nch) break;
        const uint32_t* u = half ? u1 : u0;
        const int base = cc * 32;
        uint32_t pk[16];
        if (base + 31 <= i_eff) {
          #pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float p0 = exp2f(fmaf(__uint_as_float(u[e]), sl2, -ms));
            const float p1 = exp2f(fmaf(__uint_as_float(u[e + 1]), sl2, -ms));
            l4[(e >> 1) & 3] += p0 + p1;
            pk[e >> 1] = pack_bf16(p0, p1);
          }
        } else if (base <= hi) {
          #pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const bool v0 = visible(i, base + e, S, hi, my_bid, sm.bid);
            const bool v1 = visible(i, base + e + 1, S, hi, my_bid, sm.bid);
            const float p0 = v0 ? exp2f(fmaf(__uint_as_float(u[e]), sl2, -ms)) : 0.f;
            const float p1 = v1 ? exp2f(fmaf(__uint_as_float(u[e + 1]), sl2, -ms)) : 0.f;
            l4[(e >> 1) & 3] += p0 + p1;
            pk[e >> 1] = pack_bf16(p0, p1);
          }
        } else {
          #pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = 0u;
        }
        uint8_t* blk = P + (cc >> 1) * (128 * 128);
        const int cbase = (cc & 1) * 32;
        #pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(blk + sw128(r, cbase + q * 8)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
    }
    const float l = (l4[0] + l4[1]) + (l4[2] + l4[3]);
    fence_proxy_async();
    tc_fence_before();
    mbar_arrive(&sm.bar_p);
    // epilogue: O / l
    mbar_wait(&sm.bar_o, 0, abort_flag);
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint32_t o0[32], o1[32];
    tmem_ld_x32_nowait(trow, o0);
    tmem_ld_x32_nowait(trow + 32, o1);
    tmem_wait_ld();
    if (row_ok) {
      uint4* dst = reinterpret_cast<uint4*>(a.out + (long long)(row_base + i) * E + h * kHd);
      #pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t* o = q < 4 ? o0 : o1;
        const int b = (q & 3) * 8;
        dst[q] = make_uint4(pack_bf16(__uint_as_float(o[b]) * inv, __uint_as_float(o[b + 1]) * inv),
                            pack_bf16(__uint_as_float(o[b + 2]) * inv, __uint_as_float(o[b + 3]) * inv),
                            pack_bf16(__uint_as_float(o[b + 4]) * inv, __uint_as_float(o[b + 5]) * inv),
                            pack_bf16(__uint_as_float(o[b + 6]) * inv, __uint_as_float(o[b + 7]) * inv));
      }
      a.lse[((long long)seq * a.H + h) * S + i] = ms + log2f(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ===========================================================================
// Backward.  One CTA per (head, sequence).  Iterates over (128-key tile kt,
// 128-query half qh) pairs that contain any visible (query, key) pair:
//   MMA-A:  S^T = K_kt Q_qh^T and dP^T = V_kt dO_qh^T      (TMEM, 128 cols each)
//   EW:     P^T = exp2(S^T * c - L_q) (masked), dS^T = P^T * (dP^T - D_q),
//           written as bf16 K-major operands (key rows, 128 B = 64 queries)
//   MMA-B:  dV_kt += P^T dO_qh,  dK_kt += dS^T Q_qh,  dQ_qh += dS K_kt
//           (dS read MN-major from the dS^T buffer, dO/Q/K MN-major from
//           their TMA tiles)
// TMEM columns: [0,128) S^T, [128,256) dP^T, [256,320) dV, [320,384) dK,
// [384,512) dQ for the two query halves.  Eight elementwise warps: group g
// (warps 2+4g .. 5+4g) owns query columns [64g, 64g+64) of each half; the
// TMEM lane = key row.  dK and dQ get the 1/sqrt(64) scale and the inverse
// RoPE rotation before their bf16 store.
// ===========================================================================
struct BwdArgs {
  const __nv_bfloat16* out;
  const __nv_bfloat16* dout;
  const float* lse;
  __nv_bfloat16* dqkv;
  const int32_t* bid;
  const int32_t* first;  // [nseq - n_causal, S] first index of the row's block
  const float* rope;
  int S, H, n_causal;
};

struct BwdSmem {
  uint8_t Q[kTiles][kTileBytes];
  uint8_t K[kTiles][kTileBytes];
  uint8_t V[kTiles][kTileBytes];
  uint8_t dO[kTiles][kTileBytes];
  uint8_t PT[2][128 * 128];   // [query block][128 key rows x 64 queries]
  uint8_t dST[2][128 * 128];
  uint64_t bar_load, bar_sa, bar_ew, bar_mb, bar_epi;
  uint32_t tmem_base;
  int abort;
  float D[kMaxS];
  float L[kMaxS];
  int32_t bid[kMaxS];
  int32_t first[kMaxS];
};

constexpr int kBwdThreads = 320;

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tqkv, const __grid_constant__ CUtensorMap tdo,
                       const BwdArgs a) {
  extern __shared__ uint8_t raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int h = blockIdx.x, seq = blockIdx.y;
  const int S = a.S, E = a.H * kHd;
  const long long ld = 3ll * E;
  const bool prefix = seq >= a.n_causal;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_base = seq * S;
  const int pseq = seq - a.n_causal;
  const long long lrow = ((long long)seq * a.H + h) * S;
  volatile int* abort_flag = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar_load, 1);
    mbar_init(&sm.bar_sa, 1);
    mbar_init(&sm.bar_ew, 256);
    mbar_init(&sm.bar_mb, 1);
    mbar_init(&sm.bar_epi, 256);
    sm.abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tqkv);
    prefetch_tmap(&tdo);
    // all four 64-row tiles of every operand: rows past this sequence are the
    // next sequence's (finite) values or TMA zero fill, never stale memory
    mbar_arrive_expect_tx(&sm.bar_load, 4 * kTiles * kTileBytes);
    for (int t = 0; t < kTiles; ++t) {
      const int r0 = row_base + t * kTileRows;
      tma_load_2d(sm.Q[t], &tqkv, &sm.bar_load, h * kHd, r0);
      tma_load_2d(sm.K[t], &tqkv, &sm.bar_load, E + h * kHd, r0);
      tma_load_2d(sm.V[t], &tqkv, &sm.bar_load, 2 * E + h * kHd, r0);
      tma_load_2d(sm.dO[t], &tdo, &sm.bar_load, h * kHd, r0);
    }
  }
  for (int i = threadIdx.x; i < kMaxS; i += blockDim.x) {
    const bool ok = i < S;
    sm.bid[i] = ok ? (prefix ? a.bid[(long long)pseq * S + i] : i) : -1;
    sm.first[i] = ok ? (prefix ? a.first[(long long)pseq * S + i] : i) : S;
    float d = 0.f, l = 0.f;
    if (ok) {
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
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // (key tile, query half) iteration list, identical in every thread
  const int n_kt = (S + 127) / 128;
  uint32_t codes = 0;  // 2 bits per iteration: kt * 2 + qh (kept in a register, not local memory)
  int nit = 0;
  for (int kt = 0; kt < n_kt; ++kt) {
    int mf = S;
    for (int r = lane; r < 128; r += 32) {
      const int j = kt * 128 + r;
      if (j < S) mf = min(mf, sm.first[j]);
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) mf = min(mf, __shfl_xor_sync(0xffffffffu, mf, o));
    for (int qh = 0; qh < n_kt; ++qh)
      if (qh >= kt || mf < (qh + 1) * 128) codes |= (uint32_t)(kt * 2 + qh) << (2 * nit++);
  }

  if (warp == 1) {
    if (lane == 0) {
      mbar_wait(&sm.bar_load, 0, abort_flag);
      tc_fence_after();
      const uint32_t qb = smem_u32(sm.Q[0]), kb = smem_u32(sm.K[0]), vb = smem_u32(sm.V[0]),
                     ob = smem_u32(sm.dO[0]);
      const uint32_t ptb = smem_u32(sm.PT[0]), dsb = smem_u32(sm.dST[0]);
      const uint32_t id_s = make_idesc_bf16(128, 128, false, false);
      const uint32_t id_kn = make_idesc_bf16(128, kHd, false, true);
      const uint32_t id_nn = make_idesc_bf16(128, kHd, true, true);
      auto issue_a = [&](int code) {
        const int kt = code >> 1, qh = code & 1;
        #pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          umma_f16(tmem, make_sdesc(kb + kt * 16384 + kk * 32, 16, 1024),
                   make_sdesc(qb + qh * 16384 + kk * 32, 16, 1024), id_s, kk > 0 ? 1u : 0u);
          umma_f16(tmem + 128, make_sdesc(vb + kt * 16384 + kk * 32, 16, 1024),
                   make_sdesc(ob + qh * 16384 + kk * 32, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&sm.bar_sa);
      };
      issue_a(codes & 3);
      uint32_t q_seen = 0;
      int epi_waits = 0;
      for (int it = 0; it < nit; ++it) {
        const int code = (codes >> (2 * it)) & 3;
        const int kt = code >> 1, qh = code & 1;
        const bool first_of_kt = it == 0 || (((codes >> (2 * (it - 1))) & 3) >> 1) != kt;
        mbar_wait(&sm.bar_ew, it & 1, abort_flag);
        if (first_of_kt && it > 0) mbar_wait(&sm.bar_epi, (epi_waits++) & 1, abort_flag);
        tc_fence_after();
        #pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) {  // 128 queries
          const uint32_t acc_kv = (!first_of_kt || kk > 0) ? 1u : 0u;
          const uint64_t a_pt = make_sdesc(ptb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t a_ds = make_sdesc(dsb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          umma_f16(tmem + 256, a_pt, make_sdesc(ob + qh * 16384 + kk * 2048, 8192, 1024), id_kn, acc_kv);
          umma_f16(tmem + 320, a_ds, make_sdesc(qb + qh * 16384 + kk * 2048, 8192, 1024), id_kn, acc_kv);
        }
        #pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) {  // 128 keys
          const uint32_t acc_q = (((q_seen >> qh) & 1u) || kk > 0) ? 1u : 0u;
          umma_f16(tmem + 384 + qh * kHd, make_sdesc(dsb + kk * 2048, 16384, 1024),
                   make_sdesc(kb + kt * 16384 + kk * 2048, 8192, 1024), id_nn, acc_q);
        }
        q_seen |= 1u << qh;
        tc_commit(&sm.bar_mb);
        if (it + 1 < nit) issue_a((codes >> (2 * (it + 1))) & 3);
      }
    }
  } else if (warp >= 2) {
    const int g = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sl2 = 0.125f * kLog2e;
    for (int it = 0; it < nit; ++it) {
      const int code = (codes >> (2 * it)) & 3;
      const int kt = code >> 1, qh = code & 1;
      const bool last_of_kt = it == nit - 1 || (((codes >> (2 * (it + 1))) & 3) >> 1) != kt;
      const int j = kt * 128 + r;
      const bool jok = j < S;
      const int fj = jok ? sm.first[j] : S;
      const int bj = jok ? sm.bid[j] : -2;
      mbar_wait(&sm.bar_sa, it & 1, abort_flag);
      if (it > 0) mbar_wait(&sm.bar_mb, (it - 1) & 1, abort_flag);
      tc_fence_after();
      uint32_t s0[32], s1[32], d0[32], d1[32];
      tmem_ld_x32_nowait(tmem + lane_off + g * 64, s0);
      tmem_ld_x32_nowait(tmem + lane_off + g * 64 + 32, s1);
      tmem_ld_x32_nowait(tmem + lane_off + 128 + g * 64, d0);
      tmem_ld_x32_nowait(tmem + lane_off + 128 + g * 64 + 32, d1);
      tmem_wait_ld();
      #pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const uint32_t* su = cc ? s1 : s0;
        const uint32_t* du = cc ? d1 : d0;
        const int qb = qh * 128 + g * 64 + cc * 32;
        const bool full = jok && qb >= j && qb + 31 < S;
        const bool none = !jok || qb + 31 < fj || qb >= S;
        uint32_t pk[16], dk[16];
        if (none) {
          #pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = dk[e] = 0u;
        } else {
          // L and D of these 32 queries: the same addresses in every lane (broadcast)
          const float4* L4 = reinterpret_cast<const float4*>(sm.L + qb);
          const float4* D4 = reinterpret_cast<const float4*>(sm.D + qb);
          #pragma unroll
          for (int e4 = 0; e4 < 8; ++e4) {
            const float4 l4 = L4[e4], dd4 = D4[e4];
            const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
            const float dv4[4] = {dd4.x, dd4.y, dd4.z, dd4.w};
            float pv[4], dsv[4];
            #pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int e = e4 * 4 + k;
              const float p = exp2f(fmaf(__uint_as_float(su[e]), sl2, -lv[k]));
              pv[k] = p;
              dsv[k] = p * (__uint_as_float(du[e]) - dv4[k]);
            }
            if (!full) {
              #pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int i = qb + e4 * 4 + k;
                const bool vis = i < S && (i >= j || (i >= fj && sm.bid[i] == bj));
                pv[k] = vis ? pv[k] : 0.f;
                dsv[k] = vis ? dsv[k] : 0.f;
              }
            }
            pk[e4 * 2] = pack_bf16(pv[0], pv[1]);
            pk[e4 * 2 + 1] = pack_bf16(pv[2], pv[3]);
            dk[e4 * 2] = pack_bf16(dsv[0], dsv[1]);
            dk[e4 * 2 + 1] = pack_bf16(dsv[2], dsv[3]);
          }
        }
        #pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t off = sw128(r, cc * 32 + q * 8);
          *reinterpret_cast<uint4*>(sm.PT[g] + off) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          *reinterpret_cast<uint4*>(sm.dST[g] + off) = make_uint4(dk[4 * q], dk[4 * q + 1], dk[4 * q + 2], dk[4 * q + 3]);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.bar_ew);
      if (last_of_kt) {
        // dV_kt, dK_kt complete: group g stores dims [32g, 32g+32)
        mbar_wait(&sm.bar_mb, it & 1, abort_flag);
        tc_fence_after();
        uint32_t vv[32], kv[32];
        tmem_ld_x32_nowait(tmem + lane_off + 256 + g * 32, vv);
        tmem_ld_x32_nowait(tmem + lane_off + 320 + g * 32, kv);
        tmem_wait_ld();
        if (jok) {
          float dkf[32];
          #pragma unroll
          for (int e = 0; e < 32; ++e) dkf[e] = __uint_as_float(kv[e]) * 0.125f;
          if (a.rope != nullptr) {
            const float2* cs = reinterpret_cast<const float2*>(a.rope + ((long long)j * 32 + g * 16) * 2);
            #pragma unroll
            for (int p = 0; p < 16; ++p) {
              const float2 t = cs[p];
              const float x0 = dkf[2 * p], x1 = dkf[2 * p + 1];
              dkf[2 * p] = x0 * t.x + x1 * t.y;
              dkf[2 * p + 1] = x1 * t.x - x0 * t.y;
            }
          }
          __nv_bfloat16* rowp = a.dqkv + (long long)(row_base + j) * ld;
          uint4* dkp = reinterpret_cast<uint4*>(rowp + E + h * kHd + g * 32);
          uint4* dvp = reinterpret_cast<uint4*>(rowp + 2 * E + h * kHd + g * 32);
          #pragma unroll
          for (int q = 0; q < 4; ++q) {
            dkp[q] = make_uint4(pack_bf16(dkf[8 * q], dkf[8 * q + 1]), pack_bf16(dkf[8 * q + 2], dkf[8 * q + 3]),
                                pack_bf16(dkf[8 * q + 4], dkf[8 * q + 5]), pack_bf16(dkf[8 * q + 6], dkf[8 * q + 7]));
            dvp[q] = make_uint4(pack_bf16(__uint_as_float(vv[8 * q]), __uint_as_float(vv[8 * q + 1])),
                                pack_bf16(__uint_as_float(vv[8 * q + 2]), __uint_as_float(vv[8 * q + 3])),
                                pack_bf16(__uint_as_float(vv[8 * q + 4]), __uint_as_float(vv[8 * q + 5])),
                                pack_bf16(__uint_as_float(vv[8 * q + 6]), __uint_as_float(vv[8 * q + 7])));
          }
        }
        tc_fence_before();
        mbar_arrive(&sm.bar_epi);
      }
    }
    // dQ for both query halves (lane = query row within the half)
    mbar_wait(&sm.bar_mb, (nit - 1) & 1, abort_flag);
    tc_fence_after();
    for (int qh = 0; qh < n_kt; ++qh) {
      uint32_t qv[32];
      tmem_ld_x32_nowait(tmem + lane_off + 384 + qh * kHd + g * 32, qv);
      tmem_wait_ld();
      const int i = qh * 128 + r;
      if (i < S) {
        float dqf[32];
        #pragma unroll
        for (int e = 0; e < 32; ++e) dqf[e] = __uint_as_float(qv[e]) * 0.125f;
        if (a.rope != nullptr) {
          const float2* cs = reinterpret_cast<const float2*>(a.rope + ((long long)i * 32 + g * 16) * 2);
          #pragma unroll
          for (int p = 0; p < 16; ++p) {
            const float2 t = cs[p];
            const float x0 = dqf[2 * p], x1 = dqf[2 * p + 1];
            dqf[2 * p] = x0 * t.x + x1 * t.y;
            dqf[2 * p + 1] = x1 * t.x - x0 * t.y;
          }
        }
        uint4* dqp = reinterpret_cast<uint4*>(a.dqkv + (long long)(row_base + i) * ld + h * kHd + g * 32);
        #pragma unroll
        for (int q = 0; q < 4; ++q)
          dqp[q] = make_uint4(pack_bf16(dqf[8 * q], dqf[8 * q + 1]), pack_bf16(dqf[8 * q + 2], dqf[8 * q + 3]),
                              pack_bf16(dqf[8 * q + 4], dqf[8 * q + 5]), pack_bf16(dqf[8 * q + 6], dqf[8 * q + 7]));
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

}  // namespace tcattn

// Host launcher used by cdk_attn_bwd for S <= 256.
int launch_attn_bwd_tc(const void* qkv, const void* out, const void* dout, const float* lse, void* dqkv,
                       int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                       const int32_t* meta, const float* rope, cudaStream_t stream) {
  using namespace tcattn;
  if (S > kMaxS || S <= 0) return -20;
  CUtensorMap tq, tdo;
  if (!make_tmap(&tq, qkv, 3 * H * kHd, nseq * S, 3 * H * kHd, 64, 64)) return -21;
  if (!make_tmap(&tdo, dout, H * kHd, nseq * S, H * kHd, 64, 64)) return -21;
  BwdArgs a;
  a.out = reinterpret_cast<const __nv_bfloat16*>(out);
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout);
  a.lse = lse;
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv);
  const int64_t np = nseq - n_causal;
  const int nt64 = (int)((S + kTileRows - 1) / kTileRows);
  a.bid = bid;
  a.first = np > 0 ? meta + np * 2 * nt64 : nullptr;
  a.rope = rope;
  a.S = (int)S;
  a.H = (int)H;
  a.n_causal = (int)n_causal;
  const size_t smem = sizeof(BwdSmem) + 1024;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_bwd_tc_kernel, kBwdThreads, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm * 512 > 512) return -22;
    attr_done[dev] = true;
  }
  attn_bwd_tc_kernel<<<dim3((unsigned)H, (unsigned)nseq), kBwdThreads, smem, stream>>>(tq, tdo, a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

// Host launcher used by cdk_attn_fwd for S <= 256.
int launch_attn_fwd_tc(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S, int64_t H,
                       const int32_t* bid, const int32_t* meta, cudaStream_t stream) {
  using namespace tcattn;
  if (S > kMaxS || S <= 0) return -20;
  CUtensorMap tq;
  if (!make_tmap(&tq, qkv, 3 * H * kHd, nseq * S, 3 * H * kHd, 64, 64)) return -21;
  Args a;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  const int64_t np = nseq - n_causal;
  const int nt64 = (int)((S + kTileRows - 1) / kTileRows);
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
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    // tcgen05.alloc blocks until columns are free: co-resident CTAs must fit in 512 columns
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_fwd_tc_kernel, kFwdThreads, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm * 256 > 512) return -22;
    attr_done[dev] = true;
  }
  attn_fwd_tc_kernel<<<dim3((unsigned)((S + 127) / 128), (unsigned)H, (unsigned)nseq), kFwdThreads, smem, stream>>>(tq,
                                                                                                              a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace cdk
