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
//   2. eight softmax warps (two threads per query row: the TMEM lane is the
//      row, the even / odd 32-key chunks are split between warps w and w+4)
//      read the score row back with tcgen05.ld, apply the causal /
//      block-prefix mask and a single-pass softmax (the full row is
//      resident, so no online rescaling; the two halves exchange their row
//      max and sum through shared memory), and write P in bf16 into a
//      128-byte-swizzled K-major shared-memory operand;
//   3. O = P V is issued as tcgen05.mma (M=128, N=64, K=keys, V read
//      MN-major straight from its TMA tile) into a second TMEM region;
//   4. the same warps scale O by 1/rowsum and store it, plus the base-2
//      log-sum-exp that the backward needs.
// Warp roles (320 threads): thread 0 = barriers + TMA, warp 1 = TMEM
// allocation + MMA issue, warps 2-9 = softmax / epilogue.  All waits are
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
  float red_max[2][128];           // per-half row maxima / sums of the two softmax threads of a row
  float red_sum[2][128];
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

constexpr int kFwdThreads = 320;  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-9 softmax / epilogue

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
    mbar_init(&sm.bar_p, 256);
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
    // Two threads per query row: warps w and w+4 share TMEM lane quadrant
    // (w & 3); half 0 takes the even 32-key chunks, half 1 the odd ones.
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
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
    for (int c = half; c < nch; c += 2) {
      const int base = c * 32;
      if (base > hi_w) break;
      uint32_t u[32];
      tmem_ld_x32_nowait(trow + base, u);
      tmem_wait_ld();
      if (base + 31 <= hi) {
        #pragma unroll
        for (int e = 0; e < 32; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(u[e]));
      } else if (base <= hi) {
        #pragma unroll
        for (int e = 0; e < 32; ++e)
          if (base + e <= hi) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(u[e]));
      }
    }
    sm.red_max[half][r] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float ms = fmaxf(sm.red_max[0][r], sm.red_max[1][r]) * sl2;
    // pass 2: probabilities -> bf16 P operand (overwrites Q/K), partial row sum
    float l4[4] = {0.f, 0.f, 0.f, 0.f};
    uint8_t* P = sm.qkp;
    for (int cc = half; cc < nch; cc += 2) {
      const int base = cc * 32;
      uint32_t u[32];
      const bool any = base <= hi_w;  // warp-uniform
      if (any) {
        tmem_ld_x32_nowait(trow + base, u);
        tmem_wait_ld();
      }
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
    sm.red_sum[half][r] = (l4[0] + l4[1]) + (l4[2] + l4[3]);
    fence_proxy_async();
    tc_fence_before();
    mbar_arrive(&sm.bar_p);
    // epilogue: O / l, half h stores dims [32h, 32h + 32)
    mbar_wait(&sm.bar_o, 0, abort_flag);
    asm volatile("bar.sync 1, 256;" ::: "memory");
    tc_fence_after();
    const float l = sm.red_sum[0][r] + sm.red_sum[1][r];
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint32_t o[32];
    tmem_ld_x32_nowait(trow + half * 32, o);
    tmem_wait_ld();
    if (row_ok) {
      uint4* dst = reinterpret_cast<uint4*>(a.out + (long long)(row_base + i) * E + h * kHd + half * 32);
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int b = q * 8;
        dst[q] = make_uint4(pack_bf16(__uint_as_float(o[b]) * inv, __uint_as_float(o[b + 1]) * inv),
                            pack_bf16(__uint_as_float(o[b + 2]) * inv, __uint_as_float(o[b + 3]) * inv),
                            pack_bf16(__uint_as_float(o[b + 4]) * inv, __uint_as_float(o[b + 5]) * inv),
                            pack_bf16(__uint_as_float(o[b + 6]) * inv, __uint_as_float(o[b + 7]) * inv));
      }
      if (half == 0) a.lse[((long long)seq * a.H + h) * S + i] = ms + log2f(l);
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
  uint64_t bar_load, bar_o, bar_sa, bar_ew, bar_mb, bar_epi;
  uint32_t tmem_base;
  int abort;
  alignas(16) float D[kMaxS];  // read as float4
  alignas(16) float L[kMaxS];
  float Dpart[2][kMaxS];
  int32_t bid[kMaxS];
  int32_t first[kMaxS];
};

static_assert(offsetof(BwdSmem, D) % 16 == 0 && offsetof(BwdSmem, L) % 16 == 0, "D / L are read as float4");
static_assert(offsetof(BwdSmem, PT) % 1024 == 0 && offsetof(BwdSmem, dST) % 1024 == 0,
              "TMA / UMMA operands with the 128-byte swizzle need 1024-byte alignment");

constexpr int kBwdThreads = 576;  // warp 0 TMA, warp 1 TMEM + MMA, warps 2-17 elementwise / epilogue

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tqkv, const __grid_constant__ CUtensorMap tdo,
                       const __grid_constant__ CUtensorMap tout, const BwdArgs a) {
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
    mbar_init(&sm.bar_o, 1);
    mbar_init(&sm.bar_sa, 1);
    mbar_init(&sm.bar_ew, 512);
    mbar_init(&sm.bar_mb, 1);
    mbar_init(&sm.bar_epi, 512);
    sm.abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tqkv);
    prefetch_tmap(&tdo);
    prefetch_tmap(&tout);
    // O (for D = rowsum(dO * O)) goes into the P^T buffer, which is free
    // until the first elementwise phase
    mbar_arrive_expect_tx(&sm.bar_o, kTiles * kTileBytes);
    for (int t = 0; t < kTiles; ++t)
      tma_load_2d(sm.PT[0] + t * kTileBytes, &tout, &sm.bar_o, h * kHd, row_base + t * kTileRows);
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
    sm.L[i] = ok ? a.lse[lrow + i] : 0.f;
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
        for (int kk = 0; kk < 8; ++kk) {
          // three independent accumulation chains interleaved: dV, dK over the
          // 128 queries and dQ over the 128 keys, step kk of each
          const uint32_t acc_kv = (!first_of_kt || kk > 0) ? 1u : 0u;
          const uint64_t a_pt = make_sdesc(ptb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t a_ds = make_sdesc(dsb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          umma_f16(tmem + 256, a_pt, make_sdesc(ob + qh * 16384 + kk * 2048, 8192, 1024), id_kn, acc_kv);
          umma_f16(tmem + 320, a_ds, make_sdesc(qb + qh * 16384 + kk * 2048, 8192, 1024), id_kn, acc_kv);
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
    // 16 elementwise warps: group g = (warp - 2) / 4 owns query columns
    // [32g, 32g + 32) of the 128-query half; the TMEM lane quadrant (warp & 3)
    // is the key row block.
    const int ew = warp - 2;
    const int g = ew >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sl2 = 0.125f * kLog2e;
    {
      // D[i] = rowsum(dO_i * O_i) from the swizzled O (in PT) and dO tiles:
      // two threads per row, 32 dims each; rows >= S get 0
      const int t = ew * 32 + lane;  // 0..511
      const int i = t & 255, part = t >> 8;
      mbar_wait(&sm.bar_load, 0, abort_flag);
      mbar_wait(&sm.bar_o, 0, abort_flag);
      float dsum = 0.f;
      if (i < S) {
        const uint8_t* ot = sm.PT[0] + (i >> 6) * kTileBytes;
        const uint8_t* dt = sm.dO[i >> 6];
        const int rr = i & 63;
        #pragma unroll
        for (int c = part * 4; c < part * 4 + 4; ++c) {
          const uint32_t off = (uint32_t)(rr * 128 + (((c ^ (rr & 7)) & 7) << 4));
          const uint4 wo = *reinterpret_cast<const uint4*>(ot + off);
          const uint4 wd = *reinterpret_cast<const uint4*>(dt + off);
          const __nv_bfloat162* ho = reinterpret_cast<const __nv_bfloat162*>(&wo);
          const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&wd);
          #pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fo = __bfloat1622float2(ho[e]), fd = __bfloat1622float2(hd[e]);
            dsum = fmaf(fo.x, fd.x, fmaf(fo.y, fd.y, dsum));
          }
        }
      }
      sm.Dpart[part][i] = dsum;
      asm volatile("bar.sync 1, 512;" ::: "memory");
      if (t < 256) sm.D[t] = sm.Dpart[0][t] + sm.Dpart[1][t];
      // all D written and all O reads done before P^T overwrites the buffer
      asm volatile("bar.sync 1, 512;" ::: "memory");
    }
    for (int it = 0; it < nit; ++it) {
      const int code = (codes >> (2 * it)) & 3;
      const int kt = code >> 1, qh = code & 1;
      const bool last_of_kt = it == nit - 1 || (((codes >> (2 * (it + 1))) & 3) >> 1) != kt;
      const int j = kt * 128 + r;
      const bool jok = j < S;
      const int fj = jok ? sm.first[j] : S;
      const int bj = jok ? sm.bid[j] : -2;
      const int qb = qh * 128 + g * 32;
      // per-thread classification of this 32-query chunk, and its warp-uniform form
      const bool full = jok && qb >= j && qb + 31 < S;
      const bool none = !jok || qb + 31 < fj || qb >= S;
      const bool none_w = __all_sync(0xffffffffu, none);
      mbar_wait(&sm.bar_sa, it & 1, abort_flag);
      if (it > 0) mbar_wait(&sm.bar_mb, (it - 1) & 1, abort_flag);
      tc_fence_after();
      uint8_t* pt = sm.PT[g >> 1];
      uint8_t* dst = sm.dST[g >> 1];
      const int cbase = (g & 1) * 32;
      #pragma unroll
      for (int sc = 0; sc < 2; ++sc) {
        uint32_t pk[8], dk[8];
        if (none_w || none) {
          #pragma unroll
          for (int e = 0; e < 8; ++e) pk[e] = dk[e] = 0u;
        }
        if (!none_w) {
          uint32_t su[16], du[16];
          tmem_ld_x16_nowait(tmem + lane_off + g * 32 + sc * 16, su);
          tmem_ld_x16_nowait(tmem + lane_off + 128 + g * 32 + sc * 16, du);
          tmem_wait_ld();
          if (!none) {
            // L and D of these 16 queries: the same addresses in every lane (broadcast)
            const int q0 = qb + sc * 16;
            const float4* L4 = reinterpret_cast<const float4*>(sm.L + q0);
            const float4* D4 = reinterpret_cast<const float4*>(sm.D + q0);
            #pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
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
                  const int i = q0 + e4 * 4 + k;
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
        }
        #pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t off = sw128(r, cbase + sc * 16 + q * 8);
          *reinterpret_cast<uint4*>(pt + off) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          *reinterpret_cast<uint4*>(dst + off) = make_uint4(dk[4 * q], dk[4 * q + 1], dk[4 * q + 2], dk[4 * q + 3]);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sm.bar_ew);
      if (last_of_kt) {
        // dV_kt, dK_kt complete: group g stores dims [16g, 16g + 16).  The TMEM
        // columns are released (bar_epi) as soon as they are in registers.
        mbar_wait(&sm.bar_mb, it & 1, abort_flag);
        tc_fence_after();
        uint32_t vv[16], kv[16];
        tmem_ld_x16_nowait(tmem + lane_off + 256 + g * 16, vv);
        tmem_ld_x16_nowait(tmem + lane_off + 320 + g * 16, kv);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&sm.bar_epi);
        if (jok) {
          float dkf[16];
          #pragma unroll
          for (int e = 0; e < 16; ++e) dkf[e] = __uint_as_float(kv[e]) * 0.125f;
          if (a.rope != nullptr) {
            const float4* cs = reinterpret_cast<const float4*>(a.rope + ((long long)j * 32 + g * 8) * 2);
            #pragma unroll
            for (int p = 0; p < 4; ++p) {
              const float4 t = cs[p];  // (cos, sin) of two consecutive pairs
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
    // dQ for both query halves (lane = query row within the half); group g
    // stores dims [16g, 16g + 16)
    mbar_wait(&sm.bar_mb, (nit - 1) & 1, abort_flag);
    tc_fence_after();
    for (int qh = 0; qh < n_kt; ++qh) {
      const int i = qh * 128 + r;
      float4 cs[4];
      if (a.rope != nullptr && i < S) {
        const float4* rp = reinterpret_cast<const float4*>(a.rope + ((long long)i * 32 + g * 8) * 2);
        #pragma unroll
        for (int p = 0; p < 4; ++p) cs[p] = rp[p];
      }
      uint32_t qv[16];
      tmem_ld_x16_nowait(tmem + lane_off + 384 + qh * kHd + g * 16, qv);
      tmem_wait_ld();
      if (i < S) {
        float dqf[16];
        #pragma unroll
        for (int e = 0; e < 16; ++e) dqf[e] = __uint_as_float(qv[e]) * 0.125f;
        if (a.rope != nullptr) {
          #pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float4 t = cs[p];
            float x0 = dqf[4 * p], x1 = dqf[4 * p + 1];
            dqf[4 * p] = x0 * t.x + x1 * t.y;
            dqf[4 * p + 1] = x1 * t.x - x0 * t.y;
            x0 = dqf[4 * p + 2];
            x1 = dqf[4 * p + 3];
            dqf[4 * p + 2] = x0 * t.z + x1 * t.w;
            dqf[4 * p + 3] = x1 * t.z - x0 * t.w;
          }
        }
        uint4* dqp = reinterpret_cast<uint4*>(a.dqkv + (long long)(row_base + i) * ld + h * kHd + g * 16);
        #pragma unroll
        for (int q = 0; q < 2; ++q)
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
  CUtensorMap tout;
  if (!make_tmap(&tout, out, H * kHd, nseq * S, H * kHd, 64, 64)) return -21;
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
  attn_bwd_tc_kernel<<<dim3((unsigned)H, (unsigned)nseq), kBwdThreads, smem, stream>>>(tq, tdo, tout, a);
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
