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

}  // namespace tcattn

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
