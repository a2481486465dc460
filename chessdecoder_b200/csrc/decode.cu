// KV-cache inference kernels: the batched incremental backbone of
// chessdecoder/cpp/decoder/batched_backbone.cpp over the exported KV-cache
// module chessdecoder/export/backbone_causal.py.
//
// Cache layout in HBM, per cache (causal or prefix) and layer:
//   k, v   bf16 [B][H][max_len][64]   (one 128-byte row per key, per head)
//   valid  u8   [B][max_len]          (key j of sequence b may be attended)
//   len    int32 on the device        (keys [0, len) are in the cache)
// The reference keeps an additive fp32 mask [B, 1, 1, max_seq_len] of 0 / -1e9
// per cache and concatenates fp16 K / V; here the validity is one byte per key
// and the cache is preallocated, so a step writes only its new rows.
//
// Kernels:
//   kv_append     rotary embedding of q and k at explicit per-token positions
//                 (backbone_causal.py:68-77) and the new k / v rows into the
//                 cache at [len, len + S_new) (backbone_causal.py:112-116);
//   decode_attn   softmax(q k^T / 8 + mask) v for S_new new queries per
//                 sequence over the cache keys and the new block
//                 (backbone_causal.py:121-124; masks of batched_backbone.cpp:
//                 117-150 causalForward, 160-177 causalIncremental, 192-205
//                 prefixForward, 207-225 prefixIncremental, 227-258
//                 prefixBlockForward, 264-305 probes);
//   decode_mark   marks keys valid and advances len (markCausalValid,
//                 markCausalValidRange, markPrefixValid(Range) and the cache
//                 length update of forwardImpl).
// The HBM-bound part is decode_attn: it reads each cache key row once per
// (sequence, head, 16-query chunk); kv_append and decode_mark are O(new rows).
#include <algorithm>
#include <cstddef>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "cdk.h"
#include "cdk_common.cuh"

using namespace cdk;

namespace {

constexpr int kHD = 64;      // head dim (embed 1024 / 16 heads)
constexpr int kWarps = 4;    // warps per CTA; each walks its own key tiles
constexpr int kKT = 32;      // keys per warp tile: one key per lane

__device__ __forceinline__ float2 bf2f(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ uint32_t f2bf2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One thread per (token row, head, dim pair): q / k rotated, v copied.
// qkv_f32: the projection output is fp32 [T, ldq] (q | k | v), not rotated;
// otherwise it is bf16 with q / k already rotated (a prefill through the
// training forward) and only the k / v rows are written.
__global__ void kv_append_kernel(const void* __restrict__ qkv, long long ldq, int qkv_f32,
                                 const int32_t* __restrict__ pos, const float* __restrict__ rope, int rope_len,
                                 int S_new, int H, long long max_len, const int32_t* __restrict__ len_dev,
                                 __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                 __nv_bfloat16* __restrict__ q_out, long long ldo, int qkv_out, long long total) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int pair = (int)(idx & 31);
  const long long th = idx >> 5;
  const int h = (int)(th % H);
  const long long t = th / H;
  const long long b = t / S_new;
  const int s = (int)(t % S_new);
  const long long slot = (long long)*len_dev + s;
  const int E = H * kHD;
  const int col = h * kHD + 2 * pair;
  float2 q, k, v;
  if (qkv_f32) {
    const float* row = reinterpret_cast<const float*>(qkv) + t * ldq;
    q = *reinterpret_cast<const float2*>(row + col);
    k = *reinterpret_cast<const float2*>(row + E + col);
    v = *reinterpret_cast<const float2*>(row + 2 * E + col);
    const int p = pos[t];
    if (p < 0 || p >= rope_len) {
      if (pair == 0) report_error(kErrIndex);
      return;
    }
    const float2 cs = *reinterpret_cast<const float2*>(rope + ((long long)p * 32 + pair) * 2);
    q = make_float2(q.x * cs.x - q.y * cs.y, q.y * cs.x + q.x * cs.y);
    k = make_float2(k.x * cs.x - k.y * cs.y, k.y * cs.x + k.x * cs.y);
    *reinterpret_cast<uint32_t*>(q_out + t * ldo + col) = f2bf2(q.x, q.y);
    if (qkv_out) {  // the rotated q | k | v row in the training layout (prefill through attn_fwd)
      *reinterpret_cast<uint32_t*>(q_out + t * ldo + E + col) = f2bf2(k.x, k.y);
      *reinterpret_cast<uint32_t*>(q_out + t * ldo + 2 * E + col) = f2bf2(v.x, v.y);
    }
  } else {
    const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(qkv) + t * ldq;
    k = bf2f(*reinterpret_cast<const uint32_t*>(row + E + col));
    v = bf2f(*reinterpret_cast<const uint32_t*>(row + 2 * E + col));
  }
  if (slot >= max_len) {
    if (pair == 0) report_error(kErrIndex);
    return;
  }
  const long long off = ((b * H + h) * max_len + slot) * kHD + 2 * pair;
  *reinterpret_cast<uint32_t*>(kc + off) = f2bf2(k.x, k.y);
  *reinterpret_cast<uint32_t*>(vc + off) = f2bf2(v.x, v.y);
}

struct DecodeAttnArgs {
  const __nv_bfloat16* q;
  long long ldq;
  long long max_len;
  const int32_t* len_dev;  // cache keys [0, *len_dev) precede the new block
  int S_new;
  int H;
  const uint8_t* valid;    // [B][ldv]
  long long ldv;
  int block_mode;          // CDK_BLOCK_*
  const uint8_t* active;   // [B] or null (all active)
  const int64_t* num_real; // [B] or null (all real): CAUSAL mode
  const uint8_t* full;     // [B][S_new][ldf] explicit mask over all keys, or null
  long long ldf;
  __nv_bfloat16* out;
  long long ldo;
  float scale_log2;        // softmax scale * log2(e)
};

constexpr int kStages = 3;                      // per-warp ring of key tiles
constexpr int kTileBytes = kKT * kHD * 2;       // 4 KB: 32 key rows of 128 bytes
constexpr int kStageBytes = 2 * kTileBytes;     // K tile + V tile
constexpr int kRingBytes = kWarps * kStages * kStageBytes;

// 16-byte chunk c of row r of a 128B-swizzled tile (rows of 128 bytes in a
// 1024-byte-aligned buffer): the TMA SWIZZLE_128B placement.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Several new tokens per sequence (multi-token causal steps, padded prefills,
// prefix / block steps, probes).  Grid (ceil(S_new / 16), H, B), kWarps warps.
// Warp w walks key tiles w, w + kWarps, ... of 32 keys; its lane 0 keeps
// kStages - 1 tiles of K and V in flight by TMA (2-D tiles of the cache viewed
// as [B*H*max_len, 64] bf16, 128-byte swizzle).  Per tile the warp computes the
// 16 x 32 scores S = Q K^T with mma.sync m16n8k16 (K fragments by ldmatrix from
// the swizzled tile), applies the mask and an online softmax per query row in
// registers, and accumulates O += P V (P re-packed from the score fragments
// as the A operand, V fragments by ldmatrix.trans).  The warps' partial states
// are merged through shared memory at the end.  A query with no valid key
// writes zeros.
constexpr int kMQ = 16;  // queries per CTA (one m16 tile)
constexpr int kSmemMQ = kRingBytes + kMQ * kHD * 2 + kWarps * kStages * 8 + 16 + 1024;
static_assert(kWarps * (kMQ * kHD + 2 * kMQ) * 4 <= kRingBytes, "merge area fits in the ring");

__global__ void __launch_bounds__(kWarps * 32, 2)
    decode_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const DecodeAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* qtile = smem + kRingBytes;  // [16 rows][128 bytes], swizzled like the K / V tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(qtile + kMQ * kHD * 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + kWarps * kStages);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q0 = blockIdx.x * kMQ;
  const int h = blockIdx.y;
  const long long b = blockIdx.z;
  const int nq = min(kMQ, a.S_new - q0);
  int n_cache = *a.len_dev;
  if (n_cache < 0 || (long long)n_cache + a.S_new > a.max_len) {  // host keeps len + S_new <= max_len
    if (tid == 0) report_error(kErrIndex);
    n_cache = max(0, min(n_cache, (int)a.max_len - a.S_new));
  }
  // causal new block without an explicit mask: keys past the chunk's last
  // query are visible to none of its queries
  const int total = (a.block_mode == CDK_BLOCK_CAUSAL && a.full == nullptr) ? n_cache + min(a.S_new, q0 + nq)
                                                                          : n_cache + a.S_new;
  const int row_base = (int)((b * a.H + h) * a.max_len);
  uint64_t* wbar = bars + warp * kStages;
  uint8_t* wring = ring + warp * kStages * kStageBytes;
  const int n_tiles = total > warp * kKT ? (total - warp * kKT + kWarps * kKT - 1) / (kWarps * kKT) : 0;

  if (tid == 0) *abort_flag = 0;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&wbar[s], 1);
    fence_mbar_init();
    for (int k = 0; k < kStages - 1 && k < n_tiles; ++k) {
      const int t0 = (warp + k * kWarps) * kKT;
      mbar_arrive_expect_tx(&wbar[k], kStageBytes);
      tma_load_2d(wring + k * kStageBytes, &kmap, &wbar[k], 0, row_base + t0);
      tma_load_2d(wring + k * kStageBytes + kTileBytes, &vmap, &wbar[k], 0, row_base + t0);
    }
  }
  {  // query tile: thread t loads 16 bytes (row t / 8, chunk t % 8); rows past the block are zero
    const int row = tid >> 3, c = tid & 7;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < nq) v = *reinterpret_cast<const uint4*>(a.q + (b * a.S_new + q0 + row) * a.ldq + h * kHD + c * 8);
    *reinterpret_cast<uint4*>(qtile + swz(row, c)) = v;
  }
  __syncthreads();

  const bool act = a.active == nullptr || a.active[b] != 0;
  const long long nreal = a.num_real ? a.num_real[b] : (long long)a.S_new;
  const int r0 = lane >> 2;           // this thread's rows: r0 and r0 + 8
  const int cq = (lane & 3) * 2;      // and columns cq, cq + 1 of every 8-wide n tile

  uint32_t qa[4][4];
  {
    const int mi = lane >> 3;
    const int row = (mi & 1) * 8 + (lane & 7);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      ldsm_x4(smem_u32(qtile + swz(row, 2 * kk + (mi >> 1))), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
  }
  float o[8][4];
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  for (int k = 0; k < n_tiles; ++k) {
    const int t0 = (warp + k * kWarps) * kKT;
    const int st = k % kStages;
    mbar_wait(&wbar[st], (uint32_t)((k / kStages) & 1), abort_flag);
    if (lane == 0 && k + kStages - 1 < n_tiles) {
      // the stage refilled here was read in iteration k - 1 (finished at its __syncwarp)
      const int kn = k + kStages - 1, sn = kn % kStages;
      const int tn = (warp + kn * kWarps) * kKT;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(&wbar[sn], kStageBytes);
      tma_load_2d(wring + sn * kStageBytes, &kmap, &wbar[sn], 0, row_base + tn);
      tma_load_2d(wring + sn * kStageBytes + kTileBytes, &vmap, &wbar[sn], 0, row_base + tn);
    }
    uint8_t* kt = wring + st * kStageBytes;
    uint8_t* vt = kt + kTileBytes;
    if (t0 + kKT > total) {  // keys past the sequence's end: zero V rows so that 0 * V stays 0
      if (t0 + lane >= total) {
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(vt + swz(lane, c)) = make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    // S = Q K^T: 4 n tiles of 8 keys x 4 k steps of 16 dims
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; kk += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(kt + swz(nt * 8 + (lane & 7), 2 * kk + (lane >> 3))), b0, b1, b2, b3);
        mma_bf16_16816(sc[nt], qa[kk], b0, b1);
        mma_bf16_16816(sc[nt], qa[kk + 1], b2, b3);
      }
    }
    // mask: cache keys share one validity byte per column; new keys depend on the row
    bool cok[4][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = t0 + nt * 8 + cq + e;
        cok[nt][e] = j < total && (j < n_cache || a.block_mode == CDK_BLOCK_VALID) && a.valid[b * a.ldv + j] != 0;
      }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int row = r0 + rr * 8;
      const int q = q0 + row;
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = t0 + nt * 8 + cq + e;
          bool ok;
          if (row >= nq || j >= total) {
            ok = false;
          } else if (a.full) {
            ok = j < a.ldf && a.full[(b * a.S_new + q) * a.ldf + j] != 0;
          } else if (j < n_cache || a.block_mode == CDK_BLOCK_VALID) {
            ok = cok[nt][e];
          } else if (a.block_mode == CDK_BLOCK_CAUSAL) {
            const int jt = j - n_cache;
            ok = jt <= q && jt < nreal;
          } else if (a.block_mode == CDK_BLOCK_ACTIVE) {
            ok = act;
          } else {
            ok = true;
          }
          const float v = ok ? sc[nt][rr * 2 + e] * a.scale_log2 : -INFINITY;
          sc[nt][rr * 2 + e] = v;
          mx = fmaxf(mx, v);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(m[rr], mx);
      if (mnew == -INFINITY) {  // nothing visible to this row yet
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) sc[nt][rr * 2] = sc[nt][rr * 2 + 1] = 0.f;
      } else {
        const float alpha = exp2f(m[rr] - mnew);
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float pv = exp2f(sc[nt][rr * 2 + e] - mnew);  // exp2(-inf) = 0
            sc[nt][rr * 2 + e] = pv;
            sum += pv;
          }
        l[rr] = l[rr] * alpha + sum;
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
          o[nd][rr * 2] *= alpha;
          o[nd][rr * 2 + 1] *= alpha;
        }
        m[rr] = mnew;
      }
    }
    // O += P V: P (16 x 32) from the score fragments, 2 k steps of 16 keys
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t pa[4];
      pa[0] = pack_bf16(sc[2 * ks][0], sc[2 * ks][1]);
      pa[1] = pack_bf16(sc[2 * ks][2], sc[2 * ks][3]);
      pa[2] = pack_bf16(sc[2 * ks + 1][0], sc[2 * ks + 1][1]);
      pa[3] = pack_bf16(sc[2 * ks + 1][2], sc[2 * ks + 1][3]);
      const int mi = lane >> 3;
      const int key = ks * 16 + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int nd = 0; nd < 8; nd += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(vt + swz(key, nd + (mi >> 1))), b0, b1, b2, b3);
        mma_bf16_16816(o[nd], pa, b0, b1);
        mma_bf16_16816(o[nd + 1], pa, b2, b3);
      }
    }
    __syncwarp();
  }

  // Merge the warps' partial states (every issued tile was waited for, so the
  // ring is free): per warp O [16][64], row max [16], row sum [16].
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
    l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
  }
  __syncthreads();
  float* wo = reinterpret_cast<float*>(ring) + warp * (kMQ * kHD + 2 * kMQ);
#pragma unroll
  for (int nd = 0; nd < 8; ++nd)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr)
      *reinterpret_cast<float2*>(wo + (r0 + rr * 8) * kHD + nd * 8 + cq) = make_float2(o[nd][rr * 2], o[nd][rr * 2 + 1]);
  if ((lane & 3) == 0) {
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      wo[kMQ * kHD + r0 + rr * 8] = m[rr];
      wo[kMQ * kHD + kMQ + r0 + rr * 8] = l[rr];
    }
  }
  __syncthreads();
  for (int i = tid; i < kMQ * (kHD / 2); i += blockDim.x) {
    const int row = i / (kHD / 2), d2 = i % (kHD / 2);
    if (row >= nq) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      M = fmaxf(M, reinterpret_cast<const float*>(ring)[w * (kMQ * kHD + 2 * kMQ) + kMQ * kHD + row]);
    float L = 0.f, ox = 0.f, oy = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float* ww = reinterpret_cast<const float*>(ring) + w * (kMQ * kHD + 2 * kMQ);
        const float mw = ww[kMQ * kHD + row];
        const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
        L += ww[kMQ * kHD + kMQ + row] * f;
        const float2 v = *reinterpret_cast<const float2*>(ww + row * kHD + 2 * d2);
        ox += v.x * f;
        oy += v.y * f;
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    *reinterpret_cast<uint32_t*>(a.out + (b * a.S_new + q0 + row) * a.ldo + h * kHD + 2 * d2) =
        f2bf2(ox * inv, oy * inv);
  }
}

// One query per (sequence, head): the incremental step.  Persistent: each
// CTA walks (sequence, head) items i = blockIdx.x + n * gridDim.x.  Every
// sequence has the same number of keys (len + 1), so each of the kWarps warps
// sees the same tile count per item and its TMA ring runs as one stream of
// tiles across items: while a warp merges item n, the first tiles of item n+1
// are already in flight.  Lane l owns key (tile * 32 + l): it scores it from
// its swizzled K row and, if the key is valid, folds it into its own online-
// softmax state (max, sum, 64 fp32 accumulators from its swizzled V row), so
// the key loop has no cross-lane traffic; the lane states are merged by warp
// shuffles, then across the warps through shared memory.
struct Dec1qSmem {
  float q[kWarps][kHD];          // each warp's copy of the item's scaled query
  float red[kWarps][kHD + 4];    // per-warp merged state: acc[64], max, sum (rows 16-byte aligned)
  uint64_t bar[kWarps][kStages];
  int abort;
};
static_assert(offsetof(Dec1qSmem, red) % 16 == 0 && ((kHD + 4) * 4) % 16 == 0 && offsetof(Dec1qSmem, bar) % 8 == 0,
              "float4 rows and mbarriers need their alignment");
constexpr int kSmem1q = kRingBytes + (int)sizeof(Dec1qSmem) + 1024;

__global__ void __launch_bounds__(kWarps * 32, 2)
    decode_attn_1q_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                          const DecodeAttnArgs a, int n_items) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Dec1qSmem& sm = *reinterpret_cast<Dec1qSmem*>(ring + kRingBytes);
  volatile int* abort_flag = &sm.abort;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int n_cache = *a.len_dev;
  if (n_cache < 0 || (long long)n_cache + 1 > a.max_len) {
    if (tid == 0) report_error(kErrIndex);
    n_cache = max(0, min(n_cache, (int)a.max_len - 1));
  }
  const int total = n_cache + 1;
  const int n_tiles = total > warp * kKT ? (total - warp * kKT + kWarps * kKT - 1) / (kWarps * kKT) : 0;
  const int n_local = n_items > (int)blockIdx.x ? (n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const long long stream_len = (long long)n_local * n_tiles;  // this warp's tiles over all its items
  uint64_t* wbar = sm.bar[warp];
  uint8_t* wring = ring + warp * kStages * kStageBytes;

  // tile g of this warp's stream: item blockIdx.x + (g / n_tiles) * gridDim.x, key tile g % n_tiles
  auto issue = [&](long long g) {
    const int item = (int)blockIdx.x + (int)(g / n_tiles) * (int)gridDim.x;
    const int k = (int)(g % n_tiles);
    const long long bb = item / a.H;
    const int hh = item % a.H;
    const int row = (int)((bb * a.H + hh) * a.max_len) + (warp + k * kWarps) * kKT;
    const int st = (int)(g % kStages);
    mbar_arrive_expect_tx(&wbar[st], kStageBytes);
    tma_load_2d(wring + st * kStageBytes, &kmap, &wbar[st], 0, row);
    tma_load_2d(wring + st * kStageBytes + kTileBytes, &vmap, &wbar[st], 0, row);
  };
  if (tid == 0) *abort_flag = 0;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&wbar[s], 1);
    fence_mbar_init();
    for (long long g = 0; g < kStages - 1 && g < stream_len; ++g) issue(g);
  }
  __syncthreads();

  auto key_ok = [&](long long b, int j) -> bool {
    if (j >= total) return false;
    if (a.full) return j < a.ldf && a.full[b * a.ldf + j] != 0;
    if (j < n_cache || a.block_mode == CDK_BLOCK_VALID) return a.valid[b * a.ldv + j] != 0;
    if (a.block_mode == CDK_BLOCK_CAUSAL) return a.num_real == nullptr || a.num_real[b] > 0;
    if (a.block_mode == CDK_BLOCK_ACTIVE) return a.active == nullptr || a.active[b] != 0;
    return true;
  };

  // query of the first item (two bf16 per lane), then prefetched one item ahead
  uint32_t qnext = 0;
  if (n_local > 0) {
    const int item = blockIdx.x;
    qnext = *reinterpret_cast<const uint32_t*>(a.q + (long long)(item / a.H) * a.ldq + (item % a.H) * kHD + 2 * lane);
  }
  long long g = 0;
  // validity of this lane's key in the current tile, loaded one tile ahead
  bool ok_cur = n_local > 0 && n_tiles > 0 && key_ok((int)blockIdx.x / a.H, warp * kKT + lane);
  for (int n = 0; n < n_local; ++n) {
    const int item = (int)blockIdx.x + n * (int)gridDim.x;
    const long long b = item / a.H;
    const int h = item % a.H;
    {
      const float2 qf = bf2f(qnext);
      sm.q[warp][2 * lane] = qf.x * a.scale_log2;
      sm.q[warp][2 * lane + 1] = qf.y * a.scale_log2;
      if (n + 1 < n_local) {
        const int nx = item + (int)gridDim.x;
        qnext = *reinterpret_cast<const uint32_t*>(a.q + (long long)(nx / a.H) * a.ldq + (nx % a.H) * kHD + 2 * lane);
      }
      __syncwarp();
    }
    const float* qs = sm.q[warp];
    float m = -INFINITY, l = 0.f;
    float acc[kHD];
#pragma unroll
    for (int d = 0; d < kHD; ++d) acc[d] = 0.f;
    for (int k = 0; k < n_tiles; ++k, ++g) {
      const int t0 = (warp + k * kWarps) * kKT;
      const int st = (int)(g % kStages);
      mbar_wait(&wbar[st], (uint32_t)((g / kStages) & 1), abort_flag);
      // refill the stage read in the previous step (its reads finished at that step's __syncwarp)
      if (lane == 0 && g + kStages - 1 < stream_len) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(g + kStages - 1);
      }
      bool ok_next = false;  // next tile of this item, or the first tile of the next item
      if (k + 1 < n_tiles) ok_next = key_ok(b, t0 + kWarps * kKT + lane);
      else if (n + 1 < n_local) ok_next = key_ok((item + (int)gridDim.x) / a.H, warp * kKT + lane);
      const uint8_t* kt = wring + st * kStageBytes;
      const uint8_t* vt = kt + kTileBytes;
      if (ok_cur) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 kc = *reinterpret_cast<const uint4*>(kt + swz(lane, c));
          const float4 qa = *reinterpret_cast<const float4*>(qs + c * 8);
          const float4 qb = *reinterpret_cast<const float4*>(qs + c * 8 + 4);
          float2 f = bf2f(kc.x);
          s0 = fmaf(qa.x, f.x, s0);
          s1 = fmaf(qa.y, f.y, s1);
          f = bf2f(kc.y);
          s0 = fmaf(qa.z, f.x, s0);
          s1 = fmaf(qa.w, f.y, s1);
          f = bf2f(kc.z);
          s0 = fmaf(qb.x, f.x, s0);
          s1 = fmaf(qb.y, f.y, s1);
          f = bf2f(kc.w);
          s0 = fmaf(qb.z, f.x, s0);
          s1 = fmaf(qb.w, f.y, s1);
        }
        const float sc = s0 + s1;
        if (sc > m) {  // new running max for this lane: rescale its state
          const float alpha = exp2f(m - sc);
          l *= alpha;
#pragma unroll
          for (int d = 0; d < kHD; ++d) acc[d] *= alpha;
          m = sc;
        }
        const float pv = exp2f(sc - m);
        l += pv;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 vc = *reinterpret_cast<const uint4*>(vt + swz(lane, c));
          float2 f = bf2f(vc.x);
          acc[c * 8 + 0] = fmaf(pv, f.x, acc[c * 8 + 0]);
          acc[c * 8 + 1] = fmaf(pv, f.y, acc[c * 8 + 1]);
          f = bf2f(vc.y);
          acc[c * 8 + 2] = fmaf(pv, f.x, acc[c * 8 + 2]);
          acc[c * 8 + 3] = fmaf(pv, f.y, acc[c * 8 + 3]);
          f = bf2f(vc.z);
          acc[c * 8 + 4] = fmaf(pv, f.x, acc[c * 8 + 4]);
          acc[c * 8 + 5] = fmaf(pv, f.y, acc[c * 8 + 5]);
          f = bf2f(vc.w);
          acc[c * 8 + 6] = fmaf(pv, f.x, acc[c * 8 + 6]);
          acc[c * 8 + 7] = fmaf(pv, f.y, acc[c * 8 + 7]);
        }
      }
      ok_cur = ok_next;
      __syncwarp();
    }

    // warp merge: rescale every lane to the warp max, then butterfly sums
    float wm = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
    const float f = (m == -INFINITY) ? 0.f : exp2f(m - wm);
    l *= f;
#pragma unroll
    for (int d = 0; d < kHD; ++d) acc[d] *= f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
      for (int d = 0; d < kHD; ++d) acc[d] += __shfl_xor_sync(0xffffffffu, acc[d], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int d = 0; d < kHD; d += 4)
        *reinterpret_cast<float4*>(&sm.red[warp][d]) = make_float4(acc[d], acc[d + 1], acc[d + 2], acc[d + 3]);
      sm.red[warp][kHD] = wm;
      sm.red[warp][kHD + 1] = l;
    }
    __syncthreads();
    if (warp == 0) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm.red[w][kHD]);
      float L = 0.f, ox = 0.f, oy = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          const float fw = sm.red[w][kHD] == -INFINITY ? 0.f : exp2f(sm.red[w][kHD] - M);
          L += sm.red[w][kHD + 1] * fw;
          ox += sm.red[w][2 * lane] * fw;
          oy += sm.red[w][2 * lane + 1] * fw;
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      *reinterpret_cast<uint32_t*>(a.out + b * a.ldo + h * kHD + 2 * lane) = f2bf2(ox * inv, oy * inv);
    }
    __syncthreads();  // sm.red is rewritten by the next item
  }
}

// One block: keys [base, base + count) of each sequence become valid where the
// sequence is active and the key's offset is below its real-token count, with
// base = start (start >= 0) or len; then len += advance (every thread has read
// len before thread 0 writes it).
__global__ void decode_mark_kernel(uint8_t* __restrict__ valid, long long ldv, int B, long long start, int count,
                                   int advance, int32_t* __restrict__ len_dev, const uint8_t* __restrict__ active,
                                   const int64_t* __restrict__ num_real, long long max_len) {
  const int len = *len_dev;
  const long long base = start >= 0 ? start : (long long)len;
  for (long long i = threadIdx.x; i < (long long)B * count; i += blockDim.x) {
    const long long b = i / count;
    const int s = (int)(i % count);
    const bool on = (active == nullptr || active[b] != 0) && (num_real == nullptr || s < num_real[b]);
    if (on && base + s < max_len) valid[b * ldv + base + s] = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (base + count > max_len || (long long)len + advance > max_len) report_error(kErrIndex);
    *len_dev = len + advance;
  }
}

// u[t, f] = silu(gu[t, f]) * gu[t, F + f] from fp32 projections (the split-K
// form of the small-batch SwiGLU), bf16 out.  Two columns per thread.
__global__ void swiglu_f32_kernel(const float* __restrict__ gu, long long ldg, long long T, int F,
                                  __nv_bfloat16* __restrict__ u, long long ldu) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int half = F / 2;
  if (i >= T * half) return;
  const long long t = i / half;
  const int f = (int)(i % half) * 2;
  const float2 g = *reinterpret_cast<const float2*>(gu + t * ldg + f);
  const float2 v = *reinterpret_cast<const float2*>(gu + t * ldg + F + f);
  const float a = g.x / (1.f + __expf(-g.x)) * v.x;
  const float c = g.y / (1.f + __expf(-g.y)) * v.y;
  *reinterpret_cast<uint32_t*>(u + t * ldu + f) = f2bf2(a, c);
}

// splitmix64 finaliser (Steele, Lea and Flood, "Fast splittable pseudorandom
// number generators", 2014): a counter-based stream keyed by (seed, step,
// row, column), so a replayed step draws fresh numbers from the step counter.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Next token per sequence.  temperature <= 0: idx = argmax(logits[r, :ncols])
// (lowest index on ties, as torch.argmax); otherwise a sample of
// softmax(clamp(logits, -1e4, 1e4) / temperature) by the Gumbel-max rule,
// argmax(logit / T + g) with g = -log(-log(u)), u uniform in (0, 1) from the
// counter-based stream.
// ids[r] = lut ? lut[idx] : idx; lp_out[r] = log_softmax(logits[r])[idx] (the
// unscaled log-probability, as the reference records it); the step's ids (and
// log-probs) appended at row *counter of hist (lp_hist); then pos[r] += 1 and
// *counter += 1.  One block: warp w handles rows w, w + 8, ...
__global__ void head_select_kernel(const float* __restrict__ logits, long long ldl, int rows, int ncols,
                                   float temperature, const uint64_t* __restrict__ seed,
                                   const int64_t* __restrict__ lut, int64_t* __restrict__ ids,
                                   float* __restrict__ lp_out, int64_t* __restrict__ pos, int64_t* __restrict__ hist,
                                   float* __restrict__ lp_hist, int32_t* __restrict__ counter, int max_steps) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int step = counter ? *counter : 0;
  const bool sample = temperature > 0.f;
  const float inv_t = sample ? 1.f / temperature : 0.f;
  const uint64_t key = mix64((seed ? *seed : 0ull) ^ mix64((uint64_t)step));
  const bool want_lp = lp_out != nullptr || lp_hist != nullptr;
  for (int r = warp; r < rows; r += blockDim.x >> 5) {
    const float* row = logits + (long long)r * ldl;
    const uint64_t rkey = mix64(key ^ (uint64_t)r);
    float best = -INFINITY, mx = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < ncols; c += 32) {
      const float v = row[c];
      mx = fmaxf(mx, v);
      float sc = v;
      if (sample) {
        // u = (k + 0.5) / 2^23 for a 23-bit k: exact in fp32 and strictly
        // inside (0, 1), so -log(-log(u)) is finite for every draw.  The
        // logit is clamped to [-1e4, 1e4] before the temperature (the
        // reference's sampler clamps before its softmax); the recorded
        // log-probability below uses the unclamped logits.
        const float u = ((float)(mix64(rkey ^ (uint64_t)c) >> 41) + 0.5f) * (1.f / 8388608.f);
        sc = fminf(fmaxf(v, -1e4f), 1e4f) * inv_t - logf(-logf(u));
      }
      if (sc > best || (sc == best && c < bi)) {
        best = sc;
        bi = c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    float lp = 0.f;
    if (want_lp) {
      float sum = 0.f;
      for (int c = lane; c < ncols; c += 32) sum += expf(row[c] - mx);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (bi < ncols) lp = row[bi] - mx - logf(sum);
    }
    if (lane == 0) {
      if (bi >= ncols) bi = 0;  // every logit NaN
      const int64_t id = lut ? lut[bi] : (int64_t)bi;
      ids[r] = id;
      if (lp_out) lp_out[r] = lp;
      if (pos) pos[r] += 1;
      if (hist || lp_hist) {
        if (step < max_steps) {
          if (hist) hist[(long long)step * rows + r] = id;
          if (lp_hist) lp_hist[(long long)step * rows + r] = lp;
        } else {
          report_error(kErrIndex);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && counter) *counter = step + 1;
}

// a[r, c] = mish(z[r, c]) = z * tanh(softplus(z)) in bf16: the hidden layer of
// the value heads (Linear -> Mish -> Linear, model.py:39-52), softplus passing
// through above 20 as torch's does.
__global__ void mish_bf16_kernel(const float* __restrict__ z, long long ldz, long long rows, int cols,
                                 __nv_bfloat16* __restrict__ a, long long lda) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const long long r = i / cols;
  const int c = (int)(i % cols);
  const float x = z[r * ldz + c];
  const float sp = x > 20.f ? x : log1pf(expf(x));
  a[r * lda + c] = __float2bfloat16_rn(x * tanhf(sp));
}

__global__ void decode_slots_kernel(const uint8_t* __restrict__ om, long long n, int32_t* __restrict__ slot) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) slot[t] = om[t] ? (int32_t)t : -1;
}

inline bool al(const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

}  // namespace

extern "C" int cdk_kv_append(const void* qkv, int64_t ldq, int qkv_f32, const int32_t* pos, const float* rope,
                             int64_t rope_len, int64_t B, int64_t S_new, int64_t H, void* k_cache, void* v_cache,
                             int64_t max_len, const int32_t* len_dev, void* q_out, int64_t ldo, int qkv_out,
                             void* stream) {
  if (B == 0 || S_new == 0) return 0;
  if (!qkv || !k_cache || !v_cache || !len_dev || B < 0 || S_new < 0 || H <= 0 || max_len <= 0) return -1;
  if (ldq < 3 * H * kHD || ldq % 2) return -2;
  if (qkv_f32 && (!pos || !rope || !q_out || rope_len <= 0 || ldo < (qkv_out ? 3 : 1) * H * kHD || ldo % 2))
    return -3;
  if (!al(k_cache, 16) || !al(v_cache, 16) || !al(qkv, 8)) return -4;
  const long long total = B * S_new * H * 32;
  const unsigned blocks = (unsigned)((total + 255) / 256);
  kv_append_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      qkv, ldq, qkv_f32, pos, rope, (int)rope_len, (int)S_new, (int)H, max_len, len_dev,
      reinterpret_cast<__nv_bfloat16*>(k_cache), reinterpret_cast<__nv_bfloat16*>(v_cache),
      reinterpret_cast<__nv_bfloat16*>(q_out), ldo, qkv_f32 ? qkv_out : 0, total);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_decode_attn(const void* q, int64_t ldq, const void* k_cache, const void* v_cache,
                               int64_t max_len, const int32_t* len_dev, int64_t S_new, int64_t B, int64_t H,
                               const uint8_t* valid, int64_t ldv, int block_mode, const uint8_t* active,
                               const int64_t* num_real, const uint8_t* full_mask, int64_t ldf, void* out,
                               int64_t ldo, float scale, void* stream) {
  if (B == 0 || S_new == 0) return 0;
  if (!q || !k_cache || !v_cache || !len_dev || !valid || !out || B < 0 || S_new < 0 || H <= 0) return -1;
  if (B > 65535 || H > 65535 || ldq < H * kHD || ldq % 2 || ldo < H * kHD || ldo % 2 || ldv < max_len ||
      S_new > max_len)
    return -2;
  if (full_mask && ldf < 1) return -3;
  if (block_mode < CDK_BLOCK_CAUSAL || block_mode > CDK_BLOCK_VALID) return -4;
  if (!al(k_cache, 16) || !al(v_cache, 16) || !al(out, 4)) return -5;
  if (B * H * max_len >= (1ll << 31)) return -6;
  CUtensorMap kmap, vmap;
  const uint64_t rows = (uint64_t)(B * H * max_len);
  if (!make_tmap(&kmap, k_cache, kHD, rows, kHD, kHD, kKT) || !make_tmap(&vmap, v_cache, kHD, rows, kHD, kHD, kKT))
    return -7;
  DecodeAttnArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.ldq = ldq;
  a.max_len = max_len;
  a.len_dev = len_dev;
  a.S_new = (int)S_new;
  a.H = (int)H;
  a.valid = valid;
  a.ldv = ldv;
  a.block_mode = block_mode;
  a.active = active;
  a.num_real = num_real;
  a.full = full_mask;
  a.ldf = ldf;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.scale_log2 = scale * 1.4426950408889634f;
  static bool attr_done[64] = {false};
  static int num_sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return -8;
  if (!attr_done[dev]) {
    cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMQ);
    cudaFuncSetAttribute(decode_attn_1q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem1q);
    cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    attr_done[dev] = true;
  }
  if (S_new == 1) {
    const long long n_items = B * H;
    const int grid = (int)std::min<long long>(n_items, 2ll * std::max(num_sms[dev], 1));
    decode_attn_1q_kernel<<<grid, kWarps * 32, kSmem1q, reinterpret_cast<cudaStream_t>(stream)>>>(kmap, vmap, a,
                                                                                              (int)n_items);
  } else {
    if (ldq % 8) return -9;  // 16-byte query rows
    dim3 grid((unsigned)((S_new + kMQ - 1) / kMQ), (unsigned)H, (unsigned)B);
    decode_attn_kernel<<<grid, kWarps * 32, kSmemMQ, reinterpret_cast<cudaStream_t>(stream)>>>(kmap, vmap, a);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_decode_mark(void* valid, int64_t ldv, int64_t B, int64_t start, int64_t count, int64_t advance,
                               int32_t* len_dev, const uint8_t* active, const int64_t* num_real, int64_t max_len,
                               void* stream) {
  if (!valid || !len_dev || B < 0 || count < 0 || advance < 0 || ldv < max_len || start >= max_len) return -1;
  if (B == 0 || (count == 0 && advance == 0)) return 0;
  decode_mark_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<uint8_t*>(valid), ldv, (int)B, start, (int)count, (int)advance, len_dev, active, num_real,
      max_len);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_swiglu_f32(const float* gu, int64_t ldg, int64_t T, int64_t F, void* u, int64_t ldu,
                              void* stream) {
  if (T == 0) return 0;
  if (!gu || !u || T < 0 || F <= 0 || F % 2 || ldg < 2 * F || ldg % 2 || ldu < F || ldu % 2) return -1;
  const long long n = T * (F / 2);
  swiglu_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      gu, ldg, T, (int)F, reinterpret_cast<__nv_bfloat16*>(u), ldu);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_head_select(const float* logits, int64_t ldl, int64_t rows, int64_t ncols, float temperature,
                               const uint64_t* seed, const int64_t* lut, int64_t* ids, float* lp_out, int64_t* pos,
                               int64_t* hist, float* lp_hist, int32_t* counter, int64_t max_steps, void* stream) {
  if (rows == 0) return 0;
  if (!logits || !ids || rows < 0 || ncols <= 0 || ldl < ncols || ((hist || lp_hist) && !counter)) return -1;
  if (!(temperature == temperature)) return -2;  // NaN temperature
  head_select_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ldl, (int)rows, (int)ncols, temperature, seed, lut, ids, lp_out, pos, hist, lp_hist, counter,
      (int)max_steps);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_mish_bf16(const float* z, int64_t ldz, int64_t rows, int64_t cols, void* a, int64_t lda,
                             void* stream) {
  if (rows == 0 || cols == 0) return 0;
  if (!z || !a || rows < 0 || cols < 0 || ldz < cols || lda < cols) return -1;
  const long long n = rows * cols;
  mish_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      z, ldz, rows, (int)cols, reinterpret_cast<__nv_bfloat16*>(a), lda);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_decode_slots(const uint8_t* override_mask, int64_t n, int32_t* slot, void* stream) {
  if (n == 0) return 0;
  if (!override_mask || !slot || n < 0) return -1;
  decode_slots_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      override_mask, n, slot);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}
