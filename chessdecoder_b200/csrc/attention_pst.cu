// Persistent tensor-core attention forward for sequences of at most 256
// tokens, head_dim 64 -- the pretraining shape of the reference model
// (chessdecoder/train/config.yaml: max_seq_len 256; causal and block-prefix
// masks of chessdecoder/models/model.py:158-171).
//
// One CTA per SM walks the (head, sequence) items b, b + grid, b + 2 grid, ...
// An item is the whole sequence of one head: Q, K, V (up to 256 rows of 128 B
// each) arrive by TMA in one of two item slots, so the loads of the next item
// run while this one computes.  The item's two 128-row query tiles are two
// independent pipelines:
//
//   warp 0          producer: per item, the TMA loads, then (while they
//                   fly) the row metadata (block id, last visible key) into
//                   the slot
//   warp 1 / 2      MMA issuer of query tile 0 / 1 (whole warp, one elected lane):
//                   S_t = Q_t K^T (M=128, N = keys <= 256) into TMEM region t,
//                   then O_t = P_t V with P_t read from TMEM (A operand) and V
//                   MN-major from its TMA tile
//   warps 4-11 / 12-19  softmax of tile 0 / 1, two threads per query row
//                   (the TMEM lane) each taking one half of the keys: row
//                   max (halves merged in shared memory), exp2, bf16 P
//                   written back into score columns the same thread has
//                   already read (P for keys 2c, 2c+1 in consecutive columns;
//                   the upper half from column keys/2), then
//                   O_t / rowsum -> bf16 rows in global memory and the base-2
//                   log-sum-exp for the backward.  With contiguous blocks (the
//                   loader's rows: a board block is one run of 68 rows, every
//                   other token its own block) key j is visible to row i
//                   exactly when j <= max(i, last row of i's block); other
//                   block layouts compare block ids per key
//
// TMEM (512 columns): region t = [256 t, 256 t + 256): scores in [0, keys),
// P in [0, keys / 4) and [keys / 2, 3 keys / 4), O in [192, 256) (written
// only after the row's scores have been read).  Every wait is bounded (cdk_common); a timeout sets the
// device error word and drains every role to the TMEM release.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {
namespace pstattn {

constexpr int kHd = 64;
constexpr int kMaxS = 256;
constexpr int kBox = 64 * 128;  // one TMA box: 64 rows x 128 B (64 bf16)
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kThreads = 640;   // warps 0-3 producer / MMA, 4-11 softmax of tile 0, 12-19 of tile 1

struct Slot {
  uint8_t Q[4 * kBox];
  uint8_t K[4 * kBox];
  uint8_t V[4 * kBox];
};

struct FwdSmem {
  Slot slot[2];
  int32_t bid[2][kMaxS];   // block id of each row (causal: the row index)
  int32_t hi[2][kMaxS];    // max(i, last[i]): no key beyond it is visible to row i
  int32_t nk[2][2];        // keys (multiple of 64) of query tile 0 / 1
  int32_t contig[2];       // 1: every block id of the sequence is one contiguous run of rows
  float red_max[2][2][128];  // [tile][key half][row]: partial row maxima of the two threads of a row
  float red_sum[2][2][128];  // partial row sums
  // per item slot: Q|K landed, V landed, row metadata written; Q|K free again
  // (the item's S products done), V and metadata free again (P V products done)
  uint64_t qk_full[2], v_full[2], meta_full[2], qk_empty[2], v_empty[2];
  uint64_t sfull[2], pfull[2], ofull[2], oempty[2];
  uint32_t tmem_base;
  int abort;
};
static_assert(offsetof(FwdSmem, slot) % 1024 == 0 && sizeof(Slot) % 1024 == 0,
              "TMA / UMMA operands with the 128-byte swizzle need 1024-byte alignment");

struct Args {
  __nv_bfloat16* out;
  float* lse;
  const int32_t* bid;         // [nseq - n_causal, S]
  const int32_t* first;       // [nseq - n_causal, S]
  const int32_t* last;        // [nseq - n_causal, S]
  const int32_t* tile_kv_hi;  // [nseq - n_causal][2 * nt64]: exclusive key bound per 64-row query tile
  int S, H, n_causal, nt64, n_items;
};

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// tcgen05.wait::ld that also names the loaded registers, so that no use of
// them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld_dep(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

__device__ __forceinline__ void zero16(uint32_t (&pk)[16]) {
  #pragma unroll
  for (int e = 0; e < 16; ++e) pk[e] = 0u;
}

// Running max of the scores of keys [base, base + 32) that are <= hi.
__device__ __forceinline__ void row_max_chunk(const uint32_t (&v)[32], int base, int hi, float (&mx4)[4]) {
  if (base + 31 <= hi) {
    #pragma unroll
    for (int e = 0; e < 32; ++e) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(v[e]));
  } else if (base <= hi) {
    #pragma unroll
    for (int e = 0; e < 32; ++e)
      if (base + e <= hi) mx4[e & 3] = fmaxf(mx4[e & 3], __uint_as_float(v[e]));
  }
}

// bf16 probabilities of keys [base, base + 32) (pairs packed low = even key),
// accumulating the row sum.
__device__ __forceinline__ void probs_chunk(const uint32_t (&v)[32], int base, float sl2, float ms, int full_hi,
                                            int hi, int my_bid, bool contig, const int* bid, uint32_t (&pk)[16],
                                            float (&l4)[4]) {
  if (base + 31 <= full_hi) {
    #pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const float p0 = ex2_approx(fmaf(__uint_as_float(v[e]), sl2, -ms));
      const float p1 = ex2_approx(fmaf(__uint_as_float(v[e + 1]), sl2, -ms));
      l4[(e >> 1) & 3] += p0 + p1;
      pk[e >> 1] = pack_bf16(p0, p1);
    }
  } else if (base <= hi) {
    #pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const int j0 = base + e, j1 = j0 + 1;
      const bool v0 = j0 <= full_hi || (!contig && j0 <= hi && bid[j0] == my_bid);
      const bool v1 = j1 <= full_hi || (!contig && j1 <= hi && bid[j1] == my_bid);
      const float p0 = v0 ? ex2_approx(fmaf(__uint_as_float(v[e]), sl2, -ms)) : 0.f;
      const float p1 = v1 ? ex2_approx(fmaf(__uint_as_float(v[e + 1]), sl2, -ms)) : 0.f;
      l4[(e >> 1) & 3] += p0 + p1;
      pk[e >> 1] = pack_bf16(p0, p1);
    }
  } else {
    zero16(pk);
  }
}

// Key count of query tile t of an item (a multiple of 64, at most 256: the
// K / V rows arrive in 64-row boxes, and the softmax reads 64 keys at a time).
__device__ __forceinline__ int tile_keys(const Args& a, int t, bool prefix, int pseq) {
  const int S = a.S;
  int kv = min(S, (t + 1) * 128);
  if (prefix) {
    const int* kvhi = a.tile_kv_hi + (long long)pseq * 2 * a.nt64;
    for (int q = 2 * t; q < min(2 * t + 2, a.nt64); ++q) kv = max(kv, kvhi[q]);
  }
  return min(kMaxS, (min(kv, S) + 63) / 64 * 64);
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_pst_kernel(const __grid_constant__ CUtensorMap tqkv, const Args a) {
  extern __shared__ uint8_t raw[];
  FwdSmem& sm = *reinterpret_cast<FwdSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int S = a.S, H = a.H, E = H * kHd;
  const int n_tiles = S > 128 ? 2 : 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int n_local = a.n_items > (int)blockIdx.x ? (a.n_items - (int)blockIdx.x + G - 1) / G : 0;
  volatile int* abort_flag = &sm.abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.qk_full[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.meta_full[s], 32);
      mbar_init(&sm.qk_empty[s], n_tiles);
      mbar_init(&sm.v_empty[s], n_tiles);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.sfull[t], 1);
      mbar_init(&sm.pfull[t], 256);
      mbar_init(&sm.ofull[t], 1);
      mbar_init(&sm.oempty[t], 256);
    }
    sm.abort = 0;
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

  if (warp == 0) {
    // ---- producer --------------------------------------------------------
    if (lane == 0) prefetch_tmap(&tqkv);
    const int nq64 = (S + 63) / 64;
    for (int k = 0; k < n_local; ++k) {
      const int s = k & 1, u = k >> 1;
      const int item = (int)blockIdx.x + k * G;
      const int seq = item / H, h = item - seq * H;
      const bool prefix = seq >= a.n_causal;
      const int pseq = seq - a.n_causal;
      const int row0 = seq * S;
      // Q and K as soon as the S products of the item two back have read the
      // slot's, V (and then the row metadata, which the softmax reads until P
      // is formed) once its P V products have.  The last query tile sees every
      // key, so K and V are always ceil(S / 64) boxes.
      if (u > 0) mbar_wait(&sm.qk_empty[s], (u - 1) & 1, abort_flag);
      if (lane == 0) {
        mbar_arrive_expect_tx(&sm.qk_full[s], (uint32_t)(2 * nq64) * kBox);
        for (int b = 0; b < nq64; ++b) {
          tma_load_2d(sm.slot[s].Q + b * kBox, &tqkv, &sm.qk_full[s], h * kHd, row0 + b * 64);
          tma_load_2d(sm.slot[s].K + b * kBox, &tqkv, &sm.qk_full[s], E + h * kHd, row0 + b * 64);
        }
      }
      __syncwarp();
      // the item's row metadata into registers first (all of a lane's loads in
      // one round trip, overlapping the wait for the slot's V); causal rows:
      // block id = row, last visible key = row
      constexpr int kJ = kMaxS / 32;
      int bv[kJ], lv[kJ], fv[kJ];
      #pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const int i = lane + 32 * j;
        bv[j] = lv[j] = fv[j] = i;
        if (prefix && i < S) {
          const long long o = (long long)pseq * S + i;
          bv[j] = __ldg(a.bid + o);
          lv[j] = __ldg(a.last + o);
          fv[j] = __ldg(a.first + o);
        }
      }
      const int nk0 = tile_keys(a, 0, prefix, pseq);
      const int nk1 = n_tiles > 1 ? tile_keys(a, 1, prefix, pseq) : 0;
      if (u > 0) mbar_wait(&sm.v_empty[s], (u - 1) & 1, abort_flag);
      if (lane == 0) {
        mbar_arrive_expect_tx(&sm.v_full[s], (uint32_t)nq64 * kBox);
        for (int b = 0; b < nq64; ++b)
          tma_load_2d(sm.slot[s].V + b * kBox, &tqkv, &sm.v_full[s], 2 * E + h * kHd, row0 + b * 64);
      }
      __syncwarp();
      bool runs_ok = true;  // a row whose id differs from the previous row's opens the id's first run
      #pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const int i = lane + 32 * j;
        const bool ok = i < S;
        // the previous row's id: lane - 1's, or lane 31's of the previous group
        int prev = __shfl_up_sync(0xffffffffu, bv[j], 1);
        const int prev31 = __shfl_sync(0xffffffffu, bv[j > 0 ? j - 1 : 0], 31);
        if (lane == 0) prev = prev31;
        const int b = ok ? bv[j] : -1;
        sm.bid[s][i] = b;
        sm.hi[s][i] = ok ? max(i, lv[j]) : -1;
        if (prefix && ok && i > 0 && b != prev && fv[j] != i) runs_ok = false;
      }
      runs_ok = __all_sync(0xffffffffu, runs_ok);
      if (lane == 0) {
        sm.nk[s][0] = nk0;
        sm.nk[s][1] = nk1;
        sm.contig[s] = runs_ok ? 1 : 0;
      }
      mbar_arrive(&sm.meta_full[s]);  // 32 arrivals: the slot's metadata is written
    }
  } else if (warp == 1 || warp == 2) {
    // ---- MMA issuer of query tile t --------------------------------------
    const int t = warp - 1;
    // the whole warp runs the issue loop; one elected lane issues (uniform operands)
    if (t < n_tiles) {
      const uint32_t treg = tmem + (uint32_t)(t * 256);
      const uint32_t idesc_o = make_idesc_bf16(128, kHd, false, true);
      for (int k = 0; k < n_local; ++k) {
        const int s = k & 1, u = k >> 1;
        mbar_wait(&sm.meta_full[s], u & 1, abort_flag);
        mbar_wait(&sm.qk_full[s], u & 1, abort_flag);
        if (k > 0) mbar_wait(&sm.oempty[t], (k - 1) & 1, abort_flag);
        tc_fence_after();
        const int nk = sm.nk[s][t];
        const uint32_t idesc_s = make_idesc_bf16(128, nk, false, false);
        const uint32_t qa = smem_u32(sm.slot[s].Q + t * 2 * kBox);
        const uint32_t kb = smem_u32(sm.slot[s].K);
        #pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk)
          umma_f16_w(treg, make_sdesc(qa + kk * 32, 16, 1024), make_sdesc(kb + kk * 32, 16, 1024), idesc_s,
                   kk > 0 ? 1u : 0u);
        tc_commit_w(&sm.sfull[t]);
        tc_commit_w(&sm.qk_empty[s]);
        mbar_wait(&sm.pfull[t], k & 1, abort_flag);
        mbar_wait(&sm.v_full[s], u & 1, abort_flag);
        tc_fence_after();
        const uint32_t vb = smem_u32(sm.slot[s].V);
        // P of keys [0, nk/2) sits in columns [0, nk/4), P of keys [nk/2, nk)
        // in columns [nk/2, 3 nk/4): each half written over scores its own
        // thread has read
        for (int k4 = 0; k4 < nk / 64; ++k4) {  // nk is a multiple of 64
          const uint64_t vd = make_sdesc(vb + k4 * 64 * 128, 8192, 1024);
          #pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int key0 = k4 * 64 + kk * 16;
            const uint32_t acol = (uint32_t)(key0 / 2 + (key0 >= nk / 2 ? nk / 4 : 0));
            umma_f16_ts_w(treg + 192, treg + acol, vd + (uint64_t)(kk * 16 * 128 / 16), idesc_o,
                          (k4 > 0 || kk > 0) ? 1u : 0u);
          }
        }
        tc_commit_w(&sm.ofull[t]);
        tc_commit_w(&sm.v_empty[s]);
      }
    }
  } else if (warp >= 4) {
    // ---- softmax + epilogue of query tile t ------------------------------
    // Two threads per query row: warps 4 + 8t + 4h + q (q = TMEM lane
    // quadrant) take key half h, keys [h nk/2, (h + 1) nk/2).
    const int t = (warp - 4) >> 3;
    const int hf = ((warp - 4) >> 2) & 1;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int i = t * 128 + r;
    const bool row_ok = i < S;
    const uint32_t trow = tmem + (uint32_t)(t * 256) + (static_cast<uint32_t>(quad * 32) << 16);
    const float sl2 = 0.125f * kLog2e;
    const int bar_id = 1 + t;  // named barrier of the tile's 256 softmax threads
    if (t < n_tiles) {
      for (int k = 0; k < n_local; ++k) {
        const int s = k & 1, u = k >> 1;
        const int item = (int)blockIdx.x + k * G;
        const int seq = item / H, h = item - seq * H;
        mbar_wait(&sm.meta_full[s], u & 1, abort_flag);  // row metadata of the slot
        const int nk = sm.nk[s][t];
        const int* bid = sm.bid[s];
        const int my_bid = row_ok ? bid[i] : -2;
        const int hi = row_ok ? sm.hi[s][i] : -1;
        // contiguous blocks: key j is visible to row i exactly when j <= hi;
        // otherwise a key in (i, hi] is visible only when it has row i's block id
        const bool contig = sm.contig[s] != 0;
        const int full_hi = row_ok ? (contig ? hi : i) : -1;  // keys [0, full_hi] are all visible
        // tcgen05.ld / st are warp-collective: load decisions use the
        // warp-uniform bound hi_w, per-row bounds only steer arithmetic
        int hi_w = hi;
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) hi_w = max(hi_w, __shfl_xor_sync(0xffffffffu, hi_w, o));
        const int c0 = hf * (nk / 64), c1 = c0 + nk / 64;  // this thread's 32-key chunks
        const int c1v = min(c1, hi_w >= 0 ? hi_w / 32 + 1 : 0);  // ... that hold a key <= hi_w
        mbar_wait(&sm.sfull[t], k & 1, abort_flag);
        tc_fence_after();
        // pass 1: max of the raw scores of keys <= hi (an upper bound of the
        // visible maximum; either keeps exp2 <= 1), halves merged in shared memory
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        for (int c = c0; c < c1v; ++c) {
          uint32_t va[32];
          tmem_ld_x32_nowait(trow + c * 32, va);
          tmem_wait_ld_dep(va);
          row_max_chunk(va, c * 32, hi, mx4);
        }
        sm.red_max[t][hf][r] = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        asm volatile("bar.sync %0, 256;" ::"r"(bar_id) : "memory");
        const float ms = fmaxf(sm.red_max[t][0][r], sm.red_max[t][1][r]) * sl2;
        // pass 2: bf16 probabilities of this thread's keys into score columns
        // it has already read (P of keys [base_h, ...) from column
        // hf * nk/4 + (key / 2)), partial row sum
        float l4[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c = c0; c < c1; ++c) {
          uint32_t pk[16];
          if (c < c1v) {
            uint32_t va[32];
            tmem_ld_x32_nowait(trow + c * 32, va);
            tmem_wait_ld_dep(va);
            probs_chunk(va, c * 32, sl2, ms, full_hi, hi, my_bid, contig, bid, pk, l4);
          } else {
            zero16(pk);
          }
          tmem_st_x16(trow + hf * (nk / 4) + c * 16, pk);
        }
        sm.red_sum[t][hf][r] = (l4[0] + l4[1]) + (l4[2] + l4[3]);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.pfull[t]);
        // epilogue: O / l in bf16 (half hf stores dims [32 hf, 32 hf + 32)),
        // and the base-2 log-sum-exp
        mbar_wait(&sm.ofull[t], k & 1, abort_flag);
        tc_fence_after();
        uint32_t o[32];
        tmem_ld_x32_nowait(trow + 192 + hf * 32, o);
        tmem_wait_ld_dep(o);
        tc_fence_before();
        mbar_arrive(&sm.oempty[t]);
        asm volatile("bar.sync %0, 256;" ::"r"(bar_id) : "memory");  // both partial sums written
        const float l = sm.red_sum[t][0][r] + sm.red_sum[t][1][r];
        if (row_ok) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(a.out + (long long)(seq * S + i) * E + h * kHd + hf * 32);
          #pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int b = q * 8;
            dst[q] = make_uint4(pack_bf16(__uint_as_float(o[b]) * inv, __uint_as_float(o[b + 1]) * inv),
                                pack_bf16(__uint_as_float(o[b + 2]) * inv, __uint_as_float(o[b + 3]) * inv),
                                pack_bf16(__uint_as_float(o[b + 4]) * inv, __uint_as_float(o[b + 5]) * inv),
                                pack_bf16(__uint_as_float(o[b + 6]) * inv, __uint_as_float(o[b + 7]) * inv));
          }
          if (hf == 0) a.lse[((long long)seq * H + h) * S + i] = ms + log2f(l);
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

}  // namespace pstattn

// Host launcher used by cdk_attn_fwd for S <= 256.
int launch_attn_fwd_pst(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S,
                        int64_t H, const int32_t* bid, const int32_t* meta, cudaStream_t stream) {
  using namespace pstattn;
  if (S > kMaxS || S <= 0) return -20;
  if (nseq * H > (int64_t)1 << 30) return -5;
  CUtensorMap tq;
  if (!make_tmap(&tq, qkv, 3 * H * kHd, nseq * S, 3 * H * kHd, 64, 64)) return -21;
  Args a;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.lse = lse;
  const int64_t np = nseq - n_causal;
  const int nt64 = (int)((S + 63) / 64);
  a.bid = bid;
  a.tile_kv_hi = meta;
  a.first = np > 0 ? meta + np * 2 * nt64 : nullptr;
  a.last = np > 0 ? meta + np * 2 * nt64 + np * S : nullptr;
  a.nt64 = nt64;
  a.S = (int)S;
  a.H = (int)H;
  a.n_causal = (int)n_causal;
  a.n_items = (int)(nseq * H);
  const size_t smem = sizeof(FwdSmem) + 1024;
  static int sm_count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return -24;
  if (sm_count[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_pst_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    // tcgen05.alloc blocks until columns are free: one 512-column CTA per SM
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_fwd_pst_kernel, kThreads, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm != 1) return -22;
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return (int)e;
    sm_count[dev] = sms;
  }
  const int grid = (int)(nseq * H < sm_count[dev] ? nseq * H : sm_count[dev]);
  attn_fwd_pst_kernel<<<grid, kThreads, smem, stream>>>(tq, a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace cdk
