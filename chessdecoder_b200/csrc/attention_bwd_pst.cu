// Persistent tensor-core attention backward for sequences of at most 256
// tokens, head_dim 64 (the pretraining shape; causal and block-prefix masks of
// chessdecoder/models/model.py:158-171, gradient of the SDPA in
// chessdecoder/export/backbone_causal.py:112-137).
//
// One CTA per SM walks the (head, sequence) items b, b + grid, ...  An item's
// keys form key tiles kt of 128 rows, its queries query halves qh of 128 rows;
// the work is a list of sub-units (kt, qs) with qs a 64-query sub-tile, taken
// key-tile-major in pairs (qs = 2 qh, 2 qh + 1) over the query halves that can
// see the key tile.  Per sub-unit:
//   MMA-A   S^T = K_kt Q_qs^T, dP^T = V_kt dO_qs^T           (TMEM, N = 64)
//   EW      P^T = exp2(S^T c - L), dS^T = P^T (dP^T - D)      (masked)
//   MMA-B   dV_kt += P^T dO_qs (P^T read from TMEM), dK_kt += dS^T Q_qs
//   (pair)  dQ_qh += dS K_kt  (dS read MN-major from the pair's dS^T tiles)
// S^T | dP^T are double-buffered in TMEM, so the tensor core runs MMA-B / dQ
// of one sub-unit and MMA-A of the next but one while the elementwise warps
// work on the next.  dV / dK of a key tile and dQ of both query halves stay in
// TMEM until complete and are written once (dK, dQ scaled by 1/8 with the
// inverse RoPE rotation).  The operands of an item live in shared memory in
// four 32 KB slots -- K|V of key tile 0 and 1, Q|dO of query half 0 and 1 --
// each released as soon as the item's last product that reads it has retired,
// so the next item's loads overlap this one.  D = rowsum(dO * O) comes from a
// pass before (attn_dsum).
//
//   warp 0       producer: row metadata (L, D, block bounds) and TMA loads
//   warp 1       TMEM allocation, MMA issue (whole warp, one elected lane)
//   warps 2-17   elementwise + epilogues: thread = (key row r = TMEM lane,
//                16-query group g of the sub-tile)
// TMEM: S^T|dP^T x 2 [0, 256) | dV [256, 320) | dK [320, 384) | dQ_0 [384, 448)
// | dQ_1 [448, 512).  P^T (bf16) is written over the thread's own S^T columns
// after it has read them: queries [16 g, 16 g + 16) -> columns [16 g, 16 g + 8)
// of the buffer.  Every wait is bounded (cdk_common).
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {
namespace pstbwd {

constexpr int kHd = 64;
constexpr int kMaxS = 256;
constexpr int kBox = 64 * 128;  // one TMA box: 64 rows x 128 B
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kThreads = 576;   // warp 0 producer, warp 1 MMA, warps 2-17 elementwise
constexpr int kMaxUnits = 8;    // sub-units of one item (two key tiles x two query halves x 2; 3 bits each)

struct Meta {
  alignas(16) float L[kMaxS];   // base-2 log-sum-exp of each query row (0 past S)
  alignas(16) float D[kMaxS];   // rowsum(dO * O) of each query row (0 past S)
  int32_t first[kMaxS];         // first row of each key row's block (causal: the row; S past S)
  int32_t bid[kMaxS];           // block id of each row (non-contiguous layouts only)
  int32_t contig;               // 1: every block id is one contiguous run of rows
};

struct BwdSmem {
  uint8_t KV[2][4 * kBox];      // key tile kt: K rows (2 boxes) | V rows (2 boxes)
  uint8_t QO[2][4 * kBox];      // query half qh: Q rows (2 boxes) | dO rows (2 boxes)
  uint8_t dST[2][2][128 * 128]; // [pair buffer][sub-tile]: 128 key rows x 64 queries (bf16, 128-B swizzle)
  uint8_t stage[4][32 * 128];   // epilogue transposition, per TMEM lane quadrant: 32 rows x 64 dims bf16
  Meta meta[2];
  uint64_t kvfull[2], kvempty[2], qfull[2], qempty[2], mfull[2], mempty[2];
  uint64_t sa[2], ew[2], dq[2], kvdone, kvfree, dqdone, dqfree;
  uint32_t tmem_base;
  int abort;
};
static_assert(offsetof(BwdSmem, QO) % 1024 == 0 && offsetof(BwdSmem, dST) % 1024 == 0,
              "TMA / UMMA operands with the 128-byte swizzle need 1024-byte alignment");
static_assert(offsetof(BwdSmem, meta) % 16 == 0 && sizeof(Meta) % 16 == 0, "L / D are read as float4");
static_assert(offsetof(BwdSmem, stage) % 128 == 0, "staging rows are read as 16-byte chunks");

struct Args {
  const float* lse;       // [nseq, H, S]
  const float* dsum;      // [nseq, H, S]
  __nv_bfloat16* dqkv;
  const int32_t* bid;     // [nseq - n_causal, S]
  const int32_t* first;   // [nseq - n_causal, S]
  const int32_t* q_lo;    // [nseq - n_causal][2 * nt64]; + nt64: lowest first row per 64-row tile
  const float* rope;      // [>= S, 32, 2] (cos, sin) or null
  Q8Out q8;               // q8.q set: dq|dk|dv written as 8-bit (fp8 recipe) instead of bf16
  int S, H, n_causal, nt64, n_items;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void tmem_wait_ld_dep16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// The sub-units of an item: key tile kt (k-major), query sub-tile qs; pairs of
// sub-tiles (2 qh, 2 qh + 1) from the first query half that can see the key
// tile.  Packed into one register word (3 bits per sub-unit: kt << 2 | qs) so
// that a runtime sub-unit index never touches local memory.
struct Units {
  int n;
  uint32_t code;
  __device__ __forceinline__ int kt(int u) const { return (int)((code >> (3 * u + 2)) & 1u); }
  __device__ __forceinline__ int qs(int u) const { return (int)((code >> (3 * u)) & 3u); }
};

__device__ __forceinline__ Units item_units(const Args& a, bool prefix, int pseq) {
  Units u;
  u.n = 0;
  u.code = 0;
  const int nkt = (a.S + 127) / 128;
  for (int kt = 0; kt < nkt; ++kt) {
    int qh0 = kt;
    if (prefix) {
      const int* ql = a.q_lo + (long long)pseq * 2 * a.nt64 + a.nt64;
      int q0 = kt * 128;
      for (int t = 2 * kt; t < min(2 * kt + 2, a.nt64); ++t) q0 = min(q0, ql[t]);
      qh0 = q0 / 128;
    }
    for (int qh = qh0; qh < nkt; ++qh) {
      u.code |= (uint32_t)((kt << 2) | (2 * qh)) << (3 * u.n);
      u.code |= (uint32_t)((kt << 2) | (2 * qh + 1)) << (3 * (u.n + 1));
      u.n += 2;
    }
  }
  return u;
}

// (cos, sin) pairs of the 16 dims [c0, c0 + 16) of position pos, or the
// identity when rope == null.  Loaded before the epilogue's wait on the
// accumulator so that the table read overlaps the last MMAs.
struct Rope16 {
  float4 cs[4];
};
__device__ __forceinline__ Rope16 load_rope16(const float* rope, int pos, int c0, bool ok) {
  Rope16 r;
  if (rope != nullptr && ok) {
    const float4* p = reinterpret_cast<const float4*>(rope + ((long long)pos * 32 + c0 / 2) * 2);
    #pragma unroll
    for (int q = 0; q < 4; ++q) r.cs[q] = p[q];
  } else {
    #pragma unroll
    for (int q = 0; q < 4; ++q) r.cs[q] = make_float4(1.f, 0.f, 1.f, 0.f);
  }
  return r;
}

// 16 consecutive dims of a dX row: value * scale, then the inverse RoPE
// rotation given by rp (the identity for V or without RoPE), packed to bf16.
__device__ __forceinline__ void rotate16(const uint32_t (&v)[16], float scale, const Rope16& rp, float (&f)[16]) {
  #pragma unroll
  for (int e = 0; e < 16; ++e) f[e] = __uint_as_float(v[e]) * scale;
  #pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float4 t = rp.cs[p];  // (cos, sin) of two consecutive pairs
    float x0 = f[4 * p], x1 = f[4 * p + 1];
    f[4 * p] = x0 * t.x + x1 * t.y;
    f[4 * p + 1] = x1 * t.x - x0 * t.y;
    x0 = f[4 * p + 2];
    x1 = f[4 * p + 3];
    f[4 * p + 2] = x0 * t.z + x1 * t.w;
    f[4 * p + 3] = x1 * t.z - x0 * t.w;
  }
}
__device__ __forceinline__ void rotate_pack16(const uint32_t (&v)[16], float scale, const Rope16& rp,
                                              uint32_t (&w)[8]) {
  float f[16];
  rotate16(v, scale, rp, f);
  #pragma unroll
  for (int q = 0; q < 8; ++q) w[q] = pack_bf16(f[2 * q], f[2 * q + 1]);
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Stores one 32-row x 64-dim bf16 block of dQ, dK or dV (the rows of one TMEM
// lane quadrant; each of the quadrant's 4 warps holds 16 dims of every row).
// Row-per-thread stores would touch 32 rows per instruction; instead the four
// warps transpose the block through shared memory (128-byte rows, chunks
// XOR-swizzled by the row) and each warp stores 8 whole rows, 4 per
// instruction.  All 128 threads of the quadrant call it (two named barriers).
__device__ __forceinline__ void quad_store(uint8_t* stg, int bar_id, int lane, int g4, const uint32_t (&w)[8],
                                           __nv_bfloat16* row0, long long pitch, int rows_valid) {
  #pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int chunk = g4 * 2 + q;
    *reinterpret_cast<uint4*>(stg + lane * 128 + ((chunk ^ (lane & 7)) << 4)) =
        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
  named_bar_sync(bar_id, 128);
  #pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int rr = g4 * 8 + it * 4 + (lane >> 3), c = lane & 7;
    if (rr < rows_valid) {
      const uint4 x = *reinterpret_cast<const uint4*>(stg + rr * 128 + ((c ^ (rr & 7)) << 4));
      *reinterpret_cast<uint4*>(row0 + (long long)rr * pitch + c * 8) = x;
    }
  }
  named_bar_sync(bar_id, 128);  // the staging rows are free again
}

// The same block written as 8-bit values q = saturate(v * qs) (64-byte rows:
// each of the quadrant's 4 warps holds one 16-byte chunk of every row, chunks
// XOR-swizzled by the row); returns max |v| of this thread's 16 values.
__device__ __forceinline__ float quad_store_q8(uint8_t* stg, int bar_id, int lane, int g4, const float (&f)[16],
                                               float qs, int fmt, uint8_t* row0, long long pitch, int rows_valid) {
  uint32_t w[4];
  float m = 0.f;
  #pragma unroll
  for (int q = 0; q < 4; ++q) {
    w[q] = q8_pack4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3], qs, fmt);
    m = abs_max4(m, f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
  }
  *reinterpret_cast<uint4*>(stg + lane * 64 + ((g4 ^ (lane & 3)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
  named_bar_sync(bar_id, 128);
  const int rr = g4 * 8 + (lane >> 2), c = lane & 3;
  if (rr < rows_valid)
    *reinterpret_cast<uint4*>(row0 + (long long)rr * pitch + c * 16) =
        *reinterpret_cast<const uint4*>(stg + rr * 64 + ((c ^ (rr & 3)) << 4));
  named_bar_sync(bar_id, 128);
  return m;
}

// P^T and dS^T of one thread's 16 queries: P = exp2(S * scale - L),
// dS = P (dP - D), bf16-packed; with MASK, queries outside [e_lo, e_hi) get 0.
template <bool MASK>
__device__ __forceinline__ void ew16(const uint32_t (&su)[16], const uint32_t (&du)[16], const float* L, const float* D,
                                     float sl2, int e_lo, int e_hi, uint32_t (&pk)[8], uint32_t (&dk)[8]) {
  const float4* L4 = reinterpret_cast<const float4*>(L);
  const float4* D4 = reinterpret_cast<const float4*>(D);
  #pragma unroll
  for (int e4 = 0; e4 < 4; ++e4) {
    const float4 l4 = L4[e4], d4 = D4[e4];
    float pv[4], dsv[4];
    pv[0] = ex2_approx(fmaf(__uint_as_float(su[4 * e4 + 0]), sl2, -l4.x));
    pv[1] = ex2_approx(fmaf(__uint_as_float(su[4 * e4 + 1]), sl2, -l4.y));
    pv[2] = ex2_approx(fmaf(__uint_as_float(su[4 * e4 + 2]), sl2, -l4.z));
    pv[3] = ex2_approx(fmaf(__uint_as_float(su[4 * e4 + 3]), sl2, -l4.w));
    dsv[0] = pv[0] * (__uint_as_float(du[4 * e4 + 0]) - d4.x);
    dsv[1] = pv[1] * (__uint_as_float(du[4 * e4 + 1]) - d4.y);
    dsv[2] = pv[2] * (__uint_as_float(du[4 * e4 + 2]) - d4.z);
    dsv[3] = pv[3] * (__uint_as_float(du[4 * e4 + 3]) - d4.w);
    if (MASK) {
      #pragma unroll
      for (int kq = 0; kq < 4; ++kq) {
        const int e = 4 * e4 + kq;
        const bool vis = e >= e_lo && e < e_hi;
        pv[kq] = vis ? pv[kq] : 0.f;
        dsv[kq] = vis ? dsv[kq] : 0.f;
      }
    }
    pk[e4 * 2] = pack_bf16(pv[0], pv[1]);
    pk[e4 * 2 + 1] = pack_bf16(pv[2], pv[3]);
    dk[e4 * 2] = pack_bf16(dsv[0], dsv[1]);
    dk[e4 * 2 + 1] = pack_bf16(dsv[2], dsv[3]);
  }
}

template <bool Q8>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_pst_kernel(const __grid_constant__ CUtensorMap tqkv, const __grid_constant__ CUtensorMap tdo,
                        const Args a) {
  extern __shared__ uint8_t raw[];
  BwdSmem& sm = *reinterpret_cast<BwdSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int S = a.S, H = a.H, E = H * kHd;
  const int nkt = (S + 127) / 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const int n_local = a.n_items > (int)blockIdx.x ? (a.n_items - (int)blockIdx.x + G - 1) / G : 0;
  volatile int* abort_flag = &sm.abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.kvfull[s], 1);
      mbar_init(&sm.kvempty[s], 1);
      mbar_init(&sm.qfull[s], 1);
      mbar_init(&sm.qempty[s], 1);
      mbar_init(&sm.mfull[s], 32);
      mbar_init(&sm.mempty[s], 512);
      mbar_init(&sm.sa[s], 1);
      mbar_init(&sm.ew[s], 512);
      mbar_init(&sm.dq[s], 1);
    }
    mbar_init(&sm.kvdone, 1);
    mbar_init(&sm.kvfree, 512);
    mbar_init(&sm.dqdone, 1);
    mbar_init(&sm.dqfree, 512);
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
    // ---- producer ----------------------------------------------------------
    if (lane == 0) {
      prefetch_tmap(&tqkv);
      prefetch_tmap(&tdo);
    }
    for (int k = 0; k < n_local; ++k) {
      const int item = (int)blockIdx.x + k * G;
      const int seq = item / H, h = item - seq * H;
      const bool prefix = seq >= a.n_causal;
      const int pseq = seq - a.n_causal;
      const int row0 = seq * S;
      const long long lrow = ((long long)seq * H + h) * S;
      // row metadata (double-buffered per item): all of a lane's global loads
      // first (one round trip, overlapping the wait for the buffer); causal
      // rows: block id = first row of the block = row
      constexpr int kJ = kMaxS / 32;
      float Lv[kJ], Dv[kJ];
      int fv[kJ], bv[kJ];
      #pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const int i = lane + 32 * j;
        Lv[j] = 0.f;
        Dv[j] = 0.f;
        fv[j] = bv[j] = i;
        if (i < S) {
          Lv[j] = __ldg(a.lse + lrow + i);
          Dv[j] = __ldg(a.dsum + lrow + i);
          if (prefix) {
            const long long o = (long long)pseq * S + i;
            fv[j] = __ldg(a.first + o);
            bv[j] = __ldg(a.bid + o);
          }
        }
      }
      const int m = k & 1;
      if (k >= 2) mbar_wait(&sm.mempty[m], ((k >> 1) - 1) & 1, abort_flag);
      Meta& mt = sm.meta[m];
      bool runs_ok = true;  // a row whose id differs from the previous row's opens that id's first run
      #pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const int i = lane + 32 * j;
        const bool ok = i < S;
        // the previous row's id: lane - 1's, or lane 31's of the previous group
        int prev = __shfl_up_sync(0xffffffffu, bv[j], 1);
        const int prev31 = __shfl_sync(0xffffffffu, bv[j > 0 ? j - 1 : 0], 31);
        if (lane == 0) prev = prev31;
        mt.L[i] = Lv[j];
        mt.D[i] = Dv[j];
        mt.first[i] = ok ? fv[j] : S;
        const int b = ok ? bv[j] : -1;
        mt.bid[i] = b;
        if (prefix && ok && i > 0 && b != prev && fv[j] != i) runs_ok = false;
      }
      runs_ok = __all_sync(0xffffffffu, runs_ok);
      if (lane == 0) mt.contig = runs_ok ? 1 : 0;
      mbar_arrive(&sm.mfull[m]);
      // operand slots, in the order the item's first sub-units need them
      auto load_kv = [&](int kt) {
        if (k >= 1) mbar_wait(&sm.kvempty[kt], (k - 1) & 1, abort_flag);
        if (lane == 0) {
          mbar_arrive_expect_tx(&sm.kvfull[kt], 4 * kBox);
          for (int b = 0; b < 2; ++b) {
            const int r = row0 + kt * 128 + b * 64;
            tma_load_2d(sm.KV[kt] + b * kBox, &tqkv, &sm.kvfull[kt], E + h * kHd, r);
            tma_load_2d(sm.KV[kt] + (2 + b) * kBox, &tqkv, &sm.kvfull[kt], 2 * E + h * kHd, r);
          }
        }
      };
      auto load_q = [&](int qh) {
        if (k >= 1) mbar_wait(&sm.qempty[qh], (k - 1) & 1, abort_flag);
        if (lane == 0) {
          mbar_arrive_expect_tx(&sm.qfull[qh], 4 * kBox);
          for (int b = 0; b < 2; ++b) {
            const int r = row0 + qh * 128 + b * 64;
            tma_load_2d(sm.QO[qh] + b * kBox, &tqkv, &sm.qfull[qh], h * kHd, r);
            tma_load_2d(sm.QO[qh] + (2 + b) * kBox, &tdo, &sm.qfull[qh], h * kHd, r);
          }
        }
      };
      load_kv(0);
      load_q(0);
      if (nkt > 1) {
        load_q(1);
        load_kv(1);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue -----------------------------------------------------------
    // the whole warp runs the issue loop; one elected lane issues (uniform operands)
    {
      const uint32_t id_s = make_idesc_bf16(128, 64, false, false);   // S^T, dP^T: N = 64 queries
      const uint32_t id_kn = make_idesc_bf16(128, kHd, false, true);  // dV, dK: B read MN-major
      const uint32_t id_nn = make_idesc_bf16(128, kHd, true, true);   // dQ: A (dS) and B (K) MN-major
      int g_issued = 0;    // global index of the next sub-unit whose MMA-A is to be issued
      int ka = 0, ua = 0;  // its item and unit
      Units units_a;
      bool have_a = false;
      auto next_a = [&]() {  // advance (ka, ua) to the next sub-unit; false when none is left
        while (true) {
          if (!have_a) {
            if (ka >= n_local) return false;
            const int item = (int)blockIdx.x + ka * G;
            const int seq = item / H;
            units_a = item_units(a, seq >= a.n_causal, seq - a.n_causal);
            have_a = true;
            ua = 0;
          }
          if (ua < units_a.n) return true;
          have_a = false;
          ++ka;
        }
      };
      // Issues MMA-A of the next sub-unit not yet issued, unless it belongs to
      // an item after `max_item`: the next item's operands are loaded into
      // slots this item releases, so its MMA-A waits for loads that can only
      // start after this item's release commits.
      auto issue_a = [&](int max_item) {
        if (!next_a() || ka > max_item) return;
        const int kt = units_a.kt(ua), qs = units_a.qs(ua), qh = qs >> 1;
        const int b = g_issued & 1;
        mbar_wait(&sm.kvfull[kt], ka & 1, abort_flag);
        mbar_wait(&sm.qfull[qh], ka & 1, abort_flag);
        tc_fence_after();
        const uint32_t kb = smem_u32(sm.KV[kt]), vb = kb + 2 * kBox;
        const uint32_t qb = smem_u32(sm.QO[qh]) + (qs & 1) * kBox, ob = smem_u32(sm.QO[qh]) + (2 + (qs & 1)) * kBox;
        #pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          umma_f16_w(tmem + b * 128, make_sdesc(kb + kk * 32, 16, 1024), make_sdesc(qb + kk * 32, 16, 1024), id_s,
                   kk > 0 ? 1u : 0u);
          umma_f16_w(tmem + b * 128 + 64, make_sdesc(vb + kk * 32, 16, 1024), make_sdesc(ob + kk * 32, 16, 1024),
                   id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit_w(&sm.sa[b]);
        ++g_issued;
        ++ua;
      };
      issue_a(0);
      issue_a(0);
      int g = 0;   // global sub-unit index
      int c = 0;   // global key-tile block index (dV / dK accumulations)
      for (int k = 0; k < n_local; ++k) {
        const int item = (int)blockIdx.x + k * G;
        const int seq = item / H;
        const Units un = item_units(a, seq >= a.n_causal, seq - a.n_causal);
        // last sub-unit reading each query slot
        int last_q0 = -1, last_q1 = -1;
        for (int u = 0; u < un.n; ++u) {
          if ((un.qs(u) >> 1) == 0) last_q0 = u;
          else last_q1 = u;
        }
        uint32_t dq_seen = 0;
        for (int u = 0; u < un.n; ++u, ++g) {
          const int kt = un.kt(u), qs = un.qs(u), qh = qs >> 1;
          const int b = g & 1, pb = (g >> 1) & 1;
          const bool first_kt = u == 0 || un.kt(u - 1) != kt;
          const bool last_kt = u == un.n - 1 || un.kt(u + 1) != kt;
          mbar_wait(&sm.ew[b], (g >> 1) & 1, abort_flag);
          if (first_kt && c > 0) mbar_wait(&sm.kvfree, (c - 1) & 1, abort_flag);
          tc_fence_after();
          const uint32_t qb = smem_u32(sm.QO[qh]) + (qs & 1) * kBox, ob = smem_u32(sm.QO[qh]) + (2 + (qs & 1)) * kBox;
          const uint32_t dsb = smem_u32(sm.dST[pb][qs & 1]);
          #pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 64 queries, 16 per step
            const uint32_t acc = (!first_kt || kk > 0) ? 1u : 0u;
            const uint32_t pcol = (uint32_t)(b * 128 + kk * 16);
            umma_f16_ts_w(tmem + 256, tmem + pcol, make_sdesc(ob + kk * 2048, 8192, 1024), id_kn, acc);
            umma_f16_w(tmem + 320, make_sdesc(dsb + kk * 32, 16, 1024), make_sdesc(qb + kk * 2048, 8192, 1024), id_kn,
                     acc);
          }
          if (qs & 1) {
            // dQ_qh += dS K_kt over the pair's 128 queries (A: the two dS^T tiles, MN-major)
            if (dq_seen == 0 && k > 0) mbar_wait(&sm.dqfree, (k - 1) & 1, abort_flag);
            tc_fence_after();
            const uint32_t pair = smem_u32(sm.dST[pb][0]);
            const uint32_t kb = smem_u32(sm.KV[kt]);
            const bool first_q = ((dq_seen >> qh) & 1u) == 0;
            #pragma unroll
            for (int kk = 0; kk < 8; ++kk)  // 128 keys
              umma_f16_w(tmem + 384 + qh * 64, make_sdesc(pair + kk * 2048, 16384, 1024),
                       make_sdesc(kb + kk * 2048, 8192, 1024), id_nn, (!first_q || kk > 0) ? 1u : 0u);
            dq_seen |= 1u << qh;
            tc_commit_w(&sm.dq[pb]);
          }
          if (last_kt) {
            tc_commit_w(&sm.kvdone);
            tc_commit_w(&sm.kvempty[kt]);
            ++c;
          }
          if (u == last_q0) tc_commit_w(&sm.qempty[0]);
          if (u == last_q1) tc_commit_w(&sm.qempty[1]);
          if (u == un.n - 1) tc_commit_w(&sm.dqdone);
          // keep MMA-A two sub-units ahead; across an item boundary only once
          // every release commit of this item has been issued
          const int max_item = u == un.n - 1 ? k + 1 : k;
          while (g_issued < g + 3 && next_a() && ka <= max_item) issue_a(max_item);
        }
      }
    }
  } else {
    // ---- elementwise + epilogues -------------------------------------------
    const int quad = warp & 3;
    const int g4 = (warp - 2) >> 2;  // 16-query group of the 64-query sub-tile
    const int r = quad * 32 + lane;  // key row within the key tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    uint8_t* stg = sm.stage[quad];
    const int qbar = 1 + quad;  // named barrier of the 4 warps that own this lane quadrant
    const float sl2 = 0.125f * kLog2e;
    int g = 0, c = 0;
    // The epilogues run one sub-unit late: after the last sub-unit of a key
    // tile (or of an item) the warps go on with the next sub-unit, whose MMA-A
    // is already in flight, while that tile's last products retire.
    int kv_pend = -1, kv_j0 = 0, kv_h = 0;  // pending dV / dK store: block index, first key row, head
    long long kv_row0 = 0;  // global row of the pending key tile's sequence start
    int dq_pend = -1, dq_h = 0;             // pending dQ store: item index, head
    long long dq_row0 = 0;
    // one 32-row x 64-dim block of dQ / dK / dV (rows from global row row0, columns
    // [col, col + 64) of q|k|v): bf16, or 8-bit with its amax (fp8 recipe)
    float q8m = 0.f;
    auto emit = [&](const uint32_t (&v)[16], float scale, const Rope16& rp, long long row0, int col, int nvalid) {
      const bool mine = lane < nvalid;  // this thread's own row (row0 + lane) lies inside the sequence
      if constexpr (Q8) {
        float f[16];
        rotate16(v, scale, rp, f);
        const float qm = quad_store_q8(stg, qbar, lane, g4, f, *a.q8.qscale, a.q8.fmt,
                                       a.q8.q + row0 * a.q8.ldq + col, a.q8.ldq, nvalid);
        if (mine) q8m = fmaxf(q8m, qm);
      } else {
        uint32_t w[8];
        rotate_pack16(v, scale, rp, w);
        quad_store(stg, qbar, lane, g4, w, a.dqkv + row0 * 3 * E + col, 3 * E, nvalid);
      }
    };
    auto kv_epilogue = [&]() {
      // dV, dK of the key tile complete: this thread stores dims [16 g, 16 g + 16) of its key row
      const int j = kv_j0 + r;
      const Rope16 rk = load_rope16(a.rope, j, g4 * 16, j < S);
      mbar_wait(&sm.kvdone, kv_pend & 1, abort_flag);
      tc_fence_after();
      uint32_t vv[16], kv[16];
      tmem_ld_x16_nowait(tmem + lane_off + 256 + g4 * 16, vv);
      tmem_ld_x16_nowait(tmem + lane_off + 320 + g4 * 16, kv);
      tmem_wait_ld_dep16(vv);
      tmem_wait_ld_dep16(kv);
      tc_fence_before();
      mbar_arrive(&sm.kvfree);
      const int jq = kv_j0 + quad * 32;  // first key row of this quadrant
      const int nvalid = min(max(S - jq, 0), 32);
      emit(kv, 0.125f, rk, kv_row0 + jq, E + kv_h * kHd, nvalid);
      emit(vv, 1.f, load_rope16(nullptr, 0, 0, false), kv_row0 + jq, 2 * E + kv_h * kHd, nvalid);
      kv_pend = -1;
    };
    auto dq_epilogue = [&]() {
      // dQ of both query halves (lane = query row within the half)
      const Rope16 r0 = load_rope16(a.rope, r, g4 * 16, r < S);
      const Rope16 r1 = load_rope16(a.rope, 128 + r, g4 * 16, nkt > 1 && 128 + r < S);
      mbar_wait(&sm.dqdone, dq_pend & 1, abort_flag);
      tc_fence_after();
      uint32_t q0v[16], q1v[16];
      tmem_ld_x16_nowait(tmem + lane_off + 384 + g4 * 16, q0v);
      if (nkt > 1) tmem_ld_x16_nowait(tmem + lane_off + 448 + g4 * 16, q1v);
      tmem_wait_ld_dep16(q0v);
      if (nkt > 1) tmem_wait_ld_dep16(q1v);
      tc_fence_before();
      mbar_arrive(&sm.dqfree);
      emit(q0v, 0.125f, r0, dq_row0 + quad * 32, dq_h * kHd, min(max(S - quad * 32, 0), 32));
      if (nkt > 1) emit(q1v, 0.125f, r1, dq_row0 + 128 + quad * 32, dq_h * kHd, min(max(S - 128 - quad * 32, 0), 32));
      dq_pend = -1;
    };
    for (int k = 0; k < n_local; ++k) {
      const int item = (int)blockIdx.x + k * G;
      const int seq = item / H, h = item - seq * H;
      const bool prefix = seq >= a.n_causal;
      const Units un = item_units(a, prefix, seq - a.n_causal);
      const int m = k & 1;
      mbar_wait(&sm.mfull[m], (k >> 1) & 1, abort_flag);
      const Meta& mt = sm.meta[m];
      const bool contig = mt.contig != 0;
      const long long rowbase = (long long)seq * S;
      for (int u = 0; u < un.n; ++u, ++g) {
        const int kt = un.kt(u), qs = un.qs(u);
        const int b = g & 1, P = g >> 1, pb = P & 1;
        const bool last_kt = u == un.n - 1 || un.kt(u + 1) != kt;
        const int j = kt * 128 + r;
        const bool jok = j < S;
        const int fj = jok ? mt.first[j] : S;
        const int bj = jok ? mt.bid[j] : -2;
        const int q0 = qs * 64 + g4 * 16;  // this thread's 16 queries
        // a key row j sees the queries i >= first_j (< S) when the blocks are
        // contiguous; otherwise i >= j, or first_j <= i < j with j's block id
        // (the interval [first_j, S) is masked further below)
        const bool none = !jok || q0 + 15 < fj || q0 >= S;
        const bool none_w = __all_sync(0xffffffffu, none);
        // every lane's 16 queries visible (below the diagonal): no interval mask
        const bool full_w = __all_sync(0xffffffffu, jok && fj <= q0 && q0 + 16 <= S);
        // the pair buffer is free once the dQ product of pair P - 2 has retired
        if ((u & 1) == 0 && P >= 2) mbar_wait(&sm.dq[pb], ((P >> 1) - 1) & 1, abort_flag);
        mbar_wait(&sm.sa[b], (g >> 1) & 1, abort_flag);
        tc_fence_after();
        uint32_t pk[8], dk[8];
        #pragma unroll
        for (int e = 0; e < 8; ++e) pk[e] = dk[e] = 0u;
        if (!none_w) {
          uint32_t su[16], du[16];
          tmem_ld_x16_nowait(tmem + lane_off + b * 128 + g4 * 16, su);
          tmem_ld_x16_nowait(tmem + lane_off + b * 128 + 64 + g4 * 16, du);
          tmem_wait_ld_dep16(su);
          tmem_wait_ld_dep16(du);
          if (!none) {
            const int e_lo = max(fj - q0, 0), e_hi = min(S - q0, 16);
            if (full_w) ew16<false>(su, du, mt.L + q0, mt.D + q0, sl2, e_lo, e_hi, pk, dk);
            else ew16<true>(su, du, mt.L + q0, mt.D + q0, sl2, e_lo, e_hi, pk, dk);
            if (!contig) {
              // a query before the key row sees it only within the key's block
              #pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int i = q0 + e;
                if (i < j && i >= fj && mt.bid[i] != bj) {
                  const uint32_t keep = (e & 1) ? 0x0000ffffu : 0xffff0000u;
                  pk[e >> 1] &= keep;
                  dk[e >> 1] &= keep;
                }
              }
            }
          }
        }
        // P^T over this thread's own (already read) S^T columns; dS^T into the pair buffer
        tmem_st_x8(tmem + lane_off + b * 128 + g4 * 16, pk);
        uint8_t* dst = sm.dST[pb][qs & 1];
        #pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int chunk = g4 * 2 + q;  // 16-byte chunk of the 128-byte row
          *reinterpret_cast<uint4*>(dst + r * 128 + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(dk[4 * q], dk[4 * q + 1], dk[4 * q + 2], dk[4 * q + 3]);
        }
        tmem_wait_st();
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(&sm.ew[b]);
        if (kv_pend >= 0) kv_epilogue();
        if (dq_pend >= 0) dq_epilogue();
        if (last_kt) {
          kv_pend = c++;
          kv_j0 = kt * 128;
          kv_h = h;
          kv_row0 = rowbase;
        }
      }
      mbar_arrive(&sm.mempty[m]);
      dq_pend = k;
      dq_h = h;
      dq_row0 = rowbase;
    }
    if (kv_pend >= 0) kv_epilogue();
    if (dq_pend >= 0) dq_epilogue();
    if (Q8 && a.q8.amax) {
      const float m = warp_max(q8m);
      if (lane == 0 && m > 0.f) atomicMax(reinterpret_cast<int*>(a.q8.amax), __float_as_int(m));
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

}  // namespace pstbwd

int launch_attn_dsum(const void* out, const void* dout, float* dsum, int64_t T, int64_t S, int64_t H,
                     cudaStream_t stream);

// Host launcher used by cdk_attn_bwd for S <= 256.
int launch_attn_bwd_pst(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum,
                        void* dqkv, int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid,
                        const int32_t* meta, const float* rope, cudaStream_t stream, const Q8Out* q8) {
  using namespace pstbwd;
  if (S > kMaxS || S <= 0) return -20;
  if (nseq * H > (int64_t)1 << 30) return -5;
  CUtensorMap tq, tdo;
  if (!make_tmap(&tq, qkv, 3 * H * kHd, nseq * S, 3 * H * kHd, 64, 64)) return -21;
  if (!make_tmap(&tdo, dout, H * kHd, nseq * S, H * kHd, 64, 64)) return -21;
  int rc = launch_attn_dsum(out, dout, dsum, nseq * S, S, H, stream);
  if (rc != 0) return rc;
  Args a;
  a.lse = lse;
  a.dsum = dsum;
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv);
  a.q8.q = nullptr;
  a.q8.ldq = 0;
  a.q8.fmt = 0;
  a.q8.qscale = nullptr;
  a.q8.amax = nullptr;
  if (q8 != nullptr) a.q8 = *q8;
  if (a.q8.q == nullptr && dqkv == nullptr) return -1;
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
  a.n_items = (int)(nseq * H);
  const size_t smem = sizeof(BwdSmem) + 1024;
  static int sm_count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return -24;
  if (sm_count[dev] == 0) {
    for (auto k : {attn_bwd_pst_kernel<false>, attn_bwd_pst_kernel<true>}) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
      // tcgen05.alloc blocks until columns are free: one 512-column CTA per SM
      int per_sm = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem);
      if (e != cudaSuccess) return (int)e;
      if (per_sm != 1) return -22;
    }
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return (int)e;
    sm_count[dev] = sms;
  }
  const int grid = (int)(nseq * H < sm_count[dev] ? nseq * H : sm_count[dev]);
  if (a.q8.q) attn_bwd_pst_kernel<true><<<grid, kThreads, smem, stream>>>(tq, tdo, a);
  else attn_bwd_pst_kernel<false><<<grid, kThreads, smem, stream>>>(tq, tdo, a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace cdk
