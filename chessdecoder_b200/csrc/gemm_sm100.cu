// Warp-specialised persistent bf16 / fp8 GEMM for sm_100a: TMA -> shared-memory
// ring -> tcgen05.mma (issued by one elect.sync lane of the MMA warp) ->
// double-buffered TMEM accumulators -> eight epilogue warps with fused
// epilogues (RoPE, SwiGLU forward / backward, residual add, split-K bulk
// reduce-add).
//
// Replaces the nn.Linear forward/backward calls of the reference model
// (chessdecoder/models/model.py:96-108, 119-136) that PyTorch dispatches to
// cuBLAS.  Roles inside one CTA (320 threads, 352 with the TMA-fed / TMA-stored
// epilogues, one CTA per SM):
//   warp 0      TMA producer (lane 0)
//   warp 1      TMEM allocator + MMA issuer (whole warp, one elected lane)
//   warps 2..9  epilogue; warp w owns TMEM lanes 32*(w%4) .. +31, warps w and
//               w+4 split the columns of those rows
//   warp 10     epilogue operand / output streaming (lane 0), when present
// CTA-pair form (the default where M is a multiple of 256): clusters of two
// CTAs walk 256-row units; each loads its 128 A rows and half of the B tile,
// the even CTA issues tcgen05.mma.cta_group::2 with M=256, and each CTA's
// epilogue reads its own 128 accumulator rows.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

#include <cstdlib>
#include <cstring>
#include <mutex>

namespace cdk {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = 128 B = one swizzle row (128 fp8 elements in the fp8 instantiations)
constexpr int kThreads = 320;
// TMA-fed epilogue (residual add, SwiGLU backward): an 11th warp streams the
// epilogue's global operand through 64 KB of shared-memory slots (boxes of
// 128 rows x 128 bytes) and writes the results back by TMA store; the
// mainloop ring gives up one (BN=256) stage for it.
constexpr int kThreadsTE = 352;
constexpr int kTeSlots = 8;
constexpr int kTeSlotBytes = 8192;
// Store-only form for the bf16 epilogues (plain store, RoPE, SwiGLU forward):
// the epilogue warps write 64-column x 128-row bf16 boxes (128-byte swizzle)
// into 2 x 16 KB slots and the 11th warp stores them with TMA, so the output
// leaves as full 128-byte row segments.
constexpr int kTe2Slots = 2;
constexpr int kTe2SlotBytes = 16384;

template <int BN>
struct GemmCfg {
  static constexpr int kBytesA = kBM * kBK * 2;
  static constexpr int kBytesB = BN * kBK * 2;
  static constexpr int kStageBytes = kBytesA + kBytesB;
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kStagingBytes = 8 * 2560;  // per epilogue warp: 32 rows x 80 B transpose buffer
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + kBarrierBytes + kStagingBytes;
  static constexpr int kStagesTE = BN == 256 ? 3 : 5;
  static constexpr int kSmemBytesTE = kStagesTE * kStageBytes + 1024 + kTeSlots * kTeSlotBytes + kBarrierBytes;
  static constexpr int kSmemBytesTE2 = kStages * kStageBytes + 1024 + kTe2Slots * kTe2SlotBytes + kBarrierBytes;
  // CTA-pair form (BN = 256): each CTA holds its 128 A rows and half of the B
  // rows of a stage, so a stage is 32 KB and the ring six deep (five with the
  // TMA-fed epilogue's 64 KB of slots)
  static constexpr int kStageBytesPair = kBytesA + kBytesB / 2;
  // pair = 2: the SwiGLU store form (three output boxes per 64 columns)
  // trades a stage for two more 16 KB output slots
  static constexpr int stages_pair(int tem, int pair) { return tem == 1 || pair == 2 ? 5 : 6; }
  static constexpr int te2_slots_pair(int pair) { return pair == 2 ? 4 : kTe2Slots; }
  static constexpr int slot_area_pair(int tem, int pair) {
    return tem == 1 ? kTeSlots * kTeSlotBytes : te2_slots_pair(pair) * kTe2SlotBytes;
  }
  static constexpr int smem_pair(int tem, int pair) {
    return stages_pair(tem, pair) * kStageBytesPair + 1024 + slot_area_pair(tem, pair) + kBarrierBytes;
  }
};

struct EpiDev {
  int kind;
  int seq_len;
  int rope_cols;
  int vec;  // 1: full 16-column chunks with 16-byte aligned rows -> warp-cooperative (coalesced) path
  void* out;
  long long ldo;
  const float* bias;
  const float* resid;
  long long ldr;
  void* out2;
  long long ldo2;
  const __nv_bfloat16* aux;
  long long ldaux;
  long long half_n;
  const float* rope;
};

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, splits, k_tiles, k_per_split;
  int dual;      // SWIGLU: B tile = rows [n0, n0+BN/2) and [n0+b_off, ...)
  int b_off;
  uint32_t idesc_f8;           // fp8 instantiations: kind::f8f6f4 descriptor (operand formats)
  int pair;                    // 1: clusters of 2 CTAs issuing 2-SM (M=256) MMAs; m_tiles counts 256-row tiles
  const float* scale_inv_a;    // fp8: dequantisation factors (device scalars), else null
  const float* scale_inv_b;
  EpiDev epi;
};

// Unit walk of a CTA: one unit per CTA pair in the 2-SM form (both CTAs walk
// the same units), each CTA's own 128-row tile of the unit's 256 rows.
__device__ __forceinline__ int unit_start(const GemmParams& p) { return p.pair ? (int)blockIdx.x >> 1 : (int)blockIdx.x; }
__device__ __forceinline__ int unit_stride(const GemmParams& p) { return p.pair ? (int)gridDim.x >> 1 : (int)gridDim.x; }
__device__ __forceinline__ int tile_row0(const GemmParams& p, int mt) {
  return (p.pair ? mt * 2 + (int)cluster_ctarank() : mt) * kBM;
}

__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_fast(x); }

// ---- epilogue store helpers (one thread = one row, kC consecutive columns) --
constexpr int kC = 16;  // columns per epilogue chunk (one tcgen05.ld.32x32b.x16)

__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const float (&v)[kC], int ncols) {
  if (ncols >= kC && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    #pragma unroll
    for (int q = 0; q < kC / 8; ++q) {
      uint4 w;
      w.x = pack_bf16(v[8 * q + 0], v[8 * q + 1]);
      w.y = pack_bf16(v[8 * q + 2], v[8 * q + 3]);
      w.z = pack_bf16(v[8 * q + 4], v[8 * q + 5]);
      w.w = pack_bf16(v[8 * q + 6], v[8 * q + 7]);
      d4[q] = w;
    }
  } else {
    #pragma unroll
    for (int i = 0; i < kC; ++i)
      if (i < ncols) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

__device__ __forceinline__ void store_row_f32(float* dst, const float (&v)[kC], int ncols) {
  if (ncols >= kC && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    float4* d4 = reinterpret_cast<float4*>(dst);
    #pragma unroll
    for (int q = 0; q < kC / 4; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
    #pragma unroll
    for (int i = 0; i < kC; ++i)
      if (i < ncols) dst[i] = v[i];
  }
}

__device__ __forceinline__ void load_row_f32(const float* src, float (&v)[kC], int ncols) {
  if (ncols >= kC && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
    #pragma unroll
    for (int q = 0; q < kC / 4; ++q) {
      float4 t = s4[q];
      v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
    }
  } else {
    #pragma unroll
    for (int i = 0; i < kC; ++i) v[i] = i < ncols ? src[i] : 0.f;
  }
}

__device__ __forceinline__ void load_row_bf16(const __nv_bfloat16* src, float (&v)[kC]) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  #pragma unroll
  for (int q = 0; q < kC / 8; ++q) {
    uint4 w = s4[q];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      v[8 * q + 2 * j] = f.x;
      v[8 * q + 2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void atomic_row_f32(float* dst, const float (&v)[kC], int ncols) {
  if (ncols >= kC && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    float4* d4 = reinterpret_cast<float4*>(dst);
    #pragma unroll
    for (int q = 0; q < kC / 4; ++q) atomicAdd(d4 + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
  } else {
    #pragma unroll
    for (int i = 0; i < kC; ++i)
      if (i < ncols) atomicAdd(dst + i, v[i]);
  }
}

// 16 accumulator columns of this thread's row, times the dequantisation
// factor `sc` (1 for bf16 operands; 1/(scale_a * scale_b) for fp8 operands).
__device__ __forceinline__ void tmem_ld_f16cols(uint32_t taddr, float (&v)[kC], float sc) {
  uint32_t u[kC];
  tmem_ld_x16_nowait(taddr, u);
  tmem_wait_ld();
  #pragma unroll
  for (int i = 0; i < kC; ++i) v[i] = __uint_as_float(u[i]) * sc;
}

// L2 prefetch of the global operand an epilogue tile will read (residual /
// accumulator rows, or the gate|up rows of the SwiGLU backward): one prefetch
// per 128-byte line of this thread's row segment, issued a tile ahead so that
// the DRAM latency overlaps the mainloop instead of the epilogue.
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

template <int BN>
__device__ __forceinline__ void epi_prefetch(const EpiDev& e, const GemmParams& p, int row, int n0, int half) {
  if (row >= p.M) return;
  if (e.kind == CDK_EPI_RESID_F32 || e.kind == CDK_EPI_ACCUM_F32) {
    const float* base = e.kind == CDK_EPI_RESID_F32 ? e.resid + (long long)row * e.ldr
                                                    : reinterpret_cast<const float*>(e.out) + (long long)row * e.ldo;
    #pragma unroll
    for (int c = half; c < BN / 32; c += 2)
      if (n0 + c * 32 < p.N) prefetch_l2(base + n0 + c * 32);
  } else if (e.kind == CDK_EPI_DSWIGLU) {
    const __nv_bfloat16* base = e.aux + (long long)row * e.ldaux;
    #pragma unroll
    for (int c = half; c < BN / 64; c += 2)
      if (n0 + c * 64 < p.N) {
        prefetch_l2(base + n0 + c * 64);
        prefetch_l2(base + e.half_n + n0 + c * 64);
      }
  }
}

// ---- warp-cooperative row transfers ------------------------------------------
// A warp's 32 epilogue rows (lane = row) x 16 columns go through a per-warp
// shared-memory buffer so that global accesses are row-contiguous: a store
// instruction writes 8 rows x 64 B (fp32) or 16 rows x 32 B (bf16) instead of
// 32 scattered 16-byte pieces.  Row strides of 20 / 12 words make both the
// row-wise and the transposed 16-byte accesses conflict-free.
constexpr int kStgF32 = 20;
constexpr int kStgB16 = 12;
constexpr int kStgWords = 32 * kStgF32;

__device__ __forceinline__ void warp_store_f32(uint32_t* stg, const float (&v)[kC], float* g, long long ld,
                                               int nvalid, int lane) {
  float4* my = reinterpret_cast<float4*>(stg + lane * kStgF32);
  #pragma unroll
  for (int q = 0; q < 4; ++q) my[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __syncwarp();
  const int c = lane & 3;
  #pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = k * 8 + (lane >> 2);
    const float4 t = *reinterpret_cast<const float4*>(stg + r * kStgF32 + c * 4);
    if (r < nvalid) *reinterpret_cast<float4*>(g + (long long)r * ld + c * 4) = t;
  }
  __syncwarp();
}

__device__ __forceinline__ void warp_store_bf16(uint32_t* stg, const float (&v)[kC], __nv_bfloat16* g, long long ld,
                                                int nvalid, int lane) {
  uint4* my = reinterpret_cast<uint4*>(stg + lane * kStgB16);
  my[0] = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
  my[1] = make_uint4(pack_bf16(v[8], v[9]), pack_bf16(v[10], v[11]), pack_bf16(v[12], v[13]),
                     pack_bf16(v[14], v[15]));
  __syncwarp();
  const int c = lane & 1;
  #pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int r = k * 16 + (lane >> 1);
    const uint4 t = *reinterpret_cast<const uint4*>(stg + r * kStgB16 + c * 4);
    if (r < nvalid) *reinterpret_cast<uint4*>(g + (long long)r * ld + c * 8) = t;
  }
  __syncwarp();
}

// Row-contiguous fp32 loads of 32 rows x 16 columns: issue() starts them,
// finish() transposes through shared memory so that lane = row again.
__device__ __forceinline__ void warp_load_f32_issue(float4 (&t)[4], const float* g, long long ld, int nvalid,
                                                    int lane) {
  const int c = lane & 3;
  #pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = k * 8 + (lane >> 2);
    t[k] = r < nvalid ? __ldg(reinterpret_cast<const float4*>(g + (long long)r * ld + c * 4))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}
__device__ __forceinline__ void warp_load_f32_finish(uint32_t* stg, const float4 (&t)[4], float (&v)[kC], int lane) {
  const int c = lane & 3;
  #pragma unroll
  for (int k = 0; k < 4; ++k) *reinterpret_cast<float4*>(stg + (k * 8 + (lane >> 2)) * kStgF32 + c * 4) = t[k];
  __syncwarp();
  const float4* my = reinterpret_cast<const float4*>(stg + lane * kStgF32);
  #pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 x = my[q];
    v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
  }
  __syncwarp();
}

// Row-contiguous bf16 loads of 32 rows x 16 columns (two lanes per row),
// transposed through shared memory so that lane = row.
__device__ __forceinline__ void warp_load_bf16_issue(uint4 (&t)[2], const __nv_bfloat16* g, long long ld, int nvalid,
                                                     int lane) {
  const int c = lane & 1;
  #pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int r = k * 16 + (lane >> 1);
    t[k] = r < nvalid ? __ldg(reinterpret_cast<const uint4*>(g + (long long)r * ld + c * 8)) : make_uint4(0, 0, 0, 0);
  }
}
__device__ __forceinline__ void warp_load_bf16_finish(uint32_t* stg, const uint4 (&t)[2], float (&v)[kC], int lane) {
  const int c = lane & 1;
  #pragma unroll
  for (int k = 0; k < 2; ++k) *reinterpret_cast<uint4*>(stg + (k * 16 + (lane >> 1)) * kStgB16 + c * 4) = t[k];
  __syncwarp();
  #pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 w = *reinterpret_cast<const uint4*>(stg + lane * kStgB16 + q * 4);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[8 * q + 2 * j] = f.x;
      v[8 * q + 2 * j + 1] = f.y;
    }
  }
  __syncwarp();
}

// Coalesced variants of the forward epilogues (row0 = the warp's first row).
// Software-pipelined: the TMEM load of chunk c+1 is in flight while chunk c is
// converted and stored, and the residual rows arrive two chunks ahead.
__device__ __forceinline__ void unpack_scaled(const uint32_t (&u)[kC], float (&v)[kC], float sc) {
  #pragma unroll
  for (int i = 0; i < kC; ++i) v[i] = __uint_as_float(u[i]) * sc;
}

template <int BN, bool F8>
__device__ __forceinline__ void epi_vec(const EpiDev& e, const GemmParams& p, uint32_t tbase, int row0, int n0,
                                        int half, uint32_t* stg, int lane, float sc) {
  const int nvalid = min(32, p.M - row0);
  const int row = row0 + lane;
  if (e.kind == CDK_EPI_SWIGLU) {
    __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(e.out2) + (long long)row0 * e.ldo2;
    __nv_bfloat16* uo = reinterpret_cast<__nv_bfloat16*>(e.out) + (long long)row0 * e.ldo;
    const int nch = min(BN / 64, (p.N - n0 - half * kC + 31) / 32);
    uint32_t ug[kC], uu[kC];
    if (nch > 0) {
      tmem_ld_x16_nowait(tbase + half * kC, ug);
      tmem_ld_x16_nowait(tbase + BN / 2 + half * kC, uu);
    }
    #pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      const int col = n0 + c * 32 + half * kC;
      float g[kC], up[kC], h[kC];
      tmem_wait_ld();
      unpack_scaled(ug, g, sc);
      unpack_scaled(uu, up, sc);
      if (c + 1 < nch) {
        tmem_ld_x16_nowait(tbase + (c + 1) * 32 + half * kC, ug);
        tmem_ld_x16_nowait(tbase + BN / 2 + (c + 1) * 32 + half * kC, uu);
      }
      #pragma unroll
      for (int i = 0; i < kC; ++i) h[i] = silu_f(g[i]) * up[i];
      warp_store_bf16(stg, g, gu + col, e.ldo2, nvalid, lane);
      warp_store_bf16(stg, up, gu + e.half_n + col, e.ldo2, nvalid, lane);
      warp_store_bf16(stg, h, uo + col, e.ldo, nvalid, lane);
    }
    return;
  }
  const int nch = min(BN / 32, (p.N - n0 - half * kC + 31) / 32);
  if (nch <= 0) return;
  uint32_t ua[kC];
  tmem_ld_x16_nowait(tbase + half * kC, ua);
  if (!F8 && e.kind == CDK_EPI_DSWIGLU) {  // (the host keeps fp8 DSWIGLU launches off this path)
    // acc = d(silu(g) * u) for columns n0..; aux = [g | u]; out = [dg | du]
    const __nv_bfloat16* abase = e.aux + (long long)row0 * e.ldaux;
    __nv_bfloat16* obase = reinterpret_cast<__nv_bfloat16*>(e.out) + (long long)row0 * e.ldo;
    uint4 g0[2], u0[2];
    warp_load_bf16_issue(g0, abase + n0 + half * kC, e.ldaux, nvalid, lane);
    warp_load_bf16_issue(u0, abase + e.half_n + n0 + half * kC, e.ldaux, nvalid, lane);
    #pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      const int col = n0 + c * 32 + half * kC;
      float g[kC], up[kC], v[kC];
      warp_load_bf16_finish(stg, g0, g, lane);
      warp_load_bf16_finish(stg, u0, up, lane);
      if (c + 1 < nch) {  // the next chunk's gate / up rows (L2-prefetched a tile ahead)
        warp_load_bf16_issue(g0, abase + col + 32, e.ldaux, nvalid, lane);
        warp_load_bf16_issue(u0, abase + e.half_n + col + 32, e.ldaux, nvalid, lane);
      }
      tmem_wait_ld();
      unpack_scaled(ua, v, sc);
      if (c + 1 < nch) tmem_ld_x16_nowait(tbase + (c + 1) * 32 + half * kC, ua);
      float dg[kC], du[kC];
      #pragma unroll
      for (int i = 0; i < kC; ++i) {
        const float sg = sigmoid_fast(g[i]);
        du[i] = v[i] * g[i] * sg;
        dg[i] = v[i] * up[i] * (sg * (1.f + g[i] * (1.f - sg)));
      }
      warp_store_bf16(stg, dg, obase + col, e.ldo, nvalid, lane);
      warp_store_bf16(stg, du, obase + e.half_n + col, e.ldo, nvalid, lane);
    }
    return;
  }
  if (e.kind == CDK_EPI_RESID_F32) {
    const float* rbase = e.resid + (long long)row0 * e.ldr;
    float* obase = reinterpret_cast<float*>(e.out) + (long long)row0 * e.ldo;
    float4 pre0[4], pre1[4];
    warp_load_f32_issue(pre0, rbase + n0 + half * kC, e.ldr, nvalid, lane);
    if (nch > 1) warp_load_f32_issue(pre1, rbase + n0 + 32 + half * kC, e.ldr, nvalid, lane);
    #pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      const int col = n0 + c * 32 + half * kC;
      float r[kC], v[kC];
      warp_load_f32_finish(stg, pre0, r, lane);
      #pragma unroll
      for (int q = 0; q < 4; ++q) pre0[q] = pre1[q];
      if (c + 2 < nch) warp_load_f32_issue(pre1, rbase + col + 64, e.ldr, nvalid, lane);
      tmem_wait_ld();
      unpack_scaled(ua, v, sc);
      if (c + 1 < nch) tmem_ld_x16_nowait(tbase + (c + 1) * 32 + half * kC, ua);
      #pragma unroll
      for (int i = 0; i < kC; ++i) v[i] += r[i] + (e.bias != nullptr ? __ldg(e.bias + col + i) : 0.f);
      warp_store_f32(stg, v, obase + col, e.ldo, nvalid, lane);
    }
    return;
  }
  // CDK_EPI_STORE_BF16 / CDK_EPI_ROPE_BF16
  __nv_bfloat16* obase = reinterpret_cast<__nv_bfloat16*>(e.out) + (long long)row0 * e.ldo;
  const int pos = row % max(e.seq_len, 1);
  #pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int col = n0 + c * 32 + half * kC;
    float r[kC];
    const bool rope = e.kind == CDK_EPI_ROPE_BF16 && col < e.rope_cols;
    if (rope && lane < nvalid) {
      const float4* cs = reinterpret_cast<const float4*>(e.rope + ((long long)pos * 32 + ((col & 63) >> 1)) * 2);
      #pragma unroll
      for (int q = 0; q < kC / 4; ++q) {
        const float4 t = __ldg(cs + q);
        r[4 * q] = t.x; r[4 * q + 1] = t.y; r[4 * q + 2] = t.z; r[4 * q + 3] = t.w;
      }
    }
    float v[kC];
    tmem_wait_ld();
    unpack_scaled(ua, v, sc);
    if (c + 1 < nch) tmem_ld_x16_nowait(tbase + (c + 1) * 32 + half * kC, ua);
    if (e.bias != nullptr) {
      #pragma unroll
      for (int i = 0; i < kC; ++i) v[i] += __ldg(e.bias + col + i);
    }
    if (rope && lane < nvalid) {
      #pragma unroll
      for (int i = 0; i < kC / 2; ++i) {
        const float c0 = r[2 * i], s0 = r[2 * i + 1];
        const float x0 = v[2 * i], x1 = v[2 * i + 1];
        v[2 * i] = x0 * c0 - x1 * s0;
        v[2 * i + 1] = x1 * c0 + x0 * s0;
      }
    }
    warp_store_bf16(stg, v, obase + col, e.ldo, nvalid, lane);
  }
}

// ---- epilogue tile routines ---------------------------------------------------
// One thread = one accumulator row; the two epilogue warps of a TMEM lane
// quadrant split each 32-column block: half h takes columns [32c + 16h, +16).
// Global operands of a chunk (residual, gate/up, RoPE table) are requested
// before the chunk's TMEM load so that their latency overlaps it.
template <int BN>
__device__ __forceinline__ void epi_swiglu(const EpiDev& e, const GemmParams& p, uint32_t tbase, int row,
                                           bool row_ok, int n0, int half, float sc) {
  // TMEM columns [0, BN/2) = gate, [BN/2, BN) = up, for output columns n0 ...
  __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(e.out2) + (long long)row * e.ldo2;
  __nv_bfloat16* uo = reinterpret_cast<__nv_bfloat16*>(e.out) + (long long)row * e.ldo;
  #pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    const int tc = c * 32 + half * kC;
    const int col = n0 + tc;
    if (col >= p.N) break;
    float g[kC], up[kC];
    tmem_ld_f16cols(tbase + tc, g, sc);
    tmem_ld_f16cols(tbase + BN / 2 + tc, up, sc);
    if (row_ok) {
      const int nc = min(kC, p.N - col);
      store_row_bf16(gu + col, g, nc);
      store_row_bf16(gu + e.half_n + col, up, nc);
      float h[kC];
      #pragma unroll
      for (int i = 0; i < kC; ++i) h[i] = silu_f(g[i]) * up[i];
      store_row_bf16(uo + col, h, nc);
    }
  }
}

template <int BN, int KIND>
__device__ __forceinline__ void epi_tile(const EpiDev& e, const GemmParams& p, uint32_t tbase, int row, bool row_ok,
                                         int n0, int half, float sc) {
  const long long orow = (long long)row * e.ldo;
  const int pos = KIND == CDK_EPI_ROPE_BF16 ? row % e.seq_len : 0;
  #pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    const int tc = c * 32 + half * kC;
    const int col = n0 + tc;
    if (col >= p.N) break;
    const int nc = min(kC, p.N - col);
    // prefetch this chunk's global operand
    float r[kC];
    float a2[kC];
    if (row_ok) {
      if constexpr (KIND == CDK_EPI_RESID_F32) load_row_f32(e.resid + (long long)row * e.ldr + col, r, nc);
      if constexpr (KIND == CDK_EPI_ACCUM_F32) load_row_f32(reinterpret_cast<float*>(e.out) + orow + col, r, nc);
      if constexpr (KIND == CDK_EPI_DSWIGLU) {
        const __nv_bfloat16* gsrc = e.aux + (long long)row * e.ldaux;
        load_row_bf16(gsrc + col, r);
        load_row_bf16(gsrc + e.half_n + col, a2);
      }
      if constexpr (KIND == CDK_EPI_ROPE_BF16) {
        if (col < e.rope_cols) {
          const float4* cs = reinterpret_cast<const float4*>(e.rope + ((long long)pos * 32 + ((col & 63) >> 1)) * 2);
          #pragma unroll
          for (int q = 0; q < kC / 4; ++q) {
            const float4 t = __ldg(cs + q);
            r[4 * q] = t.x; r[4 * q + 1] = t.y; r[4 * q + 2] = t.z; r[4 * q + 3] = t.w;
          }
        }
      }
    }
    float v[kC];
    tmem_ld_f16cols(tbase + tc, v, sc);
    if (!row_ok) continue;
    if (e.bias != nullptr) {
      #pragma unroll
      for (int i = 0; i < kC; ++i)
        if (i < nc) v[i] += __ldg(e.bias + col + i);
    }
    if constexpr (KIND == CDK_EPI_STORE_BF16) {
      store_row_bf16(reinterpret_cast<__nv_bfloat16*>(e.out) + orow + col, v, nc);
    } else if constexpr (KIND == CDK_EPI_STORE_F32) {
      store_row_f32(reinterpret_cast<float*>(e.out) + orow + col, v, nc);
    } else if constexpr (KIND == CDK_EPI_RESID_F32 || KIND == CDK_EPI_ACCUM_F32) {
      #pragma unroll
      for (int i = 0; i < kC; ++i) v[i] += r[i];
      store_row_f32(reinterpret_cast<float*>(e.out) + orow + col, v, nc);
    } else if constexpr (KIND == CDK_EPI_ATOMIC_F32) {
      atomic_row_f32(reinterpret_cast<float*>(e.out) + orow + col, v, nc);
    } else if constexpr (KIND == CDK_EPI_ROPE_BF16) {
      if (col < e.rope_cols) {
        #pragma unroll
        for (int i = 0; i < kC / 2; ++i) {
          const float c0 = r[2 * i], s0 = r[2 * i + 1];
          const float x0 = v[2 * i], x1 = v[2 * i + 1];
          v[2 * i] = x0 * c0 - x1 * s0;
          v[2 * i + 1] = x1 * c0 + x0 * s0;
        }
      }
      store_row_bf16(reinterpret_cast<__nv_bfloat16*>(e.out) + orow + col, v, nc);
    } else if constexpr (KIND == CDK_EPI_DSWIGLU) {
      float dg[kC], du[kC];
      #pragma unroll
      for (int i = 0; i < kC; ++i) {
        const float g = r[i], up = a2[i];
        const float sg = sigmoid_fast(g);
        du[i] = v[i] * g * sg;
        dg[i] = v[i] * up * (sg * (1.f + g * (1.f - sg)));
      }
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(e.out) + orow;
      store_row_bf16(o + col, dg, nc);
      store_row_bf16(o + e.half_n + col, du, nc);
    }
  }
}

// ---- TMA-fed epilogue (residual add, SwiGLU backward) ----------------------
// Boxes of 128 rows with 128-byte rows (128-byte swizzle: 16-byte piece q of
// row r at q ^ (r & 7)): the residual as fp32 boxes of 32 columns (16 KB, 4
// slots), the SwiGLU backward as a gate box and an up box of 64 bf16 columns
// (32 KB, 2 slots).  Every role walks the CTA's tiles in the same order; the
// k-th box of the walk uses slot k % slots.  Half h of the epilogue warps owns
// pieces 4h .. 4h+3 of each row; results are written back in place.
struct TeCursor {
  int u, j, nch, m0, n0;
};
__device__ __forceinline__ int te_cols(const GemmParams& p) { return p.epi.kind == CDK_EPI_DSWIGLU ? 64 : 32; }
template <int BN>
__device__ __forceinline__ void te_tile(TeCursor& c, const GemmParams& p) {
  const int units = p.m_tiles * p.n_tiles;
  while (c.u < units) {
    const int mt = c.u / p.n_tiles, nt = c.u - mt * p.n_tiles;
    c.m0 = tile_row0(p, mt);
    c.n0 = nt * BN;
    c.nch = min(BN, p.N - c.n0) / te_cols(p);
    c.j = 0;
    if (c.nch > 0) return;
    c.u += unit_stride(p);
  }
}
template <int BN>
__device__ __forceinline__ void te_next(TeCursor& c, const GemmParams& p) {
  if (++c.j == c.nch) {
    c.u += unit_stride(p);
    te_tile<BN>(c, p);
  }
}
__device__ __forceinline__ void te_fence_proxy() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// The streaming warp (one thread): loads box k into its slot once the TMA
// store of box k - slots has left it, and stores box k once the epilogue warps
// have written it.
template <int BN>
__device__ void te_stream(const CUtensorMap* te_in, const CUtensorMap* te_out, const GemmParams& p, uint8_t* slots,
                          uint64_t* sfull, uint64_t* sdone, volatile int* abort_flag, int area) {
  const bool dsw = p.epi.kind == CDK_EPI_DSWIGLU;
  const int hn = (int)p.epi.half_n;
  const int units = p.m_tiles * p.n_tiles;
  const int sbytes = dsw ? 32768 : 16384;
  const int nslots = area / sbytes;
  const int w = te_cols(p);
  TeCursor L{unit_start(p), 0, 0, 0, 0};
  te_tile<BN>(L, p);
  TeCursor S = L;
  int kl = 0, ks = 0;
  while (S.u < units) {
    while (L.u < units && kl < ks + nslots) {
      const int slot = kl % nslots;
      if (kl >= nslots) {
        // bulk groups committed after the store of box kl - nslots: ks - 1 - (kl - nslots)
        switch (ks - kl + nslots - 1) {
          case 0: bulk_wait_read<0>(); break;
          case 1: bulk_wait_read<1>(); break;
          case 2: bulk_wait_read<2>(); break;
          default: bulk_wait_read<3>(); break;
        }
      }
      uint8_t* dst = slots + slot * sbytes;
      const int x = L.n0 + L.j * w;
      mbar_arrive_expect_tx(&sfull[slot], sbytes);
      tma_load_2d(dst, te_in, &sfull[slot], x, L.m0);
      if (dsw) tma_load_2d(dst + sbytes / 2, te_in, &sfull[slot], hn + x, L.m0);
      te_next<BN>(L, p);
      ++kl;
    }
    const int slot = ks % nslots;
    mbar_wait(&sdone[slot], (ks / nslots) & 1, abort_flag);
    const uint8_t* src = slots + slot * sbytes;
    const int x = S.n0 + S.j * w;
    tma_store_2d(te_out, src, x, S.m0);
    if (dsw) tma_store_2d(te_out, src + sbytes / 2, hn + x, S.m0);
    bulk_commit();
    te_next<BN>(S, p);
    ++ks;
  }
  bulk_wait0();
}

__device__ __forceinline__ void epi_te_tile(const EpiDev& e, uint32_t tbase, int r, int n0, int nch, int half,
                                            int kbase, uint8_t* slots, uint64_t* sfull, uint64_t* sdone,
                                            volatile int* abort_flag, float sc, int area) {
  const bool dsw = e.kind == CDK_EPI_DSWIGLU;
  const int sbytes = dsw ? 32768 : 16384;
  const int nslots = area / sbytes;
  const int w = dsw ? 64 : 32;  // box columns; this thread takes w / 2 of them
  #pragma unroll 1
  for (int j = 0; j < nch; ++j) {
    const int k = kbase + j, slot = k % nslots;
    const int c0 = j * w + half * (w / 2);
    uint32_t a0[kC], a1[kC];
    tmem_ld_x16_nowait(tbase + c0, a0);
    if (dsw) tmem_ld_x16_nowait(tbase + c0 + kC, a1);
    mbar_wait(&sfull[slot], (k / nslots) & 1, abort_flag);
    tmem_wait_ld();
    uint8_t* sl = slots + slot * sbytes;
    if (!dsw) {
      float4* row = reinterpret_cast<float4*>(sl + r * 128);
      const int col = n0 + c0;
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int pc = (half * 4 + q) ^ (r & 7);
        float4 t = row[pc];
        t.x += __uint_as_float(a0[4 * q]) * sc;
        t.y += __uint_as_float(a0[4 * q + 1]) * sc;
        t.z += __uint_as_float(a0[4 * q + 2]) * sc;
        t.w += __uint_as_float(a0[4 * q + 3]) * sc;
        if (e.bias != nullptr) {
          t.x += __ldg(e.bias + col + 4 * q);
          t.y += __ldg(e.bias + col + 4 * q + 1);
          t.z += __ldg(e.bias + col + 4 * q + 2);
          t.w += __ldg(e.bias + col + 4 * q + 3);
        }
        row[pc] = t;
      }
    } else {
      uint4* gr = reinterpret_cast<uint4*>(sl + r * 128);
      uint4* ur = reinterpret_cast<uint4*>(sl + sbytes / 2 + r * 128);
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int pc = (half * 4 + q) ^ (r & 7);
        const uint4 gw = gr[pc], uw = ur[pc];
        const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&gw);
        const __nv_bfloat162* hu = reinterpret_cast<const __nv_bfloat162*>(&uw);
        const uint32_t* acc = q < 2 ? a0 : a1;
        uint32_t og[4], ou[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 g = __bfloat1622float2(hg[i]), u = __bfloat1622float2(hu[i]);
          const int ai = (q & 1) * 8 + 2 * i;
          const float d0 = __uint_as_float(acc[ai]) * sc, d1 = __uint_as_float(acc[ai + 1]) * sc;
          const float s0 = sigmoid_fast(g.x), s1 = sigmoid_fast(g.y);
          og[i] = pack_bf16(d0 * u.x * (s0 * (1.f + g.x * (1.f - s0))), d1 * u.y * (s1 * (1.f + g.y * (1.f - s1))));
          ou[i] = pack_bf16(d0 * g.x * s0, d1 * g.y * s1);
        }
        gr[pc] = make_uint4(og[0], og[1], og[2], og[3]);
        ur[pc] = make_uint4(ou[0], ou[1], ou[2], ou[3]);
      }
    }
    te_fence_proxy();
    mbar_arrive(&sdone[slot]);
  }
}

// ---- TMA-stored bf16 epilogue (store-only form) ------------------------------
// Output boxes of 64 columns: plain store / RoPE: one box per 64 output columns;
// SwiGLU forward: per 64 output columns three boxes, g and u into out2 (gate |
// up halves), silu(g) * u into out.  The k-th box of the CTA's walk uses slot
// k % 2; the epilogue warps wait until the TMA store of box k - 2 has left the
// slot (sfree), write their rows, and arrive on sdone; the streaming thread
// stores the box and frees the slot once the store has read it.
template <int BN, int NS = kTe2Slots>
__device__ void te2_stream(const CUtensorMap* map_a, const CUtensorMap* map_b, const GemmParams& p, uint8_t* slots,
                           uint64_t* sdone, uint64_t* sfree, volatile int* abort_flag) {
  const bool sw = p.epi.kind == CDK_EPI_SWIGLU;
  const bool red = p.epi.kind == CDK_EPI_ATOMIC_F32;  // fp32 boxes of 32 columns, bulk reduce-add (split-K)
  const int hn = (int)p.epi.half_n;
  const int tiles_mn = p.m_tiles * p.n_tiles;
  const int units = tiles_mn * p.splits;
  const int n_step = sw ? BN / 2 : BN;
  const int box = red ? 32 : 64;
  int k = 0;
  for (int u = unit_start(p); u < units; u += unit_stride(p)) {
    const int rem = u % tiles_mn;
    const int mt = rem / p.n_tiles, nt = rem - mt * p.n_tiles;
    const int m0 = tile_row0(p, mt), n0 = nt * n_step;
    const int nq = min(n_step, p.N - n0) / box;
    for (int j = 0; j < nq; ++j) {
      for (int o = 0; o < (sw ? 3 : 1); ++o, ++k) {
        const int slot = k & (NS - 1);
        mbar_wait(&sdone[slot], (k / NS) & 1, abort_flag);
        const uint8_t* src = slots + slot * kTe2SlotBytes;
        const int x = n0 + j * box;
        if (red) tma_reduce_add_2d(map_b, src, x, m0);
        else if (!sw || o == 2) tma_store_2d(map_b, src, x, m0);
        else tma_store_2d(map_a, src, o == 0 ? x : hn + x, m0);
        bulk_commit();
        bulk_wait_read<0>();
        mbar_arrive(&sfree[slot]);
      }
    }
  }
  bulk_wait0();
}

// One thread's 32 bf16 (64 bytes) of row r into box k: half h owns 16-byte
// pieces 4h .. 4h+3 of the 128-byte row (128-byte swizzle: piece q at q ^ (r & 7)).
template <int NS = kTe2Slots>
__device__ __forceinline__ void te2_put(uint8_t* slots, uint64_t* sdone, uint64_t* sfree, int k, int r, int half,
                                        const uint32_t (&w)[16], volatile int* abort_flag) {
  static_assert((NS & (NS - 1)) == 0, "slots: a power of two");
  const int slot = k & (NS - 1);
  if (k >= NS) mbar_wait(&sfree[slot], ((k / NS) - 1) & 1, abort_flag);
  uint4* row = reinterpret_cast<uint4*>(slots + slot * kTe2SlotBytes + r * 128);
  #pragma unroll
  for (int q = 0; q < 4; ++q) row[(half * 4 + q) ^ (r & 7)] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  te_fence_proxy();
  mbar_arrive(&sdone[slot]);
}

template <int BN, int NS = kTe2Slots>
__device__ __forceinline__ void epi_te2_tile(const EpiDev& e, const GemmParams& p, uint32_t tbase, int r, int row, float sc,
                                             int n0, int half, int& k, uint8_t* slots, uint64_t* sdone,
                                             uint64_t* sfree, volatile int* abort_flag) {
  const bool sw = e.kind == CDK_EPI_SWIGLU;
  const int n_step = sw ? BN / 2 : BN;
  if (e.kind == CDK_EPI_ATOMIC_F32) {
    // fp32 partial sums, 32-column boxes (16 columns per half) for the bulk reduce-add
    const int nb = min(BN, p.N - n0) / 32;
    uint32_t a[kC];
    if (nb > 0) tmem_ld_x16_nowait(tbase + half * kC, a);
    #pragma unroll 1
    for (int j = 0; j < nb; ++j) {
      tmem_wait_ld();
      uint32_t w[16];
      #pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(__uint_as_float(a[i]) * sc);
      if (j + 1 < nb) tmem_ld_x16_nowait(tbase + (j + 1) * 32 + half * kC, a);
      te2_put<NS>(slots, sdone, sfree, k++, r, half, w, abort_flag);
    }
    return;
  }
  const int nq = min(n_step, p.N - n0) / 64;
  // RoPE: the (cos, sin) pairs of this thread's 32 columns within a head are
  // the same for every head of the tile: load them once
  float cs[32];
  const bool rope_tile = e.kind == CDK_EPI_ROPE_BF16 && n0 < e.rope_cols;
  if (rope_tile) {
    const int pos = (row < p.M ? row : 0) % max(e.seq_len, 1);
    const float4* t = reinterpret_cast<const float4*>(e.rope + ((long long)pos * 32 + half * 16) * 2);
    #pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 x = __ldg(t + q);
      cs[4 * q] = x.x; cs[4 * q + 1] = x.y; cs[4 * q + 2] = x.z; cs[4 * q + 3] = x.w;
    }
  }
  #pragma unroll 1
  for (int j = 0; j < nq; ++j) {
    const int c0 = j * 64 + half * 32;  // first TMEM / output column of this thread's 32
    uint32_t a0[kC], a1[kC];
    tmem_ld_x16_nowait(tbase + c0, a0);
    tmem_ld_x16_nowait(tbase + c0 + kC, a1);
    if (!sw) {
      tmem_wait_ld();
      float v[32];
      #pragma unroll
      for (int i = 0; i < kC; ++i) {
        v[i] = __uint_as_float(a0[i]) * sc;
        v[kC + i] = __uint_as_float(a1[i]) * sc;
      }
      const int col = n0 + c0;
      if (e.bias != nullptr) {
        #pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += __ldg(e.bias + col + i);
      }
      if (rope_tile && col < e.rope_cols) {
        #pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float c = cs[2 * i], s_ = cs[2 * i + 1];
          const float x0 = v[2 * i], x1 = v[2 * i + 1];
          v[2 * i] = x0 * c - x1 * s_;
          v[2 * i + 1] = x1 * c + x0 * s_;
        }
      }
      uint32_t w[16];
      #pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
      te2_put<NS>(slots, sdone, sfree, k++, r, half, w, abort_flag);
    } else {
      uint32_t b0[kC], b1[kC];
      tmem_ld_x16_nowait(tbase + BN / 2 + c0, b0);
      tmem_ld_x16_nowait(tbase + BN / 2 + c0 + kC, b1);
      tmem_wait_ld();
      uint32_t wg[16], wu[16], wh[16];
      #pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t* ga = i < 8 ? a0 : a1;
        const uint32_t* ua = i < 8 ? b0 : b1;
        const int ii = (i & 7) * 2;
        const float g0 = __uint_as_float(ga[ii]) * sc, g1 = __uint_as_float(ga[ii + 1]) * sc;
        const float u0 = __uint_as_float(ua[ii]) * sc, u1 = __uint_as_float(ua[ii + 1]) * sc;
        wg[i] = pack_bf16(g0, g1);
        wu[i] = pack_bf16(u0, u1);
        wh[i] = pack_bf16(silu_f(g0) * u0, silu_f(g1) * u1);
      }
      te2_put<NS>(slots, sdone, sfree, k++, r, half, wg, abort_flag);
      te2_put<NS>(slots, sdone, sfree, k++, r, half, wu, abort_flag);
      te2_put<NS>(slots, sdone, sfree, k++, r, half, wh, abort_flag);
    }
  }
}

// PAIR (1, or 2 with four output slots): clusters of two CTAs; the even CTA
// issues M=256 MMAs over both CTAs' shared memory (its 128 A rows and B rows
// [n0, n0+BN/2), the odd CTA's 128 A rows and B rows [n0+BN/2, n0+BN)), and
// each CTA's TMEM receives its own 128 accumulator rows, so the epilogue warps
// are the same in both.
template <int BN, bool A_MN, bool B_MN, bool VEC, bool F8 = false, int TEM = 0, int PAIR = 0>
__global__ void __launch_bounds__(TEM ? kThreadsTE : kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap te_in, const __grid_constant__ CUtensorMap te_out,
                     const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  // TEM 1: TMA-fed form with 64 KB of slots (3-stage ring at BN=256); TEM 4: the
  // same for the residual add with 2 x 16 KB slots and the full ring
  constexpr bool TE = TEM == 1 || TEM == 4;
  static_assert(!PAIR || (BN == 256 && (A_MN ? !F8 && B_MN && TEM == 3 : TEM == 1 || TEM == 2 || TEM == 3)),
                "pair form");
  static_assert(PAIR != 2 || TEM == 2, "wide output slots: store-only form");
  constexpr int kStages = PAIR ? Cfg::stages_pair(TEM, PAIR) : TEM == 1 ? Cfg::kStagesTE : Cfg::kStages;
  constexpr int kBytesB = PAIR ? Cfg::kBytesB / 2 : Cfg::kBytesB;
  constexpr int kStageBytes = Cfg::kBytesA + kBytesB;
  constexpr bool TE2 = TEM == 2 || TEM == 3;  // store-only / reduce-add forms share the slots and the stream
  constexpr int kNs2 = PAIR && TEM == 2 ? Cfg::te2_slots_pair(PAIR) : kTe2Slots;  // store-only output slots
  constexpr int kSlotArea =
      PAIR != 0 ? Cfg::slot_area_pair(TEM, PAIR)
      : TEM == 1 ? kTeSlots * kTeSlotBytes : TEM == 4 ? 32768 : TE2 ? kNs2 * kTe2SlotBytes : 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kBytesA;
  uint8_t* te_slots = smem + kStages * kStageBytes;  // TE: 8 x 8 KB / store-only: 2 x 16 KB, 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + kSlotArea);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  // TMA-fed form: a barrier pair per slot of its smallest box (16 KB)
  constexpr int kSlotBars = TEM == 1 ? kSlotArea / 16384 : TEM == 4 ? 2 : TE2 ? kNs2 : 0;
  uint64_t* sfull = tempty + 2;      // TE / store-only forms
  uint64_t* sdone = sfull + kSlotBars;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sdone + kSlotBars);
  static_assert((2 * kStages + 4 + 2 * kSlotBars) * 8 + 8 <= Cfg::kBarrierBytes, "barrier area");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 512 : 256);  // pair: both CTAs' epilogue threads, on the even CTA's barrier
    }
    if constexpr (TE) {
      for (int a = 0; a < kSlotBars; ++a) {
        mbar_init(&sfull[a], 1);
        mbar_init(&sdone[a], 256);
      }
    }
    if constexpr (TE2) {  // sfull = slot freed by the store (streaming thread), sdone = box written (256)
      for (int a = 0; a < kNs2; ++a) {
        mbar_init(&sfull[a], 1);
        mbar_init(&sdone[a], 256);
      }
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  if (warp == 1) {
    if constexpr (PAIR != 0) {
      tmem_alloc_pair(tmem_holder, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR != 0) cluster_sync();  // the peer's barriers are initialised before any signal reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;

  const int tiles_mn = p.m_tiles * p.n_tiles;
  const int units = tiles_mn * p.splits;
  const int n_step = p.dual ? BN / 2 : BN;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int u = unit_start(p); u < units; u += unit_stride(p)) {
        const int ks = u / tiles_mn;
        const int rem = u - ks * tiles_mn;
        const int mt = rem / p.n_tiles;
        const int nt = rem - mt * p.n_tiles;
        const int m0 = tile_row0(p, mt), n0 = nt * n_step;
        const int kt0 = ks * p.k_per_split;
        const int kt1 = min(kt0 + p.k_per_split, p.k_tiles);
        for (int kt = kt0; kt < kt1; ++kt) {
          mbar_wait(&empty[stage], phase ^ 1u, abort_flag);
          uint8_t* a_dst = sA + stage * Cfg::kBytesA;
          uint8_t* b_dst = sB + stage * kBytesB;
          if constexpr (PAIR != 0) {
            // both CTAs' loads complete on the even CTA's barrier, which expects both
            const uint32_t bar0 = mapa_shared(&full[stage], 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * kStageBytes);
            const int k0 = kt * (F8 ? 2 * kBK : kBK);  // element coordinate of this 128-byte k block
            if constexpr (A_MN) {  // this CTA's 128 rows as two 64-row groups of kBK k rows
              tma_load_2d_pair(a_dst, &tma_a, bar0, m0, k0);
              tma_load_2d_pair(a_dst + 8192, &tma_a, bar0, m0 + 64, k0);
            } else {
              tma_load_2d_pair(a_dst, &tma_a, bar0, k0, m0);
            }
            if constexpr (B_MN) {  // this CTA's BN/2 columns as 128-byte-wide groups (64 bf16 / 128 fp8)
              constexpr int kGrpE = F8 ? 128 : 64, kGrpB = F8 ? 16384 : 8192;
              #pragma unroll
              for (int i = 0; i < (BN / 2) / kGrpE; ++i)
                tma_load_2d_pair(b_dst + i * kGrpB, &tma_b, bar0, n0 + (int)rank * (BN / 2) + kGrpE * i, k0);
            } else {
              tma_load_2d_pair(b_dst, &tma_b, bar0, k0,
                               p.dual ? n0 + (rank ? p.b_off : 0) : n0 + (int)rank * (BN / 2));
            }
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          const int k0 = kt * (F8 ? 2 * kBK : kBK);  // element coordinate of this 128-byte k block
          // MN-major operands arrive as 128-byte-wide MN groups (64 bf16 / 128 fp8
          // elements) of kRowsK k rows each
          constexpr int kGrpE = F8 ? 128 : 64;
          constexpr int kGrpB = F8 ? 16384 : 8192;
          if (!A_MN) {
            tma_load_2d(a_dst, &tma_a, &full[stage], k0, m0);
          } else {
            #pragma unroll
            for (int g = 0; g < kBM / kGrpE; ++g) tma_load_2d(a_dst + g * kGrpB, &tma_a, &full[stage], m0 + g * kGrpE, k0);
          }
          if (!B_MN) {
            if (p.dual) {
              tma_load_2d(b_dst, &tma_b, &full[stage], k0, n0);
              tma_load_2d(b_dst + (BN / 2) * 128, &tma_b, &full[stage], k0, n0 + p.b_off);
            } else {
              tma_load_2d(b_dst, &tma_b, &full[stage], k0, n0);
            }
          } else {
            #pragma unroll
            for (int i = 0; i < BN / kGrpE; ++i) tma_load_2d(b_dst + i * kGrpB, &tma_b, &full[stage], n0 + kGrpE * i, k0);
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if constexpr (PAIR != 0) {
        // the even CTA's MMAs read this CTA's stages: wait until the last use of
        // each has been released before the CTA may leave
        for (int i = 0; i < kStages; ++i) {
          mbar_wait(&empty[stage], phase ^ 1u, abort_flag);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // the whole warp runs the issue loop and one elected lane issues: operands
    // stay warp-uniform (one thread of a diverged warp computing descriptors
    // issues an MMA per 75-150 cycles, about what an N=256 MMA takes)
    if (rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(PAIR ? 2 * kBM : kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int u = unit_start(p); u < units; u += unit_stride(p), ++local) {
        const int ks = u / tiles_mn;
        const int kt0 = ks * p.k_per_split;
        const int kt1 = min(kt0 + p.k_per_split, p.k_tiles);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kt = kt0; kt < kt1; ++kt) {
          mbar_wait(&full[stage], phase, abort_flag);
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::kBytesA);
          const uint32_t b_base = smem_u32(sB + stage * kBytesB);
          #pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // MN-major: one MMA consumes 16 (bf16) / 32 (fp8) k rows of 128 B
            constexpr uint32_t kKStep = F8 ? 4096 : 2048, kLbo = F8 ? 16384 : 8192;
            const uint64_t ad =
                A_MN ? make_sdesc(a_base + kk * kKStep, kLbo, 1024) : make_sdesc(a_base + kk * 32, 16, 1024);
            const uint64_t bd =
                B_MN ? make_sdesc(b_base + kk * kKStep, kLbo, 1024) : make_sdesc(b_base + kk * 32, 16, 1024);
            if constexpr (F8 && PAIR != 0) umma_f8_pair_w(d_tmem, ad, bd, p.idesc_f8, (kt > kt0 || kk > 0) ? 1u : 0u);
            else if constexpr (F8) umma_f8_w(d_tmem, ad, bd, p.idesc_f8, (kt > kt0 || kk > 0) ? 1u : 0u);
            else if constexpr (PAIR != 0) umma_f16_pair_w(d_tmem, ad, bd, idesc, (kt > kt0 || kk > 0) ? 1u : 0u);
            else umma_f16_w(d_tmem, ad, bd, idesc, (kt > kt0 || kk > 0) ? 1u : 0u);
          }
          if constexpr (PAIR != 0) tc_commit_pair_w(&empty[stage]);
          else tc_commit_w(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if constexpr (PAIR != 0) tc_commit_pair_w(&tfull[acc]);
        else tc_commit_w(&tfull[acc]);
      }
    }
  } else if (TEM && warp == 10) {
    // ---------------- epilogue operand streaming (TE) / output stores ----------------
    if (lane == 0) {
      prefetch_tmap(&te_in);
      prefetch_tmap(&te_out);
      if constexpr (TE) te_stream<BN>(&te_in, &te_out, p, te_slots, sfull, sdone, abort_flag, kSlotArea);
      else te2_stream<BN, kNs2>(&te_in, &te_out, p, te_slots, sdone, sfull, abort_flag);
    }
  } else {
    // ---------------- epilogue warps ----------------
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const EpiDev& e = p.epi;
    uint32_t* stg = reinterpret_cast<uint32_t*>(smem + kStages * kStageBytes + Cfg::kBarrierBytes) +
                    (warp - 2) * kStgWords;
    float sc = 1.f;
    if constexpr (F8) sc = *p.scale_inv_a * *p.scale_inv_b;
    int local = 0;
    int te_k = 0;  // TE: chunks of the CTA's earlier tiles
    for (int u = unit_start(p); u < units; u += unit_stride(p), ++local) {
      const int rem = u % tiles_mn;
      const int mt = rem / p.n_tiles;
      const int nt = rem - mt * p.n_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (e.kind == CDK_EPI_RESID_F32 || e.kind == CDK_EPI_ACCUM_F32 || e.kind == CDK_EPI_DSWIGLU) {
        if (local == 0) epi_prefetch<BN>(e, p, tile_row0(p, mt) + quad * 32 + lane, nt * BN, half);
        const int un = u + unit_stride(p);
        if (un < units) {
          const int rn = un % tiles_mn;
          const int mtn = rn / p.n_tiles;
          epi_prefetch<BN>(e, p, tile_row0(p, mtn) + quad * 32 + lane, (rn - mtn * p.n_tiles) * BN, half);
        }
      }
      mbar_wait(&tfull[acc], acc_phase, abort_flag);
      tc_fence_after();
      const int row = tile_row0(p, mt) + quad * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;

      if constexpr (TE) {
        const int nch = min(BN, p.N - nt * BN) / (e.kind == CDK_EPI_DSWIGLU ? 64 : 32);
        epi_te_tile(e, tbase, quad * 32 + lane, nt * BN, nch, half, te_k, te_slots, sfull, sdone, abort_flag, sc,
                    kSlotArea);
        te_k += nch;
      } else if constexpr (TE2) {
        epi_te2_tile<BN, kNs2>(e, p, tbase, quad * 32 + lane, row, sc, e.kind == CDK_EPI_SWIGLU ? nt * (BN / 2) : nt * BN,
                         half, te_k, te_slots, sdone, sfull, abort_flag);
      } else if constexpr (VEC) {
        const int row0 = tile_row0(p, mt) + quad * 32;
        if (row0 < p.M)
          epi_vec<BN, F8>(e, p, tbase, row0, e.kind == CDK_EPI_SWIGLU ? nt * (BN / 2) : nt * BN, half, stg, lane,
                          sc);
      } else switch (e.kind) {
        case CDK_EPI_SWIGLU: epi_swiglu<BN>(e, p, tbase, row, row_ok, nt * (BN / 2), half, sc); break;
        case CDK_EPI_STORE_BF16: epi_tile<BN, CDK_EPI_STORE_BF16>(e, p, tbase, row, row_ok, nt * BN, half, sc); break;
        case CDK_EPI_STORE_F32: epi_tile<BN, CDK_EPI_STORE_F32>(e, p, tbase, row, row_ok, nt * BN, half, sc); break;
        case CDK_EPI_RESID_F32: epi_tile<BN, CDK_EPI_RESID_F32>(e, p, tbase, row, row_ok, nt * BN, half, sc); break;
        case CDK_EPI_ACCUM_F32: epi_tile<BN, CDK_EPI_ACCUM_F32>(e, p, tbase, row, row_ok, nt * BN, half, sc); break;
        case CDK_EPI_ATOMIC_F32: epi_tile<BN, CDK_EPI_ATOMIC_F32>(e, p, tbase, row, row_ok, nt * BN, half, sc); break;
        case CDK_EPI_ROPE_BF16: epi_tile<BN, CDK_EPI_ROPE_BF16>(e, p, tbase, row, row_ok, nt * BN, half, sc); break;
        case CDK_EPI_DSWIGLU: epi_tile<BN, CDK_EPI_DSWIGLU>(e, p, tbase, row, row_ok, nt * BN, half, sc); break;
        default: break;
      }
      tc_fence_before();
      if constexpr (PAIR != 0) mbar_arrive_cluster(mapa_shared(&tempty[acc], 0));
      else mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR != 0) cluster_sync();  // neither CTA leaves while the pair's MMAs or signals may touch it
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR != 0) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    else tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map, 128-byte swizzle: dims {inner, outer}, row pitch in elements.
bool make_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch,
               uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D fp32 tensor map, 128-byte swizzle; pitch in elements.
bool make_tmap_f32(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch,
                   uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D uint8 (fp8 payload) tensor map, 128-byte swizzle; pitch in bytes.
static bool make_tmap_u8(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch,
                         uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D tensor map with a chosen element type and swizzle (TMA-fed epilogue boxes).
static bool make_tmap_sw(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                         uint64_t outer, uint64_t pitch, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || base == nullptr) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// CDK_GEMM_TE=0 turns the TMA-fed epilogue off (the register-staged epilogue runs instead).
static bool te_enabled() {
  static const bool on = [] {
    const char* v = getenv("CDK_GEMM_TE");
    return !(v && v[0] == '0');
  }();
  return on;
}

static bool te_resid_deep() {
  static const bool on = [] {
    const char* v = getenv("CDK_GEMM_TE_RESID_SLOTS");
    return v && v[0] == '4';
  }();
  return on;
}

static int num_sms(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

template <int BN, bool A_MN, bool B_MN, bool VEC, bool F8 = false, int TE = 0, int PAIR = 0>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& te_in,
                       const CUtensorMap& te_out, const GemmParams& p, int grid, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  constexpr int threads = TE ? kThreadsTE : kThreads;
  constexpr int smem =
      PAIR ? Cfg::smem_pair(TE, PAIR) : TE == 1 ? Cfg::kSmemBytesTE : TE >= 2 ? Cfg::kSmemBytesTE2 : Cfg::kSmemBytes;
  static_assert(TE != 4 || Cfg::kSmemBytesTE2 == Cfg::kStages * Cfg::kStageBytes + 1024 + 32768 + Cfg::kBarrierBytes,
                "TEM 4 uses the store-only form's layout");
  static_assert(smem <= 232448, "shared memory");
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kfn = gemm_bf16_kernel<BN, A_MN, B_MN, VEC, F8, TE, PAIR>;
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    // tcgen05.alloc blocks until columns are free: co-resident CTAs must fit in 512 columns
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, threads, smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm * Cfg::kTmemCols > 512) return -12;
    attr_set[dev] = true;
  }
  if constexpr (PAIR != 0) {
    if (!p.pair || (grid & 1)) return -14;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, ta, tb, te_in, te_out, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
  } else {
    if (p.pair) return -14;
    kfn<<<grid, threads, smem, stream>>>(ta, tb, te_in, te_out, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
  }
}

// Clusters of two CTAs with the pair form's shared memory that can be resident
// at once (0 if the query fails).
static int pair_clusters(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 0;
  if (!cache[dev]) {
    using Cfg = GemmCfg<256>;
    auto kfn = gemm_bf16_kernel<256, false, false, true, false, 2, 1>;
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::smem_pair(2, 1)) != cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kThreadsTE);
    cfg.dynamicSmemBytes = Cfg::smem_pair(2, 1);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return 0;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

// CTA-pair form (K-major A): on by default; CDK_GEMM_PAIR=0 keeps every GEMM
// on the one-CTA form.
static bool pair_enabled() {
  static const bool on = [] {
    const char* v = getenv("CDK_GEMM_PAIR");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <int BN>
static int dispatch_major(bool a_mn, bool b_mn, int te, const CUtensorMap& ta, const CUtensorMap& tb,
                          const CUtensorMap& te_in, const CUtensorMap& te_out, const GemmParams& p, int grid,
                          cudaStream_t s) {
  const CUtensorMap &ti = te_in, &to = te_out;
  // the coalesced epilogues (forward kinds and bf16 stores) have their own instantiations
  if (p.scale_inv_a != nullptr) {  // fp8 operands
    if (p.pair) {
      if constexpr (BN == 256) {
        if (te == 2 && !a_mn && !b_mn && p.dual)
          return launch_gemm<256, false, false, true, true, 2, 2>(ta, tb, ti, to, p, grid, s);
        if (te == 2 && !a_mn && !b_mn) return launch_gemm<256, false, false, true, true, 2, 1>(ta, tb, ti, to, p, grid, s);
        if (te == 1 && !a_mn && !b_mn) return launch_gemm<256, false, false, true, true, 1, 1>(ta, tb, ti, to, p, grid, s);
        if (te == 2 && !a_mn && b_mn) return launch_gemm<256, false, true, true, true, 2, 1>(ta, tb, ti, to, p, grid, s);
        if (te == 3 && !a_mn && !b_mn) return launch_gemm<256, false, false, false, true, 3, 1>(ta, tb, ti, to, p, grid, s);
      }
      return -14;
    }
    if (te == 1 && !a_mn && !b_mn) return launch_gemm<BN, false, false, true, true, 1>(ta, tb, ti, to, p, grid, s);
    if (te == 4 && !a_mn && !b_mn) return launch_gemm<BN, false, false, true, true, 4>(ta, tb, ti, to, p, grid, s);
    if (te == 2 && !a_mn && !b_mn) return launch_gemm<BN, false, false, true, true, 2>(ta, tb, ti, to, p, grid, s);
    if (te == 2 && !a_mn && b_mn) return launch_gemm<BN, false, true, true, true, 2>(ta, tb, ti, to, p, grid, s);
    if (te == 3 && a_mn && b_mn) return launch_gemm<BN, true, true, false, true, 3>(ta, tb, ti, to, p, grid, s);
    if (te == 3 && !a_mn && !b_mn) return launch_gemm<BN, false, false, false, true, 3>(ta, tb, ti, to, p, grid, s);
    if (p.epi.vec && !a_mn && !b_mn) return launch_gemm<BN, false, false, true, true>(ta, tb, ti, to, p, grid, s);
    if (p.epi.vec && !a_mn && b_mn) return launch_gemm<BN, false, true, true, true>(ta, tb, ti, to, p, grid, s);
    if (!a_mn && !b_mn) return launch_gemm<BN, false, false, false, true>(ta, tb, ti, to, p, grid, s);
    if (!a_mn && b_mn) return launch_gemm<BN, false, true, false, true>(ta, tb, ti, to, p, grid, s);
    if (a_mn && !b_mn) return launch_gemm<BN, true, false, false, true>(ta, tb, ti, to, p, grid, s);
    return launch_gemm<BN, true, true, false, true>(ta, tb, ti, to, p, grid, s);
  }
  if constexpr (BN == 256) {
    if (p.pair && te == 2 && !a_mn && !b_mn && p.dual)
      return launch_gemm<256, false, false, true, false, 2, 2>(ta, tb, ti, to, p, grid, s);
    if (p.pair && te == 2 && !a_mn && !b_mn) return launch_gemm<256, false, false, true, false, 2, 1>(ta, tb, ti, to, p, grid, s);
    if (p.pair && te == 2 && !a_mn && b_mn) return launch_gemm<256, false, true, true, false, 2, 1>(ta, tb, ti, to, p, grid, s);
    if (p.pair && te == 1 && !a_mn && b_mn) return launch_gemm<256, false, true, true, false, 1, 1>(ta, tb, ti, to, p, grid, s);
    if (p.pair && te == 1 && !a_mn && !b_mn) return launch_gemm<256, false, false, true, false, 1, 1>(ta, tb, ti, to, p, grid, s);
    if (p.pair && te == 3 && a_mn && b_mn) return launch_gemm<256, true, true, false, false, 3, 1>(ta, tb, ti, to, p, grid, s);
    if (p.pair && te == 3 && !a_mn && !b_mn) return launch_gemm<256, false, false, false, false, 3, 1>(ta, tb, ti, to, p, grid, s);
  }
  if (p.pair) return -14;
  // TMA-fed epilogue (residual add / SwiGLU backward; K-major A)
  if (te == 1 && !a_mn && !b_mn) return launch_gemm<BN, false, false, true, false, 1>(ta, tb, ti, to, p, grid, s);
  if (te == 4 && !a_mn && !b_mn) return launch_gemm<BN, false, false, true, false, 4>(ta, tb, ti, to, p, grid, s);
  if (te == 1 && !a_mn && b_mn) return launch_gemm<BN, false, true, true, false, 1>(ta, tb, ti, to, p, grid, s);
  if (te == 2 && !a_mn && !b_mn) return launch_gemm<BN, false, false, true, false, 2>(ta, tb, ti, to, p, grid, s);
  if (te == 2 && !a_mn && b_mn) return launch_gemm<BN, false, true, true, false, 2>(ta, tb, ti, to, p, grid, s);
  if (te == 3 && a_mn && b_mn) return launch_gemm<BN, true, true, false, false, 3>(ta, tb, ti, to, p, grid, s);
  if (te == 3 && !a_mn && !b_mn) return launch_gemm<BN, false, false, false, false, 3>(ta, tb, ti, to, p, grid, s);
  if (p.epi.vec && !a_mn && !b_mn) return launch_gemm<BN, false, false, true>(ta, tb, ti, to, p, grid, s);
  if (p.epi.vec && !a_mn && b_mn) return launch_gemm<BN, false, true, true>(ta, tb, ti, to, p, grid, s);
  if (!a_mn && !b_mn) return launch_gemm<BN, false, false, false>(ta, tb, ti, to, p, grid, s);
  if (!a_mn && b_mn) return launch_gemm<BN, false, true, false>(ta, tb, ti, to, p, grid, s);
  if (a_mn && !b_mn) return launch_gemm<BN, true, false, false>(ta, tb, ti, to, p, grid, s);
  return launch_gemm<BN, true, true, false>(ta, tb, ti, to, p, grid, s);
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace cdk

namespace cdk {
// Shared host path of cdk_gemm_bf16 and cdk_gemm_fp8 (f8: 8-bit K-major operands
// with formats a_fmt / b_fmt and device dequantisation scalars sa / sb).
static int gemm_impl(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, int64_t M,
                     int64_t N, int64_t K, const CdkGemmEpilogue* epi, int split_k, void* stream, bool f8, int a_fmt,
                     int b_fmt, const float* sa, const float* sb) {
  if (!a || !b || !epi || !epi->out) return -1;
  if (M <= 0 || N <= 0 || K <= 0) return -2;
  if (M > (1ll << 31) || N > (1ll << 31) || K > (1ll << 31)) return -2;
  if (!aligned16(a) || !aligned16(b)) return -3;
  if (f8 ? ((lda % 16) || (ldb % 16)) : ((lda % 8) || (ldb % 8))) return -3;
  if (f8 && (!sa || !sb || a_fmt < 0 || a_fmt > 1 || b_fmt < 0 || b_fmt > 1)) return -13;
  const int kind = epi->kind;
  if (kind < CDK_EPI_STORE_BF16 || kind > CDK_EPI_ACCUM_F32) return -4;
  const bool dual = kind == CDK_EPI_SWIGLU;
  if (dual && (b_mn || epi->half_n != N || (N % 128) || !epi->out2)) return -5;
  if (kind == CDK_EPI_DSWIGLU && (!epi->aux || epi->half_n < N || (N % 32) || (epi->ldaux % 8) ||
                                  !aligned16(epi->aux)))
    return -5;
  if (kind == CDK_EPI_ROPE_BF16 && (!epi->rope || epi->seq_len <= 0 || (epi->rope_cols % 64))) return -6;
  if (kind == CDK_EPI_RESID_F32 && !epi->resid) return -7;
  if (split_k > 1 && kind != CDK_EPI_ATOMIC_F32) return -8;

  // Leading-dimension sanity (the contiguous extent must fit in the pitch).
  if (!a_mn ? lda < K : lda < M) return -9;
  if (!b_mn ? ldb < K : ldb < (dual ? 2 * N : N)) return -9;

  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = num_sms(dev);

  // Tile width: 256 unless the grid would be badly under-filled.
  int BN = 256;
  const long long m_tiles = (M + kBM - 1) / kBM;
  if (!dual) {
    const long long t256 = m_tiles * ((N + 255) / 256);
    const long long t128 = m_tiles * ((N + 127) / 128);
    if (N <= 128) BN = 128;
    else if (t256 < sms && kind != CDK_EPI_ATOMIC_F32 && t128 > t256) BN = 128;
  }
  const int n_step = dual ? BN / 2 : BN;
  const long long n_tiles = (N + n_step - 1) / n_step;
  const int bk = f8 ? 2 * kBK : kBK;  // elements per 128-byte k block
  const long long k_tiles = (K + bk - 1) / bk;

  // Split-K (ATOMIC_F32 only): the split that best fills whole waves of `slots`
  // (SMs, or CTA pairs) with `tiles` output tiles while keeping >= 8 k-tiles per unit.
  auto choose_splits = [&](long long tiles, long long slots) {
    int best_s = 1;
    if (kind != CDK_EPI_ATOMIC_F32) return 1;
    if (split_k > 0) return split_k;
    double best = -1.0;
    for (int s = 1; s <= 32; ++s) {
      if (k_tiles / s < 8 && s > 1) break;
      const long long units = tiles * s;
      const long long waves = (units + slots - 1) / slots;
      const double eff = (double)units / (double)(waves * slots);
      if (eff > best + 0.02) {
        best = eff;
        best_s = s;
      }
      if (eff > 0.97) break;
    }
    return best_s;
  };
  int splits = choose_splits(m_tiles * n_tiles, sms);
  long long k_per = (k_tiles + splits - 1) / splits;
  splits = (int)((k_tiles + k_per - 1) / k_per);

  CUtensorMap ta, tb;
  bool ok;
  if (f8 && !a_mn) ok = make_tmap_u8(&ta, a, K, M, lda, bk, kBM);
  else if (f8) ok = make_tmap_u8(&ta, a, M, K, lda, 128, bk);
  else if (!a_mn) ok = make_tmap(&ta, a, K, M, lda, kBK, kBM);
  else ok = make_tmap(&ta, a, M, K, lda, 64, kBK);
  if (!ok) return -10;
  if (f8 && !b_mn) ok = make_tmap_u8(&tb, b, K, dual ? 2 * N : N, ldb, bk, dual ? BN / 2 : BN);
  else if (f8) ok = make_tmap_u8(&tb, b, N, K, ldb, 128, bk);
  else if (!b_mn) ok = make_tmap(&tb, b, K, dual ? 2 * N : N, ldb, kBK, dual ? BN / 2 : BN);
  else ok = make_tmap(&tb, b, N, K, ldb, 64, kBK);
  if (!ok) return -11;

  GemmParams p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.m_tiles = (int)m_tiles;
  p.n_tiles = (int)n_tiles;
  p.splits = splits;
  p.k_tiles = (int)k_tiles;
  p.k_per_split = (int)k_per;
  p.dual = dual ? 1 : 0;
  p.pair = 0;
  p.b_off = dual ? (int)N : 0;
  p.idesc_f8 = f8 ? make_idesc_f8(kBM, BN, a_fmt, b_fmt, a_mn != 0, b_mn != 0) : 0u;
  p.scale_inv_a = f8 ? sa : nullptr;
  p.scale_inv_b = f8 ? sb : nullptr;
  p.epi.kind = kind;
  p.epi.seq_len = epi->seq_len;
  p.epi.rope_cols = epi->rope_cols;
  p.epi.out = epi->out;
  p.epi.ldo = epi->ldo;
  p.epi.bias = epi->bias;
  p.epi.resid = epi->resid;
  p.epi.ldr = epi->ldr;
  p.epi.out2 = epi->out2;
  p.epi.ldo2 = epi->ldo2;
  p.epi.aux = reinterpret_cast<const __nv_bfloat16*>(epi->aux);
  p.epi.ldaux = epi->ldaux;
  p.epi.half_n = epi->half_n;
  p.epi.rope = epi->rope;
  {
    auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    bool v = N % 16 == 0 && al16(epi->out);
    if (kind == CDK_EPI_RESID_F32) v = v && epi->ldo % 4 == 0 && epi->ldr % 4 == 0 && al16(epi->resid);
    else if (kind == CDK_EPI_STORE_BF16 || kind == CDK_EPI_ROPE_BF16) v = v && epi->ldo % 8 == 0;
    else if (kind == CDK_EPI_SWIGLU) v = v && epi->ldo % 8 == 0 && epi->ldo2 % 8 == 0 && epi->half_n % 8 == 0 && al16(epi->out2);
    else if (kind == CDK_EPI_DSWIGLU) v = v && !f8 && epi->ldo % 8 == 0 && epi->ldaux % 8 == 0 && epi->half_n % 8 == 0 && al16(epi->aux);
    else v = false;
    if (kind == CDK_EPI_ROPE_BF16) v = v && epi->seq_len > 0;
    p.epi.vec = v && !a_mn ? 1 : 0;
  }

  // TMA-fed epilogue for the residual add and the SwiGLU backward: 16-column x
  // 128-row boxes of the epilogue operand in and of the result out
  CUtensorMap te_in, te_out;
  std::memset(&te_in, 0, sizeof(te_in));
  std::memset(&te_out, 0, sizeof(te_out));
  bool te = p.epi.vec && splits == 1 && !dual && N % 16 == 0 && te_enabled() &&
            (kind == CDK_EPI_RESID_F32 || (kind == CDK_EPI_DSWIGLU && !f8));
  // store-only form: 64-column bf16 boxes (N a multiple of 64); split-K fp32
  // partial sums: 32-column boxes reduce-added by TMA
  bool te2 = p.epi.vec && splits == 1 && N % 64 == 0 && te_enabled() &&
             (kind == CDK_EPI_STORE_BF16 || kind == CDK_EPI_ROPE_BF16 || kind == CDK_EPI_SWIGLU);
  bool te3 = kind == CDK_EPI_ATOMIC_F32 && N % 32 == 0 && epi->bias == nullptr && epi->ldo % 4 == 0 &&
             (reinterpret_cast<uintptr_t>(epi->out) & 15) == 0 && te_enabled();
  if (te3) {
    te3 = make_tmap_sw(&te_out, epi->out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, epi->ldo, 32, kBM,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    te_in = te_out;
  }
  if (te2 && kind == CDK_EPI_SWIGLU) {
    te2 = make_tmap_sw(&te_in, epi->out2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 2 * epi->half_n, M, epi->ldo2, 64, kBM,
                       CU_TENSOR_MAP_SWIZZLE_128B) &&
          make_tmap_sw(&te_out, epi->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, epi->ldo, 64, kBM,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  } else if (te2) {
    te2 = make_tmap_sw(&te_out, epi->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, epi->ldo, 64, kBM,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    te_in = te_out;
  }
  if (te && kind == CDK_EPI_RESID_F32) {
    te = N % 32 == 0 &&
         make_tmap_sw(&te_in, epi->resid, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, epi->ldr, 32, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_tmap_sw(&te_out, epi->out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, epi->ldo, 32, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  } else if (te) {
    te = N % 64 == 0 &&
         make_tmap_sw(&te_in, epi->aux, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, epi->half_n + N, M, epi->ldaux, 64,
                      kBM, CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_tmap_sw(&te_out, epi->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, epi->half_n + N, M, epi->ldo, 64, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  }

  long long units = m_tiles * n_tiles * splits;
  int grid = (int)(units < sms ? units : sms);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the residual add keeps the full mainloop ring (its mainloop is the slower half)
  // unless CDK_GEMM_TE_RESID_SLOTS=4 asks for the 4-slot / 3-stage layout
  int tem = te ? (kind == CDK_EPI_RESID_F32 && !te_resid_deep() ? 4 : 1) : te2 ? 2 : te3 ? 3 : 0;
  // CTA-pair form: 256-row units, B split between the two CTAs of a cluster
  // (M a multiple of 256: no CTA of a pair holds a tile wholly below the last row)
  // (B MN-major: the 64-column groups are loaded as before, half of them per CTA)
  // (its 32 KB stages leave room for the residual's 64 KB four-slot layout,
  // which the one-CTA form can only have at three stages).  Weight gradients
  // (both operands MN-major, split-K reduce-add) re-choose the split for the
  // pairs.
  // (8-bit operands: K-major A; the forward, residual, dX and K-major
  // weight-gradient forms)
  const bool pair_form =
      a_mn ? (!f8 && b_mn && tem == 3)
           : tem == 3 ? !b_mn
                      : splits == 1 && (b_mn ? (tem == 2 || (!f8 && tem == 1)) : tem == 1 || tem == 2 || tem == 4);
  if (BN == 256 && pair_form && M % (2 * kBM) == 0 && pair_enabled()) {
    const int clusters = pair_clusters(dev);
    if (clusters > 0) {
      if (!b_mn && (f8 ? !make_tmap_u8(&tb, b, K, dual ? 2 * N : N, ldb, bk, BN / 2)
                       : !make_tmap(&tb, b, K, dual ? 2 * N : N, ldb, kBK, BN / 2)))
        return -11;
      p.pair = 1;
      if (f8) p.idesc_f8 = make_idesc_f8(2 * kBM, BN, a_fmt, b_fmt, false, b_mn != 0);
      if (tem == 4) tem = 1;
      p.m_tiles = (int)((M + 2 * kBM - 1) / (2 * kBM));
      if (kind == CDK_EPI_ATOMIC_F32) {
        int s2 = choose_splits((long long)p.m_tiles * n_tiles, clusters);
        const long long kp = (k_tiles + s2 - 1) / s2;
        p.k_per_split = (int)kp;
        p.splits = (int)((k_tiles + kp - 1) / kp);
      }
      units = (long long)p.m_tiles * n_tiles * p.splits;
      grid = 2 * (int)(units < clusters ? units : clusters);
    }
  }
  if (BN == 256) return dispatch_major<256>(a_mn, b_mn, tem, ta, tb, te_in, te_out, p, grid, s);
  return dispatch_major<128>(a_mn, b_mn, tem, ta, tb, te_in, te_out, p, grid, s);
}
}  // namespace cdk

extern "C" int cdk_gemm_bf16(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, int64_t M,
                             int64_t N, int64_t K, const CdkGemmEpilogue* epi, int split_k, void* stream) {
  return cdk::gemm_impl(a, lda, a_mn, b, ldb, b_mn, M, N, K, epi, split_k, stream, false, 0, 0, nullptr, nullptr);
}

extern "C" int cdk_gemm_pair_clusters(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return cdk::pair_enabled() ? cdk::pair_clusters(dev) : 0;
}

extern "C" int cdk_gemm_fp8(const void* a, int64_t lda, int a_mn, int a_fmt, const void* b, int64_t ldb, int b_mn,
                            int b_fmt, int64_t M, int64_t N, int64_t K, const float* scale_inv_a,
                            const float* scale_inv_b, const CdkGemmEpilogue* epi, int split_k, void* stream) {
  return cdk::gemm_impl(a, lda, a_mn, b, ldb, b_mn, M, N, K, epi, split_k, stream, true, a_fmt, b_fmt, scale_inv_a,
                        scale_inv_b);
}
