// Mixture-of-experts MLP support for the MoE variant of the step: routing
// (softmax over the router logits, top-2, weights renormalised over the two),
// capacity-limited slot assignment, token dispatch into expert-major buffers,
// the weighted combine into the residual stream, and their backward.
//
// The reference has no MoE; the variant's semantics (restated by the oracle):
//   p = softmax(x Wr^T) over X experts; (e1, e2) = top-2 of p (lower index on
//   ties); w_k = p_ek / (p_e1 + p_e2);
//   tokens are split into n_seg equal segments (one per forward pass); inside a
//   segment every expert has `cap` slots, filled first by the k = 0 choices in
//   token order, then by the k = 1 choices in token order; a choice that finds
//   its expert full is dropped (it contributes nothing);
//   y_t = resid_t + sum_k kept_k * w_k * FFN_ek(x_t).
// Slot s of expert e in segment g lives at row e * (n_seg * cap) + g * cap + s
// of the expert-major buffers, so each expert's rows are contiguous.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {

// One warp per token: softmax, top-2, renormalised weights.
__global__ void moe_topk_kernel(const float* __restrict__ logits, long long T, int X, int32_t* __restrict__ expert,
                                float* __restrict__ weight, float* __restrict__ probs) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const float z = lane < X ? logits[t * X + lane] : -INFINITY;
  float m = z;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float ez = lane < X ? __expf(z - m) : 0.f;
  float s = ez;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float p = ez / s;
  if (lane < X) probs[t * X + lane] = p;
  // top-2 by (value desc, index asc)
  float v1 = lane < X ? p : -1.f;
  int i1 = lane;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v1, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i1, o);
    if (ov > v1 || (ov == v1 && oi < i1)) {
      v1 = ov;
      i1 = oi;
    }
  }
  float v2 = (lane < X && lane != i1) ? p : -1.f;
  int i2 = lane;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v2, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i2, o);
    if (ov > v2 || (ov == v2 && oi < i2)) {
      v2 = ov;
      i2 = oi;
    }
  }
  if (lane == 0) {
    const float den = v1 + v2;
    expert[2 * t] = i1;
    expert[2 * t + 1] = i2;
    weight[2 * t] = v1 / den;
    weight[2 * t + 1] = v2 / den;
  }
}

// Slot assignment, three phases over chunks of 1024 tokens of one segment.
constexpr int kChunk = 1024;

__device__ __forceinline__ int block_excl_scan_1024(int v, int* sh, int* total) {
  // inclusive warp scan, then the warp sums, then add the warp prefix
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
  #pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = sh[lane];
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sh[lane] = w;  // inclusive prefix of the warp sums
  }
  __syncthreads();
  const int excl = x - v + (warp > 0 ? sh[warp - 1] : 0);
  if (total) *total = sh[31];
  __syncthreads();
  return excl;
}

// Phase 1: per chunk, per (k, expert) counts.  grid = (n_chunks, n_seg), 1024 threads.
__global__ void __launch_bounds__(kChunk) moe_count_kernel(const int32_t* __restrict__ expert, long long seg_len,
                                                           int X, int32_t* __restrict__ counts) {
  __shared__ int sh[32];
  const int chunk = blockIdx.x, seg = blockIdx.y;
  const long long t = (long long)seg * seg_len + (long long)chunk * kChunk + threadIdx.x;
  const bool ok = (long long)chunk * kChunk + threadIdx.x < seg_len;
  int32_t* out = counts + ((long long)seg * gridDim.x + chunk) * 2 * X;
  for (int k = 0; k < 2; ++k) {
    const int e = ok ? expert[2 * t + k] : -1;
    for (int x = 0; x < X; ++x) {
      int tot;
      block_excl_scan_1024(e == x ? 1 : 0, sh, &tot);
      if (threadIdx.x == 0) out[k * X + x] = tot;
    }
  }
}

// Phase 2: exclusive offsets over chunks, k-major (all k=0 before k=1), per expert and segment.
__global__ void moe_offsets_kernel(int32_t* __restrict__ counts, int n_chunks, int X) {
  const int seg = blockIdx.x;
  const int x = threadIdx.x;
  if (x >= X) return;
  int32_t* base = counts + (long long)seg * n_chunks * 2 * X;
  int run = 0;
  for (int k = 0; k < 2; ++k)
    for (int c = 0; c < n_chunks; ++c) {
      const int v = base[(long long)c * 2 * X + k * X + x];
      base[(long long)c * 2 * X + k * X + x] = run;
      run += v;
    }
}

// Phase 3: positions; slot[t][k] = row in the expert-major buffers or -1 (dropped);
// src[row] = token (rows never filled keep -1 from the host-side fill).
__global__ void __launch_bounds__(kChunk) moe_slot_kernel(const int32_t* __restrict__ expert, long long seg_len,
                                                          int X, int n_seg, long long cap,
                                                          const int32_t* __restrict__ offsets,
                                                          int32_t* __restrict__ slot, int32_t* __restrict__ src) {
  __shared__ int sh[32];
  const int chunk = blockIdx.x, seg = blockIdx.y;
  const long long local = (long long)chunk * kChunk + threadIdx.x;
  const bool ok = local < seg_len;
  const long long t = (long long)seg * seg_len + local;
  const int32_t* off = offsets + ((long long)seg * gridDim.x + chunk) * 2 * X;
  for (int k = 0; k < 2; ++k) {
    const int e = ok ? expert[2 * t + k] : -1;
    int pos = -1;
    for (int x = 0; x < X; ++x) {
      const int pre = block_excl_scan_1024(e == x ? 1 : 0, sh, nullptr);
      if (e == x) pos = off[k * X + x] + pre;
    }
    if (ok) {
      if (e >= 0 && e < X && pos < cap) {
        const long long row = (long long)e * n_seg * cap + (long long)seg * cap + pos;
        slot[2 * t + k] = (int32_t)row;
        src[row] = (int32_t)t;
      } else {
        slot[2 * t + k] = -1;
      }
    }
  }
}

// xe[row] = x[src[row]] (zero row when src < 0); one warp per row.
__global__ void moe_dispatch_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                    const int32_t* __restrict__ src, long long rows, int dim8,
                                    __nv_bfloat16* __restrict__ xe) {
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const long long t = src[r];
  uint4* d = reinterpret_cast<uint4*>(xe + r * (long long)dim8 * 8);
  if (t < 0) {
    for (int i = lane; i < dim8; i += 32) d[i] = make_uint4(0u, 0u, 0u, 0u);
  } else {
    const uint4* s = reinterpret_cast<const uint4*>(x + t * ldx);
    for (int i = lane; i < dim8; i += 32) d[i] = s[i];
  }
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 w, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 v = __bfloat1622float2(h[j]);
    f[2 * j] = v.x;
    f[2 * j + 1] = v.y;
  }
}

// out[t] = resid[t] + sum_k w_k ye[slot_k]; one warp per token, 8 columns per lane step.
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ ye, const int32_t* __restrict__ slot,
                                   const float* __restrict__ weight, const float* __restrict__ resid,
                                   float* __restrict__ out, long long T, int dim8) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int s0 = slot[2 * t], s1 = slot[2 * t + 1];
  const float w0 = weight[2 * t], w1 = weight[2 * t + 1];
  const long long dim = (long long)dim8 * 8;
  for (int i = lane; i < dim8; i += 32) {
    float acc[8];
    const float4* r4 = reinterpret_cast<const float4*>(resid + t * dim + i * 8);
    const float4 a = r4[0], b = r4[1];
    acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
    acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
    if (s0 >= 0) {
      float f[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(ye + (long long)s0 * dim)[i], f);
      #pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(w0, f[j], acc[j]);
    }
    if (s1 >= 0) {
      float f[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(ye + (long long)s1 * dim)[i], f);
      #pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(w1, f[j], acc[j]);
    }
    float4* o4 = reinterpret_cast<float4*>(out + t * dim + i * 8);
    o4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// Backward of the combine: dye[slot_k] = w_k * dout[t] (bf16), dweight[t][k] =
// dout[t] . ye[slot_k] (0 when dropped).  Rows of dye that no token owns are
// zeroed by the host beforehand.
__global__ void moe_combine_bwd_kernel(const float* __restrict__ dout, const __nv_bfloat16* __restrict__ ye,
                                       const int32_t* __restrict__ slot, const float* __restrict__ weight,
                                       __nv_bfloat16* __restrict__ dye, float* __restrict__ dweight, long long T,
                                       int dim8) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const long long dim = (long long)dim8 * 8;
  for (int k = 0; k < 2; ++k) {
    const int s = slot[2 * t + k];
    const float w = weight[2 * t + k];
    float dot = 0.f;
    if (s >= 0) {
      for (int i = lane; i < dim8; i += 32) {
        const float4* d4 = reinterpret_cast<const float4*>(dout + t * dim + i * 8);
        const float4 a = d4[0], b = d4[1];
        const float g[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        float f[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(ye + (long long)s * dim)[i], f);
        #pragma unroll
        for (int j = 0; j < 8; ++j) dot = fmaf(g[j], f[j], dot);
        reinterpret_cast<uint4*>(dye + (long long)s * dim)[i] =
            make_uint4(pack_bf16(w * g[0], w * g[1]), pack_bf16(w * g[2], w * g[3]), pack_bf16(w * g[4], w * g[5]),
                       pack_bf16(w * g[6], w * g[7]));
      }
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) dweight[2 * t + k] = dot;
  }
}

// Router backward: through w_k = p_ek / (p_e1 + p_e2) and the softmax.  One
// warp per token; dlogits in bf16 [T, ldd] (the next GEMMs' operand).
__global__ void moe_route_bwd_kernel(const float* __restrict__ probs, const int32_t* __restrict__ expert,
                                     const float* __restrict__ dweight, long long T, int X,
                                     __nv_bfloat16* __restrict__ dlogits, long long ldd) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int e1 = expert[2 * t], e2 = expert[2 * t + 1];
  const float p1 = probs[t * X + e1], p2 = probs[t * X + e2];
  const float dw1 = dweight[2 * t], dw2 = dweight[2 * t + 1];
  const float s = p1 + p2;
  const float dp1 = p2 * (dw1 - dw2) / (s * s);
  const float dp2 = p1 * (dw2 - dw1) / (s * s);
  const float p = lane < X ? probs[t * X + lane] : 0.f;
  const float dp = lane == e1 ? dp1 : (lane == e2 ? dp2 : 0.f);
  float sum = p * dp;
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane < ldd) dlogits[t * ldd + lane] = __float2bfloat16_rn(lane < X ? p * (dp - sum) : 0.f);
}

// out[t] (=/+=) sum_k dxe[slot_k] (fp32 out, bf16 dxe); one warp per token.
__global__ void moe_gather_sum_kernel(const __nv_bfloat16* __restrict__ dxe, const int32_t* __restrict__ slot,
                                      float* __restrict__ out, long long T, int dim8, int accumulate) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int s0 = slot[2 * t], s1 = slot[2 * t + 1];
  const long long dim = (long long)dim8 * 8;
  for (int i = lane; i < dim8; i += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float4* o4 = reinterpret_cast<float4*>(out + t * dim + i * 8);
    if (accumulate) {
      const float4 a = o4[0], b = o4[1];
      acc[0] = a.x; acc[1] = a.y; acc[2] = a.z; acc[3] = a.w;
      acc[4] = b.x; acc[5] = b.y; acc[6] = b.z; acc[7] = b.w;
    }
    if (s0 >= 0) {
      float f[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(dxe + (long long)s0 * dim)[i], f);
      #pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    if (s1 >= 0) {
      float f[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(dxe + (long long)s1 * dim)[i], f);
      #pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    o4[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o4[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

static inline int finish_moe() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace cdk

using namespace cdk;

extern "C" int64_t cdk_moe_route_workspace(int64_t T, int32_t n_seg, int32_t X) {
  if (n_seg <= 0 || T % n_seg) return -1;
  const int64_t chunks = (T / n_seg + kChunk - 1) / kChunk;
  return (int64_t)n_seg * chunks * 2 * X * (int64_t)sizeof(int32_t);
}

extern "C" int cdk_moe_route(const float* logits, int64_t T, int32_t X, int32_t n_seg, int64_t cap,
                             int32_t* expert, float* weight, float* probs, int32_t* slot, int32_t* src,
                             void* workspace, void* stream) {
  if (T == 0) return 0;
  if (!logits || !expert || !weight || !probs || !slot || !src || !workspace || X < 2 || X > 32 || n_seg <= 0 ||
      T % n_seg || cap <= 0)
    return -1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  moe_topk_kernel<<<(unsigned)((T + 7) / 8), 256, 0, s>>>(logits, T, X, expert, weight, probs);
  const long long seg_len = T / n_seg;
  const int chunks = (int)((seg_len + kChunk - 1) / kChunk);
  int32_t* counts = reinterpret_cast<int32_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(src, 0xff, (size_t)X * n_seg * cap * sizeof(int32_t), s);  // -1
  if (e != cudaSuccess) return (int)e;
  moe_count_kernel<<<dim3((unsigned)chunks, (unsigned)n_seg), kChunk, 0, s>>>(expert, seg_len, X, counts);
  moe_offsets_kernel<<<(unsigned)n_seg, 32, 0, s>>>(counts, chunks, X);
  moe_slot_kernel<<<dim3((unsigned)chunks, (unsigned)n_seg), kChunk, 0, s>>>(expert, seg_len, X, n_seg, cap, counts,
                                                                            slot, src);
  return finish_moe();
}

extern "C" int cdk_moe_dispatch(const void* x, int64_t ldx, const int32_t* src, int64_t rows, int64_t dim, void* xe,
                                void* stream) {
  if (rows == 0) return 0;
  if (!x || !src || !xe || dim % 8 || ldx % 8) return -1;
  moe_dispatch_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, src, rows, (int)(dim / 8), reinterpret_cast<__nv_bfloat16*>(xe));
  return finish_moe();
}

extern "C" int cdk_moe_combine(const void* ye, const int32_t* slot, const float* weight, const float* resid,
                               float* out, int64_t T, int64_t dim, void* stream) {
  if (T == 0) return 0;
  if (!ye || !slot || !weight || !resid || !out || dim % 8) return -1;
  moe_combine_kernel<<<(unsigned)((T + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(ye), slot, weight, resid, out, T, (int)(dim / 8));
  return finish_moe();
}

extern "C" int cdk_moe_combine_bwd(const float* dout, const void* ye, const int32_t* slot, const float* weight,
                                   void* dye, int64_t dye_rows, float* dweight, int64_t T, int64_t dim,
                                   void* stream) {
  if (T == 0) return 0;
  if (!dout || !ye || !slot || !weight || !dye || !dweight || dim % 8) return -1;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(dye, 0, (size_t)dye_rows * dim * 2, s);
  if (e != cudaSuccess) return (int)e;
  moe_combine_bwd_kernel<<<(unsigned)((T + 7) / 8), 256, 0, s>>>(
      dout, reinterpret_cast<const __nv_bfloat16*>(ye), slot, weight, reinterpret_cast<__nv_bfloat16*>(dye), dweight,
      T, (int)(dim / 8));
  return finish_moe();
}

extern "C" int cdk_moe_route_bwd(const float* probs, const int32_t* expert, const float* dweight, int64_t T,
                                 int32_t X, void* dlogits, int64_t ldd, void* stream) {
  if (T == 0) return 0;
  if (!probs || !expert || !dweight || !dlogits || X < 2 || X > 32 || ldd < X || ldd > 32) return -1;
  moe_route_bwd_kernel<<<(unsigned)((T + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      probs, expert, dweight, T, X, reinterpret_cast<__nv_bfloat16*>(dlogits), ldd);
  return finish_moe();
}

extern "C" int cdk_moe_gather_sum(const void* dxe, const int32_t* slot, float* out, int64_t T, int64_t dim,
                                  int accumulate, void* stream) {
  if (T == 0) return 0;
  if (!dxe || !slot || !out || dim % 8) return -1;
  moe_gather_sum_kernel<<<(unsigned)((T + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(dxe), slot, out, T, (int)(dim / 8), accumulate);
  return finish_moe();
}
