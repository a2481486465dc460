// fp8 support for the fp8 training variant: saturating casts to e4m3 / e5m2
// with an optional transposed copy (the K-major operand of the weight-gradient
// GEMM) and amax tracking, and the per-tensor delayed-scaling bookkeeping
// (amax history, scale = fmax / max(history)).
//
// The reference has no fp8 path (its GEMMs run under torch.autocast fp16,
// chessdecoder/train/train.py:168); these semantics are the variant's own and
// are restated by the oracle's fp8 simulation.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

#include <cuda_fp8.h>

namespace cdk {

__device__ __forceinline__ uint8_t to_fp8(float v, int fmt) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, fmt == 0 ? __NV_E4M3 : __NV_E5M2);
}

__device__ __forceinline__ float block_max_256(float v, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  }
  return v;  // valid in thread 0
}

// One 64 x 64 tile per block (256 threads).  Thread t covers rows
// t/16 + 16k (k < 4) and the 4 columns (t % 16) * 4 .. +3 of each.
template <int DT>
__global__ void __launch_bounds__(256) fp8_cast_kernel(const void* __restrict__ x, long long rows, long long cols,
                                                       long long ldx, const float* __restrict__ scale, int fmt,
                                                       uint8_t* __restrict__ out, long long ldo,
                                                       uint8_t* __restrict__ out_t, long long ldt,
                                                       float* __restrict__ amax) {
  __shared__ uint8_t tile[64][64 + 4];
  __shared__ float red[8];
  const long long r0 = (long long)blockIdx.y * 64, c0 = (long long)blockIdx.x * 64;
  const float s = scale ? *scale : 1.f;
  const int tr = threadIdx.x >> 4, tc = (threadIdx.x & 15) * 4;
  float mx = 0.f;
  #pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int lr = tr + 16 * k;
    const long long r = r0 + lr, c = c0 + tc;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < rows) {
      if (c + 3 < cols) {
        if constexpr (DT == 0) {
          const float* p = reinterpret_cast<const float*>(x) + r * ldx + c;
          if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
            const float4 q = *reinterpret_cast<const float4*>(p);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
          } else {
            #pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = p[j];
          }
        } else {
          const __nv_bfloat16* p = reinterpret_cast<const __nv_bfloat16*>(x) + r * ldx + c;
          if ((reinterpret_cast<uintptr_t>(p) & 7) == 0) {
            const uint2 q = *reinterpret_cast<const uint2*>(p);
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
            v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
          } else {
            #pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(p[j]);
          }
        }
      } else {
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (c + j < cols) {
            if constexpr (DT == 0) v[j] = reinterpret_cast<const float*>(x)[r * ldx + c + j];
            else v[j] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[r * ldx + c + j]);
          }
        }
      }
    }
    uint8_t q[4];
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      mx = fmaxf(mx, fabsf(v[j]));
      q[j] = to_fp8(v[j] * s, fmt);
      tile[lr][tc + j] = q[j];
    }
    if (out && r < rows) {
      uint8_t* o = out + r * ldo + c;
      if (c + 3 < cols && (reinterpret_cast<uintptr_t>(o) & 3) == 0) {
        *reinterpret_cast<uint32_t*>(o) = (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16) |
                                          ((uint32_t)q[3] << 24);
      } else {
        #pragma unroll
        for (int j = 0; j < 4; ++j)
          if (c + j < cols) o[j] = q[j];
      }
    }
  }
  if (out_t) {
    __syncthreads();
    // transposed: thread covers out_t rows (tile columns) tr + 16k, 4 tile rows from tc
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int lc = tr + 16 * k;
      const long long oc = c0 + lc;  // row of out_t
      const long long orr = r0 + tc; // first column of out_t
      if (oc >= cols) continue;
      const uint8_t q0 = tile[tc][lc], q1 = tile[tc + 1][lc], q2 = tile[tc + 2][lc], q3 = tile[tc + 3][lc];
      uint8_t* o = out_t + oc * ldt + orr;
      if (orr + 3 < rows && (reinterpret_cast<uintptr_t>(o) & 3) == 0) {
        *reinterpret_cast<uint32_t*>(o) = (uint32_t)q0 | ((uint32_t)q1 << 8) | ((uint32_t)q2 << 16) |
                                          ((uint32_t)q3 << 24);
      } else {
        const uint8_t qq[4] = {q0, q1, q2, q3};
        #pragma unroll
        for (int j = 0; j < 4; ++j)
          if (orr + j < rows) o[j] = qq[j];
      }
    }
  }
  if (amax) {
    const float m = block_max_256(mx, red);
    if (threadIdx.x == 0 && m > 0.f) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(m));
  }
}

// Row-major cast without a transposed copy: 16 consecutive elements per
// thread (two / four 16-byte loads, one 16-byte store), grid-stride.
template <int DT>
__global__ void __launch_bounds__(256) fp8_cast_rows_kernel(const void* __restrict__ x, long long rows, long long cols,
                                                            long long ldx, const float* __restrict__ scale, int fmt,
                                                            uint8_t* __restrict__ out, long long ldo,
                                                            float* __restrict__ amax) {
  __shared__ float red[8];
  const float s = scale ? *scale : 1.f;
  const long long cpr = cols / 16;  // chunks per row
  const long long n = rows * cpr;
  float mx = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cpr, c = (i - r * cpr) * 16;
    float v[16];
    if constexpr (DT == 0) {
      const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + r * ldx + c);
      #pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 t = p[q];
        v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
      }
    } else {
      const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + r * ldx + c);
      #pragma unroll
      for (int q = 0; q < 2; ++q) {
        const uint4 t = p[q];
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
          v[8 * q + 2 * j] = f.x;
          v[8 * q + 2 * j + 1] = f.y;
        }
      }
    }
    uint32_t o[4];
    #pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t word = 0;
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float f = v[4 * q + j];
        mx = fmaxf(mx, fabsf(f));
        word |= (uint32_t)to_fp8(f * s, fmt) << (8 * j);
      }
      o[q] = word;
    }
    *reinterpret_cast<uint4*>(out + r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (amax) {
    const float m = block_max_256(mx, red);
    if (threadIdx.x == 0 && m > 0.f) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(m));
  }
}

template <int DT>
__global__ void __launch_bounds__(256) fp8_amax_kernel(const void* __restrict__ x, long long rows, long long cols,
                                                       long long ldx, float* __restrict__ amax) {
  __shared__ float red[8];
  float mx = 0.f;
  const long long n = rows * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols, c = i - r * cols;
    float v;
    if constexpr (DT == 0) v = reinterpret_cast<const float*>(x)[r * ldx + c];
    else v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[r * ldx + c]);
    mx = fmaxf(mx, fabsf(v));
  }
  const float m = block_max_256(mx, red);
  if (threadIdx.x == 0 && m > 0.f) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(m));
}

__global__ void fp8_scales_kernel(float* __restrict__ amax_cur, float* __restrict__ history,
                                  float* __restrict__ scale, float* __restrict__ scale_inv,
                                  const float* __restrict__ fmax, int n, int hist_len, int mode) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float m;
  if (mode == 0) {
    float* h = history + (long long)i * hist_len;
    for (int k = hist_len - 1; k > 0; --k) h[k] = h[k - 1];
    h[0] = amax_cur[i];
    m = 0.f;
    for (int k = 0; k < hist_len; ++k) m = fmaxf(m, h[k]);
    amax_cur[i] = 0.f;
  } else {
    m = amax_cur[i];
  }
  const float sc = m > 0.f ? fmax[i] / m : 1.f;
  scale[i] = sc;
  scale_inv[i] = 1.f / sc;
}

}  // namespace cdk

using namespace cdk;

extern "C" int cdk_fp8_cast(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx, const float* scale,
                            int fmt, void* out, int64_t ldo, void* out_t, int64_t ldt, float* amax, void* stream) {
  if (rows == 0 || cols == 0) return 0;
  if (!x || rows < 0 || cols < 0 || ldx < cols || (x_dtype != 0 && x_dtype != 1) || (fmt != 0 && fmt != 1))
    return -1;
  if ((out && ldo < cols) || (out_t && ldt < rows)) return -2;
  if (rows > (1ll << 31) || cols > (1ll << 31)) return -3;
  dim3 grid((unsigned)((cols + 63) / 64), (unsigned)((rows + 63) / 64));
  if (grid.y > 65535u) return -3;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* o = reinterpret_cast<uint8_t*>(out);
  uint8_t* ot = reinterpret_cast<uint8_t*>(out_t);
  const int esz = x_dtype == 0 ? 4 : 2;
  if (!ot && o && cols % 16 == 0 && ldo % 16 == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx * esz) % 16 == 0) {
    long long blocks = (rows * (cols / 16) + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (x_dtype == 0)
      fp8_cast_rows_kernel<0><<<(unsigned)blocks, 256, 0, s>>>(x, rows, cols, ldx, scale, fmt, o, ldo, amax);
    else
      fp8_cast_rows_kernel<1><<<(unsigned)blocks, 256, 0, s>>>(x, rows, cols, ldx, scale, fmt, o, ldo, amax);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : (int)e;
  }
  if (x_dtype == 0) fp8_cast_kernel<0><<<grid, 256, 0, s>>>(x, rows, cols, ldx, scale, fmt, o, ldo, ot, ldt, amax);
  else fp8_cast_kernel<1><<<grid, 256, 0, s>>>(x, rows, cols, ldx, scale, fmt, o, ldo, ot, ldt, amax);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_fp8_amax(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx, float* amax,
                            void* stream) {
  if (rows == 0 || cols == 0) return 0;
  if (!x || !amax || rows < 0 || cols < 0 || ldx < cols || (x_dtype != 0 && x_dtype != 1)) return -1;
  long long blocks = (rows * cols + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (x_dtype == 0) fp8_amax_kernel<0><<<(unsigned)blocks, 256, 0, s>>>(x, rows, cols, ldx, amax);
  else fp8_amax_kernel<1><<<(unsigned)blocks, 256, 0, s>>>(x, rows, cols, ldx, amax);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_fp8_scales(float* amax_cur, float* history, float* scale, float* scale_inv, const float* fmax,
                              int32_t n, int32_t hist_len, int32_t mode, void* stream) {
  if (n == 0) return 0;
  if (!amax_cur || !scale || !scale_inv || !fmax || n < 0 || (mode == 0 && (!history || hist_len <= 0)) ||
      (mode != 0 && mode != 1))
    return -1;
  fp8_scales_kernel<<<(unsigned)((n + 127) / 128), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      amax_cur, history, scale, scale_inv, fmax, n, hist_len, mode);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}
