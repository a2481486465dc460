// RMSNorm forward/backward (eps 1e-6, statistics in fp32).
//
// Replaces torchtune RMSNorm as used by chessdecoder/models/model.py:112-116
// (restated torchtune-free by the reference at
// chessdecoder/export/backbone_causal.py:61-64):
//     y = x * rsqrt(mean(x^2) + eps) * scale
// One warp per row, 128-bit loads; the row stays in registers between the
// sum-of-squares and the scaling pass.  The forward writes the bf16 copy that
// feeds the next GEMM (and optionally an fp32 copy); the backward fuses the
// residual-gradient add, the bf16 copy of dx for the next GEMM and the
// per-column scale gradient.  The _q8 entry points write the fp8 recipe's
// 8-bit copy (e4m3 / e5m2 with the tensor's delayed scale, amax recorded)
// in place of the bf16 one.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

#include <type_traits>

namespace cdk {

template <int VPT, bool QOUT>  // float4 per lane; dim = 128 * VPT
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ scale,
                                                          __nv_bfloat16* __restrict__ y16, float* __restrict__ y32,
                                                          float* __restrict__ rstd, long long rows, float eps,
                                                          Q8Out q8) {
  constexpr int dim = 128 * VPT;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  float m = 0.f;  // max |y| of this lane's values (8-bit output)
  if (row < rows) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * dim);
    float4 v[VPT];
    float ss = 0.f;
    #pragma unroll
    for (int i = 0; i < VPT; ++i) {
      v[i] = xr[lane + 32 * i];
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)dim + eps);
    const float4* sc = reinterpret_cast<const float4*>(scale);
    const float qs = QOUT ? *q8.qscale : 0.f;
    #pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const float4 s = sc[lane + 32 * i];
      float4 o = make_float4(v[i].x * r * s.x, v[i].y * r * s.y, v[i].z * r * s.z, v[i].w * r * s.w);
      if (y16) {
        uint2 w;
        w.x = pack_bf16(o.x, o.y);
        w.y = pack_bf16(o.z, o.w);
        reinterpret_cast<uint2*>(y16 + row * dim)[lane + 32 * i] = w;
      }
      if (y32) reinterpret_cast<float4*>(y32 + row * dim)[lane + 32 * i] = o;
      if (QOUT) {
        reinterpret_cast<uint32_t*>(q8.q + row * q8.ldq)[lane + 32 * i] = q8_pack4(o.x, o.y, o.z, o.w, qs, q8.fmt);
        m = abs_max4(m, o.x, o.y, o.z, o.w);
      }
    }
    if (lane == 0 && rstd) rstd[row] = r;
  }
  if (QOUT && q8.amax) block_amax_atomic(m, q8.amax);  // uniform: every thread of the block takes it
}

// Generic fallback for dims that are not a multiple of 128 (dim % 4 == 0 not required).
__global__ void rmsnorm_fwd_generic(const float* __restrict__ x, const float* __restrict__ scale,
                                    __nv_bfloat16* __restrict__ y16, float* __restrict__ y32, float* __restrict__ rstd,
                                    long long rows, int dim, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * dim;
  float ss = 0.f;
  for (int i = lane; i < dim; i += 32) ss += xr[i] * xr[i];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)dim + eps);
  for (int i = lane; i < dim; i += 32) {
    const float o = xr[i] * r * scale[i];
    if (y16) y16[row * dim + i] = __float2bfloat16_rn(o);
    if (y32) y32[row * dim + i] = o;
  }
  if (lane == 0 && rstd) rstd[row] = r;
}

template <bool DY_F32>
__device__ __forceinline__ float4 load_dy4(const void* dy, long long idx4) {
  if (DY_F32) return reinterpret_cast<const float4*>(dy)[idx4];
  const uint2 w = reinterpret_cast<const uint2*>(dy)[idx4];
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// dx = dres + r * (g - xhat * mean(g * xhat)),  g = dy * scale, xhat = x * r
// dscale[c] += sum_rows dy[c] * xhat[c]
// A warp issues all of a row's loads (x, dy, dres) before its first use, so
// each warp keeps three streams in flight; the scale lives in shared memory.
template <int VPT, bool DY_F32, bool QOUT>
__global__ void __launch_bounds__(256, 2) rmsnorm_bwd_kernel(const void* __restrict__ dy, const float* __restrict__ x,
                                                             const float* __restrict__ scale,
                                                             const float* __restrict__ rstd,
                                                             const float* __restrict__ dres, float* __restrict__ dx,
                                                             __nv_bfloat16* __restrict__ dx16,
                                                             float* __restrict__ dscale, long long rows, Q8Out q8) {
  constexpr int dim = 128 * VPT;
  extern __shared__ float red[];  // [8][dim] per-warp column partials of dscale, then [dim] scale
  float* ssc = red + 8 * dim;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) ssc[c] = scale[c];
  float4* myds = reinterpret_cast<float4*>(red + warp * dim);
  #pragma unroll
  for (int i = 0; i < VPT; ++i) myds[lane + 32 * i] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  const float4* sc4 = reinterpret_cast<const float4*>(ssc);
  const float qs = QOUT ? *q8.qscale : 0.f;
  float m = 0.f;  // max |dx| of this lane's values (8-bit output)

  for (long long row = (long long)blockIdx.x * 8 + warp; row < rows; row += (long long)gridDim.x * 8) {
    float4 xv[VPT], qv[VPT];
    typename std::conditional<DY_F32, float4, uint2>::type draw[VPT];
    #pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const long long idx4 = row * (dim / 4) + lane + 32 * i;
      xv[i] = reinterpret_cast<const float4*>(x)[idx4];
      if constexpr (DY_F32) draw[i] = reinterpret_cast<const float4*>(dy)[idx4];
      else draw[i] = reinterpret_cast<const uint2*>(dy)[idx4];
      qv[i] = dres ? reinterpret_cast<const float4*>(dres)[idx4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    auto dyv = [&](int i) -> float4 {
      if constexpr (DY_F32) {
        return draw[i];
      } else {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&draw[i].x));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&draw[i].y));
        return make_float4(a.x, a.y, b.x, b.y);
      }
    };
    const float r = rstd[row];
    float dot = 0.f;
    #pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const float4 s = sc4[lane + 32 * i];
      const float4 d = dyv(i);
      xv[i] = make_float4(xv[i].x * r, xv[i].y * r, xv[i].z * r, xv[i].w * r);  // xhat
      dot += d.x * s.x * xv[i].x + d.y * s.y * xv[i].y + d.z * s.z * xv[i].z + d.w * s.w * xv[i].w;
      float4 a = myds[lane + 32 * i];
      a.x += d.x * xv[i].x;
      a.y += d.y * xv[i].y;
      a.z += d.z * xv[i].z;
      a.w += d.w * xv[i].w;
      myds[lane + 32 * i] = a;
    }
    dot = warp_sum(dot) / (float)dim;
    #pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const long long idx4 = row * (dim / 4) + lane + 32 * i;
      const float4 s = sc4[lane + 32 * i];
      const float4 d = dyv(i);
      const float4 o = make_float4(qv[i].x + r * (d.x * s.x - xv[i].x * dot), qv[i].y + r * (d.y * s.y - xv[i].y * dot),
                                   qv[i].z + r * (d.z * s.z - xv[i].z * dot), qv[i].w + r * (d.w * s.w - xv[i].w * dot));
      if (dx) reinterpret_cast<float4*>(dx)[idx4] = o;
      if (dx16) {
        uint2 w;
        w.x = pack_bf16(o.x, o.y);
        w.y = pack_bf16(o.z, o.w);
        reinterpret_cast<uint2*>(dx16)[idx4] = w;
      }
      if (QOUT) {
        reinterpret_cast<uint32_t*>(q8.q + row * q8.ldq)[lane + 32 * i] = q8_pack4(o.x, o.y, o.z, o.w, qs, q8.fmt);
        m = abs_max4(m, o.x, o.y, o.z, o.w);
      }
    }
  }
  if (QOUT && q8.amax) block_amax_atomic(m, q8.amax);
  if (dscale) {
    __syncthreads();
    for (int c = threadIdx.x; c < dim; c += blockDim.x) {
      float s = 0.f;
      #pragma unroll
      for (int w = 0; w < 8; ++w) s += red[w * dim + c];
      atomicAdd(dscale + c, s);
    }
  }
}

static int num_sms_dev() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int VPT>
static int launch_bwd(const void* dy, int dy_f32, const float* x, const float* scale, const float* rstd,
                      const float* dres, float* dx, void* dx16, float* dscale, long long rows, cudaStream_t s,
                      Q8Out q8) {
  const size_t smem = (size_t)9 * 128 * VPT * sizeof(float);
  long long blocks = (rows + 7) / 8;
  const long long cap = (long long)num_sms_dev() * 2;
  if (blocks > cap) blocks = cap;
  auto run = [&](auto k) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k<<<(unsigned)blocks, 256, smem, s>>>(dy, x, scale, rstd, dres, dx, reinterpret_cast<__nv_bfloat16*>(dx16),
                                          dscale, rows, q8);
  };
  const bool qo = q8.q != nullptr;
  if (dy_f32) {
    if (qo) run(rmsnorm_bwd_kernel<VPT, true, true>);
    else run(rmsnorm_bwd_kernel<VPT, true, false>);
  } else {
    if (qo) run(rmsnorm_bwd_kernel<VPT, false, true>);
    else run(rmsnorm_bwd_kernel<VPT, false, false>);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace cdk

using namespace cdk;

static int rmsnorm_fwd_impl(const float* x, const float* scale, void* y_bf16, float* y_f32, float* rstd,
                            int64_t rows, int64_t dim, float eps, Q8Out q8, void* stream) {
  if (!x || !scale || rows < 0 || dim <= 0) return -1;
  if (rows == 0) return 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  auto* y16 = reinterpret_cast<__nv_bfloat16*>(y_bf16);
  auto fwd = [&](auto k0, auto k1) {
    if (q8.q) k1<<<blocks, 256, 0, s>>>(x, scale, y16, y_f32, rstd, rows, eps, q8);
    else k0<<<blocks, 256, 0, s>>>(x, scale, y16, y_f32, rstd, rows, eps, q8);
  };
  switch (dim) {
    case 256: fwd(rmsnorm_fwd_kernel<2, false>, rmsnorm_fwd_kernel<2, true>); break;
    case 512: fwd(rmsnorm_fwd_kernel<4, false>, rmsnorm_fwd_kernel<4, true>); break;
    case 768: fwd(rmsnorm_fwd_kernel<6, false>, rmsnorm_fwd_kernel<6, true>); break;
    case 1024: fwd(rmsnorm_fwd_kernel<8, false>, rmsnorm_fwd_kernel<8, true>); break;
    case 2048: fwd(rmsnorm_fwd_kernel<16, false>, rmsnorm_fwd_kernel<16, true>); break;
    default:
      if (q8.q || q8.amax) return -3;  // the 8-bit output needs a width that is a multiple of 256
      rmsnorm_fwd_generic<<<blocks, 256, 0, s>>>(x, scale, y16, y_f32, rstd, rows, (int)dim, eps);
      break;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

static Q8Out make_q8(void* q, int64_t ldq, int fmt, const float* qscale, float* amax) {
  Q8Out o;
  o.q = reinterpret_cast<uint8_t*>(q);
  o.ldq = ldq;
  o.fmt = fmt;
  o.qscale = qscale;
  o.amax = amax;
  return o;
}

static bool q8_ok(void* q, int64_t ldq, int fmt, const float* qscale, int64_t dim) {
  return q && qscale && (fmt == 0 || fmt == 1) && ldq >= dim && (ldq % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(q) & 15) == 0;
}

extern "C" int cdk_rmsnorm_fwd(const float* x, const float* scale, void* y_bf16, float* y_f32, float* rstd,
                               int64_t rows, int64_t dim, float eps, void* stream) {
  return rmsnorm_fwd_impl(x, scale, y_bf16, y_f32, rstd, rows, dim, eps, make_q8(nullptr, 0, 0, nullptr, nullptr),
                          stream);
}

extern "C" int cdk_rmsnorm_fwd_q8(const float* x, const float* scale, void* y8, int64_t ldy8, int fmt,
                                  const float* qscale, float* amax, float* rstd, int64_t rows, int64_t dim, float eps,
                                  void* stream) {
  if (!q8_ok(y8, ldy8, fmt, qscale, dim)) return -2;
  return rmsnorm_fwd_impl(x, scale, nullptr, nullptr, rstd, rows, dim, eps, make_q8(y8, ldy8, fmt, qscale, amax),
                          stream);
}

static int rmsnorm_bwd_impl(const void* dy, int dy_is_f32, const float* x, const float* scale, const float* rstd,
                            const float* dres, float* dx, void* dx_bf16, float* dscale, int64_t rows, int64_t dim,
                            Q8Out q8, void* stream) {
  if (!dy || !x || !scale || !rstd || rows < 0) return -1;
  if (rows == 0) return 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dim) {
    case 256: return launch_bwd<2>(dy, dy_is_f32, x, scale, rstd, dres, dx, dx_bf16, dscale, rows, s, q8);
    case 512: return launch_bwd<4>(dy, dy_is_f32, x, scale, rstd, dres, dx, dx_bf16, dscale, rows, s, q8);
    case 768: return launch_bwd<6>(dy, dy_is_f32, x, scale, rstd, dres, dx, dx_bf16, dscale, rows, s, q8);
    case 1024: return launch_bwd<8>(dy, dy_is_f32, x, scale, rstd, dres, dx, dx_bf16, dscale, rows, s, q8);
    default: return -2;  // backbone widths are multiples of 256 up to 1024
  }
}

extern "C" int cdk_rmsnorm_bwd(const void* dy, int dy_is_f32, const float* x, const float* scale, const float* rstd,
                               const float* dres, float* dx, void* dx_bf16, float* dscale, int64_t rows, int64_t dim,
                               void* stream) {
  return rmsnorm_bwd_impl(dy, dy_is_f32, x, scale, rstd, dres, dx, dx_bf16, dscale, rows, dim,
                          make_q8(nullptr, 0, 0, nullptr, nullptr), stream);
}

extern "C" int cdk_rmsnorm_bwd_q8(const void* dy, int dy_is_f32, const float* x, const float* scale,
                                  const float* rstd, const float* dres, float* dx, void* dx8, int64_t ldx8, int fmt,
                                  const float* qscale, float* amax, float* dscale, int64_t rows, int64_t dim,
                                  void* stream) {
  if (!q8_ok(dx8, ldx8, fmt, qscale, dim)) return -3;
  return rmsnorm_bwd_impl(dy, dy_is_f32, x, scale, rstd, dres, dx, nullptr, dscale, rows, dim,
                          make_q8(dx8, ldx8, fmt, qscale, amax), stream);
}
