// Small glue kernels: row gathers / scatter-adds around the heads, casts, the
// device error word, and a tiled fp32 SIMT GEMM for the few contractions that
// are too small (or too precision-sensitive, like the Fourier projection) to
// route through the tensor-core path.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {

__device__ int g_error_flag = 0;

__global__ void gather_rows_bf16_kernel(const __nv_bfloat16* __restrict__ src, long long ld_src,
                                        const int32_t* __restrict__ rows, long long n, int dim8,
                                        __nv_bfloat16* __restrict__ dst, long long ld_dst) {
  const int lane = threadIdx.x & 31;
  const long long k = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (k >= n) return;
  const long long r = rows[k];
  const uint4* s = reinterpret_cast<const uint4*>(src + r * ld_src);
  uint4* d = reinterpret_cast<uint4*>(dst + k * ld_dst);
  for (int i = lane; i < dim8; i += 32) d[i] = s[i];
}

__global__ void scatter_add_rows_kernel(const float* __restrict__ src, long long ld_src,
                                        const int32_t* __restrict__ rows, long long n, int dim4,
                                        float* __restrict__ dst, long long ld_dst) {
  const int lane = threadIdx.x & 31;
  const long long k = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (k >= n) return;
  const long long r = rows[k];
  const float4* s = reinterpret_cast<const float4*>(src + k * ld_src);
  float4* d = reinterpret_cast<float4*>(dst + r * ld_dst);
  for (int i = lane; i < dim4; i += 32) atomicAdd(d + i, s[i]);
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

__global__ void add_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o,
                               long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    o[i] = a[i] + b[i];
}

__global__ void scale_f32_kernel(float* __restrict__ x, long long n, float s) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    x[i] *= s;
}

// SwiGLU backward (the w2(silu(w1 x) * w3 x) product of
// chessdecoder/models/model.py:104-108):  given du = dL/d(silu(g) * u) and the
// stored pre-activations gu = [g | u] (row pitch ldgu, u at column offset F),
//   dg = du * u * silu'(g),  du_up = du * silu(g)   -> dgu = [dg | du_up].
// Eight columns per thread, 16-byte loads and stores, fp32 math.
template <bool QOUT>
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ du, long long lddu,
                                  const __nv_bfloat16* __restrict__ gu, long long ldgu,
                                  __nv_bfloat16* __restrict__ dgu, long long lddgu, long long rows, int F,
                                  Q8Out q8) {
  const int f8 = F / 8;
  const long long total = rows * f8;
  const float qs = QOUT ? *q8.qscale : 0.f;
  float m = 0.f;  // max |dgu| of this thread's values (8-bit output)
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long r = idx / f8;
    const int c = (int)(idx - r * f8) * 8;
    const uint4 wd = *reinterpret_cast<const uint4*>(du + r * lddu + c);
    const uint4 wg = *reinterpret_cast<const uint4*>(gu + r * ldgu + c);
    const uint4 wu = *reinterpret_cast<const uint4*>(gu + r * ldgu + F + c);
    const __nv_bfloat162* hd = reinterpret_cast<const __nv_bfloat162*>(&wd);
    const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&wg);
    const __nv_bfloat162* hu = reinterpret_cast<const __nv_bfloat162*>(&wu);
    float fg[8], fu[8];
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 d = __bfloat1622float2(hd[j]), g = __bfloat1622float2(hg[j]), u = __bfloat1622float2(hu[j]);
      const float s0 = sigmoid_fast(g.x), s1 = sigmoid_fast(g.y);
      fg[2 * j] = d.x * u.x * (s0 * (1.f + g.x * (1.f - s0)));
      fg[2 * j + 1] = d.y * u.y * (s1 * (1.f + g.y * (1.f - s1)));
      fu[2 * j] = d.x * g.x * s0;
      fu[2 * j + 1] = d.y * g.y * s1;
    }
    if (QOUT) {
      uint8_t* q = q8.q + r * q8.ldq;
      *reinterpret_cast<uint2*>(q + c) = make_uint2(q8_pack4(fg[0], fg[1], fg[2], fg[3], qs, q8.fmt),
                                                    q8_pack4(fg[4], fg[5], fg[6], fg[7], qs, q8.fmt));
      *reinterpret_cast<uint2*>(q + F + c) = make_uint2(q8_pack4(fu[0], fu[1], fu[2], fu[3], qs, q8.fmt),
                                                        q8_pack4(fu[4], fu[5], fu[6], fu[7], qs, q8.fmt));
      #pragma unroll
      for (int j = 0; j < 2; ++j)
        m = abs_max4(abs_max4(m, fg[4 * j], fg[4 * j + 1], fg[4 * j + 2], fg[4 * j + 3]), fu[4 * j], fu[4 * j + 1],
                     fu[4 * j + 2], fu[4 * j + 3]);
    } else {
      uint32_t og[4], ou[4];
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        og[j] = pack_bf16(fg[2 * j], fg[2 * j + 1]);
        ou[j] = pack_bf16(fu[2 * j], fu[2 * j + 1]);
      }
      *reinterpret_cast<uint4*>(dgu + r * lddgu + c) = make_uint4(og[0], og[1], og[2], og[3]);
      *reinterpret_cast<uint4*>(dgu + r * lddgu + F + c) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    }
  }
  if (QOUT && q8.amax) block_amax_atomic(m, q8.amax);
}

// C[M,N] = beta*C + sum_k A(m,k) B(n,k) + bias[n]
//   A(m,k) = a_t ? A[k*lda + m] : A[m*lda + k];  B(n,k) = b_t ? B[k*ldb + n] : B[n*ldb + k]
// 64x64 tile, 16-deep k slices, 256 threads with a 4x4 micro-tile each.
// Split-K over blockIdx.z (k_per columns of K each): with more than one split
// the partial sums are atomically added (C zeroed beforehand unless
// accumulating) and split 0 adds the bias.
__global__ void __launch_bounds__(256) sgemm_kernel(const float* __restrict__ A, long long lda, int a_t,
                                                    const float* __restrict__ B, long long ldb, int b_t,
                                                    float* __restrict__ C, long long ldc, int M, int N, int K,
                                                    const float* __restrict__ bias, int accumulate, int k_per) {
  __shared__ float sA[16][64 + 4];
  __shared__ float sB[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int kb = blockIdx.z * k_per, ke = min(K, kb + k_per);
  const bool split = gridDim.z > 1;
  float acc[4][4] = {};
  for (int k0 = kb; k0 < ke; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      int kk, mm;
      if (a_t) { kk = i / 64; mm = i % 64; } else { mm = i / 16; kk = i % 16; }
      const int gm = m0 + mm, gk = k0 + kk;
      float va = 0.f;
      if (gm < M && gk < ke) va = a_t ? A[(long long)gk * lda + gm] : A[(long long)gm * lda + gk];
      sA[kk][mm] = va;
      int nn;
      if (b_t) { kk = i / 64; nn = i % 64; } else { nn = i / 16; kk = i % 16; }
      const int gn = n0 + nn, gk2 = k0 + kk;
      float vb = 0.f;
      if (gn < N && gk2 < ke) vb = b_t ? B[(long long)gk2 * ldb + gn] : B[(long long)gn * ldb + gk2];
      sB[kk][nn] = vb;
    }
    __syncthreads();
    #pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
      #pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[kk][ty * 4 + i];
      #pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sB[kk][tx * 4 + j];
      #pragma unroll
      for (int i = 0; i < 4; ++i)
        #pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  #pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float v = acc[i][j] + (bias && blockIdx.z == 0 ? bias[gn] : 0.f);
      float* c = C + (long long)gm * ldc + gn;
      if (split) atomicAdd(c, v);
      else *c = accumulate ? *c + v : v;
    }
  }
}

static inline int finish() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

static inline unsigned grid_for(long long n) {
  long long b = (n + 255) / 256;
  if (b > 148 * 16) b = 148 * 16;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace cdk

using namespace cdk;

extern "C" int cdk_version(void) { return 1; }

extern "C" int cdk_get_error(int* out_flags, int clear) {
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return (int)e;
  e = cudaMemcpyFromSymbol(&v, g_error_flag, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_error_flag, &zero, sizeof(int));
    if (e != cudaSuccess) return (int)e;
  }
  if (out_flags) *out_flags = v;
  return 0;
}

extern "C" int cdk_gather_rows_bf16(const void* src, int64_t ld_src, const int32_t* rows, int64_t n, int64_t dim,
                                    void* dst, int64_t ld_dst, void* stream) {
  if (n == 0) return 0;
  if (!src || !rows || !dst || dim % 8 || ld_src % 8 || ld_dst % 8) return -1;
  gather_rows_bf16_kernel<<<(unsigned)((n + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(src), ld_src, rows, n, (int)(dim / 8),
      reinterpret_cast<__nv_bfloat16*>(dst), ld_dst);
  return finish();
}

extern "C" int cdk_scatter_add_rows_f32(const float* src, int64_t ld_src, const int32_t* rows, int64_t n, int64_t dim,
                                        float* dst, int64_t ld_dst, void* stream) {
  if (n == 0) return 0;
  if (!src || !rows || !dst || dim % 4 || ld_src % 4 || ld_dst % 4) return -1;
  scatter_add_rows_kernel<<<(unsigned)((n + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      src, ld_src, rows, n, (int)(dim / 4), dst, ld_dst);
  return finish();
}

extern "C" int cdk_cast_f32_bf16(const float* src, void* dst, int64_t n, void* stream) {
  if (n == 0) return 0;
  if (!src || !dst) return -1;
  cast_f32_bf16_kernel<<<grid_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      src, reinterpret_cast<__nv_bfloat16*>(dst), n);
  return finish();
}

extern "C" int cdk_add_f32(const float* a, const float* b, float* out, int64_t n, void* stream) {
  if (n == 0) return 0;
  if (!a || !b || !out) return -1;
  add_f32_kernel<<<grid_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a, b, out, n);
  return finish();
}

extern "C" int cdk_scale_f32(float* x, int64_t n, float s, void* stream) {
  if (n == 0) return 0;
  if (!x) return -1;
  scale_f32_kernel<<<grid_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, n, s);
  return finish();
}

static int swiglu_bwd_impl(const void* du, int64_t lddu, const void* gu, int64_t ldgu, void* dgu, int64_t lddgu,
                           int64_t rows, int64_t F, Q8Out q8, void* stream) {
  long long blocks = (rows * (F / 8) + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  auto* d16 = reinterpret_cast<__nv_bfloat16*>(dgu);
  auto* du16 = reinterpret_cast<const __nv_bfloat16*>(du);
  auto* gu16 = reinterpret_cast<const __nv_bfloat16*>(gu);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (q8.q) swiglu_bwd_kernel<true><<<(unsigned)blocks, 256, 0, s>>>(du16, lddu, gu16, ldgu, d16, lddgu, rows, (int)F, q8);
  else swiglu_bwd_kernel<false><<<(unsigned)blocks, 256, 0, s>>>(du16, lddu, gu16, ldgu, d16, lddgu, rows, (int)F, q8);
  return finish();
}

extern "C" int cdk_swiglu_bwd(const void* du, int64_t lddu, const void* gu, int64_t ldgu, void* dgu, int64_t lddgu,
                              int64_t rows, int64_t F, void* stream) {
  if (rows == 0) return 0;
  if (!du || !gu || !dgu || F % 8 || lddu % 8 || ldgu % 8 || lddgu % 8 || rows < 0) return -1;
  if ((reinterpret_cast<uintptr_t>(du) | reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(dgu)) & 15)
    return -2;
  Q8Out q8;
  q8.q = nullptr;
  q8.ldq = 0;
  q8.fmt = 0;
  q8.qscale = nullptr;
  q8.amax = nullptr;
  return swiglu_bwd_impl(du, lddu, gu, ldgu, dgu, lddgu, rows, F, q8, stream);
}

extern "C" int cdk_swiglu_bwd_q8(const void* du, int64_t lddu, const void* gu, int64_t ldgu, void* dgu8,
                                 int64_t lddgu8, int fmt, const float* qscale, float* amax, int64_t rows, int64_t F,
                                 void* stream) {
  if (rows == 0) return 0;
  if (!du || !gu || !dgu8 || !qscale || (fmt != 0 && fmt != 1) || F % 8 || lddu % 8 || ldgu % 8 || lddgu8 % 16 ||
      lddgu8 < 2 * F || rows < 0)
    return -1;
  if ((reinterpret_cast<uintptr_t>(du) | reinterpret_cast<uintptr_t>(gu) | reinterpret_cast<uintptr_t>(dgu8)) & 15)
    return -2;
  Q8Out q8;
  q8.q = reinterpret_cast<uint8_t*>(dgu8);
  q8.ldq = lddgu8;
  q8.fmt = fmt;
  q8.qscale = qscale;
  q8.amax = amax;
  return swiglu_bwd_impl(du, lddu, gu, ldgu, nullptr, 0, rows, F, q8, stream);
}

extern "C" int cdk_gemm_f32(const float* a, int64_t lda, int a_t, const float* b, int64_t ldb, int b_t, float* c,
                            int64_t ldc, int64_t M, int64_t N, int64_t K, const float* bias, int accumulate,
                            void* stream) {
  if (M == 0 || N == 0) return 0;
  if (!a || !b || !c || M < 0 || N < 0 || K < 0) return -1;
  if (M > (1 << 24) || N > (1 << 24)) return -2;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const long long tiles = ((N + 63) / 64) * ((M + 63) / 64);
  // split K until about two blocks per SM, keeping >= 64 of K per split
  long long splits = 1;
  while (tiles * splits * 2 <= 2 * 148 && K / (splits * 2) >= 64) splits *= 2;
  const int k_per = (int)(((K + splits - 1) / splits + 15) / 16 * 16);
  splits = K > 0 ? (K + k_per - 1) / k_per : 1;
  if (splits > 1 && !accumulate) {
    cudaError_t e = cudaMemset2DAsync(c, (size_t)ldc * sizeof(float), 0, (size_t)N * sizeof(float), (size_t)M, st);
    if (e != cudaSuccess) return (int)e;
  }
  dim3 grid((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64), (unsigned)splits);
  sgemm_kernel<<<grid, 256, 0, st>>>(a, lda, a_t, b, ldb, b_t, c, ldc, (int)M, (int)N, (int)K, bias, accumulate,
                                     k_per > 0 ? k_per : 16);
  return finish();
}
