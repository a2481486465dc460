// Global-norm gradient clipping fused into AdamW, over one flat fp32 buffer.
//
// Reference: chessdecoder/train/train.py:64-68 (torch.optim.AdamW(lr, wd),
// betas (0.9, 0.999), eps 1e-8) and :248-253 (average_gradients ->
// clip_grad_norm_(max_norm=10) -> optimizer.step).  The per-rank gradient mean
// of chessdecoder/utils/distributed.py:55-67 is folded in as `grad_scale`
// (1/world_size) so that no separate division pass is needed:
//     total_norm = sqrt(sum g^2) * grad_scale
//     coef       = min(1, max_norm / (total_norm + 1e-6))
//     g'         = g * grad_scale * coef
//     p         *= 1 - lr*wd
//     m          = m + (1-b1) (g' - m)            (torch's lerp form)
//     v          = b2 v + (1-b2) g'^2
//     p         -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
// The kernel also writes the bf16 shadow copy of the updated parameters that
// the GEMMs consume, so no separate cast pass over the weights is needed.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

#include <mutex>

namespace cdk {

__global__ void sumsq_kernel(const float* __restrict__ x, long long n, float* __restrict__ partial) {
  __shared__ float red[32];
  float acc = 0.f;
  const long long n4 = n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = x4[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long long i = n4 * 4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    acc += x[i] * x[i];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}

struct AdamHyper {
  float lr, b1, b2, eps, wd, step_size, inv_bc2_sqrt, max_norm, grad_scale;
};

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ pb, long long n,
                             const float* __restrict__ partial, int n_partial, const AdamHyper h) {
  __shared__ float s_coef;
  if (threadIdx.x < 32) {
    float acc = 0.f;
    if (partial)
      for (int i = threadIdx.x; i < n_partial; i += 32) acc += partial[i];
    acc = warp_sum(acc);
    if (threadIdx.x == 0) {
      float coef = 1.f;
      if (partial && h.max_norm > 0.f) {
        const float total = sqrtf(acc) * h.grad_scale;
        coef = fminf(1.f, h.max_norm / (total + 1e-6f));
      }
      s_coef = coef * h.grad_scale;
    }
  }
  __syncthreads();
  const float gs = s_coef;
  const float decay = 1.f - h.lr * h.wd;
  const long long n4 = n / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pa = &pp.x;
    const float* ga = &gg.x;
    float* ma = &mm.x;
    float* va = &vv.x;
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = ga[j] * gs;
      pa[j] *= decay;
      ma[j] = fmaf(1.f - h.b1, gj - ma[j], ma[j]);
      va[j] = fmaf(h.b2, va[j], (1.f - h.b2) * gj * gj);
      const float denom = sqrtf(va[j]) * h.inv_bc2_sqrt + h.eps;
      pa[j] -= h.step_size * ma[j] / denom;
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (pb) {
      uint2 w;
      w.x = pack_bf16(pp.x, pp.y);
      w.y = pack_bf16(pp.z, pp.w);
      reinterpret_cast<uint2*>(pb)[i] = w;
    }
  }
  for (long long i = n4 * 4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float gj = g[i] * gs;
    float pj = p[i] * decay;
    const float mj = fmaf(1.f - h.b1, gj - m[i], m[i]);
    const float vj = fmaf(h.b2, v[i], (1.f - h.b2) * gj * gj);
    pj -= h.step_size * mj / (sqrtf(vj) * h.inv_bc2_sqrt + h.eps);
    p[i] = pj;
    m[i] = mj;
    v[i] = vj;
    if (pb) pb[i] = __float2bfloat16_rn(pj);
  }
}

}  // namespace cdk

using namespace cdk;

// ---------------------------------------------------------------------------
// Allocation-free variant of the clip + AdamW step.
//
// cdk_sumsq + cdk_adamw need a caller-provided scratch buffer for the
// per-block partial sums of the gradient norm.  Some callers cannot provide
// one: they hold only the parameter / gradient / moment buffers and have no
// way to get more device memory -- a host runtime that passes raw device
// pointers but has no CUDA allocator of its own, or a training loop running
// inside a fixed, fully pre-reserved memory pool where a new allocation would
// fail.  For them the partial sums live in the array below, which is part of
// the library image: every GPU that loads libcdk.so holds these 16 KB until
// the process exits.
//
// The array is shared by every call on a device and keeps the last call's
// contents; each call overwrites exactly the entries it then reads, so
// nothing has to be cleared first.  Calls whose kernels overlap on the GPU
// (issued on different streams of one device) race on the array: issue them
// one after another.
// ---------------------------------------------------------------------------
namespace cdk {

constexpr int kNoAllocMaxPartial = 4096;
static __device__ __align__(256) float g_noalloc_partial[kNoAllocMaxPartial];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_partial on the current device.  In host code
// the symbol names a host-side stand-in, not device memory, so the address is
// looked up once per device (with that device current) and cached.  This
// lookup happens inside the first call on each device, so that first call
// should be made before any stream capture begins.
static int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= 64) return -30;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_partial);
    if (e != cudaSuccess || ptr == nullptr) return e != cudaSuccess ? (int)e : -31;
    g_noalloc_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace cdk

extern "C" int cdk_adamw_clip_noalloc(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n,
                                      int64_t n_partial, float max_norm, float lr, float beta1, float beta2,
                                      float eps, float wd, int64_t step, float grad_scale, void* stream) {
  using namespace cdk;
  if (n_partial <= 0 || n_partial > kNoAllocMaxPartial) return -32;  // scratch holds at most 4096 partial sums
  if (n == 0) return 0;
  if (!p || !g || !m || !v || n < 0 || step < 1) return -1;
  if (((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
        reinterpret_cast<uintptr_t>(v)) & 15) ||
      (p_bf16 && (reinterpret_cast<uintptr_t>(p_bf16) & 7)))
    return -2;
  float* partial = nullptr;
  int rc = noalloc_scratch(&partial);
  if (rc != 0) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  sumsq_kernel<<<(unsigned)n_partial, 512, 0, s>>>(g, n, partial);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  return cdk_adamw(p, g, m, v, p_bf16, n, partial, n_partial, max_norm, lr, beta1, beta2, eps, wd, step, grad_scale,
                   stream);
}

extern "C" int cdk_sumsq(const float* x, int64_t n, float* partial, int64_t n_partial, void* stream) {
  if (!x || !partial || n < 0 || n_partial <= 0 || n_partial > 4096) return -1;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return -2;
  sumsq_kernel<<<(unsigned)n_partial, 512, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, n, partial);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_adamw(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n, const float* partial,
                         int64_t n_partial, float max_norm, float lr, float beta1, float beta2, float eps, float wd,
                         int64_t step, float grad_scale, void* stream) {
  if (n == 0) return 0;
  if (!p || !g || !m || !v || n < 0 || step < 1) return -1;
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
       reinterpret_cast<uintptr_t>(v)) & 15)
    return -2;
  if (p_bf16 && (reinterpret_cast<uintptr_t>(p_bf16) & 7)) return -2;
  AdamHyper h;
  h.lr = lr;
  h.b1 = beta1;
  h.b2 = beta2;
  h.eps = eps;
  h.wd = wd;
  const double bc1 = 1.0 - pow((double)beta1, (double)step);
  const double bc2 = 1.0 - pow((double)beta2, (double)step);
  h.step_size = (float)(lr / bc1);
  h.inv_bc2_sqrt = (float)(1.0 / sqrt(bc2));
  h.max_norm = max_norm;
  h.grad_scale = grad_scale;
  // SM count per device, looked up on the first call on that device
  static int sm_count[64] = {0};
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    if (sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (sm_count[dev] > 0) sms = sm_count[dev];
  }
  long long blocks = (n / 4 + 255) / 256;
  if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
  if (blocks < 1) blocks = 1;
  adamw_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      p, g, m, v, reinterpret_cast<__nv_bfloat16*>(p_bf16), n, partial, (int)n_partial, h);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}
