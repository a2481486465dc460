// Token embedding with Fourier value injection at the WL/D placeholder rows.
//
// Reference: chessdecoder/models/model.py:174-180 (h = tok_embedding(x); rows at
// wl_positions / d_positions are overwritten by FourierEncoder(value)),
// FourierEncoder at model.py:24-36 ([cos(2*pi*x*f), sin(2*pi*x*f)] -> Linear),
// and the bucket snapping of chessdecoder/utils/training.py:114-133 with
// ChessDecoder.discretize_to_bucket (model.py:189-194): the Fourier input is
// the bucket centre nearest to the target (first index on ties, like argmin).
//
// The projection Linear(2F -> E) runs as a small fp32 GEMM between
// cdk_fourier_features and cdk_embed_fwd; the embedding kernels gather / scatter
// whole 128-bit rows, one warp per token.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {

constexpr float kTwoPi = 6.283185307179586f;

__device__ __forceinline__ float snap_to_bucket(float v, const float* __restrict__ c, int n) {
  int best = 0;
  float bd = fabsf(v - c[0]);
  for (int i = 1; i < n; ++i) {
    const float d = fabsf(v - c[i]);
    if (d < bd) {
      bd = d;
      best = i;
    }
  }
  return c[best];
}

// One block per placeholder row.  values_out[k] = snapped value; feat_out[k] = [cos | sin].
__global__ void fourier_features_kernel(const float* __restrict__ wl_t, const float* __restrict__ d_t,
                                        const uint8_t* __restrict__ wl_pos, const uint8_t* __restrict__ d_pos,
                                        const float* __restrict__ wl_c, const float* __restrict__ d_c, int nb,
                                        const float* __restrict__ freqs, int nf, const int32_t* __restrict__ rows,
                                        float* __restrict__ values_out, float* __restrict__ feat) {
  __shared__ float sval;
  const long long k = blockIdx.x;
  const int t = rows[k];
  if (threadIdx.x == 0) {
    // d positions take precedence, matching the reference's overwrite order.
    // nb == 0: the values are used as given (the model forward of
    // model.py:177-180, whose inputs were snapped by the caller).
    float v = 0.f;
    if (d_pos[t]) v = nb > 0 ? snap_to_bucket(d_t[t], d_c, nb) : d_t[t];
    else if (wl_pos[t]) v = nb > 0 ? snap_to_bucket(wl_t[t], wl_c, nb) : wl_t[t];
    sval = v;
    values_out[k] = v;
  }
  __syncthreads();
  const float v = sval;
  for (int j = threadIdx.x; j < nf; j += blockDim.x) {
    const float a = kTwoPi * v * freqs[j];
    float s, c;
    sincosf(a, &s, &c);
    feat[k * 2 * nf + j] = c;
    feat[k * 2 * nf + nf + j] = s;
  }
}

// out[c * n_tok + t] = slot[t] >= 0 ? fourier_rows[slot[t]] : emb[ids[t]]  for c < n_copies.
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, long long n_tok, long long vocab,
                                 const float* __restrict__ emb, int dim4, const int32_t* __restrict__ slot,
                                 const float* __restrict__ frows, float* __restrict__ out, int n_copies) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= n_tok) return;
  const int sl = slot ? slot[t] : -1;
  const float4* src;
  bool zero = false;
  if (sl >= 0) {
    src = reinterpret_cast<const float4*>(frows) + (long long)sl * dim4;
  } else {
    long long id = ids[t];
    if (id < 0 || id >= vocab) {
      if (lane == 0) report_error(kErrIndex);
      zero = true;
      id = 0;
    }
    src = reinterpret_cast<const float4*>(emb) + id * dim4;
  }
  for (int i = lane; i < dim4; i += 32) {
    float4 v = zero ? make_float4(0.f, 0.f, 0.f, 0.f) : src[i];
    for (int c = 0; c < n_copies; ++c) reinterpret_cast<float4*>(out)[((long long)c * n_tok + t) * dim4 + i] = v;
  }
}

// demb[ids[t]] += sum_c dh[c*n_tok + t] (non-placeholder rows);
// dfrows[slot[t]] = sum_c dh[c*n_tok + t] (placeholder rows).
__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, long long n_tok, long long vocab,
                                 const float* __restrict__ dh, int dim4, int n_copies,
                                 const int32_t* __restrict__ slot, float* __restrict__ demb,
                                 float* __restrict__ dfrows) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= n_tok) return;
  const int sl = slot ? slot[t] : -1;
  const long long id = ids[t];
  if (sl < 0 && (id < 0 || id >= vocab)) {
    if (lane == 0) report_error(kErrIndex);
    return;
  }
  for (int i = lane; i < dim4; i += 32) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < n_copies; ++c) {
      const float4 v = reinterpret_cast<const float4*>(dh)[((long long)c * n_tok + t) * dim4 + i];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    if (sl >= 0) reinterpret_cast<float4*>(dfrows)[(long long)sl * dim4 + i] = s;
    else atomicAdd(reinterpret_cast<float4*>(demb) + id * dim4 + i, s);
  }
}

// dfreq[j] += sum_k 2*pi*x_k * (-dcos[k,j] * sin(a) + dsin[k,j] * cos(a)),  a = 2*pi*x_k*f_j
__global__ void fourier_bwd_kernel(const float* __restrict__ values, const float* __restrict__ freqs, int nf,
                                   const float* __restrict__ dfeat, long long n_rows, float* __restrict__ dfreq) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= nf) return;
  const float f = freqs[j];
  float acc = 0.f;
  for (long long k = blockIdx.y; k < n_rows; k += gridDim.y) {
    const float x = values[k];
    const float a = kTwoPi * x * f;
    float s, c;
    sincosf(a, &s, &c);
    acc += kTwoPi * x * (-dfeat[k * 2 * nf + j] * s + dfeat[k * 2 * nf + nf + j] * c);
  }
  atomicAdd(dfreq + j, acc);
}

}  // namespace cdk

using namespace cdk;

extern "C" int cdk_fourier_features(const float* wl_t, const float* d_t, const uint8_t* wl_pos, const uint8_t* d_pos,
                                    const float* wl_centers, const float* d_centers, int32_t n_buckets,
                                    const float* freqs, int32_t n_freq, const int32_t* rows, int64_t n_rows,
                                    float* values_out, float* feat_out, void* stream) {
  if (n_rows == 0) return 0;
  if (!wl_t || !d_t || !wl_pos || !d_pos || !freqs || !rows || !values_out || !feat_out || n_buckets < 0 ||
      n_freq <= 0 || n_rows < 0)
    return -1;
  if (n_buckets > 0 && (!wl_centers || !d_centers)) return -1;
  fourier_features_kernel<<<(unsigned)n_rows, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      wl_t, d_t, wl_pos, d_pos, wl_centers, d_centers, n_buckets, freqs, n_freq, rows, values_out, feat_out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_embed_fwd(const int64_t* ids, int64_t n_tok, int64_t vocab, const float* emb, int64_t dim,
                             const int32_t* slot, const float* fourier_rows, float* out, int64_t n_copies,
                             void* stream) {
  if (n_tok == 0) return 0;
  if (!ids || !emb || !out || dim % 4 || n_copies < 1 || n_tok < 0) return -1;
  if (slot && !fourier_rows) return -2;
  const unsigned blocks = (unsigned)((n_tok + 7) / 8);
  embed_fwd_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ids, n_tok, vocab, emb, (int)(dim / 4),
                                                                               slot, fourier_rows, out, (int)n_copies);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_embed_bwd(const int64_t* ids, int64_t n_tok, int64_t vocab, const float* dh, int64_t dim,
                             int64_t n_copies, const int32_t* slot, float* demb, float* dfourier_rows, void* stream) {
  if (n_tok == 0) return 0;
  if (!ids || !dh || !demb || dim % 4 || n_copies < 1) return -1;
  if (slot && !dfourier_rows) return -2;
  const unsigned blocks = (unsigned)((n_tok + 7) / 8);
  embed_bwd_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ids, n_tok, vocab, dh, (int)(dim / 4),
                                                                               (int)n_copies, slot, demb,
                                                                               dfourier_rows);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_fourier_bwd(const float* values, const float* freqs, int32_t n_freq, const float* dfeat,
                               int64_t n_rows, float* dfreqs, void* stream) {
  if (n_rows == 0) return 0;
  if (!values || !freqs || !dfeat || !dfreqs || n_freq <= 0) return -1;
  dim3 grid((unsigned)((n_freq + 127) / 128), (unsigned)(n_rows < 64 ? n_rows : 64));
  fourier_bwd_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(values, freqs, n_freq, dfeat, n_rows,
                                                                               dfreqs);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}
