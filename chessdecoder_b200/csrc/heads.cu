// Loss heads: softmax cross-entropy for the board / policy heads and the
// value-head tail (Mish -> Linear -> soft two-bucket cross-entropy).
//
// Board / policy (chessdecoder/train/train.py:180-207): per row
//     ce = logsumexp(logits) - logits[target]          (target -100 = ignored)
//     loss = sum_r w_r * ce_r * norm,   norm = 1 / (sum_r w_r + 1e-8)
// and the gradient written straight away as bf16 for the next GEMMs:
//     dlogits = (softmax - onehot(target)) * w_r * norm * loss_weight.
//
// Value heads (model.py:39-52, train.py:210-233, utils/training.py:24-50):
//     a = mish(z1); logits = a W2^T + b2; soft labels on the two buckets
//     around the target (linear interpolation); loss = -sum soft*log_softmax,
//     valid-masked mean.  The tail also produces dz1 for the first Linear.
#include "../../include/cdk.h"
#include "cdk_common.cuh"

namespace cdk {

// One warp per row.
__global__ void softmax_ce_kernel(const float* __restrict__ logits, long long ldl, long long rows, int ncls,
                                  const int32_t* __restrict__ target, const float* __restrict__ row_w,
                                  const float* __restrict__ norm, float loss_weight, __nv_bfloat16* __restrict__ dl,
                                  long long ldd, float* __restrict__ dbias, float* __restrict__ loss_out,
                                  int32_t* __restrict__ argmax_out) {
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* x = logits + r * ldl;
  float mx = -INFINITY;
  int amax = 0;
  for (int c = lane; c < ncls; c += 32) {
    const float v = x[c];
    if (v > mx) {
      mx = v;
      amax = c;
    }
  }
  // warp argmax, first index on ties
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o);
    const int oa = __shfl_xor_sync(0xffffffffu, amax, o);
    if (om > mx || (om == mx && oa < amax)) {
      mx = om;
      amax = oa;
    }
  }
  float se = 0.f;
  for (int c = lane; c < ncls; c += 32) se += __expf(x[c] - mx);
  se = warp_sum(se);
  const float lse = mx + __logf(se);
  const int tgt = target ? target[r] : -100;
  float w = row_w ? row_w[r] : 1.f;
  if (tgt < 0 || tgt >= ncls) w = 0.f;
  const float nrm = norm ? *norm : 1.f;
  const float coef = w * nrm * loss_weight;
  if (lane == 0) {
    if (argmax_out) argmax_out[r] = amax;
    if (loss_out && w != 0.f) atomicAdd(loss_out, w * (lse - x[tgt]) * nrm);
  }
  if (dl) {
    const float inv = 1.f / se;
    for (int c = lane; c < ncls; c += 32) {
      float g = __expf(x[c] - mx) * inv;
      if (c == tgt) g -= 1.f;
      g *= coef;
      dl[r * ldd + c] = __float2bfloat16_rn(g);
      if (dbias && coef != 0.f) atomicAdd(dbias + c, g);
    }
  }
}

// GRPO per-token policy loss on gathered action rows (one warp per row):
// lp = log_softmax(logits)[target]; with old / ref log-probs and the row's
// advantage A: r = exp(lp - old), r_ref = exp(lp - ref),
// loss = -min(r A, clamp(r, 1-eps_lo, 1+eps_hi) A) + beta ((r_ref - 1) - log(r_ref + 1e-8)),
// summed times *norm (1 / action tokens); dlogits = dloss/dlp * (onehot - softmax) * *norm.
// The gradient of min() is the reference's autograd one: r A where the
// unclipped term is the minimum (or both are equal inside the clip range), 0 where
// the clipped term is.
__global__ void grpo_token_kernel(const float* __restrict__ logits, long long ldl, long long rows, int ncls,
                                  const int32_t* __restrict__ target, const float* __restrict__ old_lp,
                                  const float* __restrict__ ref_lp, const float* __restrict__ adv,
                                  const float* __restrict__ norm, float eps_lo, float eps_hi, float beta,
                                  float* __restrict__ lp_out, __nv_bfloat16* __restrict__ dl, long long ldd,
                                  float* __restrict__ dbias, float* __restrict__ loss_out) {
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* x = logits + r * ldl;
  float mx = -INFINITY;
  for (int c = lane; c < ncls; c += 32) mx = fmaxf(mx, x[c]);
  mx = warp_max(mx);
  float se = 0.f;
  for (int c = lane; c < ncls; c += 32) se += __expf(x[c] - mx);
  se = warp_sum(se);
  const int tgt = target[r];
  const bool ok = tgt >= 0 && tgt < ncls;
  const float lp = ok ? x[tgt] - mx - __logf(se) : 0.f;
  if (lane == 0 && lp_out) lp_out[r] = lp;
  if (!old_lp) return;
  const float nrm = norm ? *norm : 1.f;
  const float A = adv[r];
  const float ratio = __expf(lp - old_lp[r]);
  const float s1 = ratio * A;
  const float rc = fminf(fmaxf(ratio, 1.f - eps_lo), 1.f + eps_hi);
  const float s2 = rc * A;
  const bool inside = ratio >= 1.f - eps_lo && ratio <= 1.f + eps_hi;
  const float rr = __expf(lp - ref_lp[r]);
  const float kl = (rr - 1.f) - __logf(rr + 1e-8f);
  const float g_obj = (s1 < s2 || (s1 == s2 && inside)) ? s1 : 0.f;
  const float dlp = ok ? (-g_obj + beta * (rr - rr / (rr + 1e-8f))) * nrm : 0.f;
  if (lane == 0 && loss_out && ok) atomicAdd(loss_out, (-fminf(s1, s2) + beta * kl) * nrm);
  if (dl) {
    const float inv = 1.f / se;
    for (int c = lane; c < ncls; c += 32) {
      float p = __expf(x[c] - mx) * inv;
      const float g = dlp * ((c == tgt ? 1.f : 0.f) - p);
      dl[r * ldd + c] = __float2bfloat16_rn(g);
      if (dbias && dlp != 0.f) atomicAdd(dbias + c, g);
    }
  }
}

__device__ __forceinline__ float softplus_t(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// One block (256 threads) per row; hidden <= 1024, nb <= 256.
__global__ void value_tail_kernel(const float* __restrict__ z1, long long rows, int hidden,
                                  const float* __restrict__ w2, const float* __restrict__ b2, int nb,
                                  const float* __restrict__ target, const float* __restrict__ valid,
                                  const float* __restrict__ centers, const float* __restrict__ norm, float loss_weight,
                                  float* __restrict__ act_out, float* __restrict__ dlogit_out,
                                  __nv_bfloat16* __restrict__ dz1, long long ldd, float* __restrict__ db1,
                                  float* __restrict__ loss_out, int32_t* __restrict__ argmax_out) {
  extern __shared__ float sm[];
  float* sa = sm;             // activations [hidden]
  float* sl = sm + hidden;    // logits / dlogits [nb]
  __shared__ float red[32];
  __shared__ int redi[32];
  const long long r = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const float* z = z1 + r * hidden;
  for (int i = tid; i < hidden; i += blockDim.x) {
    const float x = z[i];
    const float a = x * tanhf(softplus_t(x));
    sa[i] = a;
    if (act_out) act_out[r * hidden + i] = a;
  }
  __syncthreads();
  // logits: warp per output bucket
  for (int o = warp; o < nb; o += nw) {
    float acc = 0.f;
    for (int i = lane; i < hidden; i += 32) acc += sa[i] * w2[(long long)o * hidden + i];
    acc = warp_sum(acc);
    if (lane == 0) sl[o] = acc + (b2 ? b2[o] : 0.f);
  }
  __syncthreads();
  // max / argmax / sum-exp over nb (warp 0)
  if (warp == 0) {
    float mx = -INFINITY;
    int am = 0;
    for (int o = lane; o < nb; o += 32)
      if (sl[o] > mx) {
        mx = sl[o];
        am = o;
      }
    #pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, s);
      const int oa = __shfl_xor_sync(0xffffffffu, am, s);
      if (om > mx || (om == mx && oa < am)) {
        mx = om;
        am = oa;
      }
    }
    float se = 0.f;
    for (int o = lane; o < nb; o += 32) se += __expf(sl[o] - mx);
    se = warp_sum(se);
    if (lane == 0) {
      red[0] = mx;
      red[1] = __logf(se);
      redi[0] = am;
    }
  }
  __syncthreads();
  const float mx = red[0], lse = mx + red[1];
  // soft labels (two buckets around the target)
  const float t = target[r];
  const bool ok = valid ? valid[r] != 0.f : true;
  const float nrm = norm ? *norm : 1.f;
  int cnt = 0;
  for (int o = 0; o < nb; ++o) cnt += (t - centers[o] >= 0.f) ? 1 : 0;
  int lo = cnt - 1;
  lo = lo < 0 ? 0 : (lo > nb - 2 ? nb - 2 : lo);
  const int up = lo + 1;
  const float span = fmaxf(centers[up] - centers[lo], 1e-8f);
  const float wup = fminf(fmaxf((t - centers[lo]) / span, 0.f), 1.f);
  if (tid == 0) {
    if (argmax_out) argmax_out[r] = redi[0];
    if (loss_out && ok) {
      const float ll = -((1.f - wup) * (sl[lo] - lse) + wup * (sl[up] - lse));
      atomicAdd(loss_out, ll * nrm);
    }
  }
  __syncthreads();
  const float coef = ok ? nrm * loss_weight : 0.f;
  for (int o = tid; o < nb; o += blockDim.x) {
    float g = __expf(sl[o] - lse);
    if (o == lo) g -= 1.f - wup;
    if (o == up) g -= wup;
    g *= coef;
    if (dlogit_out) dlogit_out[r * nb + o] = g;
    sl[o] = g;
  }
  __syncthreads();
  // dz1 = (dlogits W2) * mish'(z1)
  for (int i = tid; i < hidden; i += blockDim.x) {
    float acc = 0.f;
    for (int o = 0; o < nb; ++o) acc += sl[o] * w2[(long long)o * hidden + i];
    const float x = z[i];
    const float sp = softplus_t(x);
    const float th = tanhf(sp);
    const float sg = 1.f / (1.f + __expf(-x));
    const float dm = th + x * (1.f - th * th) * sg;
    const float g = acc * dm;
    dz1[r * ldd + i] = __float2bfloat16_rn(g);
    if (db1 && coef != 0.f) atomicAdd(db1 + i, g);
  }
}

// Soft two-bucket cross-entropy on given logits (utils/training.py:24-50),
// one warp per row: lower = clamp(#{c <= t} - 1, 0, nb-2), upper = lower + 1,
// w_up = clamp((t - c_lo) / max(c_up - c_lo, 1e-8), 0, 1);
// loss += valid_r * -(sum soft * log_softmax) * norm;
// dlogits (f32, optional) = (softmax - soft) * valid_r * norm * loss_weight.
__global__ void soft_bucket_ce_kernel(const float* __restrict__ logits, long long ldl, long long rows, int nb,
                                      const float* __restrict__ target, const float* __restrict__ valid,
                                      const float* __restrict__ centers, const float* __restrict__ norm,
                                      float loss_weight, float* __restrict__ dl, long long ldd,
                                      float* __restrict__ loss_out) {
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* x = logits + r * ldl;
  const float t = target[r];
  float mx = -INFINITY;
  int cnt = 0;
  for (int c = lane; c < nb; c += 32) {
    mx = fmaxf(mx, x[c]);
    cnt += (t - centers[c] >= 0.f) ? 1 : 0;
  }
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  }
  float se = 0.f;
  for (int c = lane; c < nb; c += 32) se += __expf(x[c] - mx);
  se = warp_sum(se);
  const float lse = mx + __logf(se);
  int lo = cnt - 1;
  lo = lo < 0 ? 0 : (lo > nb - 2 ? nb - 2 : lo);
  const int up = lo + 1;
  const float span = fmaxf(centers[up] - centers[lo], 1e-8f);
  const float wup = fminf(fmaxf((t - centers[lo]) / span, 0.f), 1.f);
  const float vw = valid ? valid[r] : 1.f;
  const float nrm = norm ? *norm : 1.f;
  if (lane == 0 && loss_out && vw != 0.f) {
    const float ll = -((1.f - wup) * (x[lo] - lse) + wup * (x[up] - lse));
    atomicAdd(loss_out, ll * vw * nrm);
  }
  if (dl) {
    const float coef = vw * nrm * loss_weight;
    const float inv = 1.f / se;
    for (int c = lane; c < nb; c += 32) {
      float g = __expf(x[c] - mx) * inv;
      if (c == lo) g -= 1.f - wup;
      if (c == up) g -= wup;
      dl[r * ldd + c] = g * coef;
    }
  }
}

}  // namespace cdk

using namespace cdk;

extern "C" int cdk_softmax_ce(const float* logits, int64_t ldl, int64_t rows, int64_t ncls, const int32_t* target,
                              const float* row_weight, const float* norm, float loss_weight, void* dlogits_bf16,
                              int64_t ldd, float* dbias, float* loss_out, int32_t* argmax_out, void* stream) {
  if (rows == 0) return 0;
  if (!logits || rows < 0 || ncls <= 0 || ldl < ncls) return -1;
  if (dlogits_bf16 && ldd < ncls) return -2;
  softmax_ce_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ldl, rows, (int)ncls, target, row_weight, norm, loss_weight,
      reinterpret_cast<__nv_bfloat16*>(dlogits_bf16), ldd, dbias, loss_out, argmax_out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_value_tail(const float* z1, int64_t rows, int64_t hidden, const float* w2, const float* b2,
                              int64_t nb, const float* target, const float* valid, const float* centers,
                              const float* norm, float loss_weight, float* act_out, float* dlogits_out,
                              void* dz1_bf16, int64_t ldd, float* db1, float* loss_out, int32_t* argmax_out,
                              void* stream) {
  if (rows == 0) return 0;
  if (!z1 || !w2 || !target || !centers || !dz1_bf16 || hidden <= 0 || hidden > 4096 || nb < 2 || nb > 1024 ||
      ldd < hidden)
    return -1;
  const size_t smem = (size_t)(hidden + nb) * sizeof(float);
  value_tail_kernel<<<(unsigned)rows, 256, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      z1, rows, (int)hidden, w2, b2, (int)nb, target, valid, centers, norm, loss_weight, act_out, dlogits_out,
      reinterpret_cast<__nv_bfloat16*>(dz1_bf16), ldd, db1, loss_out, argmax_out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_soft_bucket_ce(const float* logits, int64_t ldl, int64_t rows, int64_t nb, const float* target,
                                  const float* valid, const float* centers, const float* norm, float loss_weight,
                                  float* dlogits, int64_t ldd, float* loss_out, void* stream) {
  if (rows == 0) return 0;
  if (!logits || !target || !centers || rows < 0 || nb < 2 || ldl < nb) return -1;
  if (dlogits && ldd < nb) return -2;
  soft_bucket_ce_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ldl, rows, (int)nb, target, valid, centers, norm, loss_weight, dlogits, ldd, loss_out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int cdk_grpo_token(const float* logits, int64_t ldl, int64_t rows, int64_t ncls, const int32_t* target,
                              const float* old_lp, const float* ref_lp, const float* adv, const float* norm,
                              float eps_low, float eps_high, float kl_coeff, float* lp_out, void* dlogits_bf16,
                              int64_t ldd, float* dbias, float* loss_out, void* stream) {
  if (rows == 0) return 0;
  if (!logits || !target || rows < 0 || ncls <= 0 || ldl < ncls) return -1;
  if (old_lp && (!ref_lp || !adv)) return -2;
  if (dlogits_bf16 && (!old_lp || ldd < ncls)) return -3;
  grpo_token_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ldl, rows, (int)ncls, target, old_lp, ref_lp, adv, norm, eps_low, eps_high, kl_coeff, lp_out,
      reinterpret_cast<__nv_bfloat16*>(dlogits_bf16), ldd, dbias, loss_out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : (int)e;
}
