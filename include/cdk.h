/*
 * cdk.h — C ABI of the chessdecoder_b200 kernel library (libcdk.so, sm_100a).
 *
 * Every entry point takes raw device pointers, int64 sizes/leading dimensions
 * and a cudaStream_t (passed as void*).  The library never allocates or frees
 * device memory and keeps no pointer past the call: the caller (PyTorch's
 * caching allocator on the Python side) owns every buffer, including scratch.
 *
 * Return value: 0 = launched; < 0 = rejected on the host before launch
 * (shape, alignment, unsupported combination); > 0 = CUDA error code from the
 * launch.  Device-side conditions (a bounded wait that timed out, an index out
 * of range) are latched in a device word read by cdk_get_error().
 *
 * The reference implements this step as PyTorch eager code on torchtune
 * modules; each group below names the reference code it replaces
 * (paths relative to the ChessDecoder repository).
 */
#ifndef CDK_H_
#define CDK_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ------------------------------------------------------------ */
int cdk_version(void);
/* Reads (and, if clear != 0, clears) the device error word of the current
 * device.  Synchronises the current device. */
int cdk_get_error(int* out_flags, int clear);

/* ---- dense contractions (tcgen05 + TMEM + TMA) ---------------------------
 * Replaces the nn.Linear calls of chessdecoder/models/model.py:96-108
 * (q/k/v/output projections, SwiGLU gate/up/down) and their autograd
 * backward, the heads at model.py:119-122 and ValueHead (model.py:39-52).
 *
 *   D[M,N] (op)= sum_k A[m,k] * B[n,k]
 *   A: a_mn == 0 -> row-major [M,K] (K contiguous), pitch lda
 *      a_mn == 1 -> row-major [K,M] (M contiguous), pitch lda
 *   B: b_mn == 0 -> row-major [N,K], pitch ldb;  b_mn == 1 -> row-major [K,N]
 * Inputs bf16, accumulation fp32, output per epilogue kind.
 */
enum {
  CDK_EPI_STORE_BF16 = 0, /* out bf16 = acc (+bias)                               */
  CDK_EPI_STORE_F32 = 1,  /* out f32  = acc (+bias)                               */
  CDK_EPI_RESID_F32 = 2,  /* out f32  = resid + acc (+bias); out may alias resid  */
  CDK_EPI_ROPE_BF16 = 3,  /* out bf16 = rope(acc) on cols < rope_cols, pos = row % seq_len */
  CDK_EPI_SWIGLU = 4,     /* B = [gate; up] (2*half_n rows, K-major); out = silu(g)*u bf16,
                             out2 = [g | u] bf16 (up at column offset half_n)      */
  CDK_EPI_DSWIGLU = 5,    /* acc = d(silu(g)*u); aux = [g | u] bf16; out = [dg | du] bf16 */
  CDK_EPI_ATOMIC_F32 = 6, /* out f32 += acc with atomics (split-K allowed)          */
  CDK_EPI_ACCUM_F32 = 7   /* out f32 += acc (plain read-modify-write, no split-K)   */
};

typedef struct CdkGemmEpilogue {
  int32_t kind;
  int32_t seq_len;   /* ROPE: rows are (sequence, position) with position = row % seq_len */
  int32_t rope_cols; /* ROPE: columns [0, rope_cols) are rotated in interleaved pairs     */
  int32_t reserved;
  void* out;
  int64_t ldo;
  const float* bias; /* optional per-column bias [N]                                     */
  const float* resid;
  int64_t ldr;
  void* out2;
  int64_t ldo2;
  const void* aux;
  int64_t ldaux;
  int64_t half_n;    /* SWIGLU / DSWIGLU: column offset of the "up" half                 */
  const float* rope; /* ROPE: table [seq_len][32][2] = (cos, sin) per position and pair  */
} CdkGemmEpilogue;

/* split_k: 0 = automatic (ATOMIC_F32 only), 1 = none, >1 = forced (ATOMIC_F32 only). */
int cdk_gemm_bf16(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, int64_t M, int64_t N,
                  int64_t K, const CdkGemmEpilogue* epi, int split_k, void* stream);
/* cdk_gemm_pair_clusters: clusters of two CTAs that the CTA-pair GEMM form
 * (M = 256 MMAs over two SMs) keeps resident on the current device, or 0 when
 * that form is off (environment CDK_GEMM_PAIR=0) or unavailable.  The pair
 * form serves GEMMs with M a multiple of 256: bf16 and 8-bit with K-major A
 * (ROPE_BF16, STORE_BF16, SWIGLU, RESID_F32; DSWIGLU and STORE_BF16 with B
 * MN-major; ATOMIC_F32 with K-major B), and bf16 ATOMIC_F32 with both operands
 * MN-major (split-K chosen for the pairs).  Results equal the one-CTA form's
 * bit for bit, except the split-K sums, whose order follows the split. */
int cdk_gemm_pair_clusters(void);

/* ---- fp8 (the fp8 training variant: e4m3 weights / activations, e5m2
 *      gradients, per-tensor delayed scaling; no counterpart in the reference,
 *      whose GEMMs run through torch.autocast fp16) ----------------------------
 * cdk_gemm_fp8: C = epilogue((A B^T) * (*scale_inv_a) * (*scale_inv_b)) with
 * 8-bit A and B laid out as in cdk_gemm_bf16 (a_mn / b_mn: MN-major; row
 * pitch lda / ldb in bytes, a multiple of 16); a_fmt /
 * b_fmt: 0 = e4m3, 1 = e5m2 (they may differ).  Same epilogue kinds and
 * split-K rules as cdk_gemm_bf16. */
int cdk_gemm_fp8(const void* a, int64_t lda, int a_mn, int a_fmt, const void* b, int64_t ldb, int b_mn, int b_fmt,
                 int64_t M, int64_t N, int64_t K, const float* scale_inv_a, const float* scale_inv_b,
                 const CdkGemmEpilogue* epi, int split_k, void* stream);
/* cdk_fp8_cast: out[r, c] = sat_fmt(x[r, c] * (*scale)) (round to nearest even,
 * saturating to the format's largest finite value); out_t (optional) [cols,
 * rows] receives the transpose (row pitch ldt bytes); amax (optional) is
 * raised to max |x| (atomic, non-negative float bits).  x_dtype: 0 = f32,
 * 1 = bf16; ldx in elements, ldo / ldt in bytes. */
int cdk_fp8_cast(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx, const float* scale, int fmt,
                 void* out, int64_t ldo, void* out_t, int64_t ldt, float* amax, void* stream);
/* cdk_fp8_amax: *amax = max(*amax, max |x|). */
int cdk_fp8_amax(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx, float* amax, void* stream);
/* cdk_fp8_scales: per-tensor delayed scaling for n tensors.  mode 0 (end of a
 * step): history[i] shifts by one and takes amax_cur[i] in slot 0, then
 * scale[i] = fmax[i] / max(history[i]) (1 when that max is 0), scale_inv[i] =
 * 1 / scale[i], amax_cur[i] = 0.  mode 1 (first use, empty history): scale
 * from amax_cur[i] alone, history untouched. */
int cdk_fp8_scales(float* amax_cur, float* history, float* scale, float* scale_inv, const float* fmax, int32_t n,
                   int32_t hist_len, int32_t mode, void* stream);

/* ---- mixture of experts (the MoE variant: X experts, top-2 routing,
 *      capacity-limited; no counterpart in the reference, whose MLP is one
 *      dense SwiGLU per layer, chessdecoder/models/model.py:104-108) ---------
 * cdk_moe_route: from router logits [T, X] (fp32): probs = softmax [T, X],
 * expert / weight [T, 2] = top-2 (lower index on ties) with weights
 * renormalised over the two; then, inside each of n_seg equal token segments,
 * every expert gets `cap` slots filled by the first choices in token order and
 * then the second choices in token order; slot [T, 2] = row of the
 * expert-major buffers (e * n_seg * cap + seg * cap + position) or -1 when the
 * expert was full; src [X * n_seg * cap] = token of each row or -1.
 * workspace: cdk_moe_route_workspace(T, n_seg, X) bytes. */
int64_t cdk_moe_route_workspace(int64_t T, int32_t n_seg, int32_t X);
int cdk_moe_route(const float* logits, int64_t T, int32_t X, int32_t n_seg, int64_t cap, int32_t* expert,
                  float* weight, float* probs, int32_t* slot, int32_t* src, void* workspace, void* stream);
/* xe[r] = x[src[r]] (bf16 rows, zero when src[r] < 0). */
int cdk_moe_dispatch(const void* x, int64_t ldx, const int32_t* src, int64_t rows, int64_t dim, void* xe,
                     void* stream);
/* out[t] = resid[t] + sum_k weight[t,k] * ye[slot[t,k]] (ye bf16, out / resid fp32; dropped slots skipped). */
int cdk_moe_combine(const void* ye, const int32_t* slot, const float* weight, const float* resid, float* out,
                    int64_t T, int64_t dim, void* stream);
/* dye (bf16, dye_rows rows, zeroed first)[slot[t,k]] = weight[t,k] * dout[t];
 * dweight[t,k] = dout[t] . ye[slot[t,k]] (0 when dropped). */
int cdk_moe_combine_bwd(const float* dout, const void* ye, const int32_t* slot, const float* weight, void* dye,
                        int64_t dye_rows, float* dweight, int64_t T, int64_t dim, void* stream);
/* dlogits (bf16 [T, ldd], ldd in [X, 32]) = d(loss)/d(router logits) through the
 * renormalised top-2 weights and the softmax. */
int cdk_moe_route_bwd(const float* probs, const int32_t* expert, const float* dweight, int64_t T, int32_t X,
                      void* dlogits, int64_t ldd, void* stream);
/* out[t] (accumulate ? += : =) sum_k dxe[slot[t,k]] (dxe bf16, out fp32). */
int cdk_moe_gather_sum(const void* dxe, const int32_t* slot, float* out, int64_t T, int64_t dim, int accumulate,
                       void* stream);

/* ---- attention -----------------------------------------------------------
 * Replaces torchtune MultiHeadAttention's SDPA call as used by
 * chessdecoder/models/model.py:158-171 (pass 1: is_causal; pass 2: bool mask
 * tril | block_id[i]==block_id[j]).  head_dim is fixed at 64.
 *
 * qkv: bf16 [nseq*S, 3*E] rows = tokens, columns [q | k | v], heads of 64.
 * Sequences [0, n_causal) use the causal mask; sequences [n_causal, nseq) use
 * the prefix mask with block ids bid[(s - n_causal)*S + i] (int32).
 * meta: int32 workspace from cdk_attn_prefix_meta (NULL if n_causal == nseq).
 */
int cdk_attn_prefix_meta(const int32_t* bid, int64_t nseq_prefix, int64_t S, int32_t* meta, void* stream);
int64_t cdk_attn_meta_elems(int64_t nseq_prefix, int64_t S);
int cdk_attn_fwd(const void* qkv, void* out, float* lse, int64_t nseq, int64_t n_causal, int64_t S, int64_t H,
                 const int32_t* bid, const int32_t* meta, void* stream);
/* Backward.  dqkv receives [dq | dk | dv] for the pre-RoPE q/k (the inverse
 * rotation with table `rope` [S][32][2] is applied in the epilogue; rope may
 * be NULL when q/k were not rotated).  dsum: f32 scratch [nseq*H*S]. */
int cdk_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum, void* dqkv,
                 int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid, const int32_t* meta,
                 const float* rope, void* stream);
/* cdk_attn_bwd_ws: cdk_attn_bwd with a caller workspace; for S > 256 the
 * tcgen05 backward accumulates dQ in fp32 there (cdk_attn_bwd_workspace bytes,
 * 16-byte aligned; 0 bytes for S <= 256) and writes D = rowsum(dO * O) into
 * dsum.  Without a workspace, or when S is not a multiple of 4, S > 256 takes
 * the mma.sync tiled kernels. */
int64_t cdk_attn_bwd_workspace(int64_t nseq, int64_t S, int64_t H);
int cdk_attn_bwd_ws(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum, void* dqkv,
                    int64_t nseq, int64_t n_causal, int64_t S, int64_t H, const int32_t* bid, const int32_t* meta,
                    const float* rope, void* workspace, int64_t workspace_bytes, void* stream);
/* cdk_attn_bwd_q8: the backward with dq|dk|dv written as 8-bit values
 * (fp8 recipe, see cdk_rmsnorm_fwd_q8): dqkv8 [nseq*S, 3*H*64] with row pitch
 * ld8 bytes, saturate(v * (*qscale)) in e4m3 (fmt 0) / e5m2 (fmt 1), amax =
 * max(amax, max |v|).  S <= 256 on the default kernel path only; returns -20
 * otherwise (the caller then uses cdk_attn_bwd_ws and a separate cast). */
int cdk_attn_bwd_q8(const void* qkv, const void* out, const void* dout, const float* lse, float* dsum, void* dqkv8,
                    int64_t ld8, int fmt, const float* qscale, float* amax, int64_t nseq, int64_t n_causal, int64_t S,
                    int64_t H, const int32_t* bid, const int32_t* meta, const float* rope, void* stream);

/* ---- RMSNorm (torchtune RMSNorm, eps 1e-6; reference restatement at
 *      chessdecoder/export/backbone_causal.py:61-64) ------------------------ */
int cdk_rmsnorm_fwd(const float* x, const float* scale, void* y_bf16, float* y_f32, float* rstd, int64_t rows,
                    int64_t dim, float eps, void* stream);
/* dx = dres + rmsnorm'(dy); dx_bf16 optional; dscale accumulated (+=).  dy bf16 or f32 (dy_is_f32). */
int cdk_rmsnorm_bwd(const void* dy, int dy_is_f32, const float* x, const float* scale, const float* rstd,
                    const float* dres, float* dx, void* dx_bf16, float* dscale, int64_t rows, int64_t dim,
                    void* stream);
/* The fp8 recipe's casts fused into the norms: the normalised output (forward)
 * or dx (backward) written as 8-bit q = saturate(v * (*qscale)) in e4m3 (fmt 0)
 * or e5m2 (fmt 1) with row pitch ldq bytes (a multiple of 16, 16-byte aligned
 * base) in place of the bf16 copy, and amax = max(amax, max |v|) (amax may be
 * null).  dim a multiple of 256.  The recipe (per-tensor delayed scaling) has
 * no counterpart in the reference, whose linears run under torch.autocast fp16
 * (chessdecoder/train/train.py:168). */
int cdk_rmsnorm_fwd_q8(const float* x, const float* scale, void* y8, int64_t ldy8, int fmt, const float* qscale,
                       float* amax, float* rstd, int64_t rows, int64_t dim, float eps, void* stream);
int cdk_rmsnorm_bwd_q8(const void* dy, int dy_is_f32, const float* x, const float* scale, const float* rstd,
                       const float* dres, float* dx, void* dx8, int64_t ldx8, int fmt, const float* qscale,
                       float* amax, float* dscale, int64_t rows, int64_t dim, void* stream);

/* ---- embedding + Fourier value injection (model.py:24-36, 174-180) and the
 *      bucket snapping of utils/training.py:114-133 / model.py:189-194 ------ */
/* values_out[k] = the value at placeholder row rows[k] (d_pos wins over wl_pos),
 * snapped to the nearest bucket centre when n_buckets > 0 and taken as given
 * when n_buckets == 0 (centre pointers may then be NULL); feat_out[k] =
 * [cos(2 pi v f) | sin(2 pi v f)]. */
int cdk_fourier_features(const float* wl_t, const float* d_t, const uint8_t* wl_pos, const uint8_t* d_pos,
                         const float* wl_centers, const float* d_centers, int32_t n_buckets, const float* freqs,
                         int32_t n_freq, const int32_t* rows, int64_t n_rows, float* values_out, float* feat_out,
                         void* stream);
int cdk_embed_fwd(const int64_t* ids, int64_t n_tok, int64_t vocab, const float* emb, int64_t dim,
                  const int32_t* slot, const float* fourier_rows, float* out, int64_t n_copies, void* stream);
int cdk_embed_bwd(const int64_t* ids, int64_t n_tok, int64_t vocab, const float* dh, int64_t dim, int64_t n_copies,
                  const int32_t* slot, float* demb, float* dfourier_rows, void* stream);
int cdk_fourier_bwd(const float* values, const float* freqs, int32_t n_freq, const float* dfeat, int64_t n_rows,
                    float* dfreqs, void* stream);

/* ---- heads: fused softmax cross-entropy (train/train.py:180-207) and the
 *      value-head tail + soft two-bucket loss (utils/training.py:24-50) -----
 * softmax_ce: per row r, ce_r = logsumexp(logits_r) - logits_r[target_r]
 * (target outside [0, ncls) contributes nothing); *loss_out += sum_r w_r*ce_r*norm;
 * dlogits (bf16, optional) = (softmax - onehot) * w_r * norm * loss_weight;
 * dbias (optional) += column sums of dlogits; argmax_out (optional) first max. */
int cdk_softmax_ce(const float* logits, int64_t ldl, int64_t rows, int64_t ncls, const int32_t* target,
                   const float* row_weight, const float* norm, float loss_weight, void* dlogits_bf16, int64_t ldd,
                   float* dbias, float* loss_out, int32_t* argmax_out, void* stream);
/* value_tail: z1 = first Linear output (bias included) [rows, hidden];
 * a = mish(z1) -> act_out; logits = a W2^T + b2 [rows, nb]; soft two-bucket CE
 * against `target` using bucket `centers`, masked by `valid` (1/0), scaled by
 * *norm; dlogits_out f32 [rows, nb] (for dW2 / db2), dz1 bf16 [rows, ldd]
 * (for dX / dW1), db1 += column sums of dz1. */
int cdk_value_tail(const float* z1, int64_t rows, int64_t hidden, const float* w2, const float* b2, int64_t nb,
                   const float* target, const float* valid, const float* centers, const float* norm,
                   float loss_weight, float* act_out, float* dlogits_out, void* dz1_bf16, int64_t ldd, float* db1,
                   float* loss_out, int32_t* argmax_out, void* stream);
/* soft_bucket_ce: the soft two-bucket cross-entropy of utils/training.py:24-50
 * on given logits [rows, nb] (row stride ldl): *loss_out += sum_r valid_r *
 * ce_r * (*norm); dlogits f32 [rows, ldd] (optional) = (softmax - soft labels)
 * * valid_r * (*norm) * loss_weight.  valid / norm may be NULL (= 1). */
int cdk_soft_bucket_ce(const float* logits, int64_t ldl, int64_t rows, int64_t nb, const float* target,
                       const float* valid, const float* centers, const float* norm, float loss_weight,
                       float* dlogits, int64_t ldd, float* loss_out, void* stream);

/* ---- gathers / scatters / casts around the heads ------------------------ */
int cdk_gather_rows_bf16(const void* src, int64_t ld_src, const int32_t* rows, int64_t n, int64_t dim, void* dst,
                         int64_t ld_dst, void* stream);
int cdk_scatter_add_rows_f32(const float* src, int64_t ld_src, const int32_t* rows, int64_t n, int64_t dim,
                             float* dst, int64_t ld_dst, void* stream);
int cdk_cast_f32_bf16(const float* src, void* dst, int64_t n, void* stream);
int cdk_add_f32(const float* a, const float* b, float* out, int64_t n, void* stream);
int cdk_scale_f32(float* x, int64_t n, float s, void* stream);
/* SwiGLU backward (FeedForward of model.py:104-108): du = dL/d(silu(g)*u) bf16
 * [rows, F]; gu = [g | u] bf16 [rows, 2F]; dgu = [du*u*silu'(g) | du*silu(g)] bf16. */
int cdk_swiglu_bwd(const void* du, int64_t lddu, const void* gu, int64_t ldgu, void* dgu, int64_t lddgu,
                   int64_t rows, int64_t F, void* stream);
/* The same with dgu written as 8-bit (fp8 recipe; see cdk_rmsnorm_fwd_q8), pitch lddgu8 bytes. */
int cdk_swiglu_bwd_q8(const void* du, int64_t lddu, const void* gu, int64_t ldgu, void* dgu8, int64_t lddgu8, int fmt,
                      const float* qscale, float* amax, int64_t rows, int64_t F, void* stream);
/* fp32 SIMT GEMM for small / precision-sensitive contractions (Fourier
 * projection, value-head second Linear): C = (accumulate ? C : 0) + op(A) op(B)^T + bias,
 * A(m,k) = a_t ? A[k*lda+m] : A[m*lda+k],  B(n,k) = b_t ? B[k*ldb+n] : B[n*ldb+k]. */
int cdk_gemm_f32(const float* a, int64_t lda, int a_t, const float* b, int64_t ldb, int b_t, float* c, int64_t ldc,
                 int64_t M, int64_t N, int64_t K, const float* bias, int accumulate, void* stream);

/* ---- optimizer: global grad-norm clip + AdamW (train/train.py:64-68,248-253)
 *      with the 1/world_size mean of utils/distributed.py:55-67 folded in --- */
/* partial[i] = sum of squares of a grid-stride slice of x; n_partial <= 4096. */
int cdk_sumsq(const float* x, int64_t n, float* partial, int64_t n_partial, void* stream);
/* One AdamW step over a flat buffer; `partial` (from cdk_sumsq over the same
 * gradients, may be NULL = no clipping) gives the global norm; p_bf16 (optional)
 * receives bf16(p) after the update. */
int cdk_adamw(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n, const float* partial,
              int64_t n_partial, float max_norm, float lr, float beta1, float beta2, float eps, float wd,
              int64_t step, float grad_scale, void* stream);

/* The same clip + AdamW step for callers that cannot allocate device memory
 * (they hold only the parameter, gradient and moment buffers -- e.g. a host
 * runtime passing raw device pointers without a CUDA allocator of its own, or
 * a loop inside a fully pre-reserved memory pool).  No counterpart in the
 * reference.  The n_partial (1..4096) gradient-norm partial sums go to a
 * 16 KB array inside libcdk.so, one per device; nothing is allocated.  Sizes
 * beyond 4096 partial sums are rejected (status -32).  Every call on a device
 * shares that array (each call overwrites what it reads, so nothing needs
 * clearing); calls that overlap on the GPU race and must be serialised.  The
 * first call on a device looks up the array's device address, so make it
 * before any stream capture. */
int cdk_adamw_clip_noalloc(float* p, const float* g, float* m, float* v, void* p_bf16, int64_t n, int64_t n_partial,
                           float max_norm, float lr, float beta1, float beta2, float eps, float wd, int64_t step,
                           float grad_scale, void* stream);

/* ---- GRPO policy loss (chessdecoder/rl/log_probs.py:58-128, rl/grpo.py:58-126)
 * On gathered action rows: lp_out[r] = log_softmax(logits[r])[target[r]].
 * With old_lp / ref_lp / adv (per row) also the per-token clipped policy loss
 * + Schulman KL, summed times *norm (1 / action tokens) into *loss_out, its
 * gradient as bf16 dlogits [rows, ldd] (optional) and dbias += column sums.
 * old_lp == NULL: log-probs only (the frozen / rollout policy). */
int cdk_grpo_token(const float* logits, int64_t ldl, int64_t rows, int64_t ncls, const int32_t* target,
                   const float* old_lp, const float* ref_lp, const float* adv, const float* norm, float eps_low,
                   float eps_high, float kl_coeff, float* lp_out, void* dlogits_bf16, int64_t ldd, float* dbias,
                   float* loss_out, void* stream);

/* ---- batch producer (host memory; no GPU involved) ------------------------
 * Tokenisation + tensorisation of pretraining games: the native counterpart of
 * chessdecoder/dataloader/data.py:7-97 (fen_to_position_tokens,
 * game_to_token_ids) and the per-game body of
 * chessdecoder/dataloader/loader.py:69-184.
 *
 * cdk_vocab_create: token strings (concatenated, offsets[n_tokens + 1]) and
 * the full -> board / full -> move sub-vocabulary maps (-1 where absent);
 * returns NULL if a structural token is missing.  The handle is immutable and
 * may be shared by threads.
 *
 * cdk_tokenize_games: n_games games, game g = plies [game_offsets[g],
 * game_offsets[g+1]) in ply order.  Per ply: FEN, played move and best move
 * (vocabulary tokens; an empty played move adds nothing, as `if played_move:`),
 * played Q and D (NaN = invalid), include_board (the reference's
 * `random.random() > skip_board_prob`; ignored for a game's first ply).  Per
 * game: start_choice = the index that `random.choice(valid_starts)` drew.
 * Outputs are [n_games, max_seq_len] row-major (bool tensors as uint8).
 * n_threads <= 0: all hardware threads.  Status: 0 ok, -1 bad argument,
 * -2 unknown move token, -3 malformed FEN, -4 start_choice out of range,
 * -5 a game without plies. */
void* cdk_vocab_create(const char* chars, const int64_t* offsets, int64_t n_tokens, const int32_t* full_to_board,
                       const int32_t* full_to_move);
void cdk_vocab_destroy(void* vocab);
int cdk_tokenize_games(const void* vocab, int64_t n_games, const int64_t* game_offsets, const char* fen_chars,
                       const int64_t* fen_offsets, const char* played_chars, const int64_t* played_offsets,
                       const char* best_chars, const int64_t* best_offsets, const double* played_q,
                       const double* played_d, const uint8_t* include_board, const int64_t* start_choice,
                       int64_t max_seq_len, int32_t n_threads, int64_t* input_ids, int64_t* board_target_ids,
                       int64_t* move_target_ids, uint8_t* move_mask, uint8_t* wl_positions, uint8_t* d_positions,
                       float* wl_targets, float* d_targets, uint8_t* wdl_valid, int64_t* block_id);

/* ---- KV-cache inference (chessdecoder/cpp/decoder/batched_backbone.hpp:17-94,
 *      over the exported module chessdecoder/export/backbone_causal.py:79-158)
 * A cache holds, per layer, k and v as bf16 [B][H][max_len][64], a validity
 * byte per key u8 [B][ldv] (the reference's 0 / -1e9 mask buffer
 * [B, 1, 1, max_seq_len]) and its length as an int32 on the device (len_dev),
 * so that a step can be captured in a CUDA graph.  A step with S_new new tokens
 * per sequence (rows t = b * S_new + s):
 *
 * cdk_kv_append: qkv_f32 != 0: qkv fp32 [T, ldq] = q | k | v projections (not
 * rotated); q and k are rotated at positions pos[t] (rope [rope_len][32][2] =
 * (cos, sin), the rope_cache of backbone_causal.py:33), q goes to q_out bf16
 * [T, ldo] and k, v to cache rows len + s; qkv_out != 0: q_out rows receive the
 * rotated q | k | v (ldo >= 3 * H * 64), the layout cdk_attn_fwd reads (a
 * prefill from an empty cache runs the training attention).  qkv_f32 == 0: qkv bf16 with q, k
 * already rotated (a prefill through the training forward): only k, v are
 * written (pos, rope, q_out unused).
 *
 * cdk_decode_attn: out[t, h] = softmax(q k^T * scale + mask) v over keys
 * [0, len + S_new) of sequence b, head h.  Keys j < len: valid[b][j].  New
 * keys (j = len + u): block_mode CDK_BLOCK_CAUSAL -> u <= s and u <
 * num_real[b] (causalForward), CDK_BLOCK_ACTIVE -> active[b]
 * (prefixBlockForward), CDK_BLOCK_ALL (probes), CDK_BLOCK_VALID -> valid[b][j]
 * like the cache keys (causal- / prefixIncremental, whose new key the caller
 * marks first, as the reference does).  full_mask
 * (u8 [B][S_new][ldf], non-zero = attend) overrides all of it (prefixForward's
 * explicit mask).  active / num_real may be NULL (all).  A query with no valid
 * key gets zeros (the reference's all -1e9 row averages every key; such rows
 * belong to inactive sequences and are never read).  Requires len + S_new <=
 * max_len; a violation sets the index error bit and clamps.
 *
 * cdk_decode_mark: keys [base, base + count) become valid where active[b] and
 * offset < num_real[b] (NULL = all), base = start (>= 0) or len (start < 0);
 * then len += advance.  One block, stream-ordered with the step's kernels.
 *
 * cdk_decode_slots: slot[t] = override_mask[t] ? t : -1 (the Fourier override
 * rows for cdk_embed_fwd, backbone_causal.py:105-109). */
enum { CDK_BLOCK_CAUSAL = 0, CDK_BLOCK_ACTIVE = 1, CDK_BLOCK_ALL = 2, CDK_BLOCK_VALID = 3 };
int cdk_kv_append(const void* qkv, int64_t ldq, int qkv_f32, const int32_t* pos, const float* rope, int64_t rope_len,
                  int64_t B, int64_t S_new, int64_t H, void* k_cache, void* v_cache, int64_t max_len,
                  const int32_t* len_dev, void* q_out, int64_t ldo, int qkv_out, void* stream);
int cdk_decode_attn(const void* q, int64_t ldq, const void* k_cache, const void* v_cache, int64_t max_len,
                    const int32_t* len_dev, int64_t S_new, int64_t B, int64_t H, const uint8_t* valid, int64_t ldv,
                    int block_mode, const uint8_t* active, const int64_t* num_real, const uint8_t* full_mask,
                    int64_t ldf, void* out, int64_t ldo, float scale, void* stream);
int cdk_decode_mark(void* valid, int64_t ldv, int64_t B, int64_t start, int64_t count, int64_t advance,
                    int32_t* len_dev, const uint8_t* active, const int64_t* num_real, int64_t max_len, void* stream);
int cdk_decode_slots(const uint8_t* override_mask, int64_t n, int32_t* slot, void* stream);
/* u[t, f] = silu(gu[t, f]) * gu[t, F + f], gu fp32 [T, ldg] (gate | up), u bf16
 * [T, ldu]: the SwiGLU of a small decode batch whose gate / up projection ran as
 * a split-K fp32 GEMM (backbone_causal.py:141-143). */
int cdk_swiglu_f32(const float* gu, int64_t ldg, int64_t T, int64_t F, void* u, int64_t ldu, void* stream);
/* Next token of a generation loop (causalBoardStep of
 * chessdecoder/cpp/decoder/torch_backbone.hpp:141-152; sampleBatched and the
 * recorded log-probabilities of batched_engine.cpp:125-180).  temperature <= 0:
 * idx = argmax over logits[r, :ncols] (lowest index on ties); temperature > 0: a
 * sample of softmax(logits / temperature) (Gumbel-max over a counter-based
 * random stream keyed by *seed, the step counter, the row and the column; seed
 * NULL = 0).  ids[r] = lut ? lut[idx] : idx (sub-vocabulary -> full vocabulary);
 * lp_out[r] = log_softmax(logits[r])[idx], unscaled by the temperature.
 * Optional: pos[r] += 1; ids / log-probs appended at row *counter of hist /
 * lp_hist (max_steps rows; beyond them the index error bit is set) and
 * *counter += 1.  One block, stream-ordered, so a captured step can feed the
 * next one without the host. */
int cdk_head_select(const float* logits, int64_t ldl, int64_t rows, int64_t ncols, float temperature,
                    const uint64_t* seed, const int64_t* lut, int64_t* ids, float* lp_out, int64_t* pos,
                    int64_t* hist, float* lp_hist, int32_t* counter, int64_t max_steps, void* stream);
/* a[r, c] = mish(z[r, c]) (bf16 out): the hidden layer of the WL / D value heads
 * (chessdecoder/models/model.py:39-52) as the decoder engine evaluates them on a
 * step's hidden states (evalWlHead / evalDHead, batched_engine.cpp:151-180). */
int cdk_mish_bf16(const float* z, int64_t ldz, int64_t rows, int64_t cols, void* a, int64_t lda, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CDK_H_ */
