"""Thin torch-tensor wrappers over the libcdk.so C ABI.

Each wrapper validates dtypes/devices, launches on the current CUDA stream and
raises ``RuntimeError`` (naming the op and the library's status code) when the
library rejects a call.  Nothing here computes on the CPU or falls back to
PyTorch kernels.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

EPI_STORE_BF16 = 0
EPI_STORE_F32 = 1
EPI_RESID_F32 = 2
EPI_ROPE_BF16 = 3
EPI_SWIGLU = 4
EPI_DSWIGLU = 5
EPI_ATOMIC_F32 = 6
EPI_ACCUM_F32 = 7


# Number of CUDA kernels this module has launched (bench.py reports it per step).
LAUNCHES = [0]


def _count(n=1):
    LAUNCHES[0] += n


class GemmTimer:
    """Per-launch CUDA-event timing of the tcgen05 GEMM (events recorded on the
    launching stream around each launch); FLOPs are the algorithmic 2*M*N*K."""

    def __init__(self):
        self.records = []

    def add(self, flops, e0, e1, key=None):
        self.records.append((flops, e0, e1, key))

    def summary(self, detail=False):
        torch.cuda.synchronize()
        ms = 0.0
        fl = 0.0
        per = {}
        for f, e0, e1, key in self.records:
            t = e0.elapsed_time(e1)
            ms += t
            fl += f
            d = per.setdefault(key, [0, 0.0, 0.0])
            d[0] += 1
            d[1] += t
            d[2] += f
        out = {"launches": len(self.records), "ms": ms, "flops": fl,
               "tflops": (fl / (ms * 1e-3) / 1e12) if ms > 0 else 0.0}
        if detail:
            out["by_shape"] = sorted(
                [{"shape": k, "n": v[0], "ms": v[1], "tflops": v[2] / (v[1] * 1e-3) / 1e12 if v[1] else 0.0}
                 for k, v in per.items()], key=lambda r: -r["ms"])
        return out


GEMM_TIMER = None

# Optional per-op CUDA-event timer (bench.py --detail): op name -> [(e0, e1)].
OP_TIMER = None


def _timed(name):
    def deco(fn):
        def wrapper(*args, **kwargs):
            t = OP_TIMER
            if t is None:
                return fn(*args, **kwargs)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            r = fn(*args, **kwargs)
            e1.record()
            t.setdefault(name, []).append((e0, e1))
            return r
        wrapper.__name__ = fn.__name__
        wrapper.__doc__ = fn.__doc__
        return wrapper
    return deco


def op_timer_summary(t):
    torch.cuda.synchronize()
    out = {k: (len(v), sum(a.elapsed_time(b) for a, b in v)) for k, v in t.items()}
    return dict(sorted(out.items(), key=lambda kv: -kv[1][1]))


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(rc: int, op: str) -> None:
    if rc != 0:
        raise RuntimeError(f"cdk op {op} failed with status {rc}")


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("chessdecoder_b200 ops need CUDA tensors (no CPU implementation exists)")


def lib():
    return _lib.load()


def get_error(clear: bool = True) -> int:
    v = C.c_int(0)
    _check(lib().cdk_get_error(C.byref(v), 1 if clear else 0), "get_error")
    return v.value


# ---------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------
def _ld(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise RuntimeError("GEMM operands must be 2-D with unit inner stride")
    return t.stride(0)


_FP8_DTYPES = (torch.uint8, torch.float8_e4m3fn, torch.float8_e5m2)
FP8_E4M3, FP8_E5M2 = 0, 1
FP8_MAX = {FP8_E4M3: 448.0, FP8_E5M2: 57344.0}


def gemm_pair_clusters() -> int:
    """Clusters of two CTAs the CTA-pair GEMM form keeps resident on the
    current device (0: the form is off or unavailable)."""
    return int(lib().cdk_gemm_pair_clusters())


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False, kind: int = EPI_STORE_BF16,
         out: torch.Tensor, bias=None, resid=None, out2=None, aux=None, half_n: int = 0, rope=None,
         seq_len: int = 0, rope_cols: int = 0, split_k: int = 0, M=None, N=None, K=None, fp8=None) -> torch.Tensor:
    """D = A @ B^T with a fused epilogue (see include/cdk.h for the kinds).

    a: [M,K] (a_mn False) or [K,M] (a_mn True); b: [N,K] (b_mn False) or [K,N].
    For SWIGLU, b is [2N, K] = [gate; up] and N is the number of output columns.
    fp8 = (a_fmt, b_fmt, scale_inv_a, scale_inv_b): 8-bit operands (FP8_E4M3 /
    FP8_E5M2, same layouts as bf16) dequantised by the two device scalars.
    """
    _need_cuda(a, b, out)
    if fp8 is None:
        if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
            raise RuntimeError("GEMM inputs must be bf16")
    else:
        if a.dtype not in _FP8_DTYPES or b.dtype not in _FP8_DTYPES:
            raise RuntimeError("fp8 GEMM inputs must be 8-bit")
    if M is None:
        M = a.shape[1] if a_mn else a.shape[0]
    if K is None:
        K = a.shape[0] if a_mn else a.shape[1]
    if N is None:
        N = b.shape[1] if b_mn else b.shape[0]
        if kind == EPI_SWIGLU:
            N //= 2
    ep = _lib.CdkGemmEpilogue()
    ep.kind = kind
    ep.seq_len = seq_len
    ep.rope_cols = rope_cols
    ep.out = out.data_ptr()
    ep.ldo = out.stride(0)
    ep.bias = bias.data_ptr() if bias is not None else None
    if resid is not None:
        ep.resid = resid.data_ptr()
        ep.ldr = resid.stride(0)
    if out2 is not None:
        ep.out2 = out2.data_ptr()
        ep.ldo2 = out2.stride(0)
    if aux is not None:
        ep.aux = aux.data_ptr()
        ep.ldaux = aux.stride(0)
    ep.half_n = half_n
    ep.rope = rope.data_ptr() if rope is not None else None
    timer = GEMM_TIMER
    if timer is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
    if fp8 is None:
        rc = lib().cdk_gemm_bf16(_p(a), _ld(a), int(a_mn), _p(b), _ld(b), int(b_mn), M, N, K, C.byref(ep), split_k,
                                 _stream())
        _check(rc, f"gemm_bf16(kind={kind}, M={M}, N={N}, K={K}, a_mn={a_mn}, b_mn={b_mn})")
    else:
        af, bf, sa, sb = fp8
        rc = lib().cdk_gemm_fp8(_p(a), a.stride(0), int(a_mn), af, _p(b), b.stride(0), int(b_mn), bf, M, N, K, _p(sa),
                                _p(sb), C.byref(ep), split_k, _stream())
        _check(rc, f"gemm_fp8(kind={kind}, M={M}, N={N}, K={K}, fmt={af}{bf})")
    _count()
    if timer is not None:
        e1.record()
        timer.add(2.0 * M * N * K * (2 if kind == EPI_SWIGLU else 1), e0, e1,
                  f"M{M} N{N} K{K} kind{kind} mn{int(a_mn)}{int(b_mn)}" + ("" if fp8 is None else " fp8"))
    return out


@_timed("fp8_cast")
def fp8_cast(x, scale, fmt, out=None, out_t=None, amax=None, rows=None, cols=None):
    """out = sat_fmt(x * scale) (8-bit), out_t its transpose, amax = max(amax, max|x|)."""
    _need_cuda(x)
    rows = x.shape[0] if rows is None else rows
    cols = x.shape[1] if cols is None else cols
    dt = 0 if x.dtype == torch.float32 else 1 if x.dtype == torch.bfloat16 else None
    if dt is None:
        raise RuntimeError("fp8_cast input must be fp32 or bf16")
    rc = lib().cdk_fp8_cast(_p(x), dt, rows, cols, x.stride(0), _p(scale), fmt, _p(out),
                            out.stride(0) if out is not None else 0, _p(out_t),
                            out_t.stride(0) if out_t is not None else 0, _p(amax), _stream())
    _check(rc, "fp8_cast")
    _count(1)


@_timed("fp8_amax")
def fp8_amax(x, amax, rows=None, cols=None):
    rows = x.shape[0] if rows is None else rows
    cols = x.shape[1] if cols is None else cols
    dt = 0 if x.dtype == torch.float32 else 1
    _check(lib().cdk_fp8_amax(_p(x), dt, rows, cols, x.stride(0), _p(amax), _stream()), "fp8_amax")
    _count(1)


@_timed("fp8_scales")
def fp8_scales(amax_cur, history, scale, scale_inv, fmax, mode=0):
    n = amax_cur.numel()
    hist_len = history.shape[1] if history is not None else 0
    _check(lib().cdk_fp8_scales(_p(amax_cur), _p(history), _p(scale), _p(scale_inv), _p(fmax), n, hist_len, mode,
                                _stream()), "fp8_scales")
    _count(1)


@_timed("gemm_f32")
def gemm_f32(a, b, c, *, a_t=False, b_t=False, bias=None, accumulate=False, M=None, N=None, K=None):
    """C (+)= op(A) op(B)^T + bias in fp32 (small contractions)."""
    _need_cuda(a, b, c)
    if M is None:
        M = a.shape[1] if a_t else a.shape[0]
    if K is None:
        K = a.shape[0] if a_t else a.shape[1]
    if N is None:
        N = b.shape[1] if b_t else b.shape[0]
    rc = lib().cdk_gemm_f32(_p(a), a.stride(0), int(a_t), _p(b), b.stride(0), int(b_t), _p(c), c.stride(0), M, N, K,
                            _p(bias), int(accumulate), _stream())
    _check(rc, "gemm_f32")
    _count(1)
    return c


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------
@_timed("attn_meta")
def attn_meta(bid32: torch.Tensor, S: int) -> torch.Tensor:
    """Per-tile bounds for the prefix mask; bid32 int32 [nseq_prefix, S]."""
    nseq = bid32.shape[0]
    n = lib().cdk_attn_meta_elems(nseq, S)
    meta = torch.empty(max(int(n), 1), dtype=torch.int32, device=bid32.device)
    _check(lib().cdk_attn_prefix_meta(_p(bid32), nseq, S, _p(meta), _stream()), "attn_prefix_meta")
    _count(1)
    return meta


@_timed("attn_fwd")
def attn_fwd(qkv, out, lse, nseq, n_causal, S, H, bid32=None, meta=None):
    _need_cuda(qkv, out, lse)
    rc = lib().cdk_attn_fwd(_p(qkv), _p(out), _p(lse), nseq, n_causal, S, H, _p(bid32), _p(meta), _stream())
    _check(rc, "attn_fwd")
    _count(1)


@_timed("attn_bwd")
def attn_bwd(qkv, out, dout, lse, dsum, dqkv, nseq, n_causal, S, H, bid32=None, meta=None, rope=None):
    _need_cuda(qkv, out, dout, lse, dsum, dqkv)
    nb = int(lib().cdk_attn_bwd_workspace(nseq, S, H))
    ws = torch.empty(max(nb, 16) // 4, dtype=torch.float32, device=qkv.device) if nb > 0 else None
    rc = lib().cdk_attn_bwd_ws(_p(qkv), _p(out), _p(dout), _p(lse), _p(dsum), _p(dqkv), nseq, n_causal, S, H,
                               _p(bid32), _p(meta), _p(rope), _p(ws), max(nb, 0), _stream())
    _check(rc, "attn_bwd")
    _count(2)


def attn_bwd_q8(qkv, out, dout, lse, dsum, q8, nseq, n_causal, S, H, bid32=None, meta=None, rope=None) -> bool:
    """The backward with dq|dk|dv written as 8-bit values: q8 = (out8, fmt,
    qscale, amax).  False (nothing launched) where only the bf16 form exists
    (S > 256, or a non-default kernel path); the caller then uses attn_bwd."""
    _need_cuda(qkv, out, dout, lse, dsum)
    o8, fmt, qs, amax = q8
    rc = lib().cdk_attn_bwd_q8(_p(qkv), _p(out), _p(dout), _p(lse), _p(dsum), _p(o8), o8.stride(0), fmt, _p(qs),
                               _p(amax), nseq, n_causal, S, H, _p(bid32), _p(meta), _p(rope), _stream())
    if rc == -20:
        return False
    _check(rc, "attn_bwd_q8")
    _count(2)
    return True


# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------
@_timed("rmsnorm_fwd")
def rmsnorm_fwd(x, scale, y16=None, y32=None, rstd=None, eps=1e-6, q8=None):
    """q8 = (out8, fmt, qscale, amax): the output written as 8-bit (fp8 recipe) in place of y16 / y32."""
    _need_cuda(x, scale)
    rows, dim = x.shape
    if q8 is None:
        rc = lib().cdk_rmsnorm_fwd(_p(x), _p(scale), _p(y16), _p(y32), _p(rstd), rows, dim, eps, _stream())
    else:
        o8, fmt, qs, amax = q8
        rc = lib().cdk_rmsnorm_fwd_q8(_p(x), _p(scale), _p(o8), o8.stride(0), fmt, _p(qs), _p(amax), _p(rstd), rows,
                                      dim, eps, _stream())
    _check(rc, "rmsnorm_fwd")
    _count(1)


@_timed("rmsnorm_bwd")
def rmsnorm_bwd(dy, x, scale, rstd, dx=None, dx16=None, dscale=None, dres=None, q8=None):
    """q8 = (out8, fmt, qscale, amax): dx written as 8-bit (fp8 recipe) in place of dx16."""
    _need_cuda(dy, x, scale, rstd)
    rows, dim = x.shape
    if q8 is None:
        rc = lib().cdk_rmsnorm_bwd(_p(dy), int(dy.dtype == torch.float32), _p(x), _p(scale), _p(rstd), _p(dres),
                                   _p(dx), _p(dx16), _p(dscale), rows, dim, _stream())
    else:
        o8, fmt, qs, amax = q8
        rc = lib().cdk_rmsnorm_bwd_q8(_p(dy), int(dy.dtype == torch.float32), _p(x), _p(scale), _p(rstd), _p(dres),
                                      _p(dx), _p(o8), o8.stride(0), fmt, _p(qs), _p(amax), _p(dscale), rows, dim,
                                      _stream())
    _check(rc, "rmsnorm_bwd")
    _count(1)


# ---------------------------------------------------------------------------
# Embedding / Fourier
# ---------------------------------------------------------------------------
@_timed("fourier_features")
def fourier_features(wl_t, d_t, wl_pos_u8, d_pos_u8, wl_c, d_c, freqs, rows32, values_out, feat_out):
    """wl_c / d_c = None: use the values as given (no bucket snapping)."""
    n = rows32.numel()
    nb = 0 if wl_c is None else wl_c.numel()
    rc = lib().cdk_fourier_features(_p(wl_t), _p(d_t), _p(wl_pos_u8), _p(d_pos_u8), _p(wl_c), _p(d_c), nb,
                                    _p(freqs), freqs.numel(), _p(rows32), n, _p(values_out), _p(feat_out), _stream())
    _check(rc, "fourier_features")
    _count(1)


@_timed("embed_fwd")
def embed_fwd(ids, emb, slot32, frows, out, n_copies=1):
    n_tok = ids.numel()
    rc = lib().cdk_embed_fwd(_p(ids), n_tok, emb.shape[0], _p(emb), emb.shape[1], _p(slot32), _p(frows), _p(out),
                             n_copies, _stream())
    _check(rc, "embed_fwd")
    _count(1)


@_timed("embed_bwd")
def embed_bwd(ids, dh, slot32, demb, dfrows, n_copies=1):
    n_tok = ids.numel()
    rc = lib().cdk_embed_bwd(_p(ids), n_tok, demb.shape[0], _p(dh), demb.shape[1], n_copies, _p(slot32), _p(demb),
                             _p(dfrows), _stream())
    _check(rc, "embed_bwd")
    _count(1)


@_timed("fourier_bwd")
def fourier_bwd(values, freqs, dfeat, dfreqs):
    rc = lib().cdk_fourier_bwd(_p(values), _p(freqs), freqs.numel(), _p(dfeat), values.numel(), _p(dfreqs),
                               _stream())
    _check(rc, "fourier_bwd")
    _count(1)


# ---------------------------------------------------------------------------
# Heads
# ---------------------------------------------------------------------------
@_timed("softmax_ce")
def softmax_ce(logits, target32, row_w, norm, loss_weight, dlogits=None, dbias=None, loss_out=None, argmax=None,
               ncls=None):
    rows = logits.shape[0]
    ncls = logits.shape[1] if ncls is None else ncls
    rc = lib().cdk_softmax_ce(_p(logits), logits.stride(0), rows, ncls, _p(target32), _p(row_w), _p(norm),
                              float(loss_weight), _p(dlogits), dlogits.stride(0) if dlogits is not None else 0,
                              _p(dbias), _p(loss_out), _p(argmax), _stream())
    _check(rc, "softmax_ce")
    _count(1)


@_timed("grpo_token")
def grpo_token(logits, target32, lp_out, old_lp=None, ref_lp=None, adv=None, norm=None, eps_low=0.2, eps_high=0.2,
               kl_coeff=0.0, dlogits=None, dbias=None, loss_out=None, ncls=None):
    """Per-token log-probs of gathered action rows, and with old / ref
    log-probs and advantages the GRPO loss and its logit gradient."""
    _need_cuda(logits, target32)
    rows = logits.shape[0]
    ncls = logits.shape[1] if ncls is None else ncls
    rc = lib().cdk_grpo_token(_p(logits), logits.stride(0), rows, ncls, _p(target32), _p(old_lp), _p(ref_lp), _p(adv),
                              _p(norm), float(eps_low), float(eps_high), float(kl_coeff), _p(lp_out), _p(dlogits),
                              dlogits.stride(0) if dlogits is not None else 0, _p(dbias), _p(loss_out), _stream())
    _check(rc, "grpo_token")
    _count(1)


@_timed("soft_bucket_ce")
def soft_bucket_ce(logits, target, valid, centers, norm, loss_weight, dlogits=None, loss_out=None):
    rows, nb = logits.shape
    rc = lib().cdk_soft_bucket_ce(_p(logits), logits.stride(0), rows, nb, _p(target), _p(valid), _p(centers), _p(norm),
                                  float(loss_weight), _p(dlogits), dlogits.stride(0) if dlogits is not None else 0,
                                  _p(loss_out), _stream())
    _check(rc, "soft_bucket_ce")
    _count(1)


@_timed("value_tail")
def value_tail(z1, w2, b2, target, valid, centers, norm, loss_weight, act_out, dlogits_out, dz1, db1=None,
               loss_out=None, argmax=None):
    rows, hidden = z1.shape
    rc = lib().cdk_value_tail(_p(z1), rows, hidden, _p(w2), _p(b2), w2.shape[0], _p(target), _p(valid), _p(centers),
                              _p(norm), float(loss_weight), _p(act_out), _p(dlogits_out), _p(dz1), dz1.stride(0),
                              _p(db1), _p(loss_out), _p(argmax), _stream())
    _check(rc, "value_tail")
    _count(1)


@_timed("gather_rows_bf16")
def gather_rows_bf16(src, rows32, dst):
    rc = lib().cdk_gather_rows_bf16(_p(src), src.stride(0), _p(rows32), rows32.numel(), src.shape[1], _p(dst),
                                    dst.stride(0), _stream())
    _check(rc, "gather_rows_bf16")
    _count(1)


@_timed("scatter_add_rows")
def scatter_add_rows(src, rows32, dst):
    rc = lib().cdk_scatter_add_rows_f32(_p(src), src.stride(0), _p(rows32), rows32.numel(), dst.shape[1], _p(dst),
                                        dst.stride(0), _stream())
    _check(rc, "scatter_add_rows_f32")
    _count(1)


@_timed("cast_bf16")
def cast_bf16(src, dst):
    _check(lib().cdk_cast_f32_bf16(_p(src), _p(dst), src.numel(), _stream()), "cast_f32_bf16")
    _count(1)


@_timed("add_f32")
def add_f32(a, b, out):
    _check(lib().cdk_add_f32(_p(a), _p(b), _p(out), a.numel(), _stream()), "add_f32")
    _count(1)


@_timed("swiglu_bwd")
def swiglu_bwd(du, gu, dgu=None, q8=None):
    """dgu = [du*u*silu'(g) | du*silu(g)] from du [T,F] and gu = [g | u] [T,2F] (all bf16);
    q8 = (out8, fmt, qscale, amax): dgu written as 8-bit (fp8 recipe) instead."""
    _need_cuda(du, gu)
    rows, F = du.shape
    if q8 is None:
        rc = lib().cdk_swiglu_bwd(_p(du), du.stride(0), _p(gu), gu.stride(0), _p(dgu), dgu.stride(0), rows, F,
                                  _stream())
    else:
        o8, fmt, qs, amax = q8
        rc = lib().cdk_swiglu_bwd_q8(_p(du), du.stride(0), _p(gu), gu.stride(0), _p(o8), o8.stride(0), fmt, _p(qs),
                                     _p(amax), rows, F, _stream())
    _check(rc, "swiglu_bwd")
    _count(1)


@_timed("scale_f32")
def scale_f32(x, s):
    _check(lib().cdk_scale_f32(_p(x), x.numel(), float(s), _stream()), "scale_f32")
    _count(1)


# ---------------------------------------------------------------------------
# Optimizer
# ---------------------------------------------------------------------------
@_timed("sumsq")
def sumsq(x, partial):
    _check(lib().cdk_sumsq(_p(x), x.numel(), _p(partial), partial.numel(), _stream()), "sumsq")
    _count(1)


@_timed("adamw")
def adamw(p, g, m, v, p_bf16, partial, *, max_norm, lr, beta1, beta2, eps, wd, step, grad_scale=1.0):
    rc = lib().cdk_adamw(_p(p), _p(g), _p(m), _p(v), _p(p_bf16), p.numel(), _p(partial),
                         partial.numel() if partial is not None else 0, float(max_norm), float(lr), float(beta1),
                         float(beta2), float(eps), float(wd), int(step), float(grad_scale), _stream())
    _check(rc, "adamw")
    _count(1)


# ---------------------------------------------------------------------------
# Mixture of experts
# ---------------------------------------------------------------------------
@_timed("moe_route")
def moe_route(logits, n_seg, cap, expert, weight, probs, slot, src, workspace):
    T, X = logits.shape
    _check(lib().cdk_moe_route(_p(logits), T, X, n_seg, cap, _p(expert), _p(weight), _p(probs), _p(slot), _p(src),
                               _p(workspace), _stream()), "moe_route")
    _count(4)


def moe_route_workspace(T, n_seg, X):
    n = int(lib().cdk_moe_route_workspace(T, n_seg, X))
    if n < 0:
        raise RuntimeError("moe_route_workspace: token count must split into equal segments")
    return n


@_timed("moe_dispatch")
def moe_dispatch(x, src, xe):
    _check(lib().cdk_moe_dispatch(_p(x), x.stride(0), _p(src), xe.shape[0], xe.shape[1], _p(xe), _stream()),
           "moe_dispatch")
    _count(1)


@_timed("moe_combine")
def moe_combine(ye, slot, weight, resid, out):
    T, dim = out.shape
    _check(lib().cdk_moe_combine(_p(ye), _p(slot), _p(weight), _p(resid), _p(out), T, dim, _stream()), "moe_combine")
    _count(1)


@_timed("moe_combine_bwd")
def moe_combine_bwd(dout, ye, slot, weight, dye, dweight):
    T, dim = dout.shape
    _check(lib().cdk_moe_combine_bwd(_p(dout), _p(ye), _p(slot), _p(weight), _p(dye), dye.shape[0], _p(dweight), T,
                                     dim, _stream()), "moe_combine_bwd")
    _count(1)


@_timed("moe_route_bwd")
def moe_route_bwd(probs, expert, dweight, dlogits):
    T, X = probs.shape
    _check(lib().cdk_moe_route_bwd(_p(probs), _p(expert), _p(dweight), T, X, _p(dlogits), dlogits.stride(0),
                                   _stream()), "moe_route_bwd")
    _count(1)


@_timed("moe_gather_sum")
def moe_gather_sum(dxe, slot, out, accumulate=False):
    T, dim = out.shape
    _check(lib().cdk_moe_gather_sum(_p(dxe), _p(slot), _p(out), T, dim, int(accumulate), _stream()), "moe_gather_sum")
    _count(1)


# ---------------------------------------------------------------------------
# KV-cache inference (csrc/decode.cu)
# ---------------------------------------------------------------------------
BLOCK_CAUSAL, BLOCK_ACTIVE, BLOCK_ALL, BLOCK_VALID = 0, 1, 2, 3


@_timed("kv_append")
def kv_append(qkv, B, S_new, H, k_cache, v_cache, len_dev, pos=None, rope=None, q_out=None, qkv_out=False):
    """qkv fp32 (rotated here at pos) or bf16 (already rotated); k / v rows into
    the cache at [len, len + S_new).  qkv_out: q_out receives the rotated
    q | k | v rows (the training attention's layout)."""
    _need_cuda(qkv, k_cache, v_cache, len_dev)
    f32 = qkv.dtype == torch.float32
    max_len = k_cache.shape[-2]
    rc = lib().cdk_kv_append(_p(qkv), qkv.stride(0), int(f32), _p(pos), _p(rope), rope.shape[0] if rope is not None
                             else 0, B, S_new, H, _p(k_cache), _p(v_cache), max_len, _p(len_dev), _p(q_out),
                             q_out.stride(0) if q_out is not None else 0, int(qkv_out), _stream())
    _check(rc, "kv_append")
    _count(1)


@_timed("decode_attn")
def decode_attn(q, k_cache, v_cache, len_dev, S_new, B, H, valid, out, block_mode=BLOCK_ACTIVE, active=None,
                num_real=None, full_mask=None, scale=0.125):
    _need_cuda(q, k_cache, v_cache, valid, out)
    max_len = k_cache.shape[-2]
    rc = lib().cdk_decode_attn(_p(q), q.stride(0), _p(k_cache), _p(v_cache), max_len, _p(len_dev), S_new, B, H,
                               _p(valid), valid.stride(0), block_mode, _p(active), _p(num_real), _p(full_mask),
                               full_mask.stride(1) if full_mask is not None else 0, _p(out), out.stride(0), scale,
                               _stream())
    _check(rc, "decode_attn")
    _count(1)


@_timed("decode_mark")
def decode_mark(valid, B, len_dev, start=-1, count=0, advance=0, active=None, num_real=None):
    """Keys [base, base + count) valid where active / real (base = start, or
    the cache length when start < 0); then the cache length += advance."""
    rc = lib().cdk_decode_mark(_p(valid), valid.stride(0), B, start, count, advance, _p(len_dev), _p(active),
                               _p(num_real), valid.shape[1], _stream())
    _check(rc, "decode_mark")
    _count(1)


@_timed("decode_slots")
def decode_slots(override_mask_u8, slot32):
    rc = lib().cdk_decode_slots(_p(override_mask_u8), override_mask_u8.numel(), _p(slot32), _stream())
    _check(rc, "decode_slots")
    _count(1)


@_timed("swiglu_f32")
def swiglu_f32(gu32, u):
    """u = silu(gate) * up from fp32 [T, 2F] (gate | up)."""
    T, F = u.shape
    rc = lib().cdk_swiglu_f32(_p(gu32), gu32.stride(0), T, F, _p(u), u.stride(0), _stream())
    _check(rc, "swiglu_f32")
    _count(1)


@_timed("head_select")
def head_select(logits, ids, temperature=0.0, seed=None, lut=None, lp=None, pos=None, hist=None, lp_hist=None,
                counter=None):
    """ids[r] = lut[argmax(logits[r])] (temperature <= 0) or a sample of
    softmax(logits[r] / temperature) (seed: device int64 [1]); lp[r] = the
    unscaled log-softmax at the chosen index; optionally pos += 1 and ids / lp
    appended to hist / lp_hist at row *counter (counter += 1)."""
    rows, ncols = logits.shape
    max_steps = hist.shape[0] if hist is not None else (lp_hist.shape[0] if lp_hist is not None else 0)
    rc = lib().cdk_head_select(_p(logits), logits.stride(0), rows, ncols, float(temperature), _p(seed), _p(lut),
                               _p(ids), _p(lp), _p(pos), _p(hist), _p(lp_hist), _p(counter), max_steps, _stream())
    _check(rc, "head_select")
    _count(1)


@_timed("mish_bf16")
def mish_bf16(z, a):
    """a = mish(z) in bf16 (z fp32 [rows, cols])."""
    rows, cols = z.shape
    _check(lib().cdk_mish_bf16(_p(z), z.stride(0), rows, cols, _p(a), a.stride(0), _stream()), "mish_bf16")
    _count(1)
