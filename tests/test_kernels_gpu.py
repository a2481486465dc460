"""Kernel-level numerics on the GPU: each CUDA kernel against a plain PyTorch
fp32 statement of the same operation on identical bf16 inputs.

Tolerances: bf16 outputs are compared by relative Frobenius error <= 1e-2 and
cosine >= 0.9999; fp32 outputs (fp32 accumulation of bf16 products) by
relative error <= 2e-3.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def cosine(a, b):
    a = a.float().flatten()
    b = b.float().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


@pytest.fixture(scope="module")
def K():
    from chessdecoder_b200 import kernels
    kernels.lib()
    return kernels


def _bf(*shape, scale=1.0, gen=None):
    return (torch.randn(*shape, generator=gen, device=DEV) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K_", [(256, 256, 128), (300, 1924, 1024), (4096, 3072, 1024), (2048, 1024, 1536),
                                    (77, 41, 1024), (128, 128, 64)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_store(K, M, N, K_, a_mn, b_mn):
    if (a_mn and M % 8) or (b_mn and N % 8):
        pytest.skip("MN-major operands need a pitch that is a multiple of 8")
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N)
    A = _bf(M, K_, gen=g)
    B = _bf(N, K_, gen=g)
    a_arg = A.t().contiguous() if a_mn else A
    b_arg = B.t().contiguous() if b_mn else B
    ref = A.float() @ B.float().t()
    out32 = torch.empty(M, N, device=DEV, dtype=torch.float32)
    K.gemm(a_arg, b_arg, a_mn=a_mn, b_mn=b_mn, kind=K.EPI_STORE_F32, out=out32, M=M, N=N, K=K_)
    torch.cuda.synchronize()
    assert rel_err(out32, ref) < 2e-3
    if N % 8 == 0:
        out16 = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
        K.gemm(a_arg, b_arg, a_mn=a_mn, b_mn=b_mn, kind=K.EPI_STORE_BF16, out=out16, M=M, N=N, K=K_)
        torch.cuda.synchronize()
        assert rel_err(out16, ref) < 1e-2
    assert K.get_error() == 0


def test_gemm_bias_resid_accum(K):
    M, N, K_ = 1000, 1024, 512
    A, B = _bf(M, K_), _bf(N, K_)
    bias = torch.randn(N, device=DEV)
    resid = torch.randn(M, N, device=DEV)
    ref = A.float() @ B.float().t()
    out = torch.empty(M, N, device=DEV)
    K.gemm(A, B, kind=K.EPI_RESID_F32, out=out, resid=resid)
    assert rel_err(out, resid + ref) < 2e-3
    out2 = torch.empty(M, N, device=DEV)
    K.gemm(A, B, kind=K.EPI_STORE_F32, out=out2, bias=bias)
    assert rel_err(out2, ref + bias) < 2e-3
    acc = resid.clone()
    K.gemm(A, B, kind=K.EPI_ACCUM_F32, out=acc)
    assert rel_err(acc, resid + ref) < 2e-3
    # in-place residual (out aliases resid)
    r2 = resid.clone()
    K.gemm(A, B, kind=K.EPI_RESID_F32, out=r2, resid=r2)
    assert rel_err(r2, resid + ref) < 2e-3
    torch.cuda.synchronize()
    assert K.get_error() == 0


@pytest.mark.parametrize("M,N,K_", [(1000, 1040, 512), (4096, 1024, 1536), (130, 96, 256)])
def test_gemm_resid_tma_epilogue(K, M, N, K_):
    """Residual epilogue (TMA-fed when the shapes allow): ragged rows, a
    partial last column tile, bias, in-place and out-of-place."""
    A, B = _bf(M, K_), _bf(N, K_)
    bias = torch.randn(N, device=DEV)
    resid = torch.randn(M, N, device=DEV)
    ref = A.float() @ B.float().t() + bias
    out = torch.full((M, N), float("nan"), device=DEV)
    K.gemm(A, B, kind=K.EPI_RESID_F32, out=out, resid=resid, bias=bias)
    r2 = resid.clone()
    K.gemm(A, B, kind=K.EPI_RESID_F32, out=r2, resid=r2, bias=bias)
    torch.cuda.synchronize()
    assert rel_err(out, resid + ref) < 2e-3
    assert rel_err(r2, resid + ref) < 2e-3
    assert K.get_error() == 0


@pytest.mark.parametrize("split", [0, 1, 3])
def test_gemm_atomic_splitk(K, split):
    M, N, K_ = 3072, 1024, 8192  # dW shape: [out, in] over K = tokens
    dY = _bf(K_, M, scale=0.5)
    X = _bf(K_, N)
    ref = dY.float().t() @ X.float()
    out = torch.zeros(M, N, device=DEV)
    K.gemm(dY, X, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=out, split_k=split)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 2e-3
    assert K.get_error() == 0


def rope_table(S, hd=64, base=10000.0):
    theta = 1.0 / (base ** (torch.arange(0, hd, 2)[: hd // 2].float() / hd))
    idx = torch.arange(S).float()
    ang = torch.outer(idx, theta)
    return torch.stack([ang.cos(), ang.sin()], dim=-1).contiguous()  # [S, 32, 2]


def apply_rope_ref(x, cache, S):
    # x [T, H*64] fp32, rows = (seq, pos)
    T, W = x.shape
    xs = x.view(T, W // 64, 32, 2)
    pos = torch.arange(T, device=x.device) % S
    c = cache[pos][:, None, :, 0]
    s = cache[pos][:, None, :, 1]
    o0 = xs[..., 0] * c - xs[..., 1] * s
    o1 = xs[..., 1] * c + xs[..., 0] * s
    return torch.stack([o0, o1], -1).view(T, W)


def test_gemm_rope(K):
    S, E = 256, 512
    T = 4 * S
    X, W = _bf(T, E), _bf(3 * E, E, scale=0.05)
    cache = rope_table(S).to(DEV)
    out = torch.empty(T, 3 * E, device=DEV, dtype=torch.bfloat16)
    K.gemm(X, W, kind=K.EPI_ROPE_BF16, out=out, rope=cache, seq_len=S, rope_cols=2 * E)
    ref = X.float() @ W.float().t()
    ref[:, : 2 * E] = apply_rope_ref(ref[:, : 2 * E].contiguous(), cache, S)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("T", [1024, 1000])
def test_gemm_swiglu_and_back(K, T):
    E, F = 512, 768
    X, W13 = _bf(T, E), _bf(2 * F, E, scale=0.05)
    u = torch.empty(T, F, device=DEV, dtype=torch.bfloat16)
    gu = torch.empty(T, 2 * F, device=DEV, dtype=torch.bfloat16)
    K.gemm(X, W13, kind=K.EPI_SWIGLU, out=u, out2=gu, half_n=F)
    ref_gu = X.float() @ W13.float().t()
    g, up = ref_gu[:, :F], ref_gu[:, F:]
    ref_u = torch.nn.functional.silu(g) * up
    torch.cuda.synchronize()
    assert rel_err(gu, ref_gu) < 1e-2
    assert rel_err(u, ref_u) < 1e-2
    # backward of the SwiGLU product through the down projection: dU = dY @ W2
    W2 = _bf(E, F, scale=0.05)
    dY = _bf(T, E)
    dgu = torch.empty(T, 2 * F, device=DEV, dtype=torch.bfloat16)
    K.gemm(dY, W2, b_mn=True, kind=K.EPI_DSWIGLU, out=dgu, aux=gu, half_n=F, N=F)
    du = dY.float() @ W2.float()
    gf, upf = gu[:, :F].float(), gu[:, F:].float()
    sg = torch.sigmoid(gf)
    ref_dg = du * upf * (sg * (1 + gf * (1 - sg)))
    ref_dup = du * gf * sg
    torch.cuda.synchronize()
    assert rel_err(dgu[:, :F], ref_dg) < 1e-2
    assert rel_err(dgu[:, F:], ref_dup) < 1e-2
    # the unfused form used by the step: bf16 du, then the elementwise SwiGLU backward
    du16 = du.to(torch.bfloat16)
    dgu2 = torch.empty(T, 2 * F, device=DEV, dtype=torch.bfloat16)
    K.swiglu_bwd(du16, gu, dgu2)
    torch.cuda.synchronize()
    assert rel_err(dgu2[:, :F], ref_dg) < 1e-2
    assert rel_err(dgu2[:, F:], ref_dup) < 1e-2


def make_bid(nseq, S, gen):
    bid = torch.empty(nseq, S, dtype=torch.int64)
    for s in range(nseq):
        ids = torch.arange(S) + 1000
        pos = int(torch.randint(0, 40, (1,), generator=gen))
        nb = 0
        while pos + 68 <= S:
            ids[pos:pos + 68] = nb
            nb += 1
            pos += 68 + int(torch.randint(3, 20, (1,), generator=gen))
        bid[s] = ids
    return bid


def ref_attention(qkv, nseq, n_causal, S, H, bid):
    x = qkv.view(nseq, S, 3, H, 64)
    q, k, v = (x[:, :, i].transpose(1, 2) for i in range(3))
    mask = torch.ones(S, S, dtype=torch.bool, device=qkv.device).tril().expand(nseq, S, S).clone()
    if n_causal < nseq:
        b = bid.to(qkv.device)
        mask[n_causal:] |= b[:, :, None] == b[:, None, :]
    sc = (q @ k.transpose(-1, -2)) * 0.125
    sc = sc.masked_fill(~mask[:, None], float("-inf"))
    o = torch.softmax(sc, -1) @ v
    return o.transpose(1, 2).reshape(nseq * S, H * 64)


@pytest.fixture(params=["default", "tc", "seq", "tiled", "long"])
def attn_path(request, monkeypatch):
    """Every attention implementation: the default (persistent tcgen05 forward
    for S <= 256), tcgen05 with one CTA per query tile (S <= 256), mma.sync
    sequence-resident (S <= 256), mma.sync tiled (any S) and the tcgen05
    long-sequence kernels forced at short S."""
    if request.param == "default":
        monkeypatch.delenv("CDK_ATTN_PATH", raising=False)
    else:
        monkeypatch.setenv("CDK_ATTN_PATH", request.param)
    return request.param


@pytest.mark.parametrize("S,nseq,n_causal", [(256, 4, 2), (100, 3, 1), (256, 2, 2), (320, 2, 0), (68, 3, 1),
                                             (136, 2, 0)])
def test_attention_fwd_bwd(K, attn_path, S, nseq, n_causal):
    H = 4
    E = H * 64
    gen = torch.Generator().manual_seed(S + nseq)
    qkv = (torch.randn(nseq * S, 3 * E, generator=gen) * 0.8).to(DEV).to(torch.bfloat16)
    bid = make_bid(nseq - n_causal, S, gen)
    bid32 = bid.to(torch.int32).to(DEV).contiguous()
    meta = K.attn_meta(bid32, S) if n_causal < nseq else None
    out = torch.empty(nseq * S, E, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(nseq * H * S, device=DEV)
    K.attn_fwd(qkv, out, lse, nseq, n_causal, S, H, bid32 if n_causal < nseq else None, meta)
    qkv_f = qkv.float().requires_grad_(True)
    ref = ref_attention(qkv_f, nseq, n_causal, S, H, bid)
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2 and cosine(out, ref) > 0.9999
    dout = (torch.randn(nseq * S, E, generator=gen) * 0.5).to(DEV).to(torch.bfloat16)
    ref.backward(dout.float())
    dqkv = torch.empty_like(qkv)
    dsum = torch.empty(nseq * H * S, device=DEV)
    K.attn_bwd(qkv, out, dout, lse, dsum, dqkv, nseq, n_causal, S, H, bid32 if n_causal < nseq else None, meta)
    torch.cuda.synchronize()
    g = qkv_f.grad
    for i, name in enumerate("qkv"):
        sl = slice(i * E, (i + 1) * E)
        assert cosine(dqkv[:, sl], g[:, sl]) > 0.999, name
        assert rel_err(dqkv[:, sl], g[:, sl]) < 3e-2, name
    assert K.get_error() == 0


@pytest.mark.parametrize("S,nseq,n_causal,H", [(256, 40, 20, 16), (100, 64, 32, 8), (136, 48, 16, 8)])
def test_attention_bwd_many_items(K, S, nseq, n_causal, H):
    """The S <= 256 forward and backward over more (head, sequence) items than
    the GPU has SMs (several waves; several items per CTA of the persistent
    forward), mixed causal / block-prefix, full and partial tiles; every output
    row and log-sum-exp written (the outputs start as NaN)."""
    E = H * 64
    gen = torch.Generator().manual_seed(S * 3 + nseq)
    qkv = (torch.randn(nseq * S, 3 * E, generator=gen) * 0.8).to(DEV).to(torch.bfloat16)
    bid = make_bid(nseq - n_causal, S, gen)
    bid32 = bid.to(torch.int32).to(DEV).contiguous()
    meta = K.attn_meta(bid32, S)
    out = torch.full((nseq * S, E), float("nan"), device=DEV, dtype=torch.bfloat16)
    lse = torch.full((nseq * H * S,), float("nan"), device=DEV)
    K.attn_fwd(qkv, out, lse, nseq, n_causal, S, H, bid32, meta)
    qkv_f = qkv.float().requires_grad_(True)
    ref = ref_attention(qkv_f, nseq, n_causal, S, H, bid)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()
    assert rel_err(out, ref) < 1e-2 and cosine(out, ref) > 0.9999
    dout = (torch.randn(nseq * S, E, generator=gen) * 0.5).to(DEV).to(torch.bfloat16)
    ref.backward(dout.float())
    dqkv = torch.full_like(qkv, float("nan"))
    dsum = torch.empty(nseq * H * S, device=DEV)
    K.attn_bwd(qkv, out, dout, lse, dsum, dqkv, nseq, n_causal, S, H, bid32, meta)
    torch.cuda.synchronize()
    g = qkv_f.grad
    assert torch.isfinite(dqkv.float()).all()
    for i, name in enumerate("qkv"):
        sl = slice(i * E, (i + 1) * E)
        assert cosine(dqkv[:, sl], g[:, sl]) > 0.999, name
        assert rel_err(dqkv[:, sl], g[:, sl]) < 3e-2, name
    assert K.get_error() == 0


def test_attention_bwd_unrope(K, attn_path):
    S, nseq, H = 128, 2, 2
    E = H * 64
    gen = torch.Generator().manual_seed(5)
    cache = rope_table(S).to(DEV)
    pre = (torch.randn(nseq * S, 3 * E, generator=gen)).to(DEV)
    pre_f = pre.clone().requires_grad_(True)
    q = apply_rope_ref(pre_f[:, :E].contiguous(), cache, S)
    k = apply_rope_ref(pre_f[:, E:2 * E].contiguous(), cache, S)
    qkv_f = torch.cat([q, k, pre_f[:, 2 * E:]], 1)
    ref = ref_attention(qkv_f, nseq, nseq, S, H, None)
    dout = torch.randn(nseq * S, E, generator=gen).to(DEV).to(torch.bfloat16)
    ref.backward(dout.float())
    qkv = qkv_f.detach().to(torch.bfloat16)
    out = torch.empty(nseq * S, E, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(nseq * H * S, device=DEV)
    K.attn_fwd(qkv, out, lse, nseq, nseq, S, H)
    dqkv = torch.empty_like(qkv)
    dsum = torch.empty(nseq * H * S, device=DEV)
    K.attn_bwd(qkv, out, dout, lse, dsum, dqkv, nseq, nseq, S, H, rope=cache)
    torch.cuda.synchronize()
    assert cosine(dqkv, pre_f.grad) > 0.999


def test_rmsnorm(K):
    T, E = 1000, 1024
    x = torch.randn(T, E, device=DEV) * 3
    s = torch.rand(E, device=DEV) + 0.5
    y16 = torch.empty(T, E, device=DEV, dtype=torch.bfloat16)
    y32 = torch.empty(T, E, device=DEV)
    rstd = torch.empty(T, device=DEV)
    K.rmsnorm_fwd(x, s, y16, y32, rstd)
    xr = x.clone().requires_grad_(True)
    ref = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * s
    torch.cuda.synchronize()
    assert rel_err(y32, ref) < 1e-5
    assert rel_err(y16, ref) < 5e-3
    dy = torch.randn(T, E, device=DEV).to(torch.bfloat16)
    dres = torch.randn(T, E, device=DEV)
    sr = s.clone().requires_grad_(True)
    ref2 = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * sr
    ref2.backward(dy.float())
    dx = torch.empty(T, E, device=DEV)
    dx16 = torch.empty(T, E, device=DEV, dtype=torch.bfloat16)
    ds = torch.zeros(E, device=DEV)
    K.rmsnorm_bwd(dy, x, s, rstd, dx=dx, dx16=dx16, dscale=ds, dres=dres)
    torch.cuda.synchronize()
    assert rel_err(dx, xr.grad + dres) < 1e-4
    assert rel_err(ds, sr.grad) < 1e-4


def test_sgemm_f32(K):
    for (M, N, Kd, at, bt) in [(100, 1024, 256, False, False), (1024, 256, 77, True, False),
                               (33, 100, 256, False, True)]:
        A = torch.randn(Kd, M, device=DEV) if at else torch.randn(M, Kd, device=DEV)
        B = torch.randn(Kd, N, device=DEV) if bt else torch.randn(N, Kd, device=DEV)
        bias = torch.randn(N, device=DEV)
        C = torch.empty(M, N, device=DEV)
        K.gemm_f32(A, B, C, a_t=at, b_t=bt, bias=bias, M=M, N=N, K=Kd)
        ref = (A.t() if at else A) @ (B if bt else B.t()) + bias
        torch.cuda.synchronize()
        assert rel_err(C, ref) < 1e-5
