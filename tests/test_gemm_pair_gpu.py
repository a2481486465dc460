"""CTA-pair GEMM form (two SMs per 256-row tile, M=256 tcgen05 MMAs): the
forward GEMMs of the training step (QKV projection with RoPE, gate|up
projection with SwiGLU, output and down projections with the fp32 residual
add, plain bf16 store), the backward's input-gradient GEMMs (MN-major
weight operand: plain bf16 store, SwiGLU backward epilogue) and its
weight-gradient GEMMs (both operands MN-major, split-K bulk reduce-add), and
the fp8 recipe's forms with 8-bit operands (e4m3 x e4m3 store, SwiGLU and
residual; e5m2 x e4m3 dX with the weight MN-major) computed with the pair form on for every form that can
use it (the default) and off (CDK_GEMM_PAIR=0), each in its own process
because the switch is read once per process.  The pair form must reproduce the one-CTA form bit for bit (each
output element is the same sequence of K=16 products accumulated in fp32) and
match a PyTorch fp32 statement of the operation (bf16 outputs: relative
Frobenius error <= 1e-2; fp32 outputs: <= 2e-3).  The weight gradients sum
split-K partial products in an order that depends on the split, so the two
forms agree there to 1e-5 (relative) instead of bit for bit.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
# (M, N, K): the step's shapes at a smaller token count, a K that is not a
# multiple of 64, an M that is not a multiple of 256 (one-CTA form in both runs)
SHAPES = [(4096, 3072, 1024), (2048, 1024, 1536), (1024, 1024, 200), (1280, 512, 512), (1000, 1024, 512)]
# weight gradients dW [M, N] = dY^T X over K tokens
WGRAD = [(3072, 1024, 8192), (1024, 1536, 4096), (1000, 512, 2048)]


def _inputs(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bf = lambda *s: (torch.randn(*s, generator=g, device="cuda") * 0.1).to(torch.bfloat16)  # noqa: E731
    return (bf(M, K), bf(N, K), bf(2 * N, K), torch.randn(M, N, generator=g, device="cuda"), bf(K, N),
            bf(M, 2 * N))


def _wgrad_inputs(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return ((torch.randn(K, M, generator=g, device="cuda") * 0.1).to(torch.bfloat16),
            (torch.randn(K, N, generator=g, device="cuda") * 0.1).to(torch.bfloat16))


def _child(out_path):
    from chessdecoder_b200 import kernels as Kn
    from chessdecoder_b200.engine import rope_table
    res = {"clusters": Kn.gemm_pair_clusters()}
    rope = rope_table(256, 64).cuda()
    for i, (M, N, K) in enumerate(SHAPES):
        X, W, W13, h, Wt, gu_in = _inputs(M, N, K, 1234 + i)
        o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(X, W, kind=Kn.EPI_STORE_BF16, out=o)
        r = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(X, W, kind=Kn.EPI_ROPE_BF16, out=r, rope=rope, seq_len=256, rope_cols=(2 * N // 3) // 64 * 64)
        u = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        gu = torch.empty(M, 2 * N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(X, W13, kind=Kn.EPI_SWIGLU, out=u, out2=gu, half_n=N)
        y = torch.empty(M, N, device="cuda")
        Kn.gemm(X, W, kind=Kn.EPI_RESID_F32, out=y, resid=h)
        dx = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(X, Wt, b_mn=True, kind=Kn.EPI_STORE_BF16, out=dx)
        dgu = torch.empty(M, 2 * N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(X, Wt, b_mn=True, kind=Kn.EPI_DSWIGLU, out=dgu, aux=gu_in, half_n=N, N=N)
        torch.cuda.synchronize()
        res[i] = {k: v.cpu() for k, v in dict(store=o, rope=r, u=u, gu=gu, resid=y, dx=dx, dgu=dgu).items()}
    for i, (M, N, K) in enumerate(WGRAD):
        dY, X = _wgrad_inputs(M, N, K, 77 + i)
        dw = torch.zeros(M, N, device="cuda")
        Kn.gemm(dY, X, a_mn=True, b_mn=True, kind=Kn.EPI_ATOMIC_F32, out=dw)
        torch.cuda.synchronize()
        res[("w", i)] = dw.cpu()
    sc = torch.ones(1, device="cuda")
    for i, (M, N, K) in enumerate(SHAPES[:3]):
        g = torch.Generator(device="cuda").manual_seed(555 + i)
        q = lambda *sh: (torch.randn(*sh, generator=g, device="cuda") * 2).to(torch.float8_e4m3fn)  # noqa: E731
        X8, W8, W13_8 = q(M, K if K % 16 == 0 else 256), q(N, K if K % 16 == 0 else 256), q(2 * N, K if K % 16 == 0 else 256)
        h = torch.randn(M, N, generator=g, device="cuda")
        o = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(X8, W8, kind=Kn.EPI_STORE_BF16, out=o, fp8=(0, 0, sc, sc))
        u = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        gu = torch.empty(M, 2 * N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(X8, W13_8, kind=Kn.EPI_SWIGLU, out=u, out2=gu, half_n=N, fp8=(0, 0, sc, sc))
        y = torch.empty(M, N, device="cuda")
        Kn.gemm(X8, W8, kind=Kn.EPI_RESID_F32, out=y, resid=h, fp8=(0, 0, sc, sc))
        G8 = (torch.randn(M, N, generator=g, device="cuda")).to(torch.float8_e5m2)
        Wd = q(N, N)  # [K = N rows, N] read MN-major
        dx = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        Kn.gemm(G8, Wd, b_mn=True, kind=Kn.EPI_STORE_BF16, out=dx, fp8=(1, 0, sc, sc))
        torch.cuda.synchronize()
        res[("f8", i)] = {k: v.cpu() for k, v in dict(store=o, u=u, gu=gu, resid=y, dx=dx).items()}
    res["error"] = Kn.get_error()
    torch.save(res, out_path)


def _run(tmp_path, pair):
    out = tmp_path / f"pair{pair}.pt"
    env = dict(os.environ, CDK_GEMM_PAIR="1" if pair else "0")
    subprocess.run([sys.executable, __file__, str(out)], env=env, cwd=ROOT, check=True, timeout=600)
    return torch.load(out)


def test_pair_form_matches_one_cta_form(tmp_path):
    from chessdecoder_b200.engine import rope_table
    on, off = _run(tmp_path, 1), _run(tmp_path, 0)
    assert on["error"] == 0 and off["error"] == 0
    assert off["clusters"] == 0
    assert on["clusters"] >= 60  # one cluster per two SMs on a B200
    rope = rope_table(256, 64)
    for i, (M, N, K) in enumerate(SHAPES):
        for k in ("store", "rope", "u", "gu", "resid", "dx", "dgu"):
            assert torch.equal(on[i][k], off[i][k]), (M, N, K, k)
        X, W, W13, h, Wt, gu_in = (t.cpu() for t in _inputs(M, N, K, 1234 + i))
        ref = X.float() @ W.float().t()
        rel = lambda a, b: ((a.float() - b).norm() / b.norm()).item()  # noqa: E731
        assert rel(on[i]["store"], ref) < 1e-2
        assert rel(on[i]["resid"], ref + h) < 2e-3
        rc = (2 * N // 3) // 64 * 64
        xs = ref[:, :rc].reshape(M, rc // 64, 32, 2)
        pos = torch.arange(M) % 256
        c, s = rope[pos][:, None, :, 0], rope[pos][:, None, :, 1]
        rot = torch.stack([xs[..., 0] * c - xs[..., 1] * s, xs[..., 1] * c + xs[..., 0] * s], -1).reshape(M, rc)
        assert rel(on[i]["rope"], torch.cat([rot, ref[:, rc:]], 1)) < 1e-2
        gu = X.float() @ W13.float().t()
        assert rel(on[i]["gu"], gu) < 1e-2
        assert rel(on[i]["u"], torch.nn.functional.silu(gu[:, :N]) * gu[:, N:]) < 1e-2
        du = X.float() @ Wt.float()
        assert rel(on[i]["dx"], du) < 1e-2
        g, up = gu_in[:, :N].float(), gu_in[:, N:].float()
        sg = torch.sigmoid(g)
        assert rel(on[i]["dgu"][:, :N], du * up * (sg * (1 + g * (1 - sg)))) < 1e-2
        assert rel(on[i]["dgu"][:, N:], du * g * sg) < 1e-2
    for i in range(3):
        for k in ("store", "u", "gu", "resid", "dx"):
            assert torch.equal(on[("f8", i)][k], off[("f8", i)][k]), ("fp8", i, k)
    for i, (M, N, K) in enumerate(WGRAD):
        dY, X = (t.cpu() for t in _wgrad_inputs(M, N, K, 77 + i))
        ref = dY.float().t() @ X.float()
        a, b = on[("w", i)], off[("w", i)]
        assert ((a - ref).norm() / ref.norm()).item() < 2e-3, (M, N, K)
        assert ((a - b).norm() / b.norm()).item() < 1e-5, (M, N, K)


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT))
    _child(sys.argv[1])
