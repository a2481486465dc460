"""The allocation-free clip + AdamW entry point (cdk_adamw_clip_noalloc).

It exists for callers that own only the parameter, gradient and moment
buffers and cannot obtain any other device memory (for instance a host
runtime that hands over raw device pointers but has no CUDA allocator, or a
training loop inside a fully pre-reserved memory pool), so it keeps its
gradient-norm partial sums in an array inside libcdk.so instead of a caller
buffer.  This test calls it through the C ABI on two optimizer steps in a row
and checks parameters, both moments and the bf16 shadow against the regular
entry points (cdk_sumsq + cdk_adamw with caller scratch) on identical inputs,
and against clip_grad_norm_ + torch.optim.AdamW on the CPU, with the
tolerance of the other optimizer tests (rtol 1e-5, atol 1e-6); the bf16
shadow, written by the same kernel from the same values, must be identical.
On the first step the clip engages (the unclipped update differs).  The file
is named to be collected last.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _vp(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def test_noalloc_adamw_matches_scratch_version_two_steps():
    from chessdecoder_b200 import _lib
    lib = _lib.load()
    dev = "cuda"
    torch.manual_seed(1)
    n = (1 << 20) + 3  # not a multiple of 4: exercises the scalar tail
    p0 = torch.randn(n, device=dev)
    m0 = torch.randn(n, device=dev).abs() * 1e-3
    v0 = torch.randn(n, device=dev).abs() * 1e-4
    p_ref, m_ref, v_ref = p0.clone(), m0.clone(), v0.clone()
    p_na, m_na, v_na = p0.clone(), m0.clone(), v0.clone()
    p_nc, m_nc, v_nc = p0.clone(), m0.clone(), v0.clone()  # no clip (partial = NULL)
    b_ref = torch.empty(n, device=dev, dtype=torch.bfloat16)
    b_na = torch.empty(n, device=dev, dtype=torch.bfloat16)
    n_partial = 512
    scratch = torch.empty(n_partial, device=dev)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    hyper = (C.c_float(10.0), C.c_float(3e-4), C.c_float(0.9), C.c_float(0.999), C.c_float(1e-8), C.c_float(0.1))
    # an independent CPU statement: clip_grad_norm_(10) + torch.optim.AdamW from the same moments
    p_cpu = p0.cpu().clone().requires_grad_(True)
    opt = torch.optim.AdamW([p_cpu], lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.1)
    opt.state[p_cpu] = {"step": torch.tensor(0.0), "exp_avg": m0.cpu().clone(), "exp_avg_sq": v0.cpu().clone()}
    for step in (1, 2):
        g = torch.randn(n, device=dev) * (3.0 if step == 1 else 0.005)  # norm ~3000 clips, ~5 does not
        rc = lib.cdk_sumsq(_vp(g), n, _vp(scratch), n_partial, stream)
        assert rc == 0
        rc = lib.cdk_adamw(_vp(p_ref), _vp(g), _vp(m_ref), _vp(v_ref), _vp(b_ref), n, _vp(scratch), n_partial,
                           *hyper, step, C.c_float(1.0), stream)
        assert rc == 0
        rc = lib.cdk_adamw_clip_noalloc(_vp(p_na), _vp(g), _vp(m_na), _vp(v_na), _vp(b_na), n, n_partial, *hyper,
                                        step, C.c_float(1.0), stream)
        assert rc == 0
        rc = lib.cdk_adamw(_vp(p_nc), _vp(g), _vp(m_nc), _vp(v_nc), None, n, None, 0, *hyper, step, C.c_float(1.0),
                           stream)
        assert rc == 0
        torch.cuda.synchronize()
        p_cpu.grad = g.cpu()
        torch.nn.utils.clip_grad_norm_([p_cpu], max_norm=10.0)
        opt.step()
        for got, ref in ((p_na, p_ref), (m_na, m_ref), (v_na, v_ref)):
            assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6)
        # the same adamw kernel on the same inputs: the bf16 shadows are identical
        assert torch.equal(b_na, b_ref)
        assert torch.allclose(p_na.cpu(), p_cpu.detach(), rtol=1e-5, atol=1e-6)
        assert torch.allclose(m_na.cpu(), opt.state[p_cpu]["exp_avg"], rtol=1e-5, atol=1e-6)
        if step == 1:
            # the clip engaged: the unclipped update differs from the allocation-free one
            assert not torch.allclose(p_nc, p_na, rtol=1e-5, atol=1e-6)
    assert not torch.allclose(p_na, p0)


def test_noalloc_rejects_oversized_scratch_request():
    from chessdecoder_b200 import _lib
    lib = _lib.load()
    x = torch.zeros(16, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.cdk_adamw_clip_noalloc(_vp(x), _vp(x), _vp(x), _vp(x), None, 16, 4097, C.c_float(10.0),
                                    C.c_float(1e-3), C.c_float(0.9), C.c_float(0.999), C.c_float(1e-8),
                                    C.c_float(0.0), 1, C.c_float(1.0), stream)
    assert rc == -32
