"""MoE variant on the GPU.

* the routing kernel against oracle/moe.py's rules (top-2 experts and
  renormalised weights, capacity slots: first choices then second choices in
  token order, per segment), dispatch / combine and their backward against
  plain PyTorch statements;
* the tiled attention kernels at the variant's long sequences (S = 1024, 4096);
* the MoE training step (8 experts, top-2, capacity 1.25, and a tight capacity
  that forces drops) against the fp32 oracle step: losses within 1e-2 relative,
  gradient cosine >= 0.999 per tensor.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def K():
    from chessdecoder_b200 import kernels
    kernels.lib()
    return kernels


def _route_ref(logits, n_seg, cap):
    """Oracle routing on fp32 logits, segment by segment."""
    T, X = logits.shape
    seg = T // n_seg
    p = torch.softmax(logits, -1)
    v, idx = torch.topk(p, 2, dim=-1)
    w = v / v.sum(-1, keepdim=True)
    slot = torch.full((T, 2), -1, dtype=torch.long)
    for g in range(n_seg):
        fill = [0] * X
        for k in range(2):
            for t in range(g * seg, (g + 1) * seg):
                e = int(idx[t, k])
                if fill[e] < cap:
                    slot[t, k] = e * n_seg * cap + g * cap + fill[e]
                fill[e] += 1
    return p, idx, w, slot


@pytest.mark.parametrize("T,X,n_seg,cf", [(3000, 8, 2, 1.25), (2048, 8, 1, 0.5), (4096, 4, 2, 2.0)])
def test_moe_route_matches_oracle_rules(K, T, X, n_seg, cf):
    g = torch.Generator().manual_seed(T + X)
    logits = torch.randn(T, X, generator=g)
    cap = math.ceil(cf * 2 * (T // n_seg) / X)
    p_ref, idx_ref, w_ref, slot_ref = _route_ref(logits, n_seg, cap)
    lg = logits.to(DEV)
    expert = torch.empty(T, 2, dtype=torch.int32, device=DEV)
    weight = torch.empty(T, 2, device=DEV)
    probs = torch.empty(T, X, device=DEV)
    slot = torch.empty(T, 2, dtype=torch.int32, device=DEV)
    R = X * n_seg * cap
    src = torch.empty(R, dtype=torch.int32, device=DEV)
    ws = torch.empty(K.moe_route_workspace(T, n_seg, X), dtype=torch.uint8, device=DEV)
    K.moe_route(lg, n_seg, cap, expert, weight, probs, slot, src, ws)
    torch.cuda.synchronize()
    assert torch.equal(expert.cpu().long(), idx_ref)
    assert torch.allclose(weight.cpu(), w_ref, atol=1e-6)
    assert torch.allclose(probs.cpu(), p_ref, atol=1e-6)
    assert torch.equal(slot.cpu().long(), slot_ref)
    # src inverts slot; unfilled rows are -1
    src_ref = torch.full((R,), -1, dtype=torch.long)
    for t in range(T):
        for k in range(2):
            if slot_ref[t, k] >= 0:
                src_ref[slot_ref[t, k]] = t
    assert torch.equal(src.cpu().long(), src_ref)
    assert K.get_error() == 0


def test_moe_dispatch_combine_and_backward(K):
    torch.manual_seed(1)
    T, E, X, n_seg = 1000, 256, 4, 1
    cap = math.ceil(1.0 * 2 * T / X)
    logits = torch.randn(T, X, device=DEV)
    expert = torch.empty(T, 2, dtype=torch.int32, device=DEV)
    weight = torch.empty(T, 2, device=DEV)
    probs = torch.empty(T, X, device=DEV)
    slot = torch.empty(T, 2, dtype=torch.int32, device=DEV)
    R = X * cap
    src = torch.empty(R, dtype=torch.int32, device=DEV)
    ws = torch.empty(K.moe_route_workspace(T, n_seg, X), dtype=torch.uint8, device=DEV)
    K.moe_route(logits, n_seg, cap, expert, weight, probs, slot, src, ws)
    x = torch.randn(T, E, device=DEV).to(torch.bfloat16)
    xe = torch.empty(R, E, device=DEV, dtype=torch.bfloat16)
    K.moe_dispatch(x, src, xe)
    s = src.long()
    ref_xe = torch.where((s >= 0)[:, None], x[s.clamp_min(0)], torch.zeros_like(x[:1]))
    assert torch.equal(xe, ref_xe)
    ye = torch.randn(R, E, device=DEV).to(torch.bfloat16)
    resid = torch.randn(T, E, device=DEV)
    out = torch.empty(T, E, device=DEV)
    K.moe_combine(ye, slot, weight, resid, out)
    sl = slot.long()
    ref = resid.clone()
    for k in range(2):
        ok = sl[:, k] >= 0
        ref[ok] += weight[ok, k:k + 1] * ye[sl[ok, k]].float()
    assert torch.allclose(out, ref, atol=1e-4, rtol=1e-5)
    # backward of the combine
    dout = torch.randn(T, E, device=DEV)
    dye = torch.empty(R, E, device=DEV, dtype=torch.bfloat16)
    dweight = torch.empty(T, 2, device=DEV)
    K.moe_combine_bwd(dout, ye, slot, weight, dye, dweight)
    ref_dye = torch.zeros(R, E, device=DEV)
    ref_dw = torch.zeros(T, 2, device=DEV)
    for k in range(2):
        ok = sl[:, k] >= 0
        ref_dye[sl[ok, k]] = weight[ok, k:k + 1] * dout[ok]
        ref_dw[ok, k] = (dout[ok] * ye[sl[ok, k]].float()).sum(1)
    assert torch.allclose(dye.float(), ref_dye, atol=2e-2, rtol=1e-2)
    assert torch.allclose(dweight, ref_dw, atol=1e-3, rtol=1e-4)
    # router backward against autograd through softmax -> top-2 renormalisation
    lg = logits.clone().requires_grad_(True)
    p = torch.softmax(lg, -1)
    v = torch.gather(p, 1, expert.long())
    w = v / v.sum(-1, keepdim=True)
    (w * dweight).sum().backward()
    dlog = torch.empty(T, 8, device=DEV, dtype=torch.bfloat16)
    K.moe_route_bwd(probs, expert, dweight, dlog)
    assert torch.allclose(dlog[:, :X].float(), lg.grad, atol=1e-3, rtol=1e-2)
    # gather-sum (un-dispatch)
    dxe = torch.randn(R, E, device=DEV).to(torch.bfloat16)
    acc = torch.empty(T, E, device=DEV)
    K.moe_gather_sum(dxe, slot, acc)
    ref_acc = torch.zeros(T, E, device=DEV)
    for k in range(2):
        ok = sl[:, k] >= 0
        ref_acc[ok] += dxe[sl[ok, k]].float()
    assert torch.allclose(acc, ref_acc, atol=1e-5)
    torch.cuda.synchronize()
    assert K.get_error() == 0


@pytest.mark.parametrize("S,nseq,n_causal", [(301, 3, 1), (1024, 2, 1), (4096, 2, 1)])
def test_attention_long_sequences(K, S, nseq, n_causal):
    """The tiled kernels (S > 256) on thinking-row block structure."""
    from chessdecoder_b200 import data
    H = 2
    E = H * 64
    g = torch.Generator().manual_seed(S)
    qkv = (torch.randn(nseq * S, 3 * E, generator=g) * 0.8).to(DEV).to(torch.bfloat16)
    bid = data.thinking_batches(1, nseq - n_causal, S, seed=2)[0]["block_id"]
    bid32 = bid.to(torch.int32).to(DEV).contiguous()
    meta = K.attn_meta(bid32, S)
    out = torch.empty(nseq * S, E, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(nseq * H * S, device=DEV)
    K.attn_fwd(qkv, out, lse, nseq, n_causal, S, H, bid32, meta)
    # reference
    q, k, v = qkv.float().view(nseq, S, 3, H, 64).unbind(2)
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool, device=DEV))
    masks = [causal] * n_causal + [causal | (bid[r].to(DEV)[:, None] == bid[r].to(DEV)[None, :])
                                   for r in range(nseq - n_causal)]
    mask = torch.stack(masks)[:, None]
    qf, kf, vf = (t.clone().requires_grad_(True) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qf, kf, vf, attn_mask=mask)
    ref_o = ref.transpose(1, 2).reshape(nseq * S, E)
    err = ((out.float() - ref_o).norm() / ref_o.norm()).item()
    assert err < 1e-2, err
    dout = (torch.randn(nseq * S, E, generator=g) * 0.5).to(DEV).to(torch.bfloat16)
    ref_o.backward(dout.float())
    dqkv = torch.empty_like(qkv)
    dsum = torch.empty(nseq * H * S, device=DEV)
    K.attn_bwd(qkv, out, dout, lse, dsum, dqkv, nseq, n_causal, S, H, bid32, meta)
    torch.cuda.synchronize()
    dq, dk, dv = dqkv.float().view(nseq, S, 3, H, 64).unbind(2)
    for got, r in ((dq, qf.grad), (dk, kf.grad), (dv, vf.grad)):
        r = r.transpose(1, 2)
        e = ((got - r).norm() / r.norm()).item()
        assert e < 2e-2, e
    assert K.get_error() == 0


MOE_SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384, moe_experts=8)


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


@pytest.mark.parametrize("capacity", [1.25, 0.5])
def test_moe_step_matches_oracle(capacity):
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import ModelConfig, TrainStep, prepare_batch
    from oracle.model import OracleChessDecoder
    from oracle.step import step_losses
    kw = dict(MOE_SMALL, moe_capacity=capacity)
    cfg = ModelConfig(**kw)
    torch.manual_seed(0)
    oracle = OracleChessDecoder(cfg.vocab_size, **kw)
    sd = {k: v.detach().clone() for k, v in oracle.state_dict().items()}
    batch = data.synthetic_batches(1, 4, cfg.max_seq_len, seed=3)[0]
    out = step_losses(oracle, batch)
    out["total"].backward()
    step = TrainStep(cfg, device="cuda", state_dict=sd)
    losses = step.forward_backward(prepare_batch(batch, "cuda")).cpu()
    for i, n in enumerate(["move", "board", "wl", "d"]):
        ref = float(out[n].detach())
        assert abs(float(losses[i]) - ref) <= 1e-2 * max(abs(ref), 1e-6), (n, float(losses[i]), ref)
    rp = dict(oracle.named_parameters())
    for name in step.store.names():
        c = cosine(step.store.grad_of(name).cpu(), rp[name].grad)
        assert c >= 0.999, (name, c)
    from chessdecoder_b200 import kernels as K
    assert K.get_error() == 0
