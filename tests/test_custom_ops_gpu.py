"""The cdk:: custom ops on the GPU: the drop-in ChessDecoder with an explicit
``input_pos`` (model.py:156-157) against the fp32 oracle, the module under
``torch.compile(fullgraph=False)`` against eager, and the backbone op releasing
its saved activations with the autograd graph."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384)


def _cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def _models(seed=0):
    from chessdecoder_b200 import vocab as V
    from chessdecoder_b200.model import ChessDecoder
    from oracle.model import OracleChessDecoder
    torch.manual_seed(seed)
    ours = ChessDecoder(V.vocab_size, **SMALL).cuda()
    torch.manual_seed(seed)
    ref = OracleChessDecoder(V.vocab_size, **SMALL).cuda()
    return ours, ref


def _batch(S=128, B=3):
    from chessdecoder_b200 import data
    b = data.synthetic_batches(1, B, S, seed=5)[0]
    return {k: v.cuda() for k, v in b.items()}


@pytest.mark.parametrize("mask_type", ["causal", "prefix"])
def test_input_pos_matches_oracle(mask_type):
    ours, ref = _models()
    b = _batch()
    B, S = b["input_ids"].shape
    # RoPE attention depends on position differences only: stretched positions
    # (a uniform shift would change nothing)
    pos = (2 * torch.arange(S, device="cuda")).unsqueeze(0).expand(B, S)
    kw = dict(input_pos=pos, mask_type=mask_type, block_id=b["block_id"])
    h = ours(b["input_ids"], **kw)
    r = ref(b["input_ids"], **kw)
    assert _cosine(h, r) > 0.9999 and ((h - r).norm() / r.norm()).item() < 1e-2
    # and it differs from the default positions: the rotation really changed
    h0 = ours(b["input_ids"], mask_type=mask_type, block_id=b["block_id"])
    assert ((h0 - h).norm() / h.norm()).item() > 1e-3
    g = torch.randn_like(h)
    (h * g).sum().backward()
    (r * g).sum().backward()
    rp = dict(ref.named_parameters())
    for n, p in ours.named_parameters():
        if rp[n].grad is not None and float(rp[n].grad.abs().max()) > 0:
            assert _cosine(p.grad, rp[n].grad) > 0.999, n
        elif p.grad is not None:  # off the oracle's graph (no value placeholders): a zero gradient here
            assert float(p.grad.abs().max()) == 0.0, n
    with pytest.raises(NotImplementedError):
        ours(b["input_ids"], input_pos=torch.stack([torch.arange(S), torch.arange(S) + 1, torch.arange(S)]).cuda())


def test_module_under_torch_compile_matches_eager():
    from chessdecoder_b200.model import ChessDecoder  # noqa: F401
    ours, _ = _models()
    b = _batch()

    def loss_fn(model, ids, bid, mt):
        h = model(ids, mask_type="prefix", block_id=bid)
        logits = model.policy_head(h)
        return F.cross_entropy(logits.reshape(-1, logits.shape[-1]), mt.reshape(-1).clamp_min(0))

    args = (b["input_ids"], b["block_id"], b["move_target_ids"])
    eager = loss_fn(ours, *args)
    eager.backward()
    g_eager = {n: p.grad.clone() for n, p in ours.named_parameters() if p.grad is not None}
    ours.zero_grad(set_to_none=True)
    compiled = torch.compile(loss_fn, fullgraph=False)
    got = compiled(ours, *args)
    got.backward()
    assert abs(float(got) - float(eager)) <= 1e-3 * abs(float(eager))
    for n, g in g_eager.items():
        p = dict(ours.named_parameters())[n]
        assert p.grad is not None, n
        if float(g.abs().max()) == 0.0:  # off this loss's graph (the Fourier encoder): zero in both
            assert float(p.grad.abs().max()) == 0.0, n
        else:
            assert _cosine(p.grad, g) > 0.9999, n


def test_backbone_activations_are_released():
    from chessdecoder_b200 import ops
    ours, _ = _models()
    b = _batch()
    n0 = ops.saved_count()
    h = ours(b["input_ids"])
    assert ops.saved_count() == n0 + 1
    h.sum().backward()
    assert ops.saved_count() == n0
    with torch.no_grad():
        ours(b["input_ids"])
    assert ops.saved_count() == n0
    h = ours(b["input_ids"])
    del h  # graph dropped without a backward
    assert ops.saved_count() == n0
