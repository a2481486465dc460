"""Training-step parity: the B200 step against the fp32 oracle step
(oracle/step.py, a restatement of chessdecoder/train/train.py:157-253) on the
same seeded synthetic batch and the same initial weights.

Gates (from the task statement for bf16): each loss within 1e-2 relative, every
parameter gradient with cosine similarity >= 0.999 against the oracle's, and
argmax agreement >= 99.9% on board rows and move rows.  One full optimizer
step is also compared against torch.optim.AdamW + clip_grad_norm_ applied to
the oracle's gradients.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384)


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def _setup(cfg_kw, B, seed=0, data_seed=3, pretrain_steps=0):
    """Same initial weights for the oracle and the B200 step.  With
    pretrain_steps > 0 the oracle is first trained for that many fp32 steps on
    its own synthetic stream (a briefly trained checkpoint, where argmax
    decisions are no longer random-init near-ties) and the B200 step starts
    from that checkpoint."""
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import ModelConfig, TrainStep
    from oracle.model import OracleChessDecoder
    from oracle.step import train_step
    cfg = ModelConfig(**cfg_kw)
    torch.manual_seed(seed)
    oracle = OracleChessDecoder(cfg.vocab_size, **cfg_kw)
    if pretrain_steps:
        opt = torch.optim.AdamW(oracle.parameters(), lr=1e-3, weight_decay=0.1)
        for b in data.synthetic_batches(pretrain_steps, 4, cfg.max_seq_len, seed=data_seed + 100):
            train_step(oracle, opt, b)
        oracle.zero_grad(set_to_none=True)
    sd = {k: v.detach().clone() for k, v in oracle.state_dict().items()}
    step = TrainStep(cfg, device="cuda", state_dict=sd)
    batch = data.synthetic_batches(1, B, cfg.max_seq_len, seed=data_seed)[0]
    return cfg, oracle, step, batch


def _top2_margin(logits):
    t = logits.detach().float().topk(2, dim=-1).values
    return t[..., 0] - t[..., 1]


@pytest.mark.parametrize("cfg_kw,B,pretrain", [(SMALL, 4, 0), (SMALL, 4, 30),
                                                (dict(SMALL, num_layers=1, max_seq_len=136), 3, 0)])
def test_step_matches_oracle(cfg_kw, B, pretrain):
    from chessdecoder_b200.engine import prepare_batch
    from oracle.step import step_losses
    cfg, oracle, step, batch = _setup(cfg_kw, B, pretrain_steps=pretrain)
    out = step_losses(oracle, batch)
    out["total"].backward()
    db = prepare_batch(batch, "cuda")
    metrics = {"board_argmax": torch.empty(db.B * db.S, dtype=torch.int32, device="cuda"),
               "move_argmax": torch.empty(max(db.prow.numel(), 1), dtype=torch.int32, device="cuda")}
    losses = step.forward_backward(db, metrics).cpu()
    names = ["move", "board", "wl", "d"]
    for i, n in enumerate(names):
        ref = float(out[n].detach())
        assert abs(float(losses[i]) - ref) <= 1e-2 * max(abs(ref), 1e-6), (n, float(losses[i]), ref)
    ref_params = dict(oracle.named_parameters())
    for name in step.store.names():
        g = step.store.grad_of(name).cpu()
        rg = ref_params[name].grad
        assert rg is not None, name
        c = cosine(g, rg)
        assert c >= 0.999, (name, c)
    # argmax agreement on supervised rows (board rows of pass 1, move rows of pass 2)
    bm = out["board_mask"].reshape(-1)
    ba = metrics["board_argmax"].cpu().long()[bm]
    bo = out["board_argmax"].reshape(-1)[bm]
    mm = out["move_mask"].reshape(-1)
    ma = metrics["move_argmax"][: int(mm.sum())].cpu().long()
    mo = out["move_argmax"].reshape(-1)[mm]
    agree_b = (ba == bo).float().mean().item()
    agree_m = (ma == mo).float().mean().item()
    if pretrain:
        assert agree_b >= 0.999, agree_b
        assert agree_m >= 0.999, agree_m
    else:
        # random init: logits are nearly flat, so a disagreement must be a near-tie of the oracle's logits
        bl = out["board_logits"].reshape(-1, out["board_logits"].shape[-1])[bm]
        assert (_top2_margin(bl)[ba != bo] < 0.02).all(), agree_b
        ml = out["move_logits"].reshape(-1, out["move_logits"].shape[-1])[mm]
        assert (_top2_margin(ml)[ma != mo] < 0.02).all(), agree_m
        assert agree_b >= 0.99 and agree_m >= 0.99
    from chessdecoder_b200 import kernels
    assert kernels.get_error() == 0


def test_optimizer_step_matches_torch_adamw():
    """Fused clip + AdamW over the flat buffers vs clip_grad_norm_ + torch.optim.AdamW."""
    from chessdecoder_b200.engine import prepare_batch
    from oracle.step import step_losses
    cfg, oracle, step, batch = _setup(SMALL, 2)
    db = prepare_batch(batch, "cuda")
    step.forward_backward(db)
    # hand the B200 gradients to a torch AdamW on a copy of the weights
    params = {n: step.store.param(n).detach().cpu().clone().requires_grad_(True) for n in step.store.names()}
    for n, p in params.items():
        p.grad = step.store.grad_of(n).detach().cpu().clone()
    opt = torch.optim.AdamW(list(params.values()), lr=3e-4, weight_decay=0.1)
    torch.nn.utils.clip_grad_norm_(list(params.values()), max_norm=10.0)
    opt.step()
    step.optimizer_step()
    for n, p in params.items():
        got = step.store.param(n).cpu()
        assert torch.allclose(got, p.detach(), rtol=1e-5, atol=1e-6), n
        # the bf16 shadow is exactly bf16(updated fp32 parameter)
        g16 = step.store.bf16(n).float().cpu()
        assert torch.equal(g16, got.to(torch.bfloat16).float()), n


def test_two_steps_loss_decreases_on_repeated_batch():
    from chessdecoder_b200.engine import prepare_batch
    cfg, oracle, step, batch = _setup(SMALL, 4)
    db = prepare_batch(batch, "cuda")
    l0 = step.total(step.forward_backward(db)).item()
    step.optimizer_step()
    for _ in range(3):
        step.forward_backward(db)
        step.optimizer_step()
    l1 = step.total(step.forward_backward(db)).item()
    assert l1 < l0
