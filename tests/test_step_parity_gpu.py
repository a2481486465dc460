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


def _setup(cfg_kw, B, seed=0, data_seed=3):
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import ModelConfig, TrainStep
    from oracle.model import OracleChessDecoder
    cfg = ModelConfig(**cfg_kw)
    torch.manual_seed(seed)
    oracle = OracleChessDecoder(cfg.vocab_size, **cfg_kw)
    sd = {k: v.clone() for k, v in oracle.state_dict().items()}
    step = TrainStep(cfg, device="cuda", state_dict=sd)
    batch = data.synthetic_batches(1, B, cfg.max_seq_len, seed=data_seed)[0]
    return cfg, oracle, step, batch


@pytest.mark.parametrize("cfg_kw,B", [(SMALL, 4), (dict(SMALL, num_layers=1, max_seq_len=136), 3)])
def test_step_matches_oracle(cfg_kw, B):
    from chessdecoder_b200.engine import prepare_batch
    from oracle.step import step_losses
    cfg, oracle, step, batch = _setup(cfg_kw, B)
    out = step_losses(oracle, batch)
    out["total"].backward()
    db = prepare_batch(batch, "cuda")
    metrics = {"board_argmax": torch.empty(db.B * db.S, dtype=torch.int32, device="cuda"),
               "move_argmax": torch.empty(max(db.prow.numel(), 1), dtype=torch.int32, device="cuda")}
    losses = step.forward_backward(db, metrics).cpu()
    names = ["move", "board", "wl", "d"]
    for i, n in enumerate(names):
        ref = float(out[n])
        assert abs(float(losses[i]) - ref) <= 1e-2 * max(abs(ref), 1e-6), (n, float(losses[i]), ref)
    ref_params = dict(oracle.named_parameters())
    for name in step.store.names():
        g = step.store.grad_of(name).cpu()
        rg = ref_params[name].grad
        assert rg is not None, name
        c = cosine(g, rg)
        assert c >= 0.999, (name, c)
    # argmax agreement on supervised rows
    bm = out["board_mask"].reshape(-1)
    ba = metrics["board_argmax"].cpu().long()
    agree = (ba[bm] == out["board_argmax"].reshape(-1)[bm]).float().mean().item()
    assert agree >= 0.999, agree
    mm = out["move_mask"].reshape(-1)
    ma = metrics["move_argmax"][: int(mm.sum())].cpu().long()
    agree_m = (ma == out["move_argmax"].reshape(-1)[mm]).float().mean().item()
    assert agree_m >= 0.999, agree_m
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
        g16 = step.store.bf16(n).float().cpu()
        assert torch.allclose(g16, p.detach().to(torch.bfloat16).float()), n


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
