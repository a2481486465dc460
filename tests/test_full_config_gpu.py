"""Training-step parity at the benchmarked model size.

The B200 step against the fp32 oracle step (oracle/step.py, a restatement of
chessdecoder/train/train.py:157-253) at the reference's default pretraining
model -- E=1024, 16 heads, 12 layers, d_ff=1536, S=256
(chessdecoder/train/config.yaml:8-20; chessdecoder/models/model.py:75-136) --
on the same seeded synthetic batch and the same weights.  The oracle runs in
fp32 on the GPU (TF32 off), so the full batch is cheap.

Gates:
* bf16, B=64 (the benchmarked batch): each loss within 1e-2 relative, every
  parameter gradient cosine >= 0.999 (one named exception, below), board and
  move argmax agreement >= 99.9% at a briefly trained checkpoint (30 oracle
  steps).  At random init the full-size model's logits are nearly flat (top-2
  margins of a few 1e-3), so there every disagreement must be an oracle
  near-tie (margin < 0.02);
* fp8 recipe, B=128: losses within 3e-2 of the fp32 oracle, gradients
  against the recipe oracle (see the test);
* MoE, S=4096: routing agreement and parity given the same routing.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

FULL = dict(embed_dim=1024, num_heads=16, num_layers=12, max_seq_len=256, d_ff=1536)


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def _top2_margin(logits):
    t = logits.detach().float().topk(2, dim=-1).values
    return t[..., 0] - t[..., 1]


def _oracle(kw, seed=0, pretrain_steps=0, pretrain_batch=8, data_seed=3):
    """fp32 oracle on the GPU, seeded like the reference's constructor; with
    pretrain_steps > 0 it is first trained on its own synthetic stream."""
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import ModelConfig
    from oracle.model import OracleChessDecoder
    from oracle.step import train_step
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    cfg = ModelConfig(**kw)
    torch.manual_seed(seed)
    oracle = OracleChessDecoder(cfg.vocab_size, **kw).cuda()
    if pretrain_steps:
        opt = torch.optim.AdamW(oracle.parameters(), lr=1e-3, weight_decay=0.1)
        for b in data.synthetic_batches(pretrain_steps, pretrain_batch, cfg.max_seq_len, seed=data_seed + 100):
            train_step(oracle, opt, b)
        del opt
    oracle.zero_grad(set_to_none=True)
    return cfg, oracle


def compare(step, oracle, batch, loss_tol):
    """Runs both steps on `batch`; returns (per-loss (got, ref), per-tensor
    gradient cosines, board / move argmax agreement and the near-tie check)."""
    from chessdecoder_b200.engine import prepare_batch
    from oracle.step import step_losses
    out = step_losses(oracle, batch)
    out["total"].backward()
    db = prepare_batch(batch, "cuda")
    metrics = {"board_argmax": torch.empty(db.B * db.S, dtype=torch.int32, device="cuda"),
               "move_argmax": torch.empty(max(db.prow.numel(), 1), dtype=torch.int32, device="cuda")}
    losses = step.forward_backward(db, metrics).cpu()
    res = {"loss": {}, "cos": {}}
    for i, n in enumerate(["move", "board", "wl", "d"]):
        res["loss"][n] = (float(losses[i]), float(out[n].detach()))
    rp = dict(oracle.named_parameters())
    for name in step.store.names():
        rg = rp[name].grad
        res["cos"][name] = cosine(step.store.grad_of(name), rg) if rg is not None else float("nan")
    bm = out["board_mask"].reshape(-1)
    ba = metrics["board_argmax"].long()[bm]
    bo = out["board_argmax"].reshape(-1)[bm]
    mm = out["move_mask"].reshape(-1)
    ma = metrics["move_argmax"][: int(mm.sum())].long()
    mo = out["move_argmax"].reshape(-1)[mm]
    res["agree_board"] = (ba == bo).float().mean().item()
    res["agree_move"] = (ma == mo).float().mean().item()
    bl = out["board_logits"].reshape(-1, out["board_logits"].shape[-1])[bm]
    ml = out["move_logits"].reshape(-1, out["move_logits"].shape[-1])[mm]
    res["board_ties_only"] = bool((_top2_margin(bl)[ba != bo] < 0.02).all())
    res["move_ties_only"] = bool((_top2_margin(ml)[ma != mo] < 0.02).all())
    return res


def check(res, loss_tol, cos_min, exceptions=None):
    """Losses within loss_tol relative; every gradient cosine >= cos_min, or
    >= exceptions[name] for the named tensors."""
    exceptions = exceptions or {}
    for n, (got, ref) in res["loss"].items():
        assert abs(got - ref) <= loss_tol * max(abs(ref), 1e-6), (n, got, ref)
    worst = sorted(res["cos"].items(), key=lambda kv: kv[1])[:5]
    assert all(c >= exceptions.get(n, cos_min) for n, c in res["cos"].items()), worst


@pytest.mark.parametrize("pretrain", [0, 30])
def test_full_config_bf16_step_matches_oracle(pretrain):
    from chessdecoder_b200 import data, kernels
    from chessdecoder_b200.engine import TrainStep
    cfg, oracle = _oracle(FULL, pretrain_steps=pretrain)
    sd = {k: v.detach().cpu().clone() for k, v in oracle.state_dict().items()}
    step = TrainStep(cfg, device="cuda", state_dict=sd)
    batch = data.synthetic_batches(1, 64, cfg.max_seq_len, seed=3)[0]
    res = compare(step, oracle, batch, 1e-2)
    # At the trained checkpoint the 128 Fourier frequencies are the one tensor
    # below 0.999 (0.9988-0.9995 over four runs; 0.99998 at random init): each
    # entry is a sum over the ~940 value-placeholder rows of 2 pi x (cos, sin)
    # terms weighted by the gradient that reaches those rows through the 12
    # bf16 layers (cosine 0.99988 to the oracle's there), and the cancelling
    # sum amplifies that error.  Every other tensor is gated at 0.999.
    check(res, 1e-2, 0.999, {"fourier_encoder.frequencies": 0.998} if pretrain else None)
    if pretrain:
        assert res["agree_board"] >= 0.999, res["agree_board"]
        assert res["agree_move"] >= 0.999, res["agree_move"]
    else:
        assert res["board_ties_only"] and res["move_ties_only"], (res["agree_board"], res["agree_move"])
    assert kernels.get_error() == 0


def test_full_config_fp8_step_matches_fp8_recipe_oracle():
    """fp8 variant at B=128.  Against the fp32 oracle each loss is within 3e-2.
    Gradients are gated against the oracle that applies the same fp8 recipe
    (oracle/fp8.py: e4m3 inputs / weights, e5m2 output gradients, per-tensor
    scaling) at cosine >= 0.995.  Not 0.999: one e5m2 rounding of a gradient
    (2 mantissa bits, relative spacing up to 2^-2) already bounds its cosine to
    the unrounded gradient near 0.998, and two implementations whose inputs
    differ at the bf16 level round about 1-2% of the elements of every cast to
    neighbouring e5m2 values; over the 24 gradient casts of a 12-layer
    backward the measured per-tensor cosines are 0.9965-0.9999 (0.9958 against
    the fp32 oracle)."""
    from chessdecoder_b200 import data, kernels
    from chessdecoder_b200.engine import TrainStep
    from oracle.fp8 import Fp8OracleChessDecoder
    cfg, oracle = _oracle(FULL)
    sd = {k: v.detach().cpu().clone() for k, v in oracle.state_dict().items()}
    batch = data.synthetic_batches(1, 128, cfg.max_seq_len, seed=3)[0]
    step = TrainStep(cfg, device="cuda", state_dict=sd, fp8=True)
    res = compare(step, oracle, batch, 3e-2)
    for n, (got, ref) in res["loss"].items():
        assert abs(got - ref) <= 3e-2 * max(abs(ref), 1e-6), (n, got, ref)
    del oracle, step
    torch.cuda.empty_cache()
    torch.manual_seed(0)
    f8o = Fp8OracleChessDecoder(cfg.vocab_size, **FULL).cuda()
    f8o.load_state_dict({k: v.cuda() for k, v in sd.items()})
    step8 = TrainStep(cfg, device="cuda", state_dict=sd, fp8=True)
    res8 = compare(step8, f8o, batch, 3e-2)
    check(res8, 3e-2, 0.995)
    assert kernels.get_error() == 0


def test_full_config_moe_step_matches_oracle():
    """MoE variant (8 experts, top-2, capacity 1.25) at S=4096 with a reduced
    batch of 2 thinking-variation sequences.  The top-2 and capacity choices
    are discrete: a bf16-vs-fp32 near-tie of two router probabilities sends a
    token to another expert.  So (1) the CUDA step's choices must agree with
    the fp32 oracle's own on >= 99% of (token, choice) decisions, and (2) given
    the CUDA step's choices (oracle/moe.py ``forced``) the oracle's losses are
    within 1e-2 and every gradient has cosine >= 0.999."""
    from chessdecoder_b200 import data, kernels
    from chessdecoder_b200.engine import TrainStep, prepare_batch
    from oracle.step import step_losses
    kw = dict(FULL, max_seq_len=4096, moe_experts=8, moe_capacity=1.25)
    cfg, oracle = _oracle(kw)
    sd = {k: v.detach().cpu().clone() for k, v in oracle.state_dict().items()}
    batch = data.thinking_batches(1, 2, cfg.max_seq_len, seed=5)[0]
    step = TrainStep(cfg, device="cuda", state_dict=sd)
    step.backbone.keep_routing = True
    db = prepare_batch(batch, "cuda")
    losses = step.forward_backward(db).cpu()
    BS = db.B * db.S
    routing = step.backbone.routing
    # (1) the oracle's own decisions, pass 1 then pass 2 of each layer
    for layer in oracle.layers:
        layer.mlp.record = []
    with torch.no_grad():
        step_losses(oracle, batch)
    agree = total = 0
    for i, layer in enumerate(oracle.layers):
        ex, sl = routing[i]
        for p, (idx, keep) in enumerate(layer.mlp.record):
            e = ex[p * BS:(p + 1) * BS].long()
            k = sl[p * BS:(p + 1) * BS] >= 0
            agree += int(((e == idx) & (k == keep)).sum())
            total += idx.numel()
        layer.mlp.record = None
    assert agree / total >= 0.99, agree / total
    # (2) parity given the CUDA step's decisions
    for i, layer in enumerate(oracle.layers):
        ex, sl = routing[i]
        layer.mlp.forced = [(ex[p * BS:(p + 1) * BS], sl[p * BS:(p + 1) * BS] >= 0) for p in range(2)]
    out = step_losses(oracle, batch)
    out["total"].backward()
    for j, n in enumerate(["move", "board", "wl", "d"]):
        ref = float(out[n].detach())
        assert abs(float(losses[j]) - ref) <= 1e-2 * max(abs(ref), 1e-6), (n, float(losses[j]), ref)
    rp = dict(oracle.named_parameters())
    cos = {name: cosine(step.store.grad_of(name), rp[name].grad) for name in step.store.names()}
    assert all(c >= 0.999 for c in cos.values()), sorted(cos.items(), key=lambda kv: kv[1])[:5]
    assert kernels.get_error() == 0
