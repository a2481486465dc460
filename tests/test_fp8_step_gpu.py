"""The fp8 variant of the training step (backbone linears on e4m3 / e5m2
tensor cores with per-tensor delayed scaling) against the fp32 oracle step.

Gates: each loss within 3e-2 relative of the oracle's (the fp8 tolerance of
the task statement); every parameter gradient with cosine >= 0.99 against the
oracle's; over several steps the fp8 step tracks the bf16 step's losses within
3e-2 and the scaling state stays finite.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384)


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def _oracle_and_sd(seed=0):
    from chessdecoder_b200.engine import ModelConfig
    from oracle.model import OracleChessDecoder
    cfg = ModelConfig(**SMALL)
    torch.manual_seed(seed)
    oracle = OracleChessDecoder(cfg.vocab_size, **SMALL)
    sd = {k: v.detach().clone() for k, v in oracle.state_dict().items()}
    return cfg, oracle, sd


def test_fp8_step_matches_oracle():
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import TrainStep, prepare_batch
    from oracle.step import step_losses
    cfg, oracle, sd = _oracle_and_sd()
    batch = data.synthetic_batches(1, 4, cfg.max_seq_len, seed=3)[0]
    out = step_losses(oracle, batch)
    out["total"].backward()
    step = TrainStep(cfg, device="cuda", state_dict=sd, fp8=True)
    losses = step.forward_backward(prepare_batch(batch, "cuda")).cpu()
    for i, n in enumerate(["move", "board", "wl", "d"]):
        ref = float(out[n].detach())
        assert abs(float(losses[i]) - ref) <= 3e-2 * max(abs(ref), 1e-6), (n, float(losses[i]), ref)
    ref_params = dict(oracle.named_parameters())
    for name in step.store.names():
        c = cosine(step.store.grad_of(name).cpu(), ref_params[name].grad)
        assert c >= 0.99, (name, c)
    from chessdecoder_b200 import kernels as K
    assert K.get_error() == 0


def test_fp8_steps_track_bf16():
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import TrainStep
    cfg, _, sd = _oracle_and_sd()
    f8 = TrainStep(cfg, device="cuda", state_dict=sd, fp8=True)
    bf = TrainStep(cfg, device="cuda", state_dict=sd)
    for b in data.synthetic_batches(6, 4, cfg.max_seq_len, seed=21):
        l8 = f8.step(b).cpu()
        lb = bf.step(b).cpu()
        for i in range(4):
            r = float(lb[i])
            assert abs(float(l8[i]) - r) <= 3e-2 * max(abs(r), 1e-6), (i, float(l8[i]), r)
    st = f8.fp8
    assert st.steps == 6
    assert torch.isfinite(st.scale).all() and (st.scale > 0).all()
    assert float(st.history[:, :6].min()) > 0.0  # every site saw a nonzero amax in every step
