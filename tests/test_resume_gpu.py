"""Gradient accumulation, YAML construction and checkpoint / resume of the
fused step (chessdecoder/train/train.py:81-104,244-253;
chessdecoder/utils/training.py:136-157)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384)
CONF = {"model": SMALL, "training": {"learning_rate": 3e-4, "weight_decay": 0.1, "gradient_accumulation_steps": 2,
                                     "use_amp": True},
        "loss": {"move_weight": 5.0, "board_weight": 1.0, "wl_weight": 1.0, "d_weight": 1.0}}


def _cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def test_accumulated_gradients_match_oracle():
    """Two micro-batches: the summed gradient equals the oracle's gradient of
    (loss_1 + loss_2) / 2 -- the flat buffer holds the sum, the 1/2 is applied
    by the optimizer kernel."""
    from chessdecoder_b200 import data
    from chessdecoder_b200.config import step_from_config
    from chessdecoder_b200.engine import prepare_batch
    from oracle.model import OracleChessDecoder
    from oracle.step import step_losses
    torch.manual_seed(0)
    oracle = OracleChessDecoder(1968, **SMALL)
    sd = {k: v.detach().clone() for k, v in oracle.state_dict().items()}
    step = step_from_config(CONF, state_dict=sd)
    assert step.grad_accum == 2 and step.lr == 3e-4
    micro = data.synthetic_batches(2, 3, 256, seed=9)
    for i, b in enumerate(micro):
        step.forward_backward(prepare_batch(b, "cuda"), zero_grad=i == 0)
        (step_losses(oracle, b)["total"] / 2).backward()
    rp = dict(oracle.named_parameters())
    for n in step.store.names():
        assert _cosine(step.store.grad_of(n).cpu() / 2, rp[n].grad) > 0.999, n


def test_checkpoint_resume_continues_identically():
    from chessdecoder_b200 import data
    from chessdecoder_b200.config import step_from_config
    from oracle.model import OracleChessDecoder
    a = step_from_config(CONF)
    batches = data.synthetic_batches(5, 2, 256, seed=21)
    for i in range(2):
        a.step_accumulated(batches[2 * i:2 * i + 2])
    ck = a.checkpoint(step=2)
    assert set(ck) >= {"step", "model_state_dict", "optimizer_state_dict", "scaler_state_dict"}
    # the reference's optimizer loads it
    ref_opt = torch.optim.AdamW(OracleChessDecoder(1968, **SMALL).parameters(), lr=3e-4, weight_decay=0.1)
    ref_opt.load_state_dict(ck["optimizer_state_dict"])
    b = step_from_config(CONF)
    assert b.load_checkpoint(ck) == 2 and b.store.step == 2
    for s in (a, b):
        s.step(batches[4])
    for n in a.store.names():
        pa, pb = a.store.param(n), b.store.param(n)
        assert torch.allclose(pa, pb, rtol=1e-4, atol=1e-6), n
    assert torch.allclose(a.store.exp_avg_sq, b.store.exp_avg_sq, rtol=1e-3, atol=1e-12)


def test_pipelined_loop_equals_stepwise():
    """TrainStep.run (batch i+1 enqueued before step i's losses are read)
    gives the losses and parameters of step() with a read after each (equal
    up to the order of the weight-gradient GEMMs' atomic split-K sums)."""
    from chessdecoder_b200 import data
    from chessdecoder_b200.config import step_from_config
    a, b = step_from_config(CONF), step_from_config(CONF)
    batches = data.synthetic_batches(4, 2, 256, seed=33)
    seq = [a.step(x).cpu() for x in batches]
    got = list(b.run(iter(batches)))
    assert [i for i, _ in got] == list(range(len(batches)))
    for (_, lv), ref in zip(got, seq):
        assert torch.allclose(lv, ref, rtol=1e-3, atol=1e-5)
    assert ((a.store.flat - b.store.flat).norm() / a.store.flat.norm()).item() < 1e-4
