"""The finetune step (chessdecoder/finetune/train.py:272-355) on the GPU
against the oracle's fp32 finetune loss: thinking-variation rows at S = 1024
(the tcgen05 long-sequence attention), a small model with the thinking head
trained; losses within 1e-2 relative, gradient cosine >= 0.999 for every
tensor (thinking head included), and one optimizer step that moves the
thinking head."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=1024, d_ff=384)


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def test_finetune_step_matches_oracle():
    from chessdecoder_b200 import data
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.engine import FINETUNE_LOSS_WEIGHTS, ModelConfig, TrainStep, prepare_batch
    from oracle.model import OracleChessDecoder
    from oracle.step import finetune_step_losses
    cfg = ModelConfig(**SMALL, finetune=True)
    torch.manual_seed(0)
    oracle = OracleChessDecoder(cfg.vocab_size, **SMALL)
    sd = {k: v.detach().clone() for k, v in oracle.state_dict().items()}
    batch = data.finetune_batches(1, 2, cfg.max_seq_len, seed=5, min_lines=2, max_lines=3, min_depth=1,
                                  max_depth=3)[0]
    assert batch["thinking_move_mask"].any() and batch["move_mask"].any()
    out = finetune_step_losses(oracle, batch, FINETUNE_LOSS_WEIGHTS)
    out["total"].backward()
    step = TrainStep(cfg, device="cuda", state_dict=sd, loss_weights=FINETUNE_LOSS_WEIGHTS, lr=3e-5)
    losses = step.forward_backward(prepare_batch(batch, "cuda")).cpu()
    for i, n in enumerate(["move", "board", "wl", "d", "think"]):
        ref = float(out[n].detach())
        assert abs(float(losses[i]) - ref) <= 1e-2 * max(abs(ref), 1e-6), (n, float(losses[i]), ref)
    rp = dict(oracle.named_parameters())
    assert "thinking_policy_head.weight" in step.store.names()
    for name in step.store.names():
        c = cosine(step.store.grad_of(name).cpu(), rp[name].grad)
        assert c >= 0.999, (name, c)
    before = step.store.param("thinking_policy_head.weight").clone()
    step.optimizer_step()
    torch.cuda.synchronize()
    assert not torch.equal(before, step.store.param("thinking_policy_head.weight"))
    assert K.get_error() == 0


def test_pretraining_leaves_thinking_head_alone():
    """Pretraining (finetune=False) keeps the thinking head out of AdamW: its
    weights are unchanged after a step, as PyTorch skips parameters without
    a gradient."""
    from chessdecoder_b200 import data
    from chessdecoder_b200.engine import ModelConfig, TrainStep
    cfg = ModelConfig(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=256, d_ff=384)
    step = TrainStep(cfg, device="cuda")
    w0 = step.store.thinking_weight.clone()
    step.step(data.synthetic_batches(1, 2, 256, seed=2)[0])
    torch.cuda.synchronize()
    assert torch.equal(w0, step.store.thinking_weight)
    assert "thinking_policy_head.weight" in step.store.state_dict()
