"""The GRPO step (chessdecoder_b200/rl.py) on the GPU against the oracle
(oracle/rl.py, the fp32 restatement of chessdecoder/rl/log_probs.py and
rl/grpo.py): per-token log-probs of the thinking and final move actions, the
loss and every parameter gradient, on thinking-variation rows at S = 1024
with rollout / reference log-probs perturbed around the current policy so that
both clipping bounds and the KL term are active."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=1024, d_ff=384)


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return (a @ b / (a.norm() * b.norm()).clamp_min(1e-30)).item()


def _rl_batch(B, S, seed):
    from chessdecoder_b200 import data
    b = data.finetune_batches(1, B, S, seed=seed, min_lines=2, max_lines=3, min_depth=1, max_depth=3)[0]
    return {"input_ids": b["input_ids"], "block_id": b["block_id"], "wl_positions": b["wl_positions"],
            "d_positions": b["d_positions"], "wl_values": b["wl_targets"], "d_values": b["d_targets"],
            "thinking_move_mask": b["thinking_move_mask"], "final_move_mask": b["move_mask"],
            "move_token_ids": b["move_target_ids"].clamp_min(0)}


def test_grpo_step_matches_oracle():
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.engine import ModelConfig
    from chessdecoder_b200.rl import GRPOStep, prepare_rl_batch
    from oracle.model import OracleChessDecoder
    from oracle import rl as R
    torch.manual_seed(0)
    oracle = OracleChessDecoder(ModelConfig().vocab_size, **SMALL)
    sd = {k: v.detach().clone() for k, v in oracle.state_dict().items()}
    batch = _rl_batch(3, SMALL["max_seq_len"], seed=9)
    with torch.no_grad():
        lp0, mask = R.prefix_log_probs(oracle, batch)
    g = torch.Generator().manual_seed(1)
    old = lp0 + torch.randn(lp0.shape, generator=g) * 0.3
    ref = lp0 + torch.randn(lp0.shape, generator=g) * 0.2
    adv = torch.randn(3, generator=g)
    eps_lo, eps_hi, kl = 0.2, 0.28, 0.04
    lp = R.prefix_log_probs(oracle, batch)[0]
    loss = R.grpo_loss(lp, old, ref, mask.float(), adv, eps_lo, eps_hi, kl)
    loss.backward()
    step = GRPOStep(ModelConfig(**SMALL), device="cuda", state_dict=sd, clip_epsilon_low=eps_lo,
                    clip_epsilon_high=eps_hi, kl_coeff=kl)
    rb = prepare_rl_batch(batch, "cuda", old, ref, adv)
    got_lp, got_mask = step.log_probs(rb)
    torch.cuda.synchronize()
    assert torch.equal(got_mask.cpu(), mask)
    assert (got_lp.cpu()[mask] - lp0[mask]).abs().max().item() < 5e-2
    got_loss, lp_cur = step.forward_backward(rb)
    torch.cuda.synchronize()
    ref_loss = loss.item()
    assert abs(float(got_loss) - ref_loss) <= 2e-2 * max(abs(ref_loss), 1e-3), (float(got_loss), ref_loss)
    assert torch.allclose(lp_cur.cpu(), got_lp.cpu(), atol=1e-5)
    rp = dict(oracle.named_parameters())
    for name in step.store.names():
        gr = rp[name].grad
        if gr is None or gr.abs().max() == 0:
            continue
        c = cosine(step.store.grad_of(name).cpu(), gr)
        assert c >= 0.99, (name, c)
    step.optimizer_step()
    torch.cuda.synchronize()
    assert K.get_error() == 0
