"""ORACLE (test infrastructure only): the reference's GRPO policy-gradient
path restated in fp32.

* ``group_advantages`` / ``normalize_advantages`` restate
  chessdecoder/rl/grpo.py:17-55;
* ``grpo_loss`` restates chessdecoder/rl/grpo.py:58-110 (per-token ratio,
  Clip-Higher clipping, Schulman KL, normalisation by the action tokens);
* ``prefix_log_probs`` restates chessdecoder/rl/log_probs.py:19-101 for the
  move actions: the prefix pass (Fourier values snapped to bucket centres),
  then log_softmax of the thinking head at ``thinking_move_mask`` rows and of
  the policy head at ``final_move_mask`` rows, gathered at ``move_token_ids``.
``grpo_loss`` and the advantage helpers are pinned against the reference's own
functions by tests/golden/rl_reference.pt.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def group_advantages(rewards: torch.Tensor, eps: float = 1e-8):
    mean = rewards.mean(dim=1, keepdim=True)
    std = rewards.std(dim=1, keepdim=True)
    diverse = std.squeeze(1) > eps
    return torch.where(diverse.unsqueeze(1), rewards - mean, torch.zeros_like(rewards)), diverse


def normalize_advantages(adv: torch.Tensor, eps: float = 1e-8):
    std = adv.std()
    if std < eps:
        return torch.zeros_like(adv)
    return (adv - adv.mean()) / (std + eps)


def grpo_loss(lp, old_lp, ref_lp, mask, adv, eps_low, eps_high, kl_coeff):
    ratio = torch.exp(lp - old_lp)
    a = adv.unsqueeze(1)
    obj = torch.min(ratio * a, torch.clamp(ratio, 1.0 - eps_low, 1.0 + eps_high) * a)
    rr = torch.exp(lp - ref_lp)
    kl = (rr - 1) - torch.log(rr + 1e-8)
    per_token = -obj + kl_coeff * kl
    return (per_token * mask).sum() / mask.sum().clamp(min=1)


def prefix_log_probs(model, batch):
    """Per-token log-probs [B, S] at the move actions and the action mask."""
    dev = next(model.parameters()).device
    b = {k: v.to(dev) for k, v in batch.items()}
    wl_pos, d_pos = b["wl_positions"], b["d_positions"]
    wl_in = torch.zeros_like(b["wl_values"])
    d_in = torch.zeros_like(b["d_values"])
    if wl_pos.any():
        wl_in[wl_pos] = model.discretize_to_bucket(b["wl_values"][wl_pos], model.wl_bucket_centers)
    if d_pos.any():
        d_in[d_pos] = model.discretize_to_bucket(b["d_values"][d_pos], model.d_bucket_centers)
    h = model(b["input_ids"], mask_type="prefix", block_id=b["block_id"], wl_values=wl_in, d_values=d_in,
              wl_positions=wl_pos, d_positions=d_pos)
    lp = torch.zeros(h.shape[:2], device=dev, dtype=h.dtype)
    mask = torch.zeros(h.shape[:2], device=dev, dtype=torch.bool)
    for key, head in (("thinking_move_mask", model.thinking_policy_head), ("final_move_mask", model.policy_head)):
        m = b[key]
        if m.any():
            logp = F.log_softmax(head(h[m]), dim=-1)
            lp[m] = logp.gather(1, b["move_token_ids"][m].unsqueeze(1)).squeeze(1)
            mask[m] = True
    return lp, mask
