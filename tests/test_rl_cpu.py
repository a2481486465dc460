"""The oracle's GRPO functions (oracle/rl.py) against the reference's own
(chessdecoder/rl/grpo.py, via tests/golden/rl_reference.pt): group
advantages, mini-batch normalisation, and the per-token clipped loss with
the KL penalty and its gradient, for three clip / KL settings."""
from pathlib import Path

import torch

from oracle import rl as R

G = torch.load(Path(__file__).parent / "golden" / "rl_reference.pt")


def test_advantages_match_reference():
    adv, diverse = R.group_advantages(G["rewards"])
    assert torch.equal(diverse, G["diverse"])
    assert torch.allclose(adv, G["adv"], atol=1e-7)
    assert torch.allclose(R.normalize_advantages(G["adv"].flatten()[:6]), G["adv_norm"], atol=1e-6)


def test_grpo_loss_matches_reference():
    for c in G["cases"]:
        x = G["lp"].clone().requires_grad_(True)
        loss = R.grpo_loss(x, G["old"], G["ref"], G["mask"], G["adv_norm"], c["eps_low"], c["eps_high"], c["kl"])
        loss.backward()
        assert torch.allclose(loss.detach(), c["loss"], rtol=1e-6, atol=1e-7)
        assert torch.allclose(x.grad, c["grad"], rtol=1e-5, atol=1e-8)
