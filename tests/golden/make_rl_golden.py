"""Generates tests/golden/rl_reference.pt from the reference's GRPO functions
(chessdecoder/rl/grpo.py imports only torch).  Run where the ChessDecoder
repository is mounted, its root given by the REFERENCE_ROOT environment
variable (required):

    REFERENCE_ROOT=<ChessDecoder checkout> python tests/golden/make_rl_golden.py
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import torch



def reference_root() -> Path:
    """The ChessDecoder checkout named by REFERENCE_ROOT (required)."""
    if not os.environ.get("REFERENCE_ROOT"):
        raise SystemExit("set REFERENCE_ROOT to the root of the ChessDecoder repository")
    return Path(os.environ["REFERENCE_ROOT"])



def main():
    sys.path.insert(0, str(reference_root()))
    from chessdecoder.rl import grpo as G
    g = torch.Generator().manual_seed(7)
    N, S = 6, 40
    lp = -torch.rand(N, S, generator=g) * 4
    old = lp + torch.randn(N, S, generator=g) * 0.3
    ref = lp + torch.randn(N, S, generator=g) * 0.2
    mask = torch.rand(N, S, generator=g) < 0.3
    rewards = torch.randn(3, 4, generator=g)
    rewards[1] = 0.5  # a constant-reward group
    adv, diverse = G.compute_group_advantages(rewards)
    adv_n = G.normalize_advantages_minibatch(adv.flatten()[:N])
    cases = []
    for eps_lo, eps_hi, kl in ((0.2, 0.2, 0.0), (0.2, 0.28, 0.04), (0.1, 0.3, 0.5)):
        x = lp.clone().requires_grad_(True)
        loss, _ = G.grpo_loss(x, old, ref, mask, adv_n, eps_lo, eps_hi, kl)
        loss.backward()
        cases.append({"eps_low": eps_lo, "eps_high": eps_hi, "kl": kl, "loss": loss.detach(), "grad": x.grad})
    torch.save({"lp": lp, "old": old, "ref": ref, "mask": mask, "rewards": rewards, "adv": adv, "diverse": diverse,
                "adv_norm": adv_n, "cases": cases}, Path(__file__).with_name("rl_reference.pt"))
    print("wrote rl_reference.pt")


if __name__ == "__main__":
    main()
