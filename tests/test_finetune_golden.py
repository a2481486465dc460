"""The finetune oracle (oracle/step.py:finetune_step_losses, a restatement
of chessdecoder/finetune/train.py:272-355) against the reference's own loss
body executed on the same model and batch (tests/golden/finetune_reference.pt,
made by tests/golden/make_finetune_golden.py): all five losses, the weighted
total and the gradients of every bias and norm scale."""
from pathlib import Path

import torch

GOLD = torch.load(Path(__file__).parent / "golden" / "finetune_reference.pt")


def test_finetune_oracle_matches_reference_loss_body():
    from oracle.model import OracleChessDecoder
    from oracle.step import finetune_step_losses
    torch.manual_seed(GOLD["seed"])
    model = OracleChessDecoder(1968, **GOLD["config"])
    w = GOLD["weights"]
    out = finetune_step_losses(model, GOLD["batch"], weights=(w["final_move_weight"], w["board_weight"],
                                                              w["wl_weight"], w["d_weight"], w["thinking_move_weight"]))
    ref = GOLD["losses"]
    pairs = {"move": "final_move_loss", "think": "thinking_move_loss", "board": "board_loss", "wl": "wl_loss",
             "d": "d_loss", "total": "total_loss"}
    for ours, theirs in pairs.items():
        assert torch.allclose(out[ours].detach(), ref[theirs], rtol=1e-5, atol=1e-6), (ours, out[ours], ref[theirs])
    assert all(float(ref[n]) > 0 for n in pairs.values())  # every term exercised
    out["total"].backward()
    params = dict(model.named_parameters())
    for n, g in GOLD["grads"].items():
        assert torch.allclose(params[n].grad, g, rtol=1e-4, atol=1e-7), n
