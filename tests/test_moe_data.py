"""Thinking-variation rows (the MoE variant's sequences) and the MoE oracle's
routing rules, on the CPU."""
import math

import torch


def test_thinking_rows_layout():
    from chessdecoder_b200 import data, vocab as V
    b = data.thinking_batches(1, 3, 4096, seed=5)[0]
    ids, bid = b["input_ids"], b["block_id"]
    tok = V.token_to_idx
    for r in range(3):
        row = ids[r]
        assert int(row[68]) == tok["start_think"]
        assert (bid[r, :68] == bid[r, 0]).all() and bid[r, 68] != bid[r, 0]   # root board = one block
        mm = b["move_mask"][r].nonzero().flatten()
        assert mm.numel() >= 7  # >= 3 lines x 2 plies + the final move
        for s in mm.tolist():
            assert int(row[s + 2]) == tok["wl_value"] and int(row[s + 3]) == tok["d_value"]
            assert V.full_idx_to_move_idx.get(int(row[s + 1])) == int(b["move_target_ids"][r, s])
        # every WL placeholder pairs with the D placeholder after it
        wl = b["wl_positions"][r].nonzero().flatten()
        dp = b["d_positions"][r].nonzero().flatten()
        assert torch.equal(wl + 1, dp)
        n = int((row != tok["pad"]).sum())
        assert int(row[n - 3]) in V.full_idx_to_move_idx and int(row[n - 4]) == tok["end_think"]


def test_oracle_moe_capacity_rules():
    """First choices fill the slots before second choices, in token order; the rest drop."""
    from oracle.moe import OracleMoE
    torch.manual_seed(0)
    m = OracleMoE(16, 32, n_experts=4, capacity=0.5)
    x = torch.randn(40, 16)
    idx, w, keep, cap = m.route(x)
    assert cap == math.ceil(0.5 * 2 * 40 / 4)
    assert torch.allclose(w.sum(1), torch.ones(40))
    for e in range(4):
        order = [(t, 0) for t in range(40) if idx[t, 0] == e] + [(t, 1) for t in range(40) if idx[t, 1] == e]
        kept = [tk for tk in order if keep[tk]]
        assert kept == order[:cap]
