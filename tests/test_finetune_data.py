"""Finetune rows and their step bookkeeping on the CPU.

* ``tensorize_variation`` against the layout facts of
  chessdecoder/finetune/data.py:144-247 and loader.py:337-440 on a hand-built
  sequence (thinking targets after ``start_think`` / a board's stm /
  ``end_var``, the final move after ``end_think``, board-target overrides,
  WL / D targets copied two tokens before the WL placeholder, block ids);
* the host index lists of a finetune batch (thinking rows, WL rows at stm+1
  of both move kinds, the board mask from the first move of either kind);
* the oracle's finetune loss reduces to the pretraining loss when no thinking
  rows exist.
"""
import numpy as np
import torch

from chessdecoder_b200 import data
from chessdecoder_b200 import vocab as V
from chessdecoder_b200.chessgen import Position


def _sequence():
    pos = Position()
    seq, blocks = [], []
    seq.extend(pos.position_tokens())
    blocks.append((0, len(seq)))
    seq.append("start_think")
    thinking, values = [], []
    p = pos
    for d in range(2):
        mv = p.legal_moves()[0]
        thinking.append((len(seq) - 1, Position.move_token(mv)))
        seq.append(Position.move_token(mv))
        p = p.apply(mv)
        values.append((len(seq), len(seq) + 1, 0.25 * (d + 1), 0.1, True))
        seq += ["wl_value", "d_value"]
        b0 = len(seq)
        seq.extend(p.position_tokens())
        blocks.append((b0, len(seq)))
    seq.append("end_var")
    mv2 = pos.legal_moves()[1]
    thinking.append((len(seq) - 1, Position.move_token(mv2)))
    seq.append(Position.move_token(mv2))
    values.append((len(seq), len(seq) + 1, -0.5, 0.2, True))
    seq += ["wl_value", "d_value"]
    b0 = len(seq)
    seq.extend(pos.apply(mv2).position_tokens())
    blocks.append((b0, len(seq)))
    seq += ["end_var", "end_think"]
    final = (len(seq) - 1, Position.move_token(pos.legal_moves()[2]))
    seq.append(final[1])
    values.append((len(seq), len(seq) + 1, 0.75, 0.05, False))
    seq += ["wl_value", "d_value"]
    return [V.token_to_idx[t] for t in seq], thinking, final, values, blocks


def test_tensorize_variation_layout():
    ids, thinking, final, values, blocks = _sequence()
    S = 512
    r = data.tensorize_variation(ids, thinking, final, values, blocks, S)
    n = len(ids)
    bt = V.board_token_to_idx
    assert r["input_ids"][:n].tolist() == ids and (r["input_ids"][n:] == V.token_to_idx["pad"]).all()
    # thinking targets: after start_think, at the first line's stm, after end_var
    tpos = [p for p, _ in thinking]
    assert ids[tpos[0]] == V.token_to_idx["start_think"] and ids[tpos[2]] == V.token_to_idx["end_var"]
    assert np.nonzero(r["thinking_move_mask"])[0].tolist() == tpos
    assert r["board_target_ids"][tpos[0]] == bt["generic_move"]
    assert r["board_target_ids"][tpos[1]] == bt["continue_var"]
    assert r["board_target_ids"][tpos[2]] == bt["new_variation"]
    for p, mv in thinking:
        assert r["move_target_ids"][p] == V.full_idx_to_move_idx[V.token_to_idx[mv]]
    # final move after end_think -> policy head
    assert ids[final[0]] == V.token_to_idx["end_think"]
    assert np.nonzero(r["move_mask"])[0].tolist() == [final[0]]
    assert r["board_target_ids"][final[0]] == bt["generic_move"]
    # other board targets are the shifted next token (board sub-vocab or ignore)
    table = np.array(V.full_to_board_table())
    special = set(tpos) | {final[0]}
    for i in range(n - 1):
        if i not in special:
            assert r["board_target_ids"][i] == table[ids[i + 1]]
    assert (r["board_target_ids"][n - 1:] == data.IGNORE_INDEX).all()
    # values: at the placeholders and two tokens before the WL placeholder
    for w, d, wl, dd, ok in values:
        assert r["wl_positions"][w] and r["d_positions"][d]
        assert r["wl_targets"][w] == np.float32(wl) and r["d_targets"][d] == np.float32(dd)
        assert r["wl_targets"][w - 2] == np.float32(wl) and r["d_targets"][w - 2] == np.float32(dd)
        assert r["wdl_valid"][w] == ok and r["wdl_valid"][w - 2] == ok
    # blocks: one id per board, unique ids elsewhere
    bid = r["block_id"]
    for k, (b0, b1) in enumerate(blocks):
        assert (bid[b0:b1] == k).all()
    outside = np.ones(S, bool)
    for b0, b1 in blocks:
        outside[b0:b1] = False
    assert (bid[outside] == np.arange(S)[outside] + len(blocks)).all()


def test_finetune_index_lists():
    from chessdecoder_b200.engine import _host_index_lists
    b = data.finetune_batches(1, 3, 1024, seed=4, min_lines=2, max_lines=3, min_depth=1, max_depth=3)[0]
    lists, Bn, S = _host_index_lists(b)
    BS = Bn * S
    mm, tm = b["move_mask"].numpy(), b["thinking_move_mask"].numpy()
    anym = mm | tm
    assert (lists["trow"] == BS + np.nonzero(tm.reshape(-1))[0]).all()
    assert (lists["tt"] == b["move_target_ids"].numpy().reshape(-1)[tm.reshape(-1)]).all()
    assert (lists["prow"] == BS + np.nonzero(mm.reshape(-1))[0]).all()
    bb, ss = np.nonzero(anym)
    assert (lists["wrow"] == BS + bb * S + np.minimum(ss + 1, S - 1)).all()
    assert np.allclose(lists["wtgt"], b["wl_targets"].numpy()[anym])
    first = np.where(anym.any(1), anym.argmax(1), S)
    bm = (b["board_target_ids"].numpy() != -100) & (np.arange(S)[None] >= first[:, None])
    assert (lists["board_w"] == bm.reshape(-1)).all()
    assert np.isclose(lists["norms"][4], 1.0 / (tm.sum() + 1e-8))


def test_oracle_finetune_reduces_to_pretraining():
    from oracle.model import OracleChessDecoder
    from oracle.step import finetune_step_losses, step_losses
    torch.manual_seed(0)
    kw = dict(embed_dim=64, num_heads=2, num_layers=1, max_seq_len=256, d_ff=96)
    model = OracleChessDecoder(V.vocab_size, **kw)
    b = data.synthetic_batches(1, 2, 256, seed=1)[0]
    b["thinking_move_mask"] = torch.zeros_like(b["move_mask"])
    ft = finetune_step_losses(model, b, weights=(5.0, 1.0, 1.0, 1.0, 3.0))
    pt = step_losses(model, b)
    for k in ("move", "board", "wl", "d", "total"):
        assert torch.allclose(ft[k], pt[k], rtol=1e-6, atol=1e-7), k
    assert float(ft["think"].detach()) == 0.0
