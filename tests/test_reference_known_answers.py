"""The reference's own structural known answers (its tests/test_vocab.py,
tests/test_data.py, tests/test_model.py), restated against this package:
vocabulary sizes and round trips, the 68-token board block layout, the
per-ply token layout, and the masks' visibility rules (GPU part)."""
import random

import pytest
import torch

from chessdecoder_b200 import vocab as V
from chessdecoder_b200.chessgen import Position, perft
from chessdecoder_b200.data import game_to_token_ids

SAMPLE_FENS = [  # the five positions of the reference's tests/conftest.py
    "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1",
    "r1bqkb1r/pppppppp/2n2n2/8/4P3/5N2/PPPP1PPP/RNBQKB1R w KQkq - 2 3",
    "8/5pk1/6p1/8/8/2B5/5PPP/6K1 w - - 0 40",
    "r1bq1rk1/pp2nppp/2n1p3/3pP3/3P4/2N2N2/PP2BPPP/R1BQ1RK1 b - - 1 10",
    "8/P7/8/8/8/8/8/4K2k w - - 0 1",
]


def test_vocab_sizes_and_roundtrips():
    assert V.vocab_size >= 1967
    assert V.board_vocab_size == 41
    assert V.move_vocab_size == 1924
    assert V.POSITION_TOKEN_LENGTH == 68
    assert len(V.token_to_idx) == V.vocab_size
    for tok, idx in V.token_to_idx.items():
        assert V.idx_to_token[idx] == tok
    for i in range(V.board_vocab_size):
        assert V.full_idx_to_board_idx[V.board_idx_to_full_idx[i]] == i
    for i in range(V.move_vocab_size):
        assert V.full_idx_to_move_idx[V.move_idx_to_full_idx[i]] == i
    assert set(V.board_idx_to_full_idx).isdisjoint(V.move_idx_to_full_idx)
    for tok in ["start_pos", "end_pos", "white_to_move", "black_to_move", "empty", "pad", "wl_value", "d_value",
                "start_think", "end_think", "end_var", "continue_var", "new_variation", "generic_move"]:
        assert tok in V.token_to_idx


@pytest.mark.parametrize("fen", SAMPLE_FENS)
def test_position_tokens_structure(fen):
    toks = Position.from_fen(fen).position_tokens()
    assert len(toks) == 68
    assert toks[0] == "start_pos" and toks[65] == "end_pos"
    assert toks[66] in V.castling_tokens
    assert toks[67] in ("white_to_move", "black_to_move")
    assert all(t in V.token_to_idx for t in toks)


def test_start_position_square_order():
    toks = Position.from_fen(SAMPLE_FENS[0]).position_tokens()
    assert toks[1] == "white_rook"      # a1
    assert toks[5] == "white_king"      # e1
    assert toks[9] == "white_pawn"      # a2
    assert toks[29] == "empty"          # e4
    assert toks[57] == "black_rook"     # a8
    assert toks[67] == "white_to_move"
    assert toks[66] == "KQkq"
    assert Position().position_tokens() == toks


def test_side_to_move_and_no_castling():
    assert Position.from_fen("rnbqkbnr/pppppppp/8/8/4P3/8/PPPP1PPP/RNBQKBNR b KQkq - 0 1").position_tokens()[67] == \
        "black_to_move"
    assert Position.from_fen("8/5pk1/6p1/8/8/2B5/5PPP/6K1 w - - 0 40").position_tokens()[66] == "no_castling_rights"


def test_game_token_layout():
    p0 = Position()
    e4 = [m for m in p0.legal_moves() if Position.move_token(m) == "e2e4"][0]
    p1 = p0.apply(e4)
    plies = [(p0.position_tokens(), "e2e4", "e2e4", 0.3 - 0.2, 0.5),
             (p1.position_tokens(), "e7e5", "e7e5", 0.4 - 0.2, 0.4)]
    ids, move_targets, blocks, values = game_to_token_ids(plies, random.Random(0), 0.0)
    assert all(0 <= t < V.vocab_size for t in ids)
    for s, e in blocks:
        assert ids[s] == V.token_to_idx["start_pos"]
        assert e - s == 68
    for wl, d, _, _, _ in values:
        assert d == wl + 1
        assert ids[wl] == V.token_to_idx["wl_value"] and ids[d] == V.token_to_idx["d_value"]
    for m_idx, best in move_targets:
        assert ids[m_idx] == V.token_to_idx[best] or V.idx_to_token[ids[m_idx]] in V.move_vocab


def test_movegen_perft_known_values():
    # standard perft counts (no promotions occur at these depths)
    assert [perft(Position(), d) for d in (1, 2, 3)] == [20, 400, 8902]
    kiwi = Position.from_fen("r3k2r/p1ppqpb1/bn2pnp1/3PN3/1p2P3/2N2Q1p/PPPBBPPP/R3K2R w KQkq - 0 1")
    assert perft(kiwi, 1) == 48 and perft(kiwi, 2) == 2039
    p3 = Position.from_fen("8/2p5/3p4/KP5r/1R3p1k/8/4P1P1/8 w - - 0 1")
    assert [perft(p3, d) for d in (1, 2, 3)] == [14, 191, 2812]


def test_castling_spelled_king_takes_rook():
    p = Position.from_fen("r3k2r/8/8/8/8/8/8/R3K2R w KQkq - 0 1")
    toks = {Position.move_token(m) for m in p.legal_moves()}
    assert "e1h1" in toks and "e1a1" in toks and "e1g1" not in toks
    assert all(t in V.move_token_to_idx for t in toks)


# ---------------------------------------------------------------------------
# tests/test_model.py:50-81 of the reference: the two masks' visibility
# ---------------------------------------------------------------------------
def _hidden(ids, bid, causal):
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.engine import ModelConfig, TrainStep, prepare_batch
    cfg = ModelConfig(embed_dim=256, num_heads=4, num_layers=2, max_seq_len=68, d_ff=384)
    step = TrainStep(cfg, device="cuda", seed=0)
    B, S = ids.shape
    z = torch.zeros(B, S, dtype=torch.bool)
    batch = {"input_ids": ids, "board_target_ids": torch.full((B, S), -100), "move_target_ids": torch.full((B, S), -100),
             "move_mask": z, "wl_positions": z, "d_positions": z, "wl_targets": torch.zeros(B, S),
             "d_targets": torch.zeros(B, S), "wdl_valid": z, "block_id": bid}
    db = prepare_batch(batch, "cuda")
    meta = K.attn_meta(db.bid, S)
    h0, _ = step.front.forward(db, n_copies=1)
    _, h32, _ = step.backbone.forward(h0, B, B if causal else 0, S, db.bid, meta, want_f32=True)
    return h32.view(B, S, -1).cpu()


@pytest.mark.gpu
def test_causal_no_future_leakage():
    ids = torch.tensor([[V.token_to_idx[t] for t in Position().position_tokens()]])
    bid = torch.zeros(1, 68, dtype=torch.long)
    h1 = _hidden(ids, bid, causal=True)
    ids2 = ids.clone()
    ids2[0, 1] = V.token_to_idx["empty"]
    h2 = _hidden(ids2, bid, causal=True)
    assert torch.equal(h1[0, 0], h2[0, 0])


@pytest.mark.gpu
def test_prefix_bidirectional_within_block():
    ids = torch.tensor([[V.token_to_idx[t] for t in Position().position_tokens()]])
    bid = torch.zeros(1, 68, dtype=torch.long)
    h1 = _hidden(ids, bid, causal=False)
    ids2 = ids.clone()
    ids2[0, 1] = V.token_to_idx["empty"]
    h2 = _hidden(ids2, bid, causal=False)
    assert not torch.allclose(h1[0, -1], h2[0, -1], atol=1e-5)
    assert not torch.allclose(h1[0, 0], h2[0, 0], atol=1e-5)  # earlier rows also see later block rows
