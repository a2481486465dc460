"""The native batch producer (cdk_tokenize_games, chessdecoder_b200/loader.py)
against the oracle's plain-Python restatement of the reference's data path
(oracle/loader.py: chessdecoder/dataloader/data.py:7-97, loader.py:30-184).
CPU only: the producer runs on host threads.

* the oracle against the reference's own known answers (its tests/test_data.py);
* the castling-rights rule of python-chess (king home + rook on the corner);
* bit-exact rows for random legal games at several sequence lengths and
  skip probabilities, including truncation inside a board block, games
  without values, missing moves and invalid (NaN) values;
* the whole iterable dataset on parquet files against the oracle's
  iteration (seeding, file / game shuffles, batching).
"""
import math
import random

import numpy as np
import pytest
import torch

from chessdecoder_b200 import vocab as V
from chessdecoder_b200.chessgen import random_game_rows
from chessdecoder_b200.loader import KEYS, GameTokenizer
from oracle import loader as OL

START = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"


def test_oracle_known_answers():
    t = OL.fen_position_tokens(START)
    assert len(t) == 68 and t[0] == "start_pos" and t[65] == "end_pos"
    assert t[1] == "white_rook" and t[5] == "white_king" and t[9] == "white_pawn" and t[29] == "empty"
    assert t[57] == "black_rook" and t[67] == "white_to_move" and t[66] == "KQkq"
    assert OL.fen_position_tokens("rnbqkbnr/pppppppp/8/8/4P3/8/PPPP1PPP/RNBQKBNR b KQkq - 0 1")[67] == "black_to_move"
    assert OL.fen_position_tokens("8/5pk1/6p1/8/8/2B5/5PPP/6K1 w - - 0 40")[66] == "no_castling_rights"
    game = {"fen": [START, "rnbqkbnr/pppppppp/8/8/4P3/8/PPPP1PPP/RNBQKBNR b KQkq e3 0 1"],
            "played_move": ["e2e4", "e7e5"], "best_move": ["e2e4", "e7e5"],
            "played_q": [None, None], "played_d": [None, None]}
    ids, moves, blocks, values = OL.game_to_token_ids(game, [1, 1])
    for s, _ in blocks:
        assert ids[s] == V.token_to_idx["start_pos"]
    for w, d, *_ in values:
        assert d == w + 1 and ids[w] == V.token_to_idx["wl_value"] and ids[d] == V.token_to_idx["d_value"]


@pytest.mark.parametrize("fen,rights", [
    ("r3k2r/8/8/8/8/8/8/R3K2R w KQkq - 0 1", "KQkq"),
    ("r3k2r/8/8/8/8/8/8/R3K1R1 w KQkq - 0 1", "Qkq"),     # no rook on h1
    ("r3k2r/8/8/8/8/8/8/1R2K2R w KQkq - 0 1", "Kkq"),     # no rook on a1
    ("r3k2r/8/8/8/8/8/8/R4K1R w KQkq - 0 1", "kq"),       # king off e1
    ("1r2k2r/8/8/8/8/8/8/R3K2R b KQkq - 0 1", "KQk"),     # no rook on a8
    ("r3k2r/8/8/8/8/8/8/R3K2R w Kq - 0 1", "Kq"),
    ("r3k2r/8/8/8/8/8/8/R3K2R w - - 0 1", "no_castling_rights"),
])
def test_castling_rights_cleaned(fen, rights):
    assert OL.fen_position_tokens(fen)[66] == rights
    tok = GameTokenizer(128, n_threads=1)
    g = {"fen": [fen], "played_move": [None], "best_move": [None], "played_q": [None], "played_d": [None]}
    out = tok([g], [(np.ones(1, np.uint8), 0)])
    assert int(out["input_ids"][0, 66]) == V.token_to_idx[rights]


def _games(rng, n, lo=1, hi=90):
    games = [random_game_rows(rng, rng.randint(lo, hi)) for _ in range(n)]
    # edge cases: a missing played move, invalid values, a one-ply game
    games[0]["played_move"][len(games[0]["fen"]) // 2] = None
    games[1]["played_q"][0] = float("nan")
    games[2]["played_d"][-1] = None
    games.append(random_game_rows(rng, 1))
    return games


@pytest.mark.parametrize("S,skip", [(256, 0.2), (64, 0.0), (1024, 0.5), (70, 0.2)])
def test_rows_match_oracle(S, skip):
    rng = random.Random(S * 7 + int(skip * 10))
    games = _games(rng, 24)
    drng = random.Random(5)
    draws = [OL.draw_decisions(g, drng, skip) for g in games]
    tok = GameTokenizer(S, n_threads=4)
    out = tok(games, [(np.asarray(i, np.uint8), st) for i, st in draws])
    for gi, (g, (inc, st)) in enumerate(zip(games, draws)):
        ref = OL.tensorize_row(*OL.game_to_token_ids(g, inc), st, S)
        for k in KEYS:
            got = out[k][gi].numpy()
            assert np.array_equal(got, ref[k].astype(got.dtype)), (gi, k)


def test_draws_follow_reference_order():
    """GameTokenizer.draw_decisions consumes the generator exactly as the oracle
    (and the reference) does."""
    rng = random.Random(3)
    games = _games(rng, 6)
    a, b = random.Random(11), random.Random(11)
    for g in games:
        i1, s1 = GameTokenizer.draw_decisions(g, a, 0.3)
        i2, s2 = OL.draw_decisions(g, b, 0.3)
        assert list(i1) == list(i2) and s1 == s2
    assert a.random() == b.random()


def test_errors_are_reported():
    tok = GameTokenizer(64, n_threads=1)
    bad = {"fen": ["not a fen"], "played_move": ["e2e4"], "best_move": ["e2e4"], "played_q": [0.1],
           "played_d": [0.2]}
    with pytest.raises(RuntimeError, match="-3"):
        tok([bad], [(np.ones(1, np.uint8), 0)])
    unk = {"fen": [START], "played_move": ["zz99"], "best_move": ["e2e4"], "played_q": [0.1], "played_d": [0.2]}
    with pytest.raises(RuntimeError, match="-2"):
        tok([unk], [(np.ones(1, np.uint8), 0)])


def test_dataset_matches_oracle_iteration(tmp_path):
    pd = pytest.importorskip("pandas")
    pytest.importorskip("pyarrow")
    from chessdecoder_b200.loader import ChessIterableDataset
    rng = random.Random(17)
    files = []
    gid = 0
    for f in range(3):
        games = [random_game_rows(rng, rng.randint(2, 60)) for _ in range(7)]
        rows = []
        for g in games:
            for ply in range(len(g["fen"])):
                rows.append({"game_id": gid, "ply": ply, **{k: g[k][ply] for k in g}})
            gid += 1
        # stored with plies shuffled: the loader sorts them
        random.Random(f).shuffle(rows)
        pd.DataFrame(rows).to_parquet(tmp_path / f"part_{f:03d}.parquet")
        files.append(games)
    ds = ChessIterableDataset(str(tmp_path), max_seq_len=128, skip_board_prob=0.2, seed=42, batch_size=5,
                              n_threads=2)
    got = list(iter(ds))
    # the oracle sees each file's games in order of first appearance in the stored (shuffled) rows
    stored = []
    for f in range(3):
        df = pd.read_parquet(tmp_path / f"part_{f:03d}.parquet")
        order = list(dict.fromkeys(df["game_id"].tolist()))
        base = sum(len(x) for x in files[:f])
        stored.append([files[f][g - base] for g in order])
    want = list(OL.iterate_batches(stored, 5, 128, 0.2, seed=42))
    assert len(got) == len(want)
    for gb, wb in zip(got, want):
        for k in KEYS:
            assert np.array_equal(gb[k].numpy(), wb[k].astype(gb[k].numpy().dtype)), k
