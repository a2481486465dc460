"""ORACLE (test infrastructure only): the reference's pretraining data path
restated in plain Python, as the checker of the native batch producer
(``cdk_tokenize_games``).

* ``fen_position_tokens`` follows chessdecoder/dataloader/data.py:7-48
  (python-chess's ``Board(fen)`` + ``has_*_castling_rights``: a right counts
  only with the king on e1 / e8 and the rook on its corner -- python-chess's
  ``clean_castling_rights`` for standard chess, version 1.11.2 pinned by the
  reference's uv.lock);
* ``game_to_token_ids`` follows data.py:50-97 with the per-ply board
  decisions passed in (``random.random() > skip_board_prob`` in the
  reference);
* ``tensorize_row`` follows the per-game body of
  chessdecoder/dataloader/loader.py:69-184 with the start index passed in
  (``random.choice(valid_starts)`` in the reference);
* ``iterate_batches`` follows ``ChessIterableDataset.__iter__``
  (loader.py:30-67) on in-memory files, single worker.
"""
from __future__ import annotations

import math
import random

import numpy as np

from chessdecoder_b200 import vocab as V

IGNORE_INDEX = -100
_NAMES = {"p": "pawn", "n": "knight", "b": "bishop", "r": "rook", "q": "queen", "k": "king"}


def fen_position_tokens(fen: str) -> list:
    placement, turn = fen.split()[:2]
    rights_field = fen.split()[2] if len(fen.split()) > 2 else "-"
    board = [None] * 64
    rank = 7
    for row in placement.split("/"):
        f = 0
        for ch in row:
            if ch.isdigit():
                f += int(ch)
            else:
                board[rank * 8 + f] = ch
                f += 1
        rank -= 1
    toks = ["start_pos"]
    for sq in range(64):
        p = board[sq]
        toks.append("empty" if p is None else ("white_" if p.isupper() else "black_") + _NAMES[p.lower()])
    toks.append("end_pos")
    ok = {"K": board[4] == "K" and board[7] == "R", "Q": board[4] == "K" and board[0] == "R",
          "k": board[60] == "k" and board[63] == "r", "q": board[60] == "k" and board[56] == "r"}
    rights = "".join(c for c in "KQkq" if c in rights_field and ok[c])
    toks.append(rights if rights else "no_castling_rights")
    toks.append("white_to_move" if turn == "w" else "black_to_move")
    return toks


def game_to_token_ids(game: dict, include_board):
    seq, moves, blocks, values = [], [], [], []
    for i in range(len(game["fen"])):
        include = i == 0 or bool(include_board[i])
        if include:
            b0 = len(seq)
            seq.extend(fen_position_tokens(game["fen"][i]))
        played = game["played_move"][i]
        if played:
            mi = len(seq)
            seq.append(played)
            if include:
                blocks.append((b0, mi))
            moves.append((mi, game["best_move"][i]))
            wl_pos = len(seq)
            seq.append("wl_value")
            d_pos = len(seq)
            seq.append("d_value")
            q, d = game["played_q"][i], game["played_d"][i]
            valid = q is not None and not (isinstance(q, float) and math.isnan(q)) and \
                d is not None and not (isinstance(d, float) and math.isnan(d))
            values.append((wl_pos, d_pos, float(q) if valid else 0.0, float(d) if valid else 0.0, valid))
    return [V.token_to_idx[t] for t in seq], moves, blocks, values


def tensorize_row(ids, moves, blocks, values, start_choice: int, S: int) -> dict:
    valid_starts = [0] + [vd[1] + 1 for vd in values[:-1]]
    start = valid_starts[start_choice]
    ids = ids[start:]
    moves = [(m - start, b) for m, b in moves if m >= start]
    values = [(w - start, d - start, wl, dd, ok) for w, d, wl, dd, ok in values if d >= start]
    adj = []
    for b0, b1 in blocks:
        a0, a1 = b0 - start, b1 - start
        if a1 > 0 and a0 < len(ids):
            adj.append((max(0, a0), min(len(ids), a1)))
    if len(ids) > S:
        ids = ids[:S]
        moves = [m for m in moves if m[0] < S]
        values = [v for v in values if v[1] < S]
        adj = [(b0, min(b1, S)) for b0, b1 in adj if b0 < S]
    values = [v for v in values if v[0] < S and v[1] < S]
    valid_moves = {v[0] - 1 for v in values}
    moves = [m for m in moves if m[0] in valid_moves]
    n = len(ids)
    out = {"input_ids": np.full(S, V.token_to_idx["pad"], np.int64),
           "board_target_ids": np.full(S, IGNORE_INDEX, np.int64),
           "move_target_ids": np.full(S, IGNORE_INDEX, np.int64),
           "move_mask": np.zeros(S, bool), "wl_positions": np.zeros(S, bool), "d_positions": np.zeros(S, bool),
           "wl_targets": np.zeros(S, np.float32), "d_targets": np.zeros(S, np.float32),
           "wdl_valid": np.zeros(S, bool)}
    out["input_ids"][:n] = ids
    for i in range(n - 1):
        out["board_target_ids"][i] = V.full_idx_to_board_idx.get(int(out["input_ids"][i + 1]), IGNORE_INDEX)
    gm = V.board_token_to_idx["generic_move"]
    for mi, best in moves:
        stm = mi - 1
        if 0 <= stm < S:
            out["board_target_ids"][stm] = gm
            out["move_target_ids"][stm] = V.full_idx_to_move_idx[V.token_to_idx[best]]
            out["move_mask"][stm] = True
    for w, d, wl, dd, ok in values:
        if w < S:
            out["wl_positions"][w], out["wl_targets"][w], out["wdl_valid"][w] = True, wl, ok
        if d < S:
            out["d_positions"][d], out["d_targets"][d], out["wdl_valid"][d] = True, dd, ok
        stm = w - 2
        if 0 <= stm < S:
            out["wl_targets"][stm], out["d_targets"][stm], out["wdl_valid"][stm] = wl, dd, ok
    bid = np.arange(S, dtype=np.int64) + len(adj)
    for k, (b0, b1) in enumerate(adj):
        bid[b0:b1] = k
    out["block_id"] = bid
    return out


def draw_decisions(game: dict, rng: random.Random, skip_board_prob: float):
    """The reference's draws for one game, in its order."""
    include = [1] + [1 if rng.random() > skip_board_prob else 0 for _ in range(1, len(game["fen"]))]
    n_values = sum(1 for m in game["played_move"] if m)
    return include, rng.choice(list(range(max(n_values, 1))))


def iterate_batches(files: list, batch_size: int, S: int, skip_board_prob: float, seed: int, epoch: int = 0,
                    rank: int = 0, world_size: int = 1, shuffle_files=True, shuffle_games=True):
    """``files``: list of lists of games (each file's games in stored order)."""
    epoch_seed = seed + epoch * 100003 + rank * 7919
    rng = random.Random(epoch_seed)
    nrng = np.random.RandomState(epoch_seed % (2 ** 32))
    order = list(range(len(files)))[rank::world_size]
    if shuffle_files:
        rng.shuffle(order)
    rows = []
    for fi in order:
        games = files[fi]
        ids = list(range(len(games)))
        if shuffle_games:
            nrng.shuffle(ids)
        for gi in ids:
            g = games[gi]
            inc, st = draw_decisions(g, rng, skip_board_prob)
            rows.append(tensorize_row(*game_to_token_ids(g, inc), st, S))
            if len(rows) == batch_size:
                yield {k: np.stack([r[k] for r in rows]) for k in rows[0]}
                rows = []
    if rows:
        yield {k: np.stack([r[k] for r in rows]) for k in rows[0]}
