"""Batch producer: seeded synthetic games -> the reference loader's 10 tensors.

Restates, for synthetic games, the tokenisation of
chessdecoder/dataloader/data.py:51-97 (``game_to_token_ids``) and the
windowing / tensorisation of chessdecoder/dataloader/loader.py:69-184
(``ChessIterableDataset.__iter__``):

* per ply: the 68-token board block (always for the first ply, otherwise kept
  with probability 1 - skip_board_prob), the move token, then ``wl_value`` and
  ``d_value`` placeholders;
* a random start among ``[0] + [d_pos + 1 ...]`` (every ply boundary except
  after the last ply), truncation to ``max_seq_len`` dropping plies whose
  WL/D placeholders were cut, padding with ``pad``;
* board targets = next token mapped to the 41-token board sub-vocabulary
  (-100 elsewhere), overridden at each kept move's stm position by
  ``generic_move``; move targets (1924 sub-vocabulary) at the stm position;
  WL/D targets at the placeholders and copied to the stm position;
* ``block_id`` = board-block index inside blocks, unique ids elsewhere.

Game content replaces the missing lc0 parquet files: uniform-random legal
playouts (see chessgen.random_game).  Each rank gets its own stream seeded with
``seed + rank * 7919`` (the rank term of loader.py:36).
"""
from __future__ import annotations

import random

import numpy as np
import torch

from . import vocab as V
from .chessgen import random_game

IGNORE_INDEX = -100
KEYS = ("input_ids", "board_target_ids", "move_target_ids", "move_mask", "wl_positions", "d_positions",
        "wl_targets", "d_targets", "wdl_valid", "block_id")

_FULL_TO_BOARD = np.array(V.full_to_board_table(), dtype=np.int64)


def game_to_token_ids(plies, rng: random.Random, skip_board_prob: float = 0.0):
    """Token ids, move targets, board-block boundaries and value data of one game.

    ``plies`` = [(position_tokens, played_move, best_move, played_q, played_d)].
    Follows chessdecoder/dataloader/data.py:51-97: one ``rng.random()`` draw per
    ply after the first decides whether the board block is emitted.
    """
    seq, move_targets, blocks, values = [], [], [], []
    for i, (pos_tokens, played, best, q, d) in enumerate(plies):
        include_board = (i == 0) or (rng.random() > skip_board_prob)
        if include_board:
            block_start = len(seq)
            seq.extend(pos_tokens)
        move_idx = len(seq)
        seq.append(played)
        if include_board:
            blocks.append((block_start, move_idx))
        move_targets.append((move_idx, best))
        wl_pos = len(seq)
        seq.append("wl_value")
        d_pos = len(seq)
        seq.append("d_value")
        values.append((wl_pos, d_pos, float(q), float(d), True))
    ids = [V.token_to_idx[t] for t in seq]
    return ids, move_targets, blocks, values


def tensorize(ids, move_targets, blocks, values, rng: random.Random, max_seq_len: int, random_start: bool = True):
    """One training row (dict of 10 numpy arrays), as loader.py:69-184 builds it
    (random_start=False keeps the sequence start, as the thinking rows need)."""
    valid_starts = [0] + [vd[1] + 1 for vd in values[:-1]]
    start = rng.choice(valid_starts) if random_start else 0
    ids = ids[start:]
    move_targets = [(m - start, b) for m, b in move_targets if m >= start]
    values = [(w - start, d - start, wl, dd, ok) for w, d, wl, dd, ok in values if d >= start]
    adj = []
    for b0, b1 in blocks:
        a0, a1 = b0 - start, b1 - start
        if a1 > 0 and a0 < len(ids):
            adj.append((max(0, a0), min(len(ids), a1)))
    if len(ids) > max_seq_len:
        ids = ids[:max_seq_len]
        move_targets = [m for m in move_targets if m[0] < max_seq_len]
        values = [v for v in values if v[1] < max_seq_len]
        adj = [(b0, min(b1, max_seq_len)) for b0, b1 in adj if b0 < max_seq_len]
    values = [v for v in values if v[0] < max_seq_len and v[1] < max_seq_len]
    valid_moves = {v[0] - 1 for v in values}
    move_targets = [m for m in move_targets if m[0] in valid_moves]

    S = max_seq_len
    n = len(ids)
    input_ids = np.full(S, V.token_to_idx["pad"], dtype=np.int64)
    input_ids[:n] = ids
    board_t = np.full(S, IGNORE_INDEX, dtype=np.int64)
    if n > 1:
        board_t[: n - 1] = _FULL_TO_BOARD[input_ids[1:n]]
    move_t = np.full(S, IGNORE_INDEX, dtype=np.int64)
    move_mask = np.zeros(S, dtype=bool)
    wl_pos = np.zeros(S, dtype=bool)
    d_pos = np.zeros(S, dtype=bool)
    wl_t = np.zeros(S, dtype=np.float32)
    d_t = np.zeros(S, dtype=np.float32)
    wdl_valid = np.zeros(S, dtype=bool)
    generic = V.board_token_to_idx["generic_move"]
    for m_idx, best in move_targets:
        stm = m_idx - 1
        if 0 <= stm < S:
            board_t[stm] = generic
            move_t[stm] = V.full_idx_to_move_idx[V.token_to_idx[best]]
            move_mask[stm] = True
    for w, d, wl, dd, ok in values:
        if w < S:
            wl_pos[w] = True
            wl_t[w] = wl
            wdl_valid[w] = ok
        if d < S:
            d_pos[d] = True
            d_t[d] = dd
            wdl_valid[d] = ok
        stm = w - 2
        if 0 <= stm < S:
            wl_t[stm] = wl
            d_t[stm] = dd
            wdl_valid[stm] = ok
    block_id = np.arange(S, dtype=np.int64) + len(adj)
    for k, (b0, b1) in enumerate(adj):
        block_id[b0:b1] = k
    return {"input_ids": input_ids, "board_target_ids": board_t, "move_target_ids": move_t, "move_mask": move_mask,
            "wl_positions": wl_pos, "d_positions": d_pos, "wl_targets": wl_t, "d_targets": d_t,
            "wdl_valid": wdl_valid, "block_id": block_id}


class SyntheticGames:
    """Endless seeded stream of training rows from random-playout games.

    ``min_plies``/``max_plies`` bound the game length (uniform).  Only the
    plies that can land in the window are generated: the start ply is drawn
    first (uniform over the game's ply boundaries, as the loader does), and
    play stops once the window is certainly full.
    """

    def __init__(self, max_seq_len=256, skip_board_prob=0.2, min_plies=8, max_plies=120, seed=0, rank=0):
        self.S = max_seq_len
        self.skip = skip_board_prob
        self.lo, self.hi = min_plies, max_plies
        self.rng = random.Random(seed + rank * 7919)

    def row(self):
        rng = self.rng
        n_plies = rng.randint(self.lo, self.hi)
        # a ply costs >= 3 tokens, so no window reaches past start + S/3 + 1 plies
        plies = random_game(rng, n_plies)
        ids, mt, blocks, values = game_to_token_ids(plies, rng, self.skip)
        return tensorize(ids, mt, blocks, values, rng, self.S)

    def batch(self, batch_size: int) -> dict:
        rows = [self.row() for _ in range(batch_size)]
        return collate(rows)


def collate(rows) -> dict:
    out = {}
    for k in KEYS:
        arr = np.stack([r[k] for r in rows])
        out[k] = torch.from_numpy(arr)
    return out


def synthetic_batches(n_batches: int, batch_size: int, max_seq_len: int = 256, seed: int = 0, rank: int = 0,
                      min_plies: int = 8, max_plies: int = 120, skip_board_prob: float = 0.2):
    src = SyntheticGames(max_seq_len, skip_board_prob, min_plies, max_plies, seed, rank)
    return [src.batch(batch_size) for _ in range(n_batches)]


# ---------------------------------------------------------------------------
# Thinking-variation rows (the MoE variant's long sequences)
# ---------------------------------------------------------------------------
def _wdl(rng: random.Random):
    w, d = rng.random(), rng.random()
    if w + d > 1.0:
        w, d = 1.0 - w, 1.0 - d
    return w - (1.0 - w - d), d


def thinking_game_to_token_ids(rng: random.Random, min_lines=3, max_lines=6, min_depth=2, max_depth=8,
                               max_opening=40):
    """One thinking-variation sequence in the layout of
    chessdecoder/finetune/data.py:144-247: root board block, ``start_think``,
    then 3-6 candidate lines, each 2-8 plies of [move][wl_value][d_value]
    [board68] and an ``end_var``, then ``end_think``, the final move and its
    wl / d placeholders.  Positions come from a seeded random opening; lines
    are seeded uniform-random legal continuations; WL / D targets are uniform
    on the simplex.  Every board is its own block; each move is predicted from
    the token before it (stm, ``start_think`` or ``end_var``, ``end_think``).
    Returns (ids, move_targets, blocks, values) as ``game_to_token_ids``."""
    from .chessgen import Position
    while True:
        pos = Position()
        for _ in range(rng.randint(0, max_opening)):
            moves = pos.legal_moves()
            if not moves:
                break
            pos = pos.apply(moves[rng.randrange(len(moves))])
        root_moves = pos.legal_moves()
        if root_moves:
            break
    seq, move_targets, blocks, values = [], [], [], []
    b0 = len(seq)
    seq.extend(pos.position_tokens())
    blocks.append((b0, len(seq)))
    seq.append("start_think")
    for _ in range(rng.randint(min_lines, max_lines)):
        p = pos
        for _ in range(rng.randint(min_depth, max_depth)):
            moves = p.legal_moves()
            if not moves:
                break
            chosen = moves[rng.randrange(len(moves))]
            mv = Position.move_token(chosen)
            move_targets.append((len(seq), mv))
            seq.append(mv)
            p = p.apply(chosen)
            wl, dd = _wdl(rng)
            values.append((len(seq), len(seq) + 1, wl, dd, True))
            seq += ["wl_value", "d_value"]
            b0 = len(seq)
            seq.extend(p.position_tokens())
            blocks.append((b0, len(seq)))
        seq.append("end_var")
    seq.append("end_think")
    mv = Position.move_token(root_moves[rng.randrange(len(root_moves))])
    move_targets.append((len(seq), mv))
    seq.append(mv)
    wl, dd = _wdl(rng)
    values.append((len(seq), len(seq) + 1, wl, dd, True))
    seq += ["wl_value", "d_value"]
    return [V.token_to_idx[t] for t in seq], move_targets, blocks, values


def thinking_batches(n_batches: int, batch_size: int, max_seq_len: int = 4096, seed: int = 0, rank: int = 0):
    """Seeded batches of thinking-variation rows, padded / truncated to max_seq_len."""
    rng = random.Random(seed + rank * 7919)
    out = []
    for _ in range(n_batches):
        rows = []
        for _ in range(batch_size):
            ids, mt, blocks, values = thinking_game_to_token_ids(rng)
            rows.append(tensorize(ids, mt, blocks, values, rng, max_seq_len, random_start=False))
        out.append(collate(rows))
    return out


# ---------------------------------------------------------------------------
# Finetune rows (thinking head + final move): chessdecoder/finetune/loader.py
# ---------------------------------------------------------------------------
FINETUNE_KEYS = KEYS + ("thinking_move_mask",)


def tensorize_variation(ids, thinking, final, values, blocks, max_seq_len: int):
    """One finetune row as ``_build_variation_tensors`` builds it
    (chessdecoder/finetune/loader.py:337-440): shifted board targets; at every
    thinking prediction position the move target, ``thinking_move_mask`` and a
    board target of ``generic_move`` (after ``start_think``), ``new_variation``
    (after ``end_var``) or ``continue_var`` (a board's stm); at the final
    prediction position (``end_think``) the move target, ``move_mask`` and
    ``generic_move``; WL / D targets at their placeholders and copied to the
    prediction position two tokens before the WL placeholder; a block id per
    board, unique ids elsewhere.

    thinking: [(predict_pos, move_token)], final: (predict_pos, move_token) or None,
    values: [(wl_pos, d_pos, wl, d, valid)], blocks: [(start, end)]."""
    S = max_seq_len
    n = min(len(ids), S)
    input_ids = np.full(S, V.token_to_idx["pad"], dtype=np.int64)
    input_ids[:n] = ids[:n]
    board_t = np.full(S, IGNORE_INDEX, dtype=np.int64)
    if n > 1:
        board_t[: n - 1] = _FULL_TO_BOARD[input_ids[1:n]]
    move_t = np.full(S, IGNORE_INDEX, dtype=np.int64)
    move_mask = np.zeros(S, dtype=bool)
    think_mask = np.zeros(S, dtype=bool)
    start_think, end_var = V.token_to_idx["start_think"], V.token_to_idx["end_var"]
    bt = V.board_token_to_idx
    for pos, mv in thinking:
        if not 0 <= pos < S:
            continue
        move_t[pos] = V.full_idx_to_move_idx[V.token_to_idx[mv]]
        think_mask[pos] = True
        tok = ids[pos]
        board_t[pos] = (bt["generic_move"] if tok == start_think else
                        bt["new_variation"] if tok == end_var else bt["continue_var"])
    if final is not None and 0 <= final[0] < S:
        move_t[final[0]] = V.full_idx_to_move_idx[V.token_to_idx[final[1]]]
        move_mask[final[0]] = True
        board_t[final[0]] = bt["generic_move"]
    wl_pos = np.zeros(S, dtype=bool)
    d_pos = np.zeros(S, dtype=bool)
    wl_t = np.zeros(S, dtype=np.float32)
    d_t = np.zeros(S, dtype=np.float32)
    valid = np.zeros(S, dtype=bool)
    for w, d, wl, dd, ok in values:
        if w < S:
            wl_pos[w], wl_t[w], valid[w] = True, wl, ok
        if d < S:
            d_pos[d], d_t[d], valid[d] = True, dd, ok
        p = w - 2
        if 0 <= p < S:
            wl_t[p], d_t[p], valid[p] = wl, dd, ok
    block_id = np.arange(S, dtype=np.int64) + len(blocks)
    for k, (b0, b1) in enumerate(blocks):
        block_id[b0:b1] = k
    return {"input_ids": input_ids, "board_target_ids": board_t, "move_target_ids": move_t, "move_mask": move_mask,
            "wl_positions": wl_pos, "d_positions": d_pos, "wl_targets": wl_t, "d_targets": d_t,
            "wdl_valid": valid, "block_id": block_id, "thinking_move_mask": think_mask}


def finetune_batches(n_batches: int, batch_size: int, max_seq_len: int = 4096, seed: int = 0, rank: int = 0,
                     min_lines: int = 3, max_lines: int = 6, min_depth: int = 2, max_depth: int = 8):
    """Seeded finetune batches: thinking-variation sequences (the layout of
    chessdecoder/finetune/data.py:144-247) in which every variation move is a
    thinking-head target and the move after ``end_think`` the policy-head
    target."""
    rng = random.Random(seed + rank * 7919)
    out = []
    for _ in range(n_batches):
        rows = []
        for _ in range(batch_size):
            ids, mt, blocks, values = thinking_game_to_token_ids(rng, min_lines, max_lines, min_depth, max_depth)
            preds = [(m - 1, mv) for m, mv in mt]  # each move is predicted from the token before it
            rows.append(tensorize_variation(ids, preds[:-1], preds[-1], values, blocks, max_seq_len))
        out.append({k: torch.from_numpy(np.stack([r[k] for r in rows])) for k in FINETUNE_KEYS})
    return out
