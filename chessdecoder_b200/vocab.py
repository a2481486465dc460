"""ChessDecoder token vocabulary (1968 tokens) and its board / move sub-vocabularies.

Same tokens, order and indices as chessdecoder/models/vocab.py (the table is an
interface: checkpoints index embedding rows and head outputs by it).  The move
list is generated from board geometry instead of being spelled out:

* for every from-square a1..h8 (index = rank*8 + file), every to-square in
  increasing index order that a queen or a knight could reach on an empty
  board (1792 moves; castling is written king-takes-rook, e.g. ``e1h1``, which
  is already a rook-line move);
* then white promotions from rank 7 to rank 8 (straight and both captures),
  each as ``q``, ``r``, ``b`` (66 tokens; knight promotions are not in the
  vocabulary);
* then black promotions from rank 2 to rank 1 in the same pattern (66 tokens).

The resulting 1924 entries are pinned against the reference table by
tests/golden/vocab_reference.json.
"""
from __future__ import annotations

import itertools

FILES = "abcdefgh"


def square_name(sq: int) -> str:
    return f"{FILES[sq % 8]}{sq // 8 + 1}"


def _queen_or_knight_reachable(frm: int, to: int) -> bool:
    fr, ff = divmod(frm, 8)
    tr, tf = divmod(to, 8)
    dr, df = tr - fr, tf - ff
    if dr == 0 and df == 0:
        return False
    if dr == 0 or df == 0 or abs(dr) == abs(df):
        return True
    return (abs(dr), abs(df)) in ((1, 2), (2, 1))


def _build_policy_index() -> list[str]:
    moves = []
    for frm in range(64):
        for to in range(64):
            if _queen_or_knight_reachable(frm, to):
                moves.append(square_name(frm) + square_name(to))
    for from_rank, to_rank in ((7, 8), (2, 1)):
        for f in range(8):
            for df in (-1, 0, 1):
                tf = f + df
                if not 0 <= tf < 8:
                    continue
                for piece in "qrb":
                    moves.append(f"{FILES[f]}{from_rank}{FILES[tf]}{to_rank}{piece}")
    return moves


policy_index = _build_policy_index()
policy_to_idx = {u: i for i, u in enumerate(policy_index)}

pieces = ["king", "queen", "rook", "bishop", "knight", "pawn"]
colors = ["white", "black"]
piece_tokens = [f"{c}_{p}" for c in colors for p in pieces]

castling_tokens = ["".join(c) for r in range(1, 5) for c in itertools.combinations("KQkq", r)] + \
    ["no_castling_rights"]
special_tokens = ["start_pos", "end_pos", "white_to_move", "black_to_move", "empty", "pad", "bos", "eos",
                  "wl_value", "d_value", "start_think", "end_think"]

vocab = policy_index + piece_tokens + special_tokens + castling_tokens + \
    ["end_var", "continue_var", "new_variation", "generic_move"]
token_to_idx = {t: i for i, t in enumerate(vocab)}
idx_to_token = {i: t for i, t in enumerate(vocab)}
vocab_size = len(vocab)

POSITION_TOKEN_LENGTH = 68

board_vocab = (piece_tokens
               + ["start_pos", "end_pos", "white_to_move", "black_to_move", "empty", "wl_value", "d_value"]
               + castling_tokens
               + ["end_var", "continue_var", "new_variation", "generic_move", "end_think", "start_think"])
board_vocab_size = len(board_vocab)
board_token_to_idx = {t: i for i, t in enumerate(board_vocab)}
board_idx_to_full_idx = [token_to_idx[t] for t in board_vocab]

move_vocab = policy_index
move_vocab_size = len(move_vocab)
move_token_to_idx = {t: i for i, t in enumerate(move_vocab)}
move_idx_to_full_idx = [token_to_idx[t] for t in move_vocab]

full_idx_to_board_idx = {token_to_idx[t]: i for i, t in enumerate(board_vocab)}
full_idx_to_move_idx = {token_to_idx[t]: i for i, t in enumerate(move_vocab)}


def full_to_board_table():
    """Dense int list: full vocab id -> board sub-vocab id, or -100."""
    t = [-100] * vocab_size
    for full, b in full_idx_to_board_idx.items():
        t[full] = b
    return t


def full_to_move_table():
    """Dense int list: full vocab id -> move sub-vocab id, or -100."""
    t = [-100] * vocab_size
    for full, m in full_idx_to_move_idx.items():
        t[full] = m
    return t
