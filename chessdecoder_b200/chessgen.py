"""Minimal legal-move generator for seeded synthetic games.

The reference trains on lc0-derived parquet files that are not available; the
benchmark instead plays uniform-random legal games from the start position.
python-chess (which the reference uses for FEN handling) is not installed, so
this module carries just enough chess to do that: a 64-square mailbox board,
pseudo-legal generation for all pieces (castling, en passant, promotions to
q/r/b), and a king-safety filter.  Moves are spelled in the model vocabulary's
form: castling as king-takes-rook (``e1h1``), like
chessdecoder/utils/uci.py:26-28 ``to_model_uci``; knight promotions are not
generated because ``a7a8n`` has no token.

Squares are indexed a1=0, b1=1, ..., h8=63 (rank*8 + file), the order of
``chess.SQUARES`` that chessdecoder/dataloader/data.py:24 walks.
"""
from __future__ import annotations

import random

EMPTY = "."
FILES = "abcdefgh"

_KNIGHT = [(1, 2), (2, 1), (2, -1), (1, -2), (-1, -2), (-2, -1), (-2, 1), (-1, 2)]
_KING = [(1, 0), (1, 1), (0, 1), (-1, 1), (-1, 0), (-1, -1), (0, -1), (1, -1)]
_ROOK = [(1, 0), (0, 1), (-1, 0), (0, -1)]
_BISHOP = [(1, 1), (1, -1), (-1, 1), (-1, -1)]


def _targets(deltas):
    out = []
    for sq in range(64):
        r, f = divmod(sq, 8)
        out.append([(r + dr) * 8 + f + df for dr, df in deltas if 0 <= r + dr < 8 and 0 <= f + df < 8])
    return out


def _rays(deltas):
    out = []
    for sq in range(64):
        r, f = divmod(sq, 8)
        rays = []
        for dr, df in deltas:
            ray, rr, ff = [], r + dr, f + df
            while 0 <= rr < 8 and 0 <= ff < 8:
                ray.append(rr * 8 + ff)
                rr += dr
                ff += df
            rays.append(ray)
        out.append(rays)
    return out


KNIGHT_T = _targets(_KNIGHT)
KING_T = _targets(_KING)
ROOK_R = _rays(_ROOK)
BISHOP_R = _rays(_BISHOP)

PIECE_NAMES = {"k": "king", "q": "queen", "r": "rook", "b": "bishop", "n": "knight", "p": "pawn"}


def sq_name(sq: int) -> str:
    return f"{FILES[sq % 8]}{sq // 8 + 1}"


class Position:
    """Board state: ``board`` list of 64 chars ('PNBRQK' white, 'pnbrqk' black, '.')."""

    __slots__ = ("board", "white", "castling", "ep")

    def __init__(self, board=None, white=True, castling="KQkq", ep=-1):
        if board is None:
            board = list("RNBQKBNR" + "P" * 8 + EMPTY * 32 + "p" * 8 + "rnbqkbnr")
        self.board = board
        self.white = white
        self.castling = castling
        self.ep = ep

    @classmethod
    def from_fen(cls, fen: str) -> "Position":
        parts = fen.split()
        rows = parts[0].split("/")
        board = [EMPTY] * 64
        for i, row in enumerate(rows):
            rank = 7 - i
            f = 0
            for ch in row:
                if ch.isdigit():
                    f += int(ch)
                else:
                    board[rank * 8 + f] = ch
                    f += 1
        white = parts[1] == "w"
        castling = "" if parts[2] == "-" else parts[2]
        ep = -1 if len(parts) < 4 or parts[3] == "-" else (int(parts[3][1]) - 1) * 8 + FILES.index(parts[3][0])
        return cls(board, white, castling, ep)

    def fen(self, halfmove: int = 0, fullmove: int = 1) -> str:
        """FEN of the position (the form the reference's parquet rows carry)."""
        rows = []
        for rank in range(7, -1, -1):
            row, run = "", 0
            for f in range(8):
                p = self.board[rank * 8 + f]
                if p == EMPTY:
                    run += 1
                else:
                    row += (str(run) if run else "") + p
                    run = 0
            rows.append(row + (str(run) if run else ""))
        ep = "-" if self.ep < 0 else sq_name(self.ep)
        cast = "".join(c for c in "KQkq" if c in self.castling) or "-"
        return f"{'/'.join(rows)} {'w' if self.white else 'b'} {cast} {ep} {halfmove} {fullmove}"

    def copy(self) -> "Position":
        return Position(self.board[:], self.white, self.castling, self.ep)

    # -- attacks -----------------------------------------------------------
    def attacked(self, sq: int, by_white: bool) -> bool:
        b = self.board
        kn, kg, pn = ("N", "K", "P") if by_white else ("n", "k", "p")
        rq = ("R", "Q") if by_white else ("r", "q")
        bq = ("B", "Q") if by_white else ("b", "q")
        for t in KNIGHT_T[sq]:
            if b[t] == kn:
                return True
        for t in KING_T[sq]:
            if b[t] == kg:
                return True
        r, f = divmod(sq, 8)
        pr = r - 1 if by_white else r + 1  # rank the attacking pawn stands on
        if 0 <= pr < 8:
            for pf in (f - 1, f + 1):
                if 0 <= pf < 8 and b[pr * 8 + pf] == pn:
                    return True
        for ray in ROOK_R[sq]:
            for t in ray:
                p = b[t]
                if p != EMPTY:
                    if p in rq:
                        return True
                    break
        for ray in BISHOP_R[sq]:
            for t in ray:
                p = b[t]
                if p != EMPTY:
                    if p in bq:
                        return True
                    break
        return False

    def king_square(self, white: bool) -> int:
        return self.board.index("K" if white else "k")

    def in_check(self) -> bool:
        return self.attacked(self.king_square(self.white), not self.white)

    # -- moves ---------------------------------------------------------------
    def _own(self, p: str) -> bool:
        return p != EMPTY and (p.isupper() == self.white)

    def _enemy(self, p: str) -> bool:
        return p != EMPTY and (p.isupper() != self.white)

    def pseudo_moves(self):
        """Yields (from, to, promo, kind) with kind in {'n','c','ep','ck','cq','d'}."""
        b = self.board
        white = self.white
        for sq in range(64):
            p = b[sq]
            if not self._own(p):
                continue
            t = p.lower()
            if t == "p":
                d = 8 if white else -8
                start_rank, promo_rank = (1, 6) if white else (6, 1)
                r, f = divmod(sq, 8)
                one = sq + d
                if b[one] == EMPTY:
                    if r == promo_rank:
                        for pr in "qrb":
                            yield sq, one, pr, "n"
                    else:
                        yield sq, one, "", "n"
                        two = sq + 2 * d
                        if r == start_rank and b[two] == EMPTY:
                            yield sq, two, "", "d"
                for df in (-1, 1):
                    if 0 <= f + df < 8:
                        to = one + df
                        if self._enemy(b[to]):
                            if r == promo_rank:
                                for pr in "qrb":
                                    yield sq, to, pr, "c"
                            else:
                                yield sq, to, "", "c"
                        elif to == self.ep:
                            yield sq, to, "", "ep"
            elif t == "n":
                for to in KNIGHT_T[sq]:
                    if not self._own(b[to]):
                        yield sq, to, "", "n"
            elif t == "k":
                for to in KING_T[sq]:
                    if not self._own(b[to]):
                        yield sq, to, "", "n"
                yield from self._castles(sq)
            else:
                rays = []
                if t in "rq":
                    rays += ROOK_R[sq]
                if t in "bq":
                    rays += BISHOP_R[sq]
                for ray in rays:
                    for to in ray:
                        q = b[to]
                        if q == EMPTY:
                            yield sq, to, "", "n"
                        else:
                            if self._enemy(q):
                                yield sq, to, "", "n"
                            break

    def _castles(self, ksq: int):
        b = self.board
        if self.white:
            if ksq != 4:
                return
            rights, rook, home = "KQ", "R", 0
        else:
            if ksq != 60:
                return
            rights, rook, home = "kq", "r", 56
        enemy_white = not self.white
        if rights[0] in self.castling and b[home + 7] == rook and b[home + 5] == EMPTY and b[home + 6] == EMPTY:
            if not any(self.attacked(s, enemy_white) for s in (home + 4, home + 5, home + 6)):
                yield ksq, home + 7, "", "ck"
        if rights[1] in self.castling and b[home] == rook and all(b[home + i] == EMPTY for i in (1, 2, 3)):
            if not any(self.attacked(s, enemy_white) for s in (home + 4, home + 3, home + 2)):
                yield ksq, home, "", "cq"

    def apply(self, mv) -> "Position":
        frm, to, promo, kind = mv
        n = self.copy()
        b = n.board
        p = b[frm]
        home = 0 if self.white else 56
        if kind in ("ck", "cq"):
            b[frm] = EMPTY
            b[to] = EMPTY
            if kind == "ck":
                b[home + 6], b[home + 5] = p, ("R" if self.white else "r")
            else:
                b[home + 2], b[home + 3] = p, ("R" if self.white else "r")
        else:
            b[frm] = EMPTY
            if kind == "ep":
                b[to - 8 if self.white else to + 8] = EMPTY
            b[to] = (promo.upper() if self.white else promo) if promo else p
        # castling rights
        cr = n.castling
        for sq, lost in ((4, "KQ"), (60, "kq"), (7, "K"), (0, "Q"), (63, "k"), (56, "q")):
            if frm == sq or to == sq:
                cr = "".join(c for c in cr if c not in lost)
        n.castling = cr
        n.ep = (frm + to) // 2 if kind == "d" else -1
        n.white = not self.white
        return n

    def legal_moves(self):
        out = []
        for mv in self.pseudo_moves():
            n = self.apply(mv)
            if not n.attacked(n.king_square(self.white), not self.white):
                out.append(mv)
        return out

    # -- spelling --------------------------------------------------------------
    @staticmethod
    def move_token(mv) -> str:
        """Model-vocabulary spelling (castling = king takes rook)."""
        frm, to, promo, _ = mv
        return sq_name(frm) + sq_name(to) + promo

    def castling_token(self) -> str:
        r = "".join(c for c in "KQkq" if c in self.castling)
        return r if r else "no_castling_rights"

    def position_tokens(self) -> list[str]:
        """The 68-token board block of chessdecoder/dataloader/data.py:7-48."""
        toks = ["start_pos"]
        for p in self.board:
            if p == EMPTY:
                toks.append("empty")
            else:
                toks.append(("white_" if p.isupper() else "black_") + PIECE_NAMES[p.lower()])
        toks.append("end_pos")
        toks.append(self.castling_token())
        toks.append("white_to_move" if self.white else "black_to_move")
        return toks


def perft(pos: Position, depth: int) -> int:
    if depth == 0:
        return 1
    return sum(perft(pos.apply(m), depth - 1) for m in pos.legal_moves()) if depth > 1 else len(pos.legal_moves())


def random_game_rows(rng: random.Random, n_plies: int) -> dict:
    """A uniform-random legal game as parquet-style columns (one entry per ply):
    ``fen``, ``played_move``, ``best_move``, ``played_q``, ``played_d`` --
    the per-ply fields chessdecoder/dataloader/data.py:50-97 reads."""
    pos = Position()
    cols = {"fen": [], "played_move": [], "best_move": [], "played_q": [], "played_d": []}
    for ply in range(n_plies):
        moves = pos.legal_moves()
        if not moves:
            break
        played = moves[rng.randrange(len(moves))]
        best = moves[rng.randrange(len(moves))]
        w, d = rng.random(), rng.random()
        if w + d > 1.0:
            w, d = 1.0 - w, 1.0 - d
        cols["fen"].append(pos.fen(0, ply // 2 + 1))
        cols["played_move"].append(Position.move_token(played))
        cols["best_move"].append(Position.move_token(best))
        cols["played_q"].append(w - (1.0 - w - d))
        cols["played_d"].append(d)
        pos = pos.apply(played)
    return cols


def random_game(rng: random.Random, n_plies: int):
    """Plays up to n_plies uniform-random legal moves from the start position.

    Returns a list of plies: (position_tokens, played_move, best_move,
    played_q, played_d).  ``best_move`` is an independent uniform legal move;
    (w, d) is uniform on the simplex w + d <= 1 and played_q = w - l.
    Stops early at checkmate / stalemate.
    """
    pos = Position()
    plies = []
    for _ in range(n_plies):
        moves = pos.legal_moves()
        if not moves:
            break
        played = moves[rng.randrange(len(moves))]
        best = moves[rng.randrange(len(moves))]
        w, d = rng.random(), rng.random()
        if w + d > 1.0:
            w, d = 1.0 - w, 1.0 - d
        l_ = 1.0 - w - d
        plies.append((pos.position_tokens(), Position.move_token(played), Position.move_token(best), w - l_, d))
        pos = pos.apply(played)
    return plies
