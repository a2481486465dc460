"""Pretraining batch producer: the reference's parquet data loader with the
per-token work in native code.

Mirrors chessdecoder/dataloader/loader.py (``ChessIterableDataset``,
``get_dataloader``): the same file sharding over ranks and workers, the same
seeding (``seed + epoch*100003 + rank*7919 + worker*997``), file and game
shuffles, and per game the same two random decisions (a board kept per ply
with probability 1 - skip_board_prob, a random start among the valid starts),
drawn from Python's ``random`` generator in the reference's order.  The FEN
parsing, tokenisation and tensorisation of a whole batch of games then run in
``cdk_tokenize_games`` (libcdk.so, host threads), which restates
chessdecoder/dataloader/data.py:7-97 and loader.py:69-184.

The dataset yields whole batches (a dict of [B, S] tensors, the reference's
10 keys); ``get_dataloader`` wraps it in a ``DataLoader`` with
``batch_size=None`` so that a batch is, as in the reference, B consecutive
rows of one worker.
"""
from __future__ import annotations

import ctypes as C
import glob
import math
import os
import random
from typing import Iterable, Optional

import numpy as np
import torch

from . import _lib
from . import vocab as V

KEYS = ("input_ids", "board_target_ids", "move_target_ids", "move_mask", "wl_positions", "d_positions",
        "wl_targets", "d_targets", "wdl_valid", "block_id")


def _pack_strings(items: Iterable[str]):
    data = bytearray()
    offs = [0]
    for s in items:
        data += s.encode()
        offs.append(len(data))
    return bytes(data) or b"\0", np.asarray(offs, dtype=np.int64)


class GameTokenizer:
    """Native tokenisation + tensorisation of pretraining games.

    ``games``: a list of games, each a dict of per-ply sequences in ply order:
    ``fen``, ``played_move`` (None / "" = no move), ``best_move``,
    ``played_q``, ``played_d`` (None / NaN = invalid).  ``draws``: per game,
    (include_board per ply, start index) -- see ``draw_decisions``."""

    def __init__(self, max_seq_len: int, n_threads: int = 0):
        self.S = int(max_seq_len)
        self.n_threads = int(n_threads)
        lib = _lib.load()
        chars, offs = _pack_strings(V.idx_to_token[i] for i in range(V.vocab_size))
        to_board = np.full(V.vocab_size, -1, dtype=np.int32)
        for full, b in V.full_idx_to_board_idx.items():
            to_board[full] = b
        to_move = np.full(V.vocab_size, -1, dtype=np.int32)
        for full, m in V.full_idx_to_move_idx.items():
            to_move[full] = m
        self._keep = (chars, offs, to_board, to_move)
        self._lib = lib
        self._vocab = lib.cdk_vocab_create(chars, offs.ctypes.data, V.vocab_size, to_board.ctypes.data,
                                           to_move.ctypes.data)
        if not self._vocab:
            raise RuntimeError("cdk_vocab_create: the vocabulary lacks a structural token")

    def __del__(self):
        if getattr(self, "_vocab", None):
            self._lib.cdk_vocab_destroy(self._vocab)
            self._vocab = None

    @staticmethod
    def draw_decisions(game: dict, rng: random.Random, skip_board_prob: float):
        """The reference's random draws for one game, in its order:
        ``random.random()`` per ply after the first (data.py:56), then
        ``random.choice(valid_starts)`` (loader.py:77)."""
        n = len(game["fen"])
        include = np.ones(n, dtype=np.uint8)
        for i in range(1, n):
            include[i] = 1 if rng.random() > skip_board_prob else 0
        n_values = sum(1 for m in game["played_move"] if m)
        starts = list(range(max(n_values, 1)))
        return include, rng.choice(starts)

    def __call__(self, games: list, draws: list) -> dict:
        B, S = len(games), self.S
        fens, played, best, q, d, inc, start = [], [], [], [], [], [], []
        game_off = [0]
        for g, (include, st) in zip(games, draws):
            n = len(g["fen"])
            fens += list(g["fen"])
            played += [m if m else "" for m in g["played_move"]]
            best += [m if m else "" for m in g["best_move"]]
            q += [np.nan if v is None else float(v) for v in g["played_q"]]
            d += [np.nan if v is None else float(v) for v in g["played_d"]]
            inc.append(np.asarray(include, dtype=np.uint8))
            start.append(int(st))
            game_off.append(game_off[-1] + n)
        fc, fo = _pack_strings(fens)
        pc, po = _pack_strings(played)
        bc, bo = _pack_strings(best)
        game_off = np.asarray(game_off, dtype=np.int64)
        q = np.asarray(q, dtype=np.float64)
        d = np.asarray(d, dtype=np.float64)
        inc = np.concatenate(inc) if inc else np.zeros(0, dtype=np.uint8)
        start = np.asarray(start, dtype=np.int64)
        out = {"input_ids": torch.empty(B, S, dtype=torch.int64),
               "board_target_ids": torch.empty(B, S, dtype=torch.int64),
               "move_target_ids": torch.empty(B, S, dtype=torch.int64),
               "move_mask": torch.empty(B, S, dtype=torch.bool),
               "wl_positions": torch.empty(B, S, dtype=torch.bool),
               "d_positions": torch.empty(B, S, dtype=torch.bool),
               "wl_targets": torch.empty(B, S, dtype=torch.float32),
               "d_targets": torch.empty(B, S, dtype=torch.float32),
               "wdl_valid": torch.empty(B, S, dtype=torch.bool),
               "block_id": torch.empty(B, S, dtype=torch.int64)}
        ptr = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
        rc = self._lib.cdk_tokenize_games(
            self._vocab, B, ptr(game_off), fc, ptr(fo), pc, ptr(po), bc, ptr(bo), ptr(q), ptr(d),
            ptr(inc) if inc.size else None, ptr(start), S, self.n_threads,
            *[out[k].data_ptr() for k in KEYS])
        if rc != 0:
            raise RuntimeError(f"cdk_tokenize_games failed with status {rc}")
        return out


def games_from_frame(df) -> list:
    """Games of one parquet file in the reference's order: grouped by
    ``game_id`` in order of first appearance, plies sorted (loader.py:59-67)."""
    out = []
    for _, g in df.groupby("game_id", sort=False):
        g = g.sort_values("ply")
        col = lambda name: list(g[name]) if name in g.columns else [None] * len(g)  # noqa: E731
        out.append({"fen": list(g["fen"]), "played_move": col("played_move"), "best_move": col("best_move"),
                    "played_q": [None if v is None or (isinstance(v, float) and math.isnan(v)) else v
                                 for v in col("played_q")],
                    "played_d": [None if v is None or (isinstance(v, float) and math.isnan(v)) else v
                                 for v in col("played_d")]})
    return out


class ChessIterableDataset(torch.utils.data.IterableDataset):
    """``chessdecoder/dataloader/loader.py:ChessIterableDataset`` yielding whole
    batches of ``batch_size`` rows built by the native producer."""

    def __init__(self, parquet_dir, max_seq_len=2048, shuffle_files=True, shuffle_games=True, skip_board_prob=0.0,
                 seed=42, rank=0, world_size=1, batch_size=16, n_threads=0):
        self.parquet_dir = parquet_dir
        self.max_seq_len = max_seq_len
        self.shuffle_files = shuffle_files
        self.shuffle_games = shuffle_games
        self.skip_board_prob = skip_board_prob
        self.pad_id = V.token_to_idx["pad"]
        self.seed = seed
        self.epoch = 0
        self.rank = rank
        self.world_size = world_size
        self.batch_size = batch_size
        self.n_threads = n_threads
        self.files = sorted(glob.glob(os.path.join(parquet_dir, "*.parquet")))

    def __iter__(self):
        import pandas as pd
        info = torch.utils.data.get_worker_info()
        worker_id = info.id if info is not None else 0
        epoch_seed = self.seed + self.epoch * 100003 + self.rank * 7919 + worker_id * 997
        rng = random.Random(epoch_seed)
        nrng = np.random.RandomState(epoch_seed % (2 ** 32))
        rank_files = self.files[self.rank::self.world_size]
        if info is None:
            files = list(rank_files)
        else:
            per = int(math.ceil(len(rank_files) / float(info.num_workers)))
            files = rank_files[worker_id * per:min(worker_id * per + per, len(rank_files))]
        if self.shuffle_files:
            rng.shuffle(files)
        tok = GameTokenizer(self.max_seq_len, self.n_threads)
        pending, draws = [], []
        for path in files:
            try:
                games = games_from_frame(pd.read_parquet(path))
            except Exception as e:  # the reference skips unreadable files
                print(f"Error reading file {path}: {e}")
                continue
            order = list(range(len(games)))
            if self.shuffle_games:
                nrng.shuffle(order)
            for gi in order:
                g = games[gi]
                pending.append(g)
                draws.append(tok.draw_decisions(g, rng, self.skip_board_prob))
                if len(pending) == self.batch_size:
                    yield tok(pending, draws)
                    pending, draws = [], []
        if pending:
            yield tok(pending, draws)


def get_dataloader(parquet_dir, batch_size=16, num_workers=0, max_seq_len=2048, skip_board_prob=0.0, seed=42,
                   rank=0, world_size=1, n_threads: Optional[int] = None):
    """``chessdecoder/dataloader/loader.py:get_dataloader`` on the native producer."""
    ds = ChessIterableDataset(parquet_dir, shuffle_files=True, shuffle_games=True, max_seq_len=max_seq_len,
                              skip_board_prob=skip_board_prob, seed=seed, rank=rank, world_size=world_size,
                              batch_size=batch_size, n_threads=1 if (n_threads is None and num_workers) else
                              (n_threads or 0))
    return torch.utils.data.DataLoader(ds, batch_size=None, num_workers=num_workers)
