"""Kernel micro-benchmarks at the training step's shapes (also the target of
the ncu captures summarised under profiles/).

    python -m chessdecoder_b200.probe gemm --kind rope      # QKV projection + RoPE epilogue
    python -m chessdecoder_b200.probe gemm --kind dw        # weight-gradient GEMM (split-K atomics)
    python -m chessdecoder_b200.probe attn --nseq 128       # attention forward + backward
    python -m chessdecoder_b200.probe adamw

Each mode allocates only its operands (a few hundred MB, larger than the
126 MB L2 so that DRAM counters are meaningful), runs --warmup untimed and
--iters timed launches, and prints one JSON line with the CUDA-event time per
launch and the achieved FLOP/s or bytes/s.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from . import kernels as K
from .engine import rope_table


def _time(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def gemm_case(kind: str, T: int = 32768, E: int = 1024, F: int = 1536):
    dev = "cuda"
    bf = lambda *s: (torch.randn(*s, device=dev) * 0.05).to(torch.bfloat16)  # noqa: E731
    if kind == "rope":
        X, W = bf(T, E), bf(3 * E, E)
        out = torch.empty(T, 3 * E, device=dev, dtype=torch.bfloat16)
        rope = rope_table(256, 64).to(dev)
        fn = lambda: K.gemm(X, W, kind=K.EPI_ROPE_BF16, out=out, rope=rope, seq_len=256, rope_cols=2 * E)  # noqa
        M, N, Kd, nbytes = T, 3 * E, E, (T * E + 3 * E * E + T * 3 * E) * 2
    elif kind == "swiglu":
        X, W = bf(T, E), bf(2 * F, E)
        u = torch.empty(T, F, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(T, 2 * F, device=dev, dtype=torch.bfloat16)
        fn = lambda: K.gemm(X, W, kind=K.EPI_SWIGLU, out=u, out2=gu, half_n=F)  # noqa
        M, N, Kd, nbytes = T, 2 * F, E, (T * E + 2 * F * E + T * 3 * F) * 2
    elif kind == "resid":
        X, W = bf(T, E), bf(E, E)
        h = torch.randn(T, E, device=dev)
        out = torch.empty(T, E, device=dev)
        fn = lambda: K.gemm(X, W, kind=K.EPI_RESID_F32, out=out, resid=h)  # noqa
        M, N, Kd, nbytes = T, E, E, (T * E + E * E) * 2 + 2 * T * E * 4
    elif kind == "resid2":  # the down projection: K = d_ff
        X, W = bf(T, F), bf(E, F)
        h = torch.randn(T, E, device=dev)
        out = torch.empty(T, E, device=dev)
        fn = lambda: K.gemm(X, W, kind=K.EPI_RESID_F32, out=out, resid=h)  # noqa
        M, N, Kd, nbytes = T, E, F, (T * F + E * F) * 2 + 2 * T * E * 4
    elif kind == "dswiglu":  # [dg | du] = SwiGLU backward of dh W2, fused into the GEMM epilogue
        dH, W2 = bf(T, E), bf(E, F)
        gu = bf(T, 2 * F)
        dgu = torch.empty(T, 2 * F, device=dev, dtype=torch.bfloat16)
        fn = lambda: K.gemm(dH, W2, b_mn=True, kind=K.EPI_DSWIGLU, out=dgu, aux=gu, half_n=F, N=F)  # noqa
        M, N, Kd, nbytes = T, F, E, (T * E + E * F + 4 * T * F) * 2
    elif kind == "dx":
        dY, W = bf(T, 3 * E), bf(3 * E, E)
        out = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        fn = lambda: K.gemm(dY, W, b_mn=True, kind=K.EPI_STORE_BF16, out=out)  # noqa
        M, N, Kd, nbytes = T, E, 3 * E, (T * 3 * E + 3 * E * E + T * E) * 2
    elif kind == "dw":
        dY, X = bf(T, 3 * E), bf(T, E)
        out = torch.zeros(3 * E, E, device=dev)
        fn = lambda: K.gemm(dY, X, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=out)  # noqa
        M, N, Kd, nbytes = 3 * E, E, T, (T * 3 * E + T * E) * 2 + 3 * E * E * 4
    else:
        raise ValueError(kind)
    return fn, 2.0 * M * N * Kd, nbytes, f"M{M} N{N} K{Kd} {kind}"


def gemm_case_fp8(kind: str, T: int = 32768, E: int = 1024, F: int = 1536):
    """The same shapes with 8-bit K-major operands (the dX / dW shapes use the
    transposed copies the fp8 recipe makes)."""
    dev = "cuda"
    q = lambda *s: (torch.randn(*s, device=dev) * 0.5).to(torch.float8_e4m3fn)  # noqa: E731
    sc = torch.ones(1, device=dev)
    f8 = (0, 0, sc, sc)
    if kind == "rope":
        X, W = q(T, E), q(3 * E, E)
        out = torch.empty(T, 3 * E, device=dev, dtype=torch.bfloat16)
        rope = rope_table(256, 64).to(dev)
        fn = lambda: K.gemm(X, W, kind=K.EPI_ROPE_BF16, out=out, rope=rope, seq_len=256, rope_cols=2 * E, fp8=f8)  # noqa
        M, N, Kd, nbytes = T, 3 * E, E, T * E + 3 * E * E + T * 3 * E * 2
    elif kind == "swiglu":
        X, W = q(T, E), q(2 * F, E)
        u = torch.empty(T, F, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(T, 2 * F, device=dev, dtype=torch.bfloat16)
        fn = lambda: K.gemm(X, W, kind=K.EPI_SWIGLU, out=u, out2=gu, half_n=F, fp8=f8)  # noqa
        M, N, Kd, nbytes = T, 2 * F, E, T * E + 2 * F * E + T * 3 * F * 2
    elif kind == "resid":
        X, W = q(T, E), q(E, E)
        h = torch.randn(T, E, device=dev)
        out = torch.empty(T, E, device=dev)
        fn = lambda: K.gemm(X, W, kind=K.EPI_RESID_F32, out=out, resid=h, fp8=f8)  # noqa
        M, N, Kd, nbytes = T, E, E, T * E + E * E + 2 * T * E * 4
    elif kind == "dx":
        dY, Wt = q(T, 3 * E), q(E, 3 * E)
        out = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        fn = lambda: K.gemm(dY, Wt, kind=K.EPI_STORE_BF16, out=out, fp8=f8)  # noqa
        M, N, Kd, nbytes = T, E, 3 * E, T * 3 * E + 3 * E * E + T * E * 2
    else:
        dYt, Xt = q(3 * E, T), q(E, T)
        out = torch.zeros(3 * E, E, device=dev)
        fn = lambda: K.gemm(dYt, Xt, kind=K.EPI_ATOMIC_F32, out=out, fp8=f8)  # noqa
        M, N, Kd, nbytes = 3 * E, E, T, T * 3 * E + T * E + 3 * E * E * 4
    return fn, 2.0 * M * N * Kd, nbytes, f"M{M} N{N} K{Kd} {kind} fp8"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["gemm", "attn", "adamw", "tokenize", "decode"])
    ap.add_argument("--batch", type=int, default=64, help="decode: sequences")
    ap.add_argument("--keys", type=int, default=542, help="decode: cached keys per sequence")
    ap.add_argument("--new", type=int, default=1, help="decode: new tokens per sequence")
    ap.add_argument("--kind", default="rope", choices=["rope", "swiglu", "resid", "resid2", "dswiglu", "dx", "dw"])
    ap.add_argument("--fp8", action="store_true", help="8-bit operands (e4m3; e5m2 x e4m3 for dx / dw)")
    ap.add_argument("--nseq", type=int, default=128)
    ap.add_argument("--seq", type=int, default=256, help="attention sequence length (> 256: thinking-row blocks)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    K.lib()
    if a.mode == "gemm":
        fn, flops, nbytes, name = (gemm_case_fp8 if a.fp8 else gemm_case)(a.kind)
        ms = _time(fn, a.warmup, a.iters)
        print(json.dumps({"probe": name, "ms": ms, "tflops": flops / ms / 1e9, "alg_bytes": nbytes,
                          "alg_gbs": nbytes / ms / 1e6}))
    elif a.mode == "decode":
        # decode attention over one layer's cache: B sequences x 16 heads x `keys`
        # cached keys (bf16 K / V rows of 128 B), `new` queries per sequence
        B, H, L0, S_new = a.batch, 16, a.keys, a.new
        max_len = L0 + S_new
        g = torch.Generator(device="cuda").manual_seed(0)
        kc = torch.randn(B, H, max_len, 64, device="cuda", generator=g).to(torch.bfloat16)
        vc = torch.randn(B, H, max_len, 64, device="cuda", generator=g).to(torch.bfloat16)
        valid = torch.ones(B, max_len, dtype=torch.uint8, device="cuda")
        len_dev = torch.tensor([L0], dtype=torch.int32, device="cuda")
        q = torch.randn(B * S_new, H * 64, device="cuda", generator=g).to(torch.bfloat16)
        out = torch.empty_like(q)
        mode = K.BLOCK_VALID if S_new == 1 else K.BLOCK_ALL
        fn = lambda: K.decode_attn(q, kc, vc, len_dev, S_new, B, H, valid, out, block_mode=mode)  # noqa: E731
        ms = _time(fn, a.warmup, a.iters)
        nbytes = B * H * (L0 + S_new) * 64 * 2 * 2
        print(json.dumps({"probe": f"decode_attn B={B} H={H} keys={L0} new={S_new}", "us": ms * 1e3,
                          "alg_bytes": nbytes, "alg_gbs": nbytes / ms / 1e6, "err": K.get_error()}))
    elif a.mode == "attn":
        S, H = a.seq, 16
        E = H * 64
        nseq, ncaus = a.nseq, a.nseq // 2
        g = torch.Generator().manual_seed(0)
        qkv = (torch.randn(nseq * S, 3 * E, generator=g) * 0.8).to("cuda").to(torch.bfloat16)
        if S > 256:  # thinking-variation rows: a board block every 71 tokens
            from .data import thinking_batches
            bid = thinking_batches(1, nseq - ncaus, S, seed=0)[0]["block_id"]
        else:
            bid = (torch.arange(S) + 1000).repeat(nseq - ncaus, 1)
            for r in range(nseq - ncaus):  # three 68-token board blocks per sequence
                bid[r, 10:78] = 0
                bid[r, 81:149] = 1
                bid[r, 152:220] = 2
        bid32 = bid.to(torch.int32).cuda().contiguous()
        meta = K.attn_meta(bid32, S)
        out = torch.empty(nseq * S, E, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(nseq * H * S, device="cuda")
        dout = torch.randn(nseq * S, E, device="cuda").to(torch.bfloat16)
        dqkv = torch.empty_like(qkv)
        dsum = torch.empty(nseq * H * S, device="cuda")
        fwd = lambda: K.attn_fwd(qkv, out, lse, nseq, ncaus, S, H, bid32, meta)  # noqa
        bwd = lambda: K.attn_bwd(qkv, out, dout, lse, dsum, dqkv, nseq, ncaus, S, H, bid32, meta)  # noqa
        fwd()
        ms_f = _time(fwd, a.warmup, a.iters)
        ms_b = _time(bwd, a.warmup, a.iters)
        bytes_f = qkv.numel() * 2 + out.numel() * 2
        bytes_b = qkv.numel() * 2 * 2 + out.numel() * 2 * 2
        # allowed (query, key) pairs -> FLOPs (fwd 4*hd per pair, bwd 10*hd)
        pairs = ncaus * S * (S + 1) // 2
        for r in range(nseq - ncaus):
            _, cnt = torch.unique(bid[r], return_counts=True)
            pairs += S * (S + 1) // 2 + int((cnt * (cnt - 1) // 2).sum())
        pairs *= H
        print(json.dumps({"probe": f"attention nseq={nseq} S={S} H={H}", "fwd_ms": ms_f, "bwd_ms": ms_b,
                          "fwd_tflops": 4 * 64 * pairs / ms_f / 1e9, "bwd_tflops": 10 * 64 * pairs / ms_b / 1e9,
                          "fwd_alg_gbs": bytes_f / ms_f / 1e6, "bwd_alg_gbs": bytes_b / ms_b / 1e6,
                          "err": K.get_error()}))
    elif a.mode == "tokenize":
        # host batch producer: 256 random games (8-120 plies) -> [256, S] rows, skip_board_prob 0.2
        import random
        import time
        import numpy as np
        from .chessgen import random_game_rows
        from .loader import GameTokenizer
        rng = random.Random(0)
        S = a.seq
        games = [random_game_rows(rng, rng.randint(8, 120)) for _ in range(256)]
        res = {"probe": f"batch producer: 256 games -> [256, {S}] rows", "host_threads": os.cpu_count()}
        for th in (1, 0):
            tok = GameTokenizer(S, n_threads=th)
            drng = random.Random(1)
            draws = [tok.draw_decisions(g, drng, 0.2) for g in games]
            tok(games, draws)
            t0 = time.perf_counter()
            for _ in range(a.iters):
                tok(games, draws)
            dt = (time.perf_counter() - t0) / a.iters
            res[f"seq_per_s_threads_{th or 'all'}"] = len(games) / dt
            res[f"tokens_per_s_threads_{th or 'all'}"] = len(games) * S / dt
        print(json.dumps(res))
    else:
        n = 111_849_344
        p, gr, m, v = (torch.randn(n, device="cuda") for _ in range(4))
        pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
        part = torch.empty(1024, device="cuda")

        def step():
            K.sumsq(gr, part)
            K.adamw(p, gr, m, v, pb, part, max_norm=10.0, lr=3e-4, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.1, step=1)
        ms = _time(step, a.warmup, a.iters)
        nbytes = n * (4 * 4 + 3 * 4 + 2)  # sumsq read g; adamw read p,g,m,v write p,m,v,bf16
        print(json.dumps({"probe": "sumsq+adamw 111.8M params", "ms": ms, "alg_gbs": nbytes / ms / 1e6}))


if __name__ == "__main__":
    main()
