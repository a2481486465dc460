"""Benchmark: ChessDecoder training step (pass-1 causal + pass-2 prefix
forward, backward, clip + AdamW) in bf16 on B200, train tokens/s.

Workload: the ~114M-parameter default pretraining model (E=1024, 16 heads, 12
layers, d_ff=1536, S=256), per-GPU batch 64 sequences of seeded synthetic
random-playout games (8-120 plies, truncated), AdamW lr 3e-4 / wd 0.1, clip 10.
With --gpus N (torchrun, one rank per GPU) each rank has its own game stream
and the gradients are averaged with bucketed NCCL all-reduces overlapped with
the backward (weak scaling: per-GPU batch fixed).

  value : tokens/s over all ranks, batch already in HBM, device time (CUDA
          events around K steps, max over ranks)
  e2e   : the same step through the public training loop (TrainStep.run /
          DataParallelStep.run: batch i+1 prepared and enqueued while step i
          runs) from pinned host batches, host index preparation +
          host-to-device copies + every step's loss read-back inside the
          timed region
  --impl reference : the reference step on the host CPU (fp32 oracle port of
          chessdecoder/train/train.py:157-253; the reference's own model
          needs torchtune and python-chess, whose import errors the line
          reports), bounded sample per step.
  gpu_eager_reference : the same step restated in PyTorch eager on this GPU
          under autocast (fp16 as shipped, and bf16) -- the eager bar.
  --probe gemm|attn|adamw|tokenize|decode : kernel micro-benchmarks at the
          step's shapes (the commands behind the ncu summaries in profiles/).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train tokens/s"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=None, help="per-GPU sequences (default 64; 128 with --fp8)")
    ap.add_argument("--fp8", action="store_true",
                    help="fp8 variant: backbone linears on e4m3 / e5m2 GEMMs with delayed scaling (per-GPU batch 128)")
    ap.add_argument("--moe", action="store_true",
                    help="MoE variant: 8 experts, top-2, capacity 1.25, thinking-variation rows, S=4096, "
                         "per-GPU batch 16")
    ap.add_argument("--finetune", action="store_true",
                    help="finetune step (chessdecoder/finetune/train.py): thinking head + 5-term loss on "
                         "thinking-variation rows, S=4096, per-GPU batch 4")
    ap.add_argument("--grpo", action="store_true",
                    help="GRPO policy-gradient step (chessdecoder/rl): prefix pass, thinking / final move heads, "
                         "clipped ratio + KL loss, S=4096, mini-batch 4")
    ap.add_argument("--decode", action="store_true",
                    help="KV-cache inference (chessdecoder/cpp/decoder BatchedBackbone): causal prefill of --seq "
                         "tokens (default 512) for --batch sequences (default 64), then timed incremental steps")
    ap.add_argument("--seq", type=int, default=None,
                    help="sequence length (default 256; 4096 with --moe / --finetune / --grpo; 512 prefill with "
                         "--decode)")
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--pool", type=int, default=4, help="distinct synthetic batches per rank")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--detail", action="store_true", help="add a per-shape GEMM breakdown to the JSON line")
    ap.add_argument("--no-eager-baseline", action="store_true",
                    help="skip the PyTorch-eager GPU context line (the oracle step under autocast)")
    ap.add_argument("--probe", choices=["gemm", "attn", "adamw", "tokenize", "decode"], default=None,
                    help="kernel micro-benchmark instead of the step: one kernel family at the step's shapes")
    ap.add_argument("--kind", default="rope", choices=["rope", "swiglu", "resid", "resid2", "dswiglu", "dx", "dw"],
                    help="--probe gemm: which GEMM form")
    ap.add_argument("--nseq", type=int, default=128, help="--probe attn: sequences (half causal, half prefix)")
    ap.add_argument("--keys", type=int, default=542, help="--probe decode: cached keys per sequence")
    ap.add_argument("--new", type=int, default=1, help="--probe decode: new tokens per sequence")
    ap.add_argument("--iters", type=int, default=10, help="--probe: timed launches")
    return ap.parse_args()


def step_flops(cfg, db_list, S):
    """Algorithmic FLOPs of one step (6 * MACs-per-token * tokens for every
    linear that the loss needs, + attention over the allowed (q,k) pairs of both
    passes), averaged over the batch pool.  MoE: each token's MLP counts twice
    (top-2 experts, no credit for dropped choices' padding) plus the router."""
    import numpy as np
    E, F, L = cfg.embed_dim, cfg.ff, cfg.num_layers
    mlp = 3 * E * F * (2 if cfg.moe_experts else 1) + E * cfg.moe_experts
    p_bb = L * (4 * E * E + mlp)
    out = []
    for b in db_list:
        B = b["input_ids"].shape[0]
        T = B * S
        bid = b["block_id"].numpy()
        pairs = B * S * (S + 1) // 2  # causal pass
        for r in range(B):
            ids = bid[r]
            # causal pairs + the extra (future, same-block) pairs of each block
            _, counts = np.unique(ids, return_counts=True)
            pairs += S * (S + 1) // 2 + int((counts * (counts - 1) // 2).sum())
        nm = int(b["move_mask"].sum())
        nt = int(b["thinking_move_mask"].sum()) if "thinking_move_mask" in b else 0  # thinking head + WL rows
        nd = int(b["wl_positions"].sum())
        pv = E * cfg.value_hidden_size + cfg.value_hidden_size * cfg.n_buckets
        f = (6 * T * (2 * p_bb + 41 * E) + 6 * (nm + nt) * (1924 * E + pv) + 6 * nd * pv
             + 3 * 4 * E * L * pairs)
        out.append(f)
    return sum(out) / len(out)


class ClockSampler:
    """nvidia-smi samples (every 200 ms) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    """(sustained bf16 TFLOP/s, burst bf16 TFLOP/s, "measured" | "fallback",
    median SM MHz of the sustained measurement)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        clk = (d.get("clocks_under_load") or {}).get("sm_mhz_median")
        return d.get("bf16_tflops_sustained", 1392.1), d.get("bf16_tflops", 1648.1), "measured", clk
    return 1400.0, 1590.0, "fallback", 1300.0


def cpu_baseline(batch, cfg_kw, steps, threads=None):
    """The oracle (fp32 port of the reference step) on the host CPU, bounded sample."""
    from oracle.model import OracleChessDecoder
    from oracle.step import train_step
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = OracleChessDecoder(1968, **cfg_kw)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
    sample = {k: v[:4] for k, v in batch.items()}
    train_step(model, opt, sample)  # warm-up
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        train_step(model, opt, sample)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    ntok = sample["input_ids"].numel()
    return {"value": ntok / t, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"one full fp32 step (both passes, backward, clip, AdamW) on 4 of the batch's sequences "
                      f"x S={sample['input_ids'].shape[1]}, median of {steps} after 1 warm-up",
            "step_s": t, "reference_imports": reference_import_status()}


def eager_gpu_baseline(pool, dev, layers, seq, steps=5, warmup=2):
    """Context line: the reference step restated in PyTorch eager (the
    oracle's torchtune-free modules, cuBLAS GEMMs and SDPA) on this GPU at the
    same batch, under autocast as chessdecoder/train/train.py:167-253 runs it
    (fp16 with GradScaler, as shipped; and bf16), clip 10, torch AdamW.
    CUDA-event time per step, batches already on the device."""
    from oracle.model import OracleChessDecoder
    from oracle.step import step_losses
    out = {}
    B = pool[0]["input_ids"].shape[0]
    batches = [{k: v.to(dev) for k, v in b.items()} for b in pool]
    for name, dt in (("fp16_autocast", torch.float16), ("bf16_autocast", torch.bfloat16)):
        torch.manual_seed(0)
        model = OracleChessDecoder(1968, embed_dim=1024, num_heads=16, num_layers=layers, max_seq_len=seq,
                                   d_ff=1536).to(dev)
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
        scaler = torch.amp.GradScaler("cuda", enabled=dt == torch.float16)

        def one(b):
            opt.zero_grad(set_to_none=True)
            with torch.autocast(device_type="cuda", dtype=dt):
                total = step_losses(model, b)["total"]
            scaler.scale(total).backward()
            scaler.unscale_(opt)
            torch.nn.utils.clip_grad_norm_(model.parameters(), 10.0)
            scaler.step(opt)
            scaler.update()
        for i in range(warmup):
            one(batches[i % len(batches)])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            one(batches[i % len(batches)])
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        out[name] = {"value": B * seq / (ms / 1000.0), "unit": UNIT, "ms_per_step": ms}
        del model, opt
        torch.cuda.empty_cache()
    out["what"] = ("oracle restatement of the reference step in PyTorch eager (cuBLAS + SDPA) on this GPU, "
                   f"same batch ({B} x {seq}), {steps} steps after {warmup}")
    return out


def reference_import_status():
    """Whether the reference's own model can run here: chessdecoder/models/model.py
    imports torchtune (0.6.1) and the data path python-chess (1.11.2)."""
    import importlib
    status = {}
    for m in ("torchtune", "chess"):
        try:
            importlib.import_module(m)
            status[m] = "ok"
        except Exception as e:  # noqa: BLE001 - the message is the report
            status[m] = f"{type(e).__name__}: {e}"
    return status


def run_reference(args, rank, world):
    """--impl reference: the reference step on the host CPU (oracle port), rank 0 only."""
    if rank != 0:
        return
    from chessdecoder_b200 import data
    cfg_kw = dict(embed_dim=1024, num_heads=16, num_layers=args.layers, max_seq_len=args.seq, d_ff=1536)
    batch = data.synthetic_batches(1, 4, args.seq, seed=0)[0]
    from oracle.model import OracleChessDecoder
    from oracle.step import train_step
    # the reference's ChessDecoder needs torchtune and python-chess; when they
    # do not import, the timed step is the oracle port, and the import errors
    # are reported in the line
    imports = reference_import_status()
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = OracleChessDecoder(1968, **cfg_kw)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.1)
    for _ in range(args.warmup):
        train_step(model, opt, batch)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        train_step(model, opt, batch)
    dt = (time.perf_counter() - t0) / args.steps
    ntok = batch["input_ids"].numel()
    v = ntok / dt
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1000, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "ChessDecoder pretraining step, default model (E=1024, 16 heads, 12 layers, "
                                   f"d_ff=1536), S={args.seq}, bounded CPU sample of 4 sequences per step",
                       "global_batch": 4, "seq_len": args.seq, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": "4 sequences per step (fp32 oracle port of train.py:157-253)",
                             "reference_imports": imports},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_grpo(args, rank, world):
    """GRPO step (prefix pass, move-action log-probs, clipped-ratio + KL loss,
    backward, clip, AdamW) on synthetic thinking rows with rollout / reference
    log-probs perturbed around the current policy; one rank, device time."""
    from chessdecoder_b200 import data, kernels as K
    from chessdecoder_b200.engine import ModelConfig
    from chessdecoder_b200.rl import GRPOStep, prepare_rl_batch
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = ModelConfig(num_layers=args.layers, max_seq_len=args.seq, finetune=True)
    step = GRPOStep(cfg, device=dev)
    rbs = []
    for b in data.finetune_batches(args.pool, args.batch, args.seq, seed=1234, rank=rank):
        rb = {"input_ids": b["input_ids"], "block_id": b["block_id"], "wl_positions": b["wl_positions"],
              "d_positions": b["d_positions"], "wl_values": b["wl_targets"], "d_values": b["d_targets"],
              "thinking_move_mask": b["thinking_move_mask"], "final_move_mask": b["move_mask"],
              "move_token_ids": b["move_target_ids"].clamp_min(0)}
        lp, _ = step.log_probs(prepare_rl_batch(rb, dev))
        g = torch.Generator(device="cpu").manual_seed(len(rbs))
        old = lp.cpu() + torch.randn(lp.shape, generator=g) * 0.1
        adv = torch.randn(args.batch, generator=g)
        rbs.append(prepare_rl_batch(rb, dev, old, lp.cpu(), adv))
    for i in range(args.warmup):
        step.forward_backward(rbs[i % len(rbs)])
        step.optimizer_step()
    torch.cuda.synchronize()
    K.LAUNCHES[0] = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        loss, _ = step.forward_backward(rbs[i % len(rbs)])
        step.optimizer_step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    tokens = args.batch * args.seq
    print(json.dumps({"metric": METRIC, "value": tokens / (ms / 1000.0), "unit": UNIT, "n_gpus": 1,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                      "data": "synthetic thinking-variation rows; rollout log-probs = current + N(0, 0.1)",
                      "config": {"workload": "ChessDecoder GRPO step (prefix pass, thinking / final move log-probs, "
                                             "clipped ratio + KL loss, bwd, clip, AdamW), default model E=1024 H=16 "
                                             "L=%d d_ff=1536" % args.layers,
                                 "global_batch": args.batch, "seq_len": args.seq, "parallelism": "dp1"},
                      "gpu_launches": K.LAUNCHES[0] // args.steps, "loss": float(loss)}))


def run_decode(args, rank, world):
    """KV-cache inference: one step = one new token for every sequence of the
    batch through the 12 layers (causal_incremental, replayed from a CUDA
    graph).  Device time over the timed steps; e2e adds, per step, the copy of
    the step's token ids from pinned host memory and the read-back of the final
    hidden states.  Replicas only: each rank decodes its own batch."""
    import numpy as np
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.decode import BatchedBackbone
    from chessdecoder_b200.engine import ModelConfig
    dev = torch.device("cuda", torch.cuda.current_device())
    B, ctx = args.batch, args.seq
    n_new = args.warmup + 2 * args.steps + 2
    max_len = ctx + n_new
    cfg = ModelConfig(num_layers=args.layers, max_seq_len=max(256, max_len))
    bb = BatchedBackbone(cfg, batch_size=B, max_seq_len=max_len, device=dev)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (B, ctx), generator=g)
    bb.causal_forward(ids, torch.arange(ctx).repeat(B, 1), None, None, None, torch.full((B,), ctx))
    toks = torch.randint(0, cfg.vocab_size, (n_new, B, 1), generator=g)
    toks_dev = toks.to(dev)
    pos = (ctx + torch.arange(n_new)).view(n_new, 1, 1).expand(n_new, B, 1).contiguous()
    pos_dev = pos.to(dev)
    act = torch.ones(B, dtype=torch.bool, device=dev)
    k = 0
    for _ in range(args.warmup):
        bb.causal_incremental(toks_dev[k], pos_dev[k], None, None, act)
        k += 1
    torch.cuda.synchronize()
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    K.LAUNCHES[0] = 0
    len0 = bb.causal_len
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        bb.causal_incremental(toks_dev[k], pos_dev[k], None, None, act)
        k += 1
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    launches = K.LAUNCHES[0] // args.steps
    # e2e: token ids from pinned host memory in, final hidden states out, every step
    ids_h = toks.pin_memory()
    pos_h = pos.pin_memory()
    out_h = torch.empty(B, cfg.embed_dim, pin_memory=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        h = bb.causal_incremental(ids_h[k], pos_h[k], None, None, act)
        out_h.copy_(h[:, 0], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        k += 1
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / args.steps
    clk = clocks.stop()
    # the dominant kernel alone: decode attention over one layer's cache at the final length
    q = torch.randn(B, cfg.embed_dim, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    c = bb.causal
    for _ in range(3):
        K.decode_attn(q, c.k[0], c.v[0], c.len_dev, 1, B, cfg.num_heads, c.valid, out, block_mode=K.BLOCK_VALID)
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    n_a = 50
    for _ in range(n_a):
        K.decode_attn(q, c.k[0], c.v[0], c.len_dev, 1, B, cfg.num_heads, c.valid, out, block_mode=K.BLOCK_VALID)
    a1.record()
    torch.cuda.synchronize()
    attn_us = a0.elapsed_time(a1) * 1000.0 / n_a
    # greedy board generation of one sequence (the single-sequence engine's
    # causalBoardStep loop): 80-token prefill, then 68 board tokens through the
    # board head, each fed back on the device
    from chessdecoder_b200 import vocab as V
    gb = BatchedBackbone(cfg, batch_size=1, max_seq_len=80 + 68, device=dev, store=bb.store)
    first = torch.full((1, 1), V.token_to_idx["start_pos"], dtype=torch.int64, device=dev)
    gids = torch.randint(0, cfg.vocab_size, (1, 80), generator=g).to(dev)
    gpos = torch.arange(80, device=dev).view(1, 80)
    n80 = torch.full((1,), 80, device=dev)
    gen_ms = []
    for rep in range(4):
        gb.reset_causal()
        gb.causal_forward(gids, gpos, None, None, None, n80)
        torch.cuda.synchronize()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        gb.generate(first, torch.full((1, 1), 80, device=dev), 68, head="board_head", lut=V.board_idx_to_full_idx)
        g1.record()
        torch.cuda.synchronize()
        if rep > 0:
            gen_ms.append(g0.elapsed_time(g1))
    gen_t = statistics.median(gen_ms)
    err = K.get_error()
    if err:
        raise SystemExit(f"device error flag {err} after the decode run")
    keys = c.len + 1
    attn_bytes = B * cfg.num_heads * keys * 64 * 2 * 2
    hbm = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("hbm_gbs") if (
        ROOT / "MEASURED_PEAKS.json").exists() else None
    peak = hbm or 6650.0
    mid = len0 + args.steps / 2.0
    E, F, L = cfg.embed_dim, cfg.ff, cfg.num_layers
    step_bytes = L * (4 * E * E + 3 * E * F) * 2 + L * B * cfg.num_heads * (mid + 1) * 64 * 2 * 2
    line = {"metric": "decode tokens/s", "value": B / (ms / 1000.0), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic token ids; random-init weights",
            "config": {"workload": "ChessDecoder KV-cache incremental decode (causal cache, one token per sequence "
                                   "per step, CUDA-graph replay), E=1024 H=16 L=%d d_ff=1536" % L,
                       "batch": B, "prefill": ctx, "cache_keys_mid": mid, "parallelism": "replicas",
                       "l2": "KV cache (%.2f GB) and weights larger than L2" % (L * B * cfg.num_heads * mid * 256
                                                                             / 1e9)},
            "e2e": {"value": B / (e2e_ms / 1000.0), "unit": "tokens/s", "h2d_bytes_per_step": B * 8 * 2,
                    "d2h_bytes_per_step": B * E * 4},
            "roofline": {"bound": "hbm", "kernel": "decode_attn_1q", "achieved": attn_bytes / attn_us / 1e3,
                         "peak": peak, "unit": "GB/s", "frac": attn_bytes / attn_us / 1e3 / peak,
                         "launch_us": attn_us, "bytes_per_launch": attn_bytes,
                         # DRAM bytes per launch: an ncu capture of the same kernel at 64 sequences x 1001
                         # keys read 263.0 MB (+ 4.6 MB written) for 262.4 MB of K / V rows; traffic grows with
                         # the rows read, so it is scaled by this launch's bytes
                         "traffic": attn_bytes * (263.0 + 4.6) / 262.4,
                         "traffic_source": "ncu capture at B=64, 1001 keys, scaled by K/V bytes",
                         "peak_kind": "measured" if hbm else "fallback",
                         "step_hbm_gbs": step_bytes / (ms / 1000.0) / 1e9},
            "gpu_launches": launches,
            "generate": {"batch": 1, "prefill": 80, "tokens": 68, "head": "board_head", "ms": gen_t,
                         "tokens_per_s": 68 / (gen_t / 1000.0), "ms_per_token": gen_t / 68}}
    if clk:
        line["clocks"] = clk
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = decode_cpu_baseline(cfg, ctx)
    print(json.dumps(line))


def decode_cpu_baseline(cfg, ctx, reps=5):
    """The oracle (numpy fp32 restatement of the exported KV-cache module) on
    the host: one incremental token of one sequence over a ctx-key cache."""
    import numpy as np
    from chessdecoder_b200.engine import init_reference_weights
    from oracle import decode as OD
    sd = init_reference_weights(cfg, 0)
    w = {k: v.float().numpy() for k, v in sd.items()}
    c = dict(num_layers=cfg.num_layers, num_heads=cfg.num_heads, embed_dim=cfg.embed_dim)
    rng = np.random.default_rng(0)
    pk = rng.standard_normal((cfg.num_layers, 1, cfg.num_heads, ctx, 64)).astype(np.float32)
    pv = rng.standard_normal(pk.shape).astype(np.float32)
    rope = OD.rope_table(ctx + 1, 64)
    args = (np.array([[5]]), np.array([[ctx]]), np.zeros((1, 1, 1, ctx + 1), np.float32), pk, pv,
            np.zeros((1, 1), np.float32), np.zeros((1, 1), bool), rope)
    OD.forward(w, c, *args)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        OD.forward(w, c, *args)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": 1.0 / t, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"one incremental token of one sequence over a {ctx}-key cache (numpy fp32 oracle of "
                      f"the exported module), median of {reps}"}


# ---------------------------------------------------------------------------
# --probe: kernel micro-benchmarks
# ---------------------------------------------------------------------------
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
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.engine import rope_table
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
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.engine import rope_table
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


def run_probe(a):
    """--probe: one kernel family at the training step's shapes, CUDA-event
    time per launch and achieved FLOP/s or bytes/s (the commands behind the
    ncu summaries in profiles/)."""
    from chessdecoder_b200 import kernels as K
    from chessdecoder_b200.engine import rope_table
    a.seq = a.seq or 256
    a.batch = a.batch or 64
    K.lib()
    if a.probe == "gemm":
        fn, flops, nbytes, name = (gemm_case_fp8 if a.fp8 else gemm_case)(a.kind)
        ms = _time(fn, a.warmup, a.iters)
        print(json.dumps({"probe": name, "ms": ms, "tflops": flops / ms / 1e9, "alg_bytes": nbytes,
                          "alg_gbs": nbytes / ms / 1e6}))
    elif a.probe == "decode":
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
    elif a.probe == "attn":
        S, H = a.seq, 16
        E = H * 64
        nseq, ncaus = a.nseq, a.nseq // 2
        g = torch.Generator().manual_seed(0)
        qkv = (torch.randn(nseq * S, 3 * E, generator=g) * 0.8).to("cuda").to(torch.bfloat16)
        if S > 256:  # thinking-variation rows: a board block every 71 tokens
            from chessdecoder_b200.data import thinking_batches
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
    elif a.probe == "tokenize":
        # host batch producer: 256 random games (8-120 plies) -> [256, S] rows, skip_board_prob 0.2
        import random
        import time
        import numpy as np
        from chessdecoder_b200.chessgen import random_game_rows
        from chessdecoder_b200.loader import GameTokenizer
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




def main():
    args = parse()
    if args.probe:
        run_probe(args)
        return
    if args.batch is None:
        args.batch = 128 if args.fp8 else 16 if args.moe else 4 if (args.finetune or args.grpo) else 64
    if args.seq is None:
        args.seq = 4096 if (args.moe or args.finetune or args.grpo) else 512 if args.decode else 256
    if args.moe + args.fp8 + args.finetune + args.grpo + args.decode > 1:
        raise SystemExit("--moe, --fp8, --finetune, --grpo and --decode are separate variants")
    from chessdecoder_b200.distributed import setup_distributed, cleanup_distributed
    rank, local_rank, world = setup_distributed() if args.gpus > 1 or "RANK" in os.environ else (0, 0, 1)
    if args.impl == "reference":
        run_reference(args, rank, world)
        cleanup_distributed()
        return
    if args.grpo or args.decode:
        # one-GPU variants: under torchrun rank 0 measures on its own GPU, the
        # other ranks exit without work
        if rank == 0:
            torch.cuda.set_device(local_rank)
            (run_grpo if args.grpo else run_decode)(args, rank, world)
        cleanup_distributed()
        return
    import torch.distributed as dist
    from chessdecoder_b200 import data, kernels as K
    from chessdecoder_b200.engine import FINETUNE_LOSS_WEIGHTS, ModelConfig, TrainStep, prepare_batch
    from chessdecoder_b200.distributed import DataParallelStep

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = ModelConfig(num_layers=args.layers, max_seq_len=args.seq, moe_experts=8 if args.moe else 0,
                      finetune=args.finetune)
    if args.finetune:  # chessdecoder/finetune/config.yaml: lr 3e-5, loss weights 3/1/3/3/3
        step = TrainStep(cfg, device=dev, seed=0, lr=3e-5, loss_weights=FINETUNE_LOSS_WEIGHTS)
    else:
        step = TrainStep(cfg, device=dev, seed=0, fp8=args.fp8)
    dp = DataParallelStep(step)
    if args.moe:
        pool = data.thinking_batches(args.pool, args.batch, args.seq, seed=1234, rank=rank)
    elif args.finetune:
        pool = data.finetune_batches(args.pool, args.batch, args.seq, seed=1234, rank=rank)
    else:
        pool = data.synthetic_batches(args.pool, args.batch, args.seq, seed=1234, rank=rank)
    dbs = [prepare_batch(b, dev) for b in pool]
    torch.cuda.synchronize()

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- value: device-resident batches ---------------------------------------
    for i in range(args.warmup):
        dp.forward_backward(dbs[i % len(dbs)])
        dp.optimizer_step()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    phys = torch.cuda.current_device()
    if visible:
        ids = [x.strip() for x in visible.split(",") if x.strip()]
        phys = int(ids[phys]) if phys < len(ids) and ids[phys].isdigit() else phys
    sampler = ClockSampler(phys)
    K.LAUNCHES[0] = 0
    sync_all()
    sampler.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        dp.forward_backward(dbs[i % len(dbs)])
        dp.optimizer_step()
    ev1.record()
    sync_all()
    clocks = sampler.stop()
    launches = K.LAUNCHES[0] // args.steps
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    # a bounded device wait that gave up (or an out-of-range index) invalidates the run
    device_error = int(max_over_ranks(float(K.get_error())))
    tokens_step = args.batch * args.seq * world
    value = tokens_step / (dev_ms / 1000.0)
    # per-launch GEMM timing (CUDA events around every GEMM launch) in a
    # separate pass after the timed region, so that `value` is not perturbed
    gemm_steps = min(args.steps, 5)
    if args.detail:
        K.OP_TIMER = {}
    gemm_timer = K.GemmTimer()
    K.GEMM_TIMER = gemm_timer
    sync_all()
    g0 = torch.cuda.Event(enable_timing=True)
    g1 = torch.cuda.Event(enable_timing=True)
    g0.record()
    for i in range(gemm_steps):
        dp.forward_backward(dbs[i % len(dbs)])
        dp.optimizer_step()
    g1.record()
    sync_all()
    K.GEMM_TIMER = None
    op_stats = K.op_timer_summary(K.OP_TIMER) if K.OP_TIMER is not None else None
    K.OP_TIMER = None
    gemm_pass_ms = g0.elapsed_time(g1) / gemm_steps
    gemm_stats = gemm_timer.summary(detail=args.detail)
    # host cost of enqueueing one step with the GPU idle (inside the timed loop the
    # host waits on the full launch queue, so its wall time there is the GPU's)
    sync_all()
    host_t0 = time.perf_counter()
    dp.forward_backward(dbs[0])
    dp.optimizer_step()
    host_enqueue_ms = (time.perf_counter() - host_t0) * 1000
    sync_all()

    # ---- e2e: public API from host batches -------------------------------------
    host_pool = []
    for b in pool:
        host_pool.append({k: (v.pin_memory() if torch.cuda.is_available() else v) for k, v in b.items()})
    for i in range(2):
        dp.step(host_pool[i % len(host_pool)])
    sync_all()
    h2d = 0
    d2h = 0
    t0 = time.perf_counter()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    # the public training loop: batch i+1 prepared and enqueued while step i
    # runs; every step's losses are read back to the host (one step behind)
    for i, lv in dp.run(host_pool[i % len(host_pool)] for i in range(args.steps)):
        d2h += lv.numel() * lv.element_size()
    e1.record()
    sync_all()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    db_tmp = prepare_batch(host_pool[0], dev)
    h2d = db_tmp.h2d_bytes
    e2e_value = tokens_step / (e2e_ms / 1000.0)

    # ---- communication timeline (N > 1), outside the timed regions -------------
    comm = None
    if world > 1 and dp.reducer is not None:
        red = dp.reducer
        red.timing = True
        recs = []
        for i in range(3):
            dp.forward_backward(dbs[i % len(dbs)])
            recs.append(red.stats())
            dp.optimizer_step()
        red.timing = False
        # the same steps with the all-reduce hooks detached: what the step costs
        # on N GPUs without communication (gradients stay per-rank here)
        hook = step.grad_hook
        step.grad_hook = None
        sync_all()
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record()
        for i in range(3):
            dp.forward_backward(dbs[i % len(dbs)])
            dp.optimizer_step()
        c1.record()
        sync_all()
        step.grad_hook = hook
        tails = sorted(r["exposed_tail_ms"] for r in recs)
        comm = {"buckets": recs[-1]["buckets"], "bytes_per_step": recs[-1]["bytes"],
                "exposed_tail_ms": max_over_ranks(tails[1]),
                "first_ready_to_last_done_ms": max_over_ranks(sorted(r["span_ms"] for r in recs)[1]),
                "ready_to_done_ms_rank0": recs[-1]["ready_to_done_ms"],
                "step_ms_without_allreduce": max_over_ranks(c0.elapsed_time(c1) / 3),
                "timing": "CUDA events: bucket ready on the compute stream, all-reduce done on the comm stream, "
                          "3 steps after the timed regions, median, max over ranks"}

    # ---- roofline of the dominant kernel (the tcgen05 GEMM) ---------------------
    peak_sust, peak_burst, peak_kind, peak_clk = measured_peaks()
    achieved = gemm_stats["tflops"]
    # The step is ~30 ms, not the seconds-long loop the sustained peak was
    # measured over (at a lower, power-capped clock), so the burst peak is the
    # denominator; the sustained peak scaled by the SM clock sampled here is
    # given beside it.
    sm_mhz = (clocks or {}).get("sm_mhz")
    sust_scaled = peak_sust * sm_mhz / peak_clk if (sm_mhz and peak_clk) else None
    roofline = {"bound": "tensor", "kernel": "gemm_bf16_kernel (tcgen05)", "achieved": achieved,
                "peak": peak_burst, "unit": "TFLOP/s", "frac": achieved / peak_burst,
                "peak_source": f"{peak_kind} bf16_tflops (burst)",
                "frac_vs_sustained_at_this_clock": (achieved / sust_scaled) if sust_scaled else None,
                "launches_per_step": gemm_stats["launches"] // max(gemm_steps, 1),
                "share_of_step": gemm_stats["ms"] / gemm_steps / gemm_pass_ms,
                "timing": f"CUDA events around each GEMM launch, {gemm_steps} steps after the timed region"}
    # DRAM bytes (read + write) of one launch of the largest GEMM shape, QKV + RoPE
    # (M=32768, N=3072, K=1024), from one `ncu --set full --clock-control none`
    # capture of `python bench.py --probe gemm --kind rope` (CTA-pair form,
    # TMA-stored epilogue): 73.5 MB read (the algorithmic A + W bytes, no
    # re-reads) + 147.6 MB written inside the launch; the launch's algorithmic
    # bytes are 275 MB.
    roofline["traffic"] = 221.1e6
    roofline["traffic_launch"] = {"shape": "M32768 N3072 K1024 (QKV + RoPE epilogue, CTA pair)",
                                  "dram_read": 73.5e6, "dram_write": 147.6e6, "algorithmic_bytes": 275.0e6}

    flops = step_flops(cfg, pool, args.seq)
    mfu_spec = flops / (dev_ms / 1000.0) / 2.25e15
    mfu_meas = flops / (dev_ms / 1000.0) / (peak_burst * 1e12)
    if args.fp8:
        roofline["kernel"] = "gemm_bf16_kernel<..., F8> (tcgen05 kind::f8f6f4)"
        roofline["note"] = ("fp8 GEMMs measured against the bf16 sustained peak (no fp8 peak is measured on this "
                            "pool; the dense fp8 spec is 4.5 PFLOP/s)")

    eager = None
    if rank == 0 and world == 1 and not args.no_eager_baseline and not (args.moe or args.finetune or args.fp8):
        eager = eager_gpu_baseline(pool, dev, args.layers, args.seq)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.moe and not args.finetune:
        cpu = cpu_baseline(pool[0], dict(embed_dim=1024, num_heads=16, num_layers=args.layers,
                                         max_seq_len=args.seq, d_ff=1536), args.cpu_steps)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None,
                "dtype": "fp8 (e4m3 activations/weights, e5m2 grads) backbone and head linears; bf16 attention"
                if args.fp8 else "bf16", "data": "synthetic thinking-variation rows" if (args.moe or args.finetune)
                else "synthetic",
                "config": {"workload": ("ChessDecoder %s step (pass-1 causal + pass-2 prefix fwd, bwd, "
                                        "clip, AdamW), default model E=1024 H=16 L=%d d_ff=1536"
                                        % ("finetune" if args.finetune else "pretraining", args.layers))
                           + (", fp8 variant (per-tensor delayed scaling, amax history 16)" if args.fp8 else "")
                           + (", MoE variant (8 experts, top-2, capacity 1.25)" if args.moe else "")
                           + (", finetune step (thinking head, 5-term loss)" if args.finetune else ""),
                           "global_batch": args.batch * world, "seq_len": args.seq,
                           "parallelism": f"dp{world}", "per_gpu_batch": args.batch,
                           "l2": "working set (activations ~11 GB) far larger than L2; no flush needed",
                           "params": int(step.store.numel)},
                "mfu": {"vs_spec_2250": mfu_spec, "vs_measured_burst": mfu_meas, "flops_per_step": flops,
                        **({"vs_fp8_spec_4500": flops / (dev_ms / 1000.0) / 4.5e15} if args.fp8 else {})},
                "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step":
                        d2h // args.steps, "ms_per_step": e2e_ms},
                "gpu_launches": launches,
                "device_error_flags": device_error,
                "host_enqueue_ms_per_step": host_enqueue_ms,
                "roofline": roofline,
                "clocks": clocks,
                "cpu_baseline": cpu}
        if eager is not None:
            line["gpu_eager_reference"] = eager
        if comm is not None:
            line["comm"] = comm
        if args.detail:
            line["gemm_by_shape"] = gemm_stats.get("by_shape")
            line["host_enqueue_ms_per_step"] = host_enqueue_ms
            # collected over the GEMM-timer pass (gemm_steps steps), as the GEMM breakdown
            line["ops_ms_per_step"] = {k: [n // gemm_steps, ms / gemm_steps] for k, (n, ms) in op_stats.items()}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
    cleanup_distributed()


if __name__ == "__main__":
    main()
