"""Data parallelism for the ChessDecoder step: the API of
chessdecoder/utils/distributed.py (setup_distributed, cleanup_distributed,
is_main_process, get_device, average_gradients, barrier, print_rank0) plus the
bucketed, backward-overlapped gradient all-reduce used by the fused step.

The reference averages gradients with one blocking ``all_reduce`` per
parameter after the backward (utils/distributed.py:55-67).  Here gradients
live in one flat buffer ordered by when the backward finishes them, so a
bucket is a contiguous slice: as soon as the backward reports a layer done,
its slice is all-reduced (SUM) on a dedicated communication stream while the
next layer is differentiated.  The 1/world_size mean is folded into the
optimizer kernel (``grad_scale``), so no division pass runs.
"""
from __future__ import annotations

import datetime
import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def setup_distributed(timeout_s: float = 120.0):
    """torchrun env -> (rank, local_rank, world_size); (0, 0, 1) without torchrun.

    Same contract as utils/distributed.py:18-34, with a finite process-group
    timeout so that a rank that dies ends its peers' collectives with an error.
    """
    if "RANK" not in os.environ:
        return 0, 0, 1
    rank = int(os.environ["RANK"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    world = int(os.environ["WORLD_SIZE"])
    if not dist.is_initialized():
        if torch.cuda.is_available():
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                    device_id=torch.device(f"cuda:{local_rank}"))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
    return rank, local_rank, world


def cleanup_distributed():
    if dist.is_initialized():
        dist.destroy_process_group()


def is_main_process():
    return not dist.is_initialized() or dist.get_rank() == 0


def get_device(local_rank):
    return torch.device(f"cuda:{local_rank}")


def barrier():
    if dist.is_initialized():
        dist.barrier()


def print_rank0(*args, **kwargs):
    if is_main_process():
        print(*args, **kwargs)


def average_gradients(model, bucket_bytes: int = 25 * 1024 * 1024):
    """After return every ``p.grad`` holds the mean over ranks (utils/distributed.py:55-67).

    Gradients are reduced in ~25 MB buckets instead of one collective per
    parameter: the backbone gradients of a chessdecoder_b200 ``ChessDecoder``
    are views of one flat buffer, reduced in place slice by slice; all other
    gradients are coalesced per bucket.  No-op when not distributed.
    """
    if not dist.is_initialized():
        return
    world = dist.get_world_size()
    done = set()
    core = getattr(model, "_core", None)
    if core is not None:
        flat = core.flat_grad_of(model)
        if flat is not None:
            n = bucket_bytes // flat.element_size()
            for s in range(0, flat.numel(), n):
                _all_reduce_mean(flat[s:s + n], world)
            done = {id(core.params[i]) for i in core.backbone_idx}
    grads = [p.grad for p in model.parameters() if p.grad is not None and id(p) not in done]
    bucket, size = [], 0
    for g in grads:
        bucket.append(g)
        size += g.numel() * g.element_size()
        if size >= bucket_bytes:
            _reduce_coalesced(bucket, world)
            bucket, size = [], 0
    if bucket:
        _reduce_coalesced(bucket, world)


def _all_reduce_mean(t: torch.Tensor, world: int):
    if t.is_cuda:
        dist.all_reduce(t, op=dist.ReduceOp.AVG)
    else:  # gloo has no AVG
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        t.div_(world)


def _reduce_coalesced(grads: List[torch.Tensor], world: int):
    flat = torch.cat([g.reshape(-1) for g in grads])
    _all_reduce_mean(flat, world)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


class BucketedAllReduce:
    """Overlapped SUM all-reduce of a flat gradient buffer.

    ``spans`` maps a backward milestone key to a [start, end) slice of
    ``flat``; ``ready(key)`` launches that slice's all-reduce on the comm
    stream after the work already queued on the compute stream.  Adjacent
    small slices are merged up to ``bucket_bytes``.  ``wait()`` makes the
    compute stream wait for every launched all-reduce.  Every rank must call
    ``ready`` with the same keys in the same order (the backward is identical
    on all ranks), so the collectives match up.
    """

    def __init__(self, flat: torch.Tensor, spans: List[Tuple[object, int, int]], group=None,
                 bucket_bytes: int = 25 * 1024 * 1024):
        self.flat = flat
        self.group = group
        self.span_of = {k: (s, e) for k, s, e in spans}
        self.order = [k for k, _, _ in spans]
        self.bucket_elems = bucket_bytes // flat.element_size()
        self.pending_start: Optional[int] = None
        self.pending_end = 0
        self.cuda = flat.is_cuda
        self.stream = torch.cuda.Stream(device=flat.device) if self.cuda else None
        self.works = []
        self.launched = 0
        # timing=True: CUDA events per bucket (ready on the compute stream, done
        # on the comm stream) and at the end of the backward; read by stats()
        self.timing = False
        self._events = []
        self._bwd_end = None
        self._bytes = 0

    def ready(self, key):
        s, e = self.span_of[key]
        if self.pending_start is None:
            self.pending_start, self.pending_end = s, e
        else:
            if s != self.pending_end:
                self._flush()
                self.pending_start = s
            self.pending_end = e
        if self.pending_end - self.pending_start >= self.bucket_elems or key == self.order[-1]:
            self._flush()

    def _flush(self):
        if self.pending_start is None:
            return
        s, e = self.pending_start, self.pending_end
        self.pending_start = None
        view = self.flat[s:e]
        if self.cuda:
            ev = torch.cuda.current_stream(self.flat.device).record_event(
                torch.cuda.Event(enable_timing=self.timing))
            self.stream.wait_event(ev)
            with torch.cuda.stream(self.stream):
                w = dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
                if self.timing:  # the comm stream waits for this collective, then marks its end
                    w.wait()
                    done = torch.cuda.Event(enable_timing=True)
                    done.record(self.stream)
                    self._events.append((ev, done))
                    self._bytes += view.numel() * view.element_size()
        else:
            w = dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        self.works.append(w)
        self.launched += 1

    def wait(self):
        if self.timing and self.cuda:
            self._bwd_end = torch.cuda.current_stream(self.flat.device).record_event(
                torch.cuda.Event(enable_timing=True))
        self._flush()
        for w in self.works:
            w.wait()
        self.works = []
        if self.cuda:
            torch.cuda.current_stream(self.flat.device).wait_stream(self.stream)


    def stats(self):
        """Per-step communication timeline of the last step run with
        ``timing=True`` (synchronises): buckets, bytes, ``ready_to_done_ms`` per
        bucket, and ``exposed_tail_ms`` = end of the backward's last kernel ->
        end of the last all-reduce (the part of the communication that the
        backward does not hide).  Clears the recorded events."""
        if not self._events:
            return None
        self._events[-1][1].synchronize()
        if self._bwd_end is not None:
            self._bwd_end.synchronize()
        out = {"buckets": len(self._events), "bytes": self._bytes,
               "ready_to_done_ms": [round(a.elapsed_time(b), 4) for a, b in self._events]}
        first_ready = self._events[0][0]
        out["span_ms"] = first_ready.elapsed_time(self._events[-1][1])
        out["exposed_tail_ms"] = (self._bwd_end.elapsed_time(self._events[-1][1])
                                  if self._bwd_end is not None else None)
        self._events, self._bwd_end, self._bytes = [], None, 0
        return out


def step_spans(store) -> List[Tuple[object, int, int]]:
    """Backward milestones of the fused step and the flat slices they finish:
    key L (heads + final norm), then per layer L-1 .. 0 the key ("mlp", i)
    (the MLP block and its norm, final first) and the key i (the attention
    block and its norm), then -1 (Fourier + embedding).  Slices tile the whole
    flat buffer in this order."""
    L = store.cfg.num_layers
    spans = []
    first_layer_start = store.layer_grad_span(L - 1)[0]
    spans.append((L, 0, first_layer_start))
    prev_end = first_layer_start
    for i in reversed(range(L)):
        for key, part in ((("mlp", i), "mlp"), (i, "attn")):
            s, e = store.layer_grad_span(i, part)
            assert s == prev_end, "layer slices must be contiguous in backward order"
            spans.append((key, s, e))
            prev_end = e
    spans.append((-1, prev_end, store.numel))
    return spans


class DataParallelStep:
    """Wraps engine.TrainStep for N ranks: bucketed overlapped all-reduce during
    the backward, then clip + AdamW with the 1/world mean folded in.  Buckets
    of >= 16 MB: each layer's MLP slice (18.9 MB at the default model) goes out
    while that layer's attention block is differentiated, which shortens the
    reduction left after the backward's last kernel."""

    def __init__(self, step, group=None, bucket_bytes: int = 16 * 1024 * 1024):
        self.step_obj = step
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.reducer = None
        if self.world > 1:
            self.reducer = BucketedAllReduce(step.store.grad, step_spans(step.store), group, bucket_bytes)
            step.grad_hook = self.reducer.ready
            step.grad_scale = 1.0 / self.world

    def forward_backward(self, db, metrics=None, zero_grad=True, sync=True):
        """sync=False: a micro-batch before the last of an accumulation (no
        all-reduce; the last micro-batch's backward reduces the sum)."""
        losses = self.step_obj.forward_backward(db, metrics, zero_grad=zero_grad, sync=sync)
        if self.reducer is not None and sync:
            self.reducer.wait()
        return losses

    def optimizer_step(self, accum: int = 1):
        self.step_obj.optimizer_step(accum)

    def step_accumulated(self, batches, metrics=None):
        from .engine import prepare_batch
        out = []
        n = len(batches)
        for i, b in enumerate(batches):
            db = prepare_batch(b, self.step_obj.device)
            out.append(self.forward_backward(db, metrics, zero_grad=i == 0, sync=i == n - 1))
        self.optimizer_step(accum=n)
        return out

    def step(self, batch, metrics=None):
        from .engine import prepare_batch
        db = prepare_batch(batch, self.step_obj.device)
        losses = self.forward_backward(db, metrics)
        self.optimizer_step()
        return losses

    def run(self, batches, metrics=None):
        """Pipelined loop over host batches (engine.TrainStep.run): yields
        (i, host losses) for every batch, one step behind the device."""
        from .engine import pipelined_steps
        return pipelined_steps(self.step, batches, metrics)
