"""Data-parallel host logic on CPU with gloo, world size 2: the bucketed
overlapped all-reduce over a flat gradient buffer, the reference-API
average_gradients, and a rank that fails before a collective (its peer must
get an error within the process-group timeout, not hang)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout=30):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout))


def _bucket_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from chessdecoder_b200.distributed import BucketedAllReduce
        flat = torch.arange(1000, dtype=torch.float32) * (rank + 1)
        spans = [("heads", 0, 100), (2, 100, 400), (1, 400, 700), (0, 700, 900), (-1, 900, 1000)]
        r = BucketedAllReduce(flat, spans, bucket_bytes=250 * 4)
        for k, _, _ in spans:
            r.ready(k)
        r.wait()
        expect = torch.arange(1000, dtype=torch.float32) * sum(range(1, world + 1))
        q.put((rank, bool(torch.equal(flat, expect)), r.launched))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), -1))


def _avg_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from chessdecoder_b200.distributed import average_gradients
        torch.manual_seed(0)
        m = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.Linear(16, 4))
        for i, p in enumerate(m.parameters()):
            p.grad = torch.full_like(p, float(rank + i))
        average_gradients(m, bucket_bytes=64)
        ok = all(torch.allclose(p.grad, torch.full_like(p, (0 + 1) / 2 + i)) for i, p in enumerate(m.parameters()))
        q.put((rank, ok, 0))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e), -1))


def _fail_worker(rank, world, port, q):
    import time
    try:
        _init(rank, world, port, timeout=5)
        dist.barrier()
        if rank == 1:
            # this rank dies between steps: it never joins the next collective
            q.put((rank, "exited", 0))
            q.close()
            q.join_thread()
            os._exit(0)
        t0 = time.time()
        try:
            dist.all_reduce(torch.ones(4))
            q.put((rank, "no error", time.time() - t0))
        except Exception as e:
            q.put((rank, "error:" + type(e).__name__, time.time() - t0))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e), -1))


def _run(target, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


def test_bucketed_allreduce_gloo():
    res = _run(_bucket_worker)
    for rank, ok, launched in res:
        assert ok is True, res
        assert launched >= 2, res


def test_average_gradients_gloo():
    res = _run(_avg_worker)
    assert all(ok is True for _, ok, _ in res), res


def test_dead_rank_gives_error_not_hang():
    res = _run(_fail_worker)
    r0 = [r for r in res if r[0] == 0][0]
    assert r0[1].startswith("error:"), res
    assert r0[2] < 60, res
