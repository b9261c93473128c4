"""Multi-process host logic of the sharded paths, on CPU with world size 2
over gloo: contiguous shards cover every unit exactly once, per-rank fp64
partials combined by one all-reduce equal the whole sum (the streaming pair's
exchange step), and a rank that fails before a collective is detected by the
other rank as an error within the process-group timeout instead of a hang."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, ROOT)
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        from bench import shard
        from oracle import oracle
        if mode == "sum":
            n = 3_000_017
            x = np.random.default_rng(11).random(n, dtype=np.float32)
            b0, b1 = shard(n, world, rank)
            part = torch.tensor([oracle.sum_f64(x[b0:b1])], dtype=torch.float64)
            dist.all_reduce(part)
            q.put((rank, "sum", float(part.item()), oracle.sum_f64(x), (b0, b1)))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("rank 1 fails before the collective")
            try:
                dist.all_reduce(torch.ones(1))
                q.put((rank, "no-error"))
            except Exception as e:  # the peer's exit surfaces as an error
                q.put((rank, "detected", type(e).__name__))
    except RuntimeError as e:
        q.put((rank, "raised", str(e)))
    finally:
        if mode != "fail" or rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(mode, world=2, timeout=90):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank process hung in mode {mode}")
    out = []
    while not q.empty():
        out.append(q.get())
    return out


def test_shard_ranges_cover_once():
    from bench import shard
    for total in (1, 7, 1024, 1 << 30, 1000003):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_sharded_sum_allreduce_world2():
    res = _run("sum")
    assert len(res) == 2
    for rank, kind, combined, full, _ in res:
        assert kind == "sum"
        assert combined == pytest.approx(full, rel=1e-12)


def test_rank_failure_detected_not_hung():
    res = _run("fail")
    by_rank = {r[0]: r[1:] for r in res}
    assert by_rank[1][0] == "raised"
    assert by_rank[0][0] == "detected"
