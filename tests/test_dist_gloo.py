"""Multi-process host logic of the sharded paths, on CPU with world size 2
over gloo: contiguous shards cover every unit exactly once, per-rank fp64
partials combined across ranks equal the whole sum, the mailbox exchange of
the in-kernel cross-GPU sum hands every rank all mailboxes in rank order
(vkcuda_b200.peer with fake device calls), and a rank that fails before a
collective is detected by the other rank as an error within the
process-group timeout instead of a hang."""
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
        elif mode == "mailboxes":
            # vkcuda_b200.peer's exchange with fake device calls: addresses
            # encode their owner, so the result shows who mapped what.
            from vkcuda_b200 import peer
            log = {"opened": [], "closed": [], "freed": []}
            own = 0x1000 + rank

            def alloc():
                return 0, own

            def get_handle(ptr):
                return 0, bytes([ptr & 0xff]) * 64

            def open_handle(h):
                log["opened"].append(h[0])
                return 0, 0x9000 + h[0]

            def close_handle(ptr):
                log["closed"].append(ptr)
                return 0

            def free(ptr):
                log["freed"].append(ptr)
                return 0

            boxes = peer.open_mailboxes(dist, rank, world, alloc, get_handle, open_handle)
            peer.close_mailboxes(dist, rank, boxes, close_handle, free)
            q.put((rank, "mailboxes", boxes, log))
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


def test_peer_mailbox_exchange_world2():
    """Host side of the in-kernel cross-GPU sum: every rank ends with all
    mailbox addresses in rank order (its own allocation at its rank, the
    others mapped from their handles), and unmaps exactly the others' and
    frees only its own."""
    res = _run("mailboxes")
    assert len(res) == 2
    for rank, kind, boxes, log in res:
        assert kind == "mailboxes"
        other = 1 - rank
        assert boxes[rank] == 0x1000 + rank
        assert boxes[other] == 0x9000 + other  # mapped from the other rank's handle
        assert log["opened"] == [other]
        assert log["closed"] == [boxes[other]]
        assert log["freed"] == [0x1000 + rank]
