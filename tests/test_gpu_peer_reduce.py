"""Cross-GPU sum inside the kernel (vc_vadd_sum_f32_allreduce) with two
ranks, one process per GPU, mailboxes shared through CUDA IPC: every epoch,
both ranks end with the same value, the sum of both ranks' fp64 sums within
1e-6. Needs two devices (skipped otherwise)."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_allreduce_through_mailboxes(gpu):
    err, count = gpu.vcGetDeviceCount()
    if count < 2:
        pytest.skip("needs two devices")
    port = _free_port()
    procs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "peer_reduce_child.py")],
                                      env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                      text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append(out)
    for rank, (p, out) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {rank}:\n{out[-3000:]}"
        assert f"rank {rank} ok" in out
