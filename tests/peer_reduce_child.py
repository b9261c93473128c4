"""One rank of the two-GPU cross-GPU sum test (run by
test_gpu_peer_reduce.py as a child process; RANK, WORLD_SIZE, MASTER_ADDR,
MASTER_PORT in the environment). Mailbox handles travel over a gloo process
group; the sums themselves only through the kernel's peer stores."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from vkcuda_b200 import vc  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    torch.cuda.set_device(rank)
    assert vc.vcInit() == 0 and vc.vcSetDevice(rank) == 0
    from vkcuda_b200 import peer
    boxes = peer.open_mailboxes(dist, rank, world)
    n = (1 << 22) + 17 * rank + 3
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    a = torch.rand(n, device="cuda", generator=g)
    b = torch.rand(n, device="cuda", generator=g)
    c = torch.empty_like(a)
    out = torch.zeros(1, dtype=torch.float64, device="cuda")
    for epoch in range(1, 7):
        b.add_(1.0 / 64)  # a different sum every epoch
        assert vc.vadd_sum_f32_allreduce(a.data_ptr(), b.data_ptr(), c.data_ptr(), n,
                                         out.data_ptr(), boxes, rank, epoch) == 0
        torch.cuda.synchronize()
        got = out.item()
        local = torch.tensor([(a + b).double().sum().item()], dtype=torch.float64)
        locals_ = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(locals_, local)
        expect = sum(t.item() for t in locals_)
        assert abs(got - expect) <= 1e-6 * abs(expect), (epoch, got, expect)
        gots = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gots, torch.tensor([got], dtype=torch.float64))
        assert all(t.item() == got for t in gots), "ranks disagree"
    assert vc.kernel_error(True) == 0
    peer.close_mailboxes(dist, rank, boxes)
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
