"""Host side of the cross-GPU sum (vc_vadd_sum_f32_allreduce), one process
per GPU.

Each rank owns one mailbox in its device memory. `open_mailboxes` exports
this rank's mailbox as a CUDA IPC handle, gathers every rank's handle over a
torch.distributed process group (any backend: only bytes travel), and maps
the others into this process, returning the world's mailbox addresses in
rank order (this rank's own at `rank`), as the kernel takes them.
`close_mailboxes` undoes it after a barrier, so that no rank still stores
into a mailbox that is being unmapped or freed.

The device calls are parameters (defaults: the library's), so the exchange
logic runs unchanged under a CPU-only process group in the tests.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple


class PeerError(RuntimeError):
    pass


def _check(err, what: str) -> None:
    if int(err) != 0:
        raise PeerError(f"{what} failed with VCError {int(err)}")


def open_mailboxes(pg, rank: int, world: int,
                   alloc: Optional[Callable[[], Tuple[int, int]]] = None,
                   get_handle: Optional[Callable[[int], Tuple[int, bytes]]] = None,
                   open_handle: Optional[Callable[[bytes], Tuple[int, int]]] = None
                   ) -> List[int]:
    """Allocate this rank's mailbox, exchange handles over `pg` (the
    torch.distributed module or an equivalent with all_gather_object) and
    return all mailbox addresses in rank order."""
    if world < 1 or not 0 <= rank < world:
        raise PeerError(f"bad rank {rank} of {world}")
    if alloc is None or get_handle is None or open_handle is None:
        from vkcuda_b200 import vc
        alloc = alloc or vc.peer_mailbox_alloc
        get_handle = get_handle or vc.peer_ipc_get_handle
        open_handle = open_handle or vc.peer_ipc_open
    err, own = alloc()
    _check(err, "vc_peer_mailbox_alloc")
    err, handle = get_handle(own)
    _check(err, "vc_peer_ipc_get_handle")
    handles = [None] * world
    pg.all_gather_object(handles, (rank, handle))
    boxes: List[int] = []
    for i, item in enumerate(handles):
        src, h = item
        if src != i:
            raise PeerError(f"handle {i} came from rank {src}")
        if i == rank:
            boxes.append(own)
        else:
            err, ptr = open_handle(h)
            _check(err, "vc_peer_ipc_open")
            boxes.append(ptr)
    return boxes


def close_mailboxes(pg, rank: int, boxes: List[int],
                    close_handle: Optional[Callable[[int], int]] = None,
                    free: Optional[Callable[[int], int]] = None) -> None:
    """Unmap the other ranks' mailboxes and free this rank's, after every
    rank has finished its calls (two barriers: nobody stores into a mailbox
    after the first; nobody frees one that another still maps before the
    second)."""
    if close_handle is None or free is None:
        from vkcuda_b200 import vc
        close_handle = close_handle or vc.peer_ipc_close
        free = free or vc.peer_mailbox_free
    pg.barrier()
    for i, ptr in enumerate(boxes):
        if i != rank:
            _check(close_handle(ptr), "vc_peer_ipc_close")
    pg.barrier()
    _check(free(boxes[rank]), "vc_peer_mailbox_free")
