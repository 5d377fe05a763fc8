"""Multi-GPU helpers on top of the C ABI: the per-rank shard split and the NVLink
ring shift between processes (one process per GPU, torch.distributed for the
host-side exchange of CUDA IPC handles only -- no collective touches the data).

The ring shift (BASELINE config 5b): rank r pushes its shard into the receive
buffer of rank (r + 1) % world with in-kernel stores over NVLink, then
release-stores a sequence number into that rank's flag word; the receiver waits
for the flag with a bounded device-side wait and reads the status word.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional

import dcopy


def exchange(obj, group=None) -> list:
    """all_gather_object of one picklable object per rank (host-side plumbing)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


@dataclass
class PeerMapping:
    """The next rank's receive buffer and flag, mapped into this process."""
    recv_ptr: int
    flag_ptr: int
    bases: List[int]
    close: Callable[[int], None]

    def release(self) -> None:
        for b in self.bases:
            self.close(b)
        self.bases = []


def map_next_peer(recv, flags, rank: int, world: int, group=None,
                  get_handle=None, open_handle=None, close_handle=None) -> PeerMapping:
    """Exchange IPC handles of every rank's receive buffer and flag word, and map
    rank (rank + 1) % world's into this process.  The handle functions are
    parameters so the exchange protocol can be exercised without a GPU."""
    get_handle = get_handle or dcopy.ipc_get_handle
    open_handle = open_handle or dcopy.ipc_open_handle
    close_handle = close_handle or dcopy.ipc_close_handle
    mine = (rank, get_handle(recv), get_handle(flags))
    table = exchange(mine, group)
    for i, entry in enumerate(table):
        if entry[0] != i:
            raise RuntimeError(f"IPC exchange out of order: slot {i} holds rank {entry[0]}")
    nxt = table[(rank + 1) % world]
    (rh, roff), (fh, foff) = nxt[1], nxt[2]
    rbase = open_handle(rh)
    try:
        fbase = rbase if fh == rh else open_handle(fh)
    except Exception:
        close_handle(rbase)
        raise
    bases = [rbase] if fbase == rbase else [rbase, fbase]
    return PeerMapping(rbase + roff, fbase + foff, bases, close_handle)


def ring_shift(src, nbytes: int, peer: PeerMapping, seq: int, stream=None) -> None:
    """Push nbytes of src into the next rank's receive buffer, then signal `seq`."""
    dcopy.p2p_copy(peer.recv_ptr, src, nbytes, stream)
    dcopy.signal(peer.flag_ptr, seq, stream)


def wait_ring(flags, seq: int, status, timeout_ns: int = 2_000_000_000, stream=None) -> None:
    """Bounded device-side wait for this rank's flag to reach `seq` (status 0 = arrived)."""
    dcopy.wait_signal(flags, seq, timeout_ns, status, stream)
