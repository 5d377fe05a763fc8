"""Host-side logic of the multi-GPU path, on CPU: shard split, and the IPC-handle
exchange between ranks run as gloo processes (world size 2) with fake handle
functions, including a rank that fails before the exchange."""
import datetime
import os
import socket
import tempfile

import pytest
import torch.multiprocessing as mp


def test_shard_range_covers_every_block_once(dcopy):
    for count in (0, 1, 7, 8, 9, 4096, 8_388_608, 2**40 + 3):
        for world in (1, 2, 3, 4, 8):
            pos = 0
            for r in range(world):
                b, c = dcopy.shard_range(count, r, world)
                assert b == pos
                assert c in (count // world, count // world + 1)
                pos += c
            assert pos == count
    with pytest.raises(dcopy.DcopyError):
        dcopy.shard_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, outdir, fail_rank):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "data-copy_b200"))
    import torch.distributed as dist
    from dcopy import multi
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=6))
    result = "ok"
    try:
        if rank == fail_rank:
            raise RuntimeError("rank failed before the exchange")
        opened, closed = [], []

        def get_handle(x):
            return (f"handle-{rank}-{x}".encode().ljust(64, b"\0"), 16 * (rank + 1))

        def open_handle(h):
            opened.append(h)
            return 0x10000 * (len(opened))

        m = multi.map_next_peer("recv", "flag", rank, world, get_handle=get_handle,
                                open_handle=open_handle, close_handle=closed.append)
        nxt = (rank + 1) % world
        assert opened == [f"handle-{nxt}-recv".encode().ljust(64, b"\0"),
                          f"handle-{nxt}-flag".encode().ljust(64, b"\0")]
        assert m.recv_ptr == 0x10000 + 16 * (nxt + 1)
        assert m.flag_ptr == 0x20000 + 16 * (nxt + 1)
        m.release()
        assert closed == [0x10000, 0x20000]
    except Exception as e:  # noqa: BLE001 - the parent checks what each rank saw
        result = f"error: {type(e).__name__}: {e}"
    finally:
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(result)
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank):
    outdir = tempfile.mkdtemp()
    mp.start_processes(_rank_main, args=(world, _free_port(), outdir, fail_rank), nprocs=world,
                       start_method="spawn", join=True)
    return [open(os.path.join(outdir, f"rank{r}.txt")).read() for r in range(world)]


def test_ipc_exchange_protocol_two_ranks():
    assert _run(2, fail_rank=-1) == ["ok", "ok"]


def test_rank_failure_is_reported_not_hung():
    res = _run(2, fail_rank=1)
    assert res[1].startswith("error: RuntimeError: rank failed")
    assert res[0].startswith("error:"), res  # the survivor's exchange times out with an error
