"""Multi-GPU paths on real GPUs.

One GPU: the bounded device-side wait times out on a flag nothing sets and then
sees a flag set earlier on the stream; a P2P copy within one device.
Two or more GPUs: per-device strided copies, the single-process ring shift over
NVLink, and the multi-process ring shift through CUDA IPC with completion flags
(one process per GPU; gloo only carries the IPC handles).  No test runs two
waiting kernels on one GPU.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _need_gpus(torch, n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def test_wait_signal_bounded(torch_cuda, dcopy):
    torch = torch_cuda
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    dcopy.wait_signal(flag, 1, 2_000_000, status)  # 2 ms; nothing sets the flag
    torch.cuda.synchronize()
    assert status.item() == 1
    dcopy.signal(flag, 1)
    dcopy.wait_signal(flag, 1, 2_000_000_000, status)
    torch.cuda.synchronize()
    assert status.item() == 0 and flag.item() == 1


def test_wait_signal_counts_a_flag_already_past(torch_cuda, dcopy):
    """A ring neighbour one step ahead has already moved the flag past the awaited
    sequence number: the wait must see it as arrived (not spin to its timeout)."""
    torch = torch_cuda
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    dcopy.signal(flag, 6)
    dcopy.wait_signal(flag, 5, 2_000_000_000, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    # Across the 2^32 wrap: 0x00000001 is past 0xFFFFFFFF.
    dcopy.signal(flag, 1)
    dcopy.wait_signal(flag, 0xFFFFFFFF, 2_000_000_000, status)
    torch.cuda.synchronize()
    assert status.item() == 0
    # A flag behind the awaited value still times out (2 ms).
    dcopy.wait_signal(flag, 3, 2_000_000, status)
    torch.cuda.synchronize()
    assert status.item() == 1


def test_p2p_copy_same_device(torch_cuda, dcopy, p2p_engine):
    torch = torch_cuda
    src = torch.randint(0, 255, (1 << 20,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros_like(src)
    dcopy.p2p_copy(dst, src, src.numel())
    torch.cuda.synchronize()
    assert torch.equal(src, dst)
    want = dcopy.P2P_ROUTE_COPY_ENGINE if p2p_engine == "copy" else dcopy.P2P_ROUTE_SM_LOAD_STORE
    assert dcopy.p2p_route(dst, src, src.numel()) == want


def test_p2p_route_to_a_peer(torch_cuda, dcopy):
    """Pushes to another GPU's allocation run on the copy engine (any size); with the
    SM engine forced, 16-byte granular pushes run the bulk-copy push and ragged ones
    the load/store kernel; a pull (launched on the receiver) stays on the load/store
    kernel."""
    torch = torch_cuda
    _need_gpus(torch, 2)
    src = torch.empty(4 << 20, dtype=torch.uint8, device="cuda:0")
    dst = torch.empty(4 << 20, dtype=torch.uint8, device="cuda:1")
    with torch.cuda.device(0):
        for n in (4 << 20, 1 << 20, 4096, 1000):
            assert dcopy.p2p_route(dst, src, n) == dcopy.P2P_ROUTE_COPY_ENGINE
        prev = dcopy.set_p2p_engine(dcopy.P2P_ENGINE_SM)
        try:
            assert dcopy.p2p_route(dst, src, 4 << 20) == dcopy.P2P_ROUTE_SM_BULK_PUSH
            assert dcopy.p2p_route(dst, src, 1000) == dcopy.P2P_ROUTE_SM_LOAD_STORE
        finally:
            dcopy.set_p2p_engine(prev)
    with torch.cuda.device(1):
        assert dcopy.p2p_route(dst, src, 4 << 20) == dcopy.P2P_ROUTE_SM_LOAD_STORE


def test_copy_ext_multi_two_devices(torch_cuda, dcopy):
    torch = torch_cuda
    _need_gpus(torch, 2)
    count, blen, gap = 4096, 2048, 2048
    srcs = [torch.randint(0, 255, (count * (blen + gap),), dtype=torch.uint8, device=f"cuda:{d}")
            for d in (0, 1)]
    dsts = [torch.zeros(count * blen, dtype=torch.uint8, device=f"cuda:{d}") for d in (0, 1)]
    dcopy.copy_ext_multi([(d, dsts[d], srcs[d], (count, blen, gap, 0), 0) for d in (0, 1)])
    for d in (0, 1):
        torch.cuda.synchronize(d)
        assert torch.equal(dsts[d], srcs[d].view(count, blen + gap)[:, :blen].reshape(-1))


@pytest.fixture(params=["auto", "sm", "copy"])
def p2p_engine(request, dcopy):
    """Each engine of dcopy_p2p_copy in turn; the former setting is restored."""
    engine = {"auto": dcopy.P2P_ENGINE_AUTO, "sm": dcopy.P2P_ENGINE_SM,
              "copy": dcopy.P2P_ENGINE_COPY}[request.param]
    prev = dcopy.set_p2p_engine(engine)
    yield request.param
    dcopy.set_p2p_engine(prev)


def test_ring_shift_single_process(torch_cuda, dcopy, p2p_engine):
    """64 MiB pushes (the copy engine under the automatic choice, the bulk-copy
    pipeline with the SM engine) and ragged ones, whole buffers compared."""
    torch = torch_cuda
    _need_gpus(torch, 2)
    n = min(torch.cuda.device_count(), 4)
    nbytes = 64 << 20
    srcs = [torch.full((nbytes,), d + 1, dtype=torch.uint8, device=f"cuda:{d}") for d in range(n)]
    dsts = [torch.zeros(nbytes, dtype=torch.uint8, device=f"cuda:{d}") for d in range(n)]
    dcopy.p2p_ring_shift(list(range(n)), srcs, dsts, nbytes)
    for d in range(n):
        torch.cuda.synchronize(d)
    for d in range(n):
        assert torch.equal(dsts[(d + 1) % n], srcs[d].to(f"cuda:{(d + 1) % n}"))
        with torch.cuda.device(d):
            assert dcopy.p2p_error() == 0
    # Ragged sizes take the load/store kernel; the result is the same bytes.
    odd = nbytes - 7
    for d in range(n):
        dsts[d].zero_()
    dcopy.p2p_ring_shift(list(range(n)), srcs, dsts, odd)
    for d in range(n):
        torch.cuda.synchronize(d)
    for d in range(n):
        got = dsts[(d + 1) % n]
        assert torch.equal(got[:odd], srcs[d][:odd].to(got.device)) and int(got[odd:].sum()) == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ipc_rank(rank, world, port, outdir):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "data-copy_b200"))
    import torch
    import torch.distributed as dist
    import dcopy
    from dcopy import multi
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    result = "ok"
    peer = None
    try:
        nbytes = 32 << 20
        src = torch.full((nbytes,), 10 + rank, dtype=torch.uint8, device="cuda")
        recv = torch.zeros(nbytes + 4096, dtype=torch.uint8, device="cuda")[4096:]  # offset view
        flags = torch.zeros(4, dtype=torch.int32, device="cuda")
        status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        dist.barrier()
        peer = multi.map_next_peer(recv, flags, rank, world)
        # The IPC mapping is another GPU's memory: a 32 MiB push goes to the copy
        # engine under the automatic choice, to the bulk-copy push with the SM engine.
        route = dcopy.p2p_route(peer.recv_ptr, src, nbytes)
        assert route == dcopy.P2P_ROUTE_COPY_ENGINE, f"route {route}"
        prev = dcopy.set_p2p_engine(dcopy.P2P_ENGINE_SM)
        route = dcopy.p2p_route(peer.recv_ptr, src, nbytes)
        dcopy.set_p2p_engine(prev)
        assert route == dcopy.P2P_ROUTE_SM_BULK_PUSH, f"SM route {route}"
        assert dcopy.p2p_route(recv, src, nbytes) == dcopy.P2P_ROUTE_SM_LOAD_STORE
        multi.ring_shift(src, nbytes, peer, seq=1)
        multi.wait_ring(flags, 1, status, timeout_ns=10_000_000_000)
        torch.cuda.synchronize()
        prev = (rank - 1) % world
        assert status.item() == 0, f"status {status.item()}"
        assert torch.equal(recv, torch.full_like(recv, 10 + prev)), "received bytes differ"
        dist.barrier()  # every rank is done reading before mappings close
    except Exception as e:  # noqa: BLE001
        result = f"error: {type(e).__name__}: {e}"
    finally:
        if peer is not None:
            peer.release()
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(result)
        dist.destroy_process_group()


def test_ring_shift_ipc_multiprocess(torch_cuda):
    torch = torch_cuda
    _need_gpus(torch, 2)
    world = min(torch.cuda.device_count(), 4)
    outdir = tempfile.mkdtemp()
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.start_processes(_ipc_rank, args=(world, _free_port(), outdir), nprocs=world,
                           start_method="spawn", join=True)
    finally:
        os.environ.clear()
        os.environ.update(env)
    res = [open(os.path.join(outdir, f"rank{r}.txt")).read() for r in range(world)]
    assert res == ["ok"] * world, res
