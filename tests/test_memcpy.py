"""The runtime memcpy task shim (rtMemcpyAsyncWithCfg shape) over the copy kernel."""
import numpy as np
import pytest


def test_memcpy_validation_on_host(dcopy):
    with pytest.raises(dcopy.DcopyError) as e:  # cnt > destMax
        dcopy.memcpy_async(0x1000, 16, 0x2000, 17, "DEVICE_TO_DEVICE")
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.memcpy_async(0x1000, 16, 0x2000, 16, 42)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.memcpy_async(0x1000, 16, 0x2000, 16, "ADDR_DEVICE_TO_DEVICE")
    assert e.value.code == dcopy.ERR_UNSUPPORTED
    dcopy.memcpy_async(0, 0, 0, 0, "DEVICE_TO_DEVICE")  # nothing to copy


@pytest.mark.gpu
def test_memcpy_kinds(torch_cuda, dcopy):
    torch = torch_cuda
    n = (8 << 20) + 5
    src = torch.randint(0, 255, (n,), dtype=torch.uint8, device="cuda")
    dst = torch.zeros(n + 64, dtype=torch.uint8, device="cuda")
    for kind in ("DEVICE_TO_DEVICE", "DEFAULT"):
        dst.zero_()
        dcopy.memcpy_async(dst.data_ptr() + 3, dst.numel() - 3, src, n, kind)
        torch.cuda.synchronize()
        assert torch.equal(dst[3:3 + n], src) and int(dst[:3].sum()) == 0
    host = np.zeros(n, dtype=np.uint8)
    dcopy.memcpy_async(host, n, src, n, "DEVICE_TO_HOST")
    torch.cuda.synchronize()
    assert host.tobytes() == src.cpu().numpy().tobytes()
    back = torch.zeros_like(src)
    dcopy.memcpy_async(back, n, host, n, "HOST_TO_DEVICE")
    torch.cuda.synchronize()
    assert torch.equal(back, src)


def test_memcpy_batch_validation_on_host(dcopy):
    """Every task is checked before anything runs; all of these fail on the host."""
    with pytest.raises(dcopy.DcopyError) as e:  # the second task's cnt > destMax
        dcopy.memcpy_async_batch([(0x1000, 16, 0x2000, 16), (0x3000, 8, 0x4000, 9)],
                                 "DEVICE_TO_DEVICE")
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.memcpy_async_batch([(0x1000, 16, 0x2000, 16)], "ADDR_DEVICE_TO_DEVICE")
    assert e.value.code == dcopy.ERR_UNSUPPORTED
    with pytest.raises(dcopy.DcopyError) as e:
        dcopy.memcpy_async_batch([(0x1000, 16, 0x2000, 16)], 42)
    assert e.value.code == dcopy.ERR_PARAM_INVALID
    assert dcopy.lib().dcopy_memcpy_async_batch(None, 2, 3, None) == dcopy.ERR_PARAM_INVALID
    dcopy.memcpy_async_batch([], "DEVICE_TO_DEVICE")
    dcopy.memcpy_async_batch([(0, 0, 0, 0)], "DEVICE_TO_DEVICE")  # nothing to copy


@pytest.mark.gpu
def test_memcpy_batch_kinds(torch_cuda, dcopy):
    """300 small tasks per kind: pinned host <-> device and device <-> device run as
    batched launches, pageable host memory and a 9 MiB task take the copy engine."""
    torch = torch_cuda
    rng = np.random.default_rng(3)
    sizes = [int(rng.integers(1, 5000)) for _ in range(300)]
    offs = np.concatenate([[0], np.cumsum([s + int(rng.integers(0, 7)) for s in sizes])])
    total = int(offs[-1]) + 64
    host_src = torch.from_numpy(rng.integers(0, 256, total, dtype=np.uint8)).pin_memory()
    dev = torch.zeros(total, dtype=torch.uint8, device="cuda")
    tasks = [(dev.data_ptr() + int(o), total - int(o), host_src.data_ptr() + int(o), s)
             for o, s in zip(offs[:-1], sizes)]
    dcopy.memcpy_async_batch(tasks, "HOST_TO_DEVICE")
    torch.cuda.synchronize()
    expect = np.zeros(total, dtype=np.uint8)
    for o, s in zip(offs[:-1], sizes):
        expect[o:o + s] = host_src.numpy()[o:o + s]
    assert dev.cpu().numpy().tobytes() == expect.tobytes()
    # Device -> pinned host, device -> device, and device -> pageable host.
    host_dst = torch.zeros(total, dtype=torch.uint8).pin_memory()
    dcopy.memcpy_async_batch([(host_dst.data_ptr() + int(o), s, dev.data_ptr() + int(o), s)
                              for o, s in zip(offs[:-1], sizes)], "DEVICE_TO_HOST")
    dev2 = torch.zeros_like(dev)
    dcopy.memcpy_async_batch([(dev2.data_ptr() + int(o), s, dev.data_ptr() + int(o), s)
                              for o, s in zip(offs[:-1], sizes)], "DEVICE_TO_DEVICE")
    pageable = np.zeros(total, dtype=np.uint8)
    dcopy.memcpy_async_batch([(pageable.ctypes.data + int(o), s, dev.data_ptr() + int(o), s)
                              for o, s in zip(offs[:-1], sizes)], "DEVICE_TO_HOST")
    torch.cuda.synchronize()
    assert host_dst.numpy().tobytes() == expect.tobytes()
    assert dev2.cpu().numpy().tobytes() == expect.tobytes()
    assert pageable.tobytes() == expect.tobytes()
    # A large host-side task (copy engine) next to small ones (kernel), kind DEFAULT.
    big = torch.randint(0, 255, (9 << 20,), dtype=torch.uint8).pin_memory()
    big_dev = torch.zeros(9 << 20, dtype=torch.uint8, device="cuda")
    small_dev = torch.zeros(100, dtype=torch.uint8, device="cuda")
    dcopy.memcpy_async_batch([(big_dev, big.numel(), big.data_ptr(), big.numel()),
                              (small_dev, 100, big.data_ptr() + 7, 100)], "DEFAULT")
    torch.cuda.synchronize()
    assert torch.equal(big_dev.cpu(), big) and torch.equal(small_dev.cpu(), big[7:107])


@pytest.mark.gpu
def test_memcpy_batch_keeps_task_order(torch_cuda, dcopy):
    """Tasks that depend on earlier tasks give the result of running them one by one:
    a chain a -> b -> c of kernel tasks, a copy-engine task (pageable host) between
    kernel tasks that reads what the first wrote, and a later kernel task that reads
    what the engine task wrote."""
    torch = torch_cuda
    n = 4096
    a = torch.randint(0, 255, (n,), dtype=torch.uint8, device="cuda")
    b = torch.zeros_like(a)
    c = torch.zeros_like(a)
    dcopy.memcpy_async_batch([(b, n, a.data_ptr(), n), (c, n, b.data_ptr(), n)],
                             "DEVICE_TO_DEVICE")
    torch.cuda.synchronize()
    assert torch.equal(b, a) and torch.equal(c, a)
    pageable = np.zeros(n, dtype=np.uint8)
    pinned = torch.zeros(n, dtype=torch.uint8).pin_memory()
    d = torch.zeros_like(a)
    e = torch.zeros_like(a)
    dcopy.memcpy_async_batch([(pinned.data_ptr(), n, a.data_ptr(), n),        # kernel
                              (pageable.ctypes.data, n, pinned.data_ptr(), n),  # engine
                              (d, n, pinned.data_ptr(), n),                    # kernel
                              (e, n, d.data_ptr(), n)], "DEFAULT")             # kernel, reads d
    torch.cuda.synchronize()
    want = a.cpu().numpy().tobytes()
    assert pageable.tobytes() == want
    assert d.cpu().numpy().tobytes() == want and e.cpu().numpy().tobytes() == want
