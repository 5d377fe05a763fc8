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
