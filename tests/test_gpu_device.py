"""The "cuda" device the reference reserves (src/runtime/device/cuda_device.py:3-33),
filled by pilm_b200.device.CudaDevice over the library's EDEV_CUDA vtable
(device/api.h:31-46): init, info, alloc, the three copies, synchronize and free."""
import numpy as np
import pytest

from pilm_b200.device import available_devices, get_device

pytestmark = pytest.mark.gpu


def test_cuda_device_vtable_round_trip():
    assert "cuda" in available_devices()
    d = get_device("cuda")
    assert d.init() == 0 and d.is_gpu and d.is_available()
    info = d.info()
    assert info.name.startswith("cuda") and 0 < info.mem_free <= info.mem_total
    n = 1 << 20
    src = np.arange(n // 4, dtype=np.float32)
    a, b = d.alloc(n), d.alloc(n, 256)
    try:
        assert a % 256 == 0 and b % 256 == 0
        d.memcpy_h2d(a, src.ctypes.data, n)
        d.memcpy_d2d(b, a, n)
        out = np.zeros_like(src)
        d.memcpy_d2h(out.ctypes.data, b, n)
        assert d.synchronize() == 0
        assert np.array_equal(out, src)
        assert d.info().mem_free <= info.mem_free  # the two buffers are held
    finally:
        d.free(a)
        d.free(b)
    with pytest.raises(KeyError):
        get_device("rocm")
