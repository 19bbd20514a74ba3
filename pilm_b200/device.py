"""CudaDevice: the device the reference reserves under "cuda".

Implements the reference's Device interface (src/runtime/device/base.py:11-23)
on the library's EDEV_CUDA vtable (include/pilm_cuda.h, device/api.h:31-46),
filling the stub of src/runtime/device/cuda_device.py:3-33.  Registered under
"cuda" by ``get_device`` like src/runtime/device/registry.py:5-15.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import bindings as abi


@dataclass
class DeviceInfo:
    name: str
    caps: int
    mem_total: int
    mem_free: int


class CudaDevice:
    def __init__(self):
        self._lib = abi._load_lib()
        self._vt = None

    def init(self) -> int:
        abi.init(device_type=abi.EDEV_CUDA)
        self._vt = self._lib.edevice_active()
        return 0

    def shutdown(self) -> int:
        abi.shutdown()
        return 0

    def _fn(self, field, restype, *argtypes):
        if self._vt is None:
            raise RuntimeError("CudaDevice.init() has not been called")
        return ctypes.cast(getattr(self._vt.contents, field), ctypes.CFUNCTYPE(restype, *argtypes))

    def alloc(self, bytes: int, alignment: int = 64) -> int:
        p = self._fn("alloc", ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t)(bytes, alignment)
        if not p:
            raise MemoryError(f"cuda alloc of {bytes} bytes failed")
        return p

    def free(self, ptr: int) -> None:
        self._fn("free", None, ctypes.c_void_p)(ptr)

    def memcpy_h2d(self, dst: int, src: int, n: int) -> None:
        self._fn("memcpy_h2d", None, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t)(dst, src, n)

    def memcpy_d2h(self, dst: int, src: int, n: int) -> None:
        self._fn("memcpy_d2h", None, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t)(dst, src, n)

    def memcpy_d2d(self, dst: int, src: int, n: int) -> None:
        self._fn("memcpy_d2d", None, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t)(dst, src, n)

    def synchronize(self) -> int:
        return self._fn("synchronize", ctypes.c_int)()

    def info(self) -> DeviceInfo:
        vt = self._vt.contents
        total = self._fn("mem_total", ctypes.c_size_t)()
        free = self._fn("mem_free", ctypes.c_size_t)()
        return DeviceInfo(name=vt.name.decode() if vt.name else "cuda", caps=vt.caps, mem_total=total, mem_free=free)

    @property
    def is_gpu(self) -> bool:
        return True

    @staticmethod
    def is_available() -> bool:
        try:
            import torch
            return torch.cuda.is_available()
        except Exception:
            return False


_REGISTRY = {"cuda": CudaDevice}


def get_device(name: str) -> CudaDevice:
    cls = _REGISTRY.get(name)
    if cls is None:
        raise KeyError(f"unknown device: {name}, available: {list(_REGISTRY)}")
    return cls()


def available_devices() -> list:
    return list(_REGISTRY)
