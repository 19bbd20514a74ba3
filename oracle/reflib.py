"""TEST INFRASTRUCTURE -- ctypes access to the UNMODIFIED reference library.

``oracle/_ref/libecpu.so`` is piLM's own C kernel library compiled from the
reference sources by ``make -C oracle ref`` (see oracle/Makefile).  Tests use it
to pin the restatement in ``oracle_kernels.c`` bit-for-bit, and bench.py's
``--impl reference`` arm times it on the host cores.  The descriptor layouts
follow the reference header src/ecpu/include/kernel/api.h:40-50.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_LIB = HERE / "_ref" / "libecpu.so"
_LIB = None


class LinearDesc(ctypes.Structure):
    """ekernel_linear_w8a32_desc_t (api.h:40-42)."""
    _fields_ = [("M", ctypes.c_size_t), ("N", ctypes.c_size_t), ("K", ctypes.c_size_t)]


class SwiGLUDesc(ctypes.Structure):
    """ekernel_w4a16_swiglu_desc_t (api.h:44-50)."""
    _fields_ = [("M", ctypes.c_size_t), ("hidden_size", ctypes.c_size_t),
                ("intermediate_size", ctypes.c_size_t), ("gate_up_in_features", ctypes.c_size_t),
                ("down_in_features", ctypes.c_size_t)]


def available() -> bool:
    return REF_LIB.exists()


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} is missing: run `make -C oracle ref` where the reference is present")
        L = ctypes.CDLL(str(REF_LIB))
        vp = ctypes.c_void_p
        for name in ("ekernel_linear_w8a32", "ekernel_linear_w8a16_bf16", "ekernel_linear_w4a16_bf16",
                     "ekernel_linear_w4a16g32_bf16", "ekernel_linear_w4a16g128_bf16"):
            fn = getattr(L, name)
            fn.argtypes = [ctypes.POINTER(LinearDesc), vp, vp, vp, vp, ctypes.c_int]
            fn.restype = ctypes.c_int
        L.ekernel_linear_w8a16_bf16_argmax.argtypes = [ctypes.POINTER(LinearDesc), vp, vp, vp,
                                                       ctypes.POINTER(ctypes.c_size_t),
                                                       ctypes.POINTER(ctypes.c_float), ctypes.c_int]
        L.ekernel_linear_w8a16_bf16_argmax.restype = ctypes.c_int
        L.ekernel_rmsnorm_bf16.argtypes = [vp, vp, vp, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float, ctypes.c_int]
        L.ekernel_swiglu_bf16.argtypes = [vp, vp, vp, ctypes.c_size_t]
        L.ekernel_swiglu_w4a16_bf16.argtypes = [ctypes.POINTER(SwiGLUDesc), vp, vp, vp, vp, vp, vp, ctypes.c_int]
        L.ekernel_detect_isa.restype = ctypes.c_int
        L.ekernel_isa_name.argtypes = [ctypes.c_int]
        L.ekernel_isa_name.restype = ctypes.c_char_p
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def isa_name() -> str:
    L = lib()
    return L.ekernel_isa_name(L.ekernel_detect_isa()).decode()


def linear(kind: str, x: np.ndarray, qw: np.ndarray, s: np.ndarray) -> np.ndarray:
    """Call ekernel_linear_<kind> with numpy buffers (bf16 as uint16 bits)."""
    M, K = x.shape
    N = qw.shape[0]
    if kind == "w8a32":
        out = np.empty((M, N), np.float32)
    else:
        out = np.empty((M, N), np.uint16)
    d = LinearDesc(M, N, K)
    fn = getattr(lib(), f"ekernel_linear_{kind}")
    rc = fn(ctypes.byref(d), _p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(qw)),
            _p(np.ascontiguousarray(s)), _p(out), 1)
    if rc != 0:
        raise RuntimeError(f"ekernel_linear_{kind} failed: rc={rc}")
    return out


def linear_w8a16_bf16_argmax(x: np.ndarray, qw: np.ndarray, s: np.ndarray) -> tuple[int, float]:
    """ekernel_linear_w8a16_bf16_argmax (api.h:66-72) for one activation row: the index
    and value of the largest output."""
    x = np.ascontiguousarray(x, np.uint16).reshape(1, -1)
    idx, val = ctypes.c_size_t(0), ctypes.c_float(0.0)
    d = LinearDesc(1, qw.shape[0], x.shape[1])
    rc = lib().ekernel_linear_w8a16_bf16_argmax(ctypes.byref(d), _p(x), _p(np.ascontiguousarray(qw)),
                                                _p(np.ascontiguousarray(s)), ctypes.byref(idx), ctypes.byref(val), 1)
    if rc != 0:
        raise RuntimeError(f"ekernel_linear_w8a16_bf16_argmax failed: rc={rc}")
    return int(idx.value), float(val.value)


def rmsnorm_bf16(x: np.ndarray, w: np.ndarray, eps: float, add_one: bool) -> np.ndarray:
    x2 = np.ascontiguousarray(x, np.uint16).reshape(-1, x.shape[-1])
    out = np.empty_like(x2)
    rc = lib().ekernel_rmsnorm_bf16(_p(x2), _p(out), _p(np.ascontiguousarray(w)), x2.shape[0], x2.shape[1],
                                    float(eps), int(add_one))
    assert rc == 0
    return out.reshape(x.shape)


def swiglu_bf16(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.uint16)
    u = np.ascontiguousarray(u, np.uint16)
    out = np.empty_like(g)
    assert lib().ekernel_swiglu_bf16(_p(g), _p(u), _p(out), g.size) == 0
    return out


def swiglu_w4a16_bf16(x, gu_qw, gu_s, d_qw, d_s, intermediate: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.uint16).reshape(1, -1)
    H = d_qw.shape[0]
    out = np.empty((1, H), np.uint16)
    d = SwiGLUDesc(1, H, intermediate, x.shape[1], intermediate)
    rc = lib().ekernel_swiglu_w4a16_bf16(ctypes.byref(d), _p(x), _p(np.ascontiguousarray(gu_qw)),
                                         _p(np.ascontiguousarray(gu_s)), _p(np.ascontiguousarray(d_qw)),
                                         _p(np.ascontiguousarray(d_s)), _p(out), 1)
    assert rc == 0
    return out
