"""TEST INFRASTRUCTURE -- the parity oracle's kernel layer, not the product.

numpy front-end for ``oracle/liboracle.so`` (the C restatement of piLM's CPU
kernels in ``oracle_kernels.c``) plus the weight quantizers that define the
packed formats the CUDA library consumes.  Only tests/, ``__graft_entry__.smoke``
and bench.py's CPU-baseline leg import this module.

Every function names the reference code it restates (paths are relative to the
piLM project root).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None

_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p


def build() -> Path:
    """Compile liboracle.so with the recipe in oracle/Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return HERE / "liboracle.so"


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        L = ctypes.CDLL(str(path))
        L.orc_gemm_f32.argtypes = [_c_size, _c_size, _c_size, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int]
        for name in ("orc_linear_w8a32", "orc_linear_w8a16_bf16", "orc_linear_w4a16_bf16"):
            getattr(L, name).argtypes = [_c_size, _c_size, _c_size, _vp, _vp, _vp, _vp]
        L.orc_linear_w4a16g_bf16.argtypes = [_c_size, _c_size, _c_size, _vp, _vp, _vp, _vp, _c_size]
        L.orc_linear_w8a16_bf16_argmax.argtypes = [_c_size, _c_size, _c_size, _vp, _vp, _vp,
                                                   ctypes.POINTER(_c_size), ctypes.POINTER(ctypes.c_float)]
        L.orc_rmsnorm_bf16.argtypes = [_vp, _vp, _vp, _c_size, _c_size, ctypes.c_float, ctypes.c_int]
        L.orc_swiglu_bf16.argtypes = [_vp, _vp, _vp, _c_size]
        L.orc_swiglu_w4a16_bf16.argtypes = [_c_size] * 5 + [_vp] * 6
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


# ---------------------------------------------------------------------------------
# bf16 helpers (kernels.c:12-25).  bf16 values are carried as uint16 bit patterns.
# ---------------------------------------------------------------------------------

def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    return (np.asarray(x, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even without NaN special-casing (kernels.c:19-25)."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bits = bits + 0x7FFF + ((bits >> 16) & 1)
    return ((bits >> 16) & 0xFFFF).astype(np.uint16)


# ---------------------------------------------------------------------------------
# Quantizers (runtime/ckernel.py:70-161).  Scales: max|w| / qmax clamped at 1e-8;
# values: round-half-to-even(w / s) clamped to +-qmax; int4 packs even k in the low
# nibble (ckernel.py:116-118).
# ---------------------------------------------------------------------------------

def quantize_i8_per_row(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """quantize_weight_i8_per_row (ckernel.py:70-75)."""
    w = np.asarray(w, dtype=np.float32)
    s = np.maximum(np.abs(w).max(axis=1) / np.float32(127.0), np.float32(1e-8)).astype(np.float32)
    q = np.clip(np.round(w / s[:, None]), -127, 127).astype(np.int8)
    return np.ascontiguousarray(q), s


def _pack_i4(q: np.ndarray) -> np.ndarray:
    rows, cols = q.shape
    if cols % 2:
        q = np.pad(q, ((0, 0), (0, 1)))
    lo = (q[:, 0::2] & 0x0F).astype(np.uint8)
    hi = ((q[:, 1::2] & 0x0F) << 4).astype(np.uint8)
    return np.ascontiguousarray(lo | hi)


def quantize_i4_per_row(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """quantize_weight_i4_per_row_chunked (ckernel.py:98-121)."""
    w = np.asarray(w, dtype=np.float32)
    s = np.maximum(np.abs(w).max(axis=1) / np.float32(7.0), np.float32(1e-8)).astype(np.float32)
    q = np.clip(np.round(w / s[:, None]), -7, 7).astype(np.int16)
    return _pack_i4(q), s


def quantize_i4_grouped(w: np.ndarray, group_size: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """quantize_weight_i4_grouped_chunked (ckernel.py:124-161): zero-padded groups."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    groups = (cols + group_size - 1) // group_size
    wp = np.pad(w, ((0, 0), (0, groups * group_size - cols))) if cols % group_size else w
    g = wp.reshape(rows, groups, group_size)
    s = np.maximum(np.abs(g).max(axis=2) / np.float32(7.0), np.float32(1e-8)).astype(np.float32)
    q = np.clip(np.round(g / s[:, :, None]), -7, 7).astype(np.int16)
    q = q.reshape(rows, groups * group_size)[:, :cols]
    return _pack_i4(q), np.ascontiguousarray(s)


def unpack_i4(qw: np.ndarray, K: int) -> np.ndarray:
    """unpack_i4_rows_to_i8 (ckernel.py:279-296): packed [N, ceil(K/2)] -> int8 [N, K]."""
    lo = (qw & 0x0F).astype(np.int8)
    hi = (qw >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty((qw.shape[0], qw.shape[1] * 2), dtype=np.int8)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out[:, :K]


# ---------------------------------------------------------------------------------
# Kernel restatements (bit-identical to the reference library; see oracle_kernels.c)
# ---------------------------------------------------------------------------------

KPAIRS_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)  # nibble position p of a word holds k = 8i + KPAIRS_ORDER[p]


def repack_w4_kpairs(qw: np.ndarray) -> np.ndarray:
    """Checker for the GPU library's own load-time layout (ekernel_repack_w4_kpairs), not a
    reference format: reference-packed int4 rows (nibble j of a row = k j, even k in the low
    nibble) rewritten so that within every 32-bit word (k = 8i .. 8i+7) nibble position p
    holds k = 8i + 2p for p < 4 and 8i + 2(p - 4) + 1 for p >= 4."""
    n, kb = qw.shape
    if kb % 4:
        raise ValueError("rows must hold whole 32-bit words (K % 8 == 0)")
    nib = np.empty((n, 2 * kb), np.uint8)
    nib[:, 0::2] = qw & 15
    nib[:, 1::2] = qw >> 4
    out = nib.reshape(n, -1, 8)[:, :, list(KPAIRS_ORDER)].reshape(n, -1)
    return (out[:, 0::2] | (out[:, 1::2] << 4)).astype(np.uint8)


def gemm_f32(a: np.ndarray, b: np.ndarray, transpose_b: bool = False) -> np.ndarray:
    """ekernel_gemm (kernels.c:396-435)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    M, K = a.shape
    N = b.shape[0] if transpose_b else b.shape[1]
    c = np.empty((M, N), np.float32)
    rc = lib().orc_gemm_f32(M, N, K, _p(a), _p(b), _p(c), 0, int(transpose_b))
    assert rc == 0
    return c


def linear_w8a32(x: np.ndarray, qw: np.ndarray, s: np.ndarray) -> np.ndarray:
    """ekernel_linear_w8a32 (kernels.c:437-467): fp32 in, fp32 out."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    N = qw.shape[0]
    c = np.empty((M, N), np.float32)
    rc = lib().orc_linear_w8a32(M, N, K, _p(x), _p(np.ascontiguousarray(qw)), _p(np.ascontiguousarray(s)), _p(c))
    assert rc == 0
    return c


def linear_w8a16_bf16(x: np.ndarray, qw: np.ndarray, s: np.ndarray) -> np.ndarray:
    """ekernel_linear_w8a16_bf16 (kernels.c:469-656): bf16 bits in/out."""
    x = np.ascontiguousarray(x, np.uint16)
    M, K = x.shape
    N = qw.shape[0]
    c = np.empty((M, N), np.uint16)
    rc = lib().orc_linear_w8a16_bf16(M, N, K, _p(x), _p(np.ascontiguousarray(qw)), _p(np.ascontiguousarray(s)), _p(c))
    assert rc == 0
    return c


def linear_w8a16_bf16_argmax(x: np.ndarray, qw: np.ndarray, s: np.ndarray) -> tuple[int, float]:
    """ekernel_linear_w8a16_bf16_argmax (kernels.c:658-737)."""
    x = np.ascontiguousarray(x, np.uint16).reshape(1, -1)
    idx = ctypes.c_size_t(0)
    val = ctypes.c_float(0.0)
    rc = lib().orc_linear_w8a16_bf16_argmax(1, qw.shape[0], x.shape[1], _p(x), _p(np.ascontiguousarray(qw)),
                                            _p(np.ascontiguousarray(s)), ctypes.byref(idx), ctypes.byref(val))
    assert rc == 0
    return int(idx.value), float(val.value)


def linear_w4a16_bf16(x: np.ndarray, qw: np.ndarray, s: np.ndarray, K: int | None = None) -> np.ndarray:
    """ekernel_linear_w4a16_bf16 (kernels.c:1002-1087): per-row scales."""
    x = np.ascontiguousarray(x, np.uint16)
    M, K = x.shape
    N = qw.shape[0]
    c = np.empty((M, N), np.uint16)
    rc = lib().orc_linear_w4a16_bf16(M, N, K, _p(x), _p(np.ascontiguousarray(qw)), _p(np.ascontiguousarray(s)), _p(c))
    assert rc == 0
    return c


def linear_w4a16g_bf16(x: np.ndarray, qw: np.ndarray, s: np.ndarray, group: int = 128) -> np.ndarray:
    """linear_w4a16g_bf16_impl (kernels.c:1089-1157): group-wise scales [N, ceil(K/group)]."""
    x = np.ascontiguousarray(x, np.uint16)
    M, K = x.shape
    N = qw.shape[0]
    c = np.empty((M, N), np.uint16)
    rc = lib().orc_linear_w4a16g_bf16(M, N, K, _p(x), _p(np.ascontiguousarray(qw)),
                                      _p(np.ascontiguousarray(s, np.float32)), _p(c), group)
    assert rc == 0
    return c


def rmsnorm_bf16(x: np.ndarray, w: np.ndarray, eps: float, add_one: bool) -> np.ndarray:
    """ekernel_rmsnorm_bf16 (kernels.c:1485-1526)."""
    x2 = np.ascontiguousarray(x, np.uint16).reshape(-1, x.shape[-1])
    out = np.empty_like(x2)
    rc = lib().orc_rmsnorm_bf16(_p(x2), _p(out), _p(np.ascontiguousarray(w, np.uint16)), x2.shape[0], x2.shape[1],
                                float(eps), int(bool(add_one)))
    assert rc == 0
    return out.reshape(x.shape)


def swiglu_bf16(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """ekernel_swiglu_bf16 (kernels.c:1580-1596)."""
    g = np.ascontiguousarray(gate, np.uint16)
    u = np.ascontiguousarray(up, np.uint16)
    out = np.empty_like(g)
    assert lib().orc_swiglu_bf16(_p(g), _p(u), _p(out), g.size) == 0
    return out


def swiglu_w4a16_bf16(x, gu_qw, gu_s, d_qw, d_s, intermediate: int) -> np.ndarray:
    """ekernel_swiglu_w4a16_bf16 (kernels.c:1598-1735), M=1 only."""
    x = np.ascontiguousarray(x, np.uint16).reshape(1, -1)
    H = d_qw.shape[0]
    out = np.empty((1, H), np.uint16)
    rc = lib().orc_swiglu_w4a16_bf16(1, H, intermediate, x.shape[1], intermediate, _p(x),
                                     _p(np.ascontiguousarray(gu_qw)), _p(np.ascontiguousarray(gu_s)),
                                     _p(np.ascontiguousarray(d_qw)), _p(np.ascontiguousarray(d_s)), _p(out))
    assert rc == 0
    return out


def set_threads(n: int) -> None:
    os.environ["OMP_NUM_THREADS"] = str(n)
