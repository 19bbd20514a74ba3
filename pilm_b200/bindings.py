"""ctypes bindings to libpilm_cuda.so.

Mirrors the reference loader/binding module (src/abi/bindings.py): the same
``_load_lib`` / ``init`` / ``version`` / ``detect_isa`` / ``runtime_info`` /
``*_ptr`` surface, so host code written against the Ecpu library can switch to
the B200 library by importing this module instead.  The library is chosen by
``PILM_CUDA_LIB`` (analogue of ``PILM_ECPU_LIB``), else the in-tree build next
to this file.  Every ``*_ptr`` function takes DEVICE pointers and returns the C
return code (0 = ok), exactly like its reference counterpart.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_lib = None
_lib_path = None
_stream = None

HERE = Path(__file__).resolve().parent

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i32 = ctypes.c_int

KERNEL_SYMBOLS = [
    "ekernel_gemm",
    "ekernel_linear_w8a32",
    "ekernel_linear_w8a16_bf16",
    "ekernel_linear_w8a16_bf16_argmax",
    "ekernel_linear_w4a16_bf16",
    "ekernel_linear_w4a16g32_bf16",
    "ekernel_linear_w4a16g128_bf16",
    "ekernel_swiglu_bf16",
    "ekernel_swiglu_w4a16_bf16",
    "ekernel_rmsnorm_bf16",
    # verify-path extensions (no reference counterpart)
    "ekernel_set_stream",
    "ekernel_get_stream",
    "ekernel_synchronize",
    "ekernel_launch_count",
    "ekernel_alloc_count",
    "ekernel_set_wait_limit",
    "ekernel_embedding_bf16",
    "ekernel_add_rmsnorm_bf16",
    "ekernel_silu_mul_bf16",
    "ekernel_qk_norm_rope_kv_append",
    "ekernel_paged_attention_verify",
    "ekernel_paged_attention_verify_noalloc",
    "ekernel_argmax_top2_f32",
    "ekernel_argmax_top2_bf16",
    "ekernel_verify_accept_greedy",
    "ekernel_verify_accept_rejection",
    "ekernel_verify_accept_rejection_bf16",
    "ekernel_linear_bf16",
    "ekernel_repack_w4_kpairs",
    "ekernel_linear_w4a16g128_bf16_kpairs",
    "ekernel_linear_w4a16_bf16_kpairs",
    "ekernel_linear_w4a16g128_bf16_kpairs_deferred",
    "ekernel_linear_w4a16g128_partials_bytes",
    "ekernel_linear_w4a16g128_bf16_kpairs_argmax",
    "ekernel_verify_accept_greedy_keys",
    "ekernel_add_rmsnorm_bf16_splitk",
    "ekernel_qk_norm_rope_kv_append_splitk",
    "ekernel_mtp_fc_input_bf16",
    "ekernel_self_attention_bf16",
    "ekernel_embedding_f32",
    "ekernel_add_rmsnorm_f32",
    "ekernel_qk_norm_rope_kv_append_f32",
    "ekernel_paged_attention_verify_f32",
    "ekernel_silu_mul_f32",
]


class EcpuConfig(ctypes.Structure):
    """ecpu_config_t (ecpu.h:23-31)."""
    _fields_ = [
        ("n_threads", ctypes.c_int),
        ("numa_policy", ctypes.c_int),
        ("disable_amx", ctypes.c_int),
        ("disable_avx512", ctypes.c_int),
        ("eram_budget_bytes", ctypes.c_size_t),
        ("kv_cache_budget_bytes", ctypes.c_size_t),
        ("device_type", ctypes.c_int),
    ]


class EdeviceVtable(ctypes.Structure):
    """edevice_vtable_t (device/api.h:31-46)."""
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("id", ctypes.c_int),
        ("caps", ctypes.c_uint64),
        ("alloc", ctypes.c_void_p),
        ("free", ctypes.c_void_p),
        ("memcpy_h2d", ctypes.c_void_p),
        ("memcpy_d2h", ctypes.c_void_p),
        ("memcpy_d2d", ctypes.c_void_p),
        ("synchronize", ctypes.c_void_p),
        ("mem_total", ctypes.c_void_p),
        ("mem_free", ctypes.c_void_p),
        ("init", ctypes.c_void_p),
        ("shutdown", ctypes.c_void_p),
    ]


class EkernelGemmDesc(ctypes.Structure):
    _fields_ = [("M", _sz), ("N", _sz), ("K", _sz), ("a_prec", _i32), ("b_prec", _i32), ("out_prec", _i32),
                ("transpose_a", _i32), ("transpose_b", _i32)]


class EkernelLinearW8A32Desc(ctypes.Structure):
    _fields_ = [("M", _sz), ("N", _sz), ("K", _sz)]


class EkernelW4A16SwiGLUDesc(ctypes.Structure):
    _fields_ = [("M", _sz), ("hidden_size", _sz), ("intermediate_size", _sz), ("gate_up_in_features", _sz),
                ("down_in_features", _sz)]


class PagedAttnDesc(ctypes.Structure):
    """ekernel_paged_attn_desc_t (include/pilm_cuda.h)."""
    _fields_ = [("num_seqs", _sz), ("total_q", _sz), ("max_q_len", _sz), ("n_heads", _sz), ("n_kv_heads", _sz),
                ("head_dim", _sz), ("block_size", _sz), ("num_blocks", _sz), ("max_blocks_per_seq", _sz),
                ("max_context", _sz), ("qkv_stride", _sz), ("rope_rows", _sz), ("rot_dim", _sz),
                ("eps", ctypes.c_float), ("add_one", _i32), ("output_gate", _i32)]


class AcceptDesc(ctypes.Structure):
    """ekernel_accept_desc_t (include/pilm_cuda.h)."""
    _fields_ = [("num_seqs", _sz), ("total_q", _sz), ("vocab", _sz)]


EDEV_ECPU = 0
EDEV_CUDA = 1
ECPU_PRECISION_F32 = 0
ECPU_PRECISION_BF16 = 2
ISA_NAMES = {0: "scalar", 1: "avx2", 2: "avx512", 3: "amx", 4: "neon", 5: "sve", 16: "sm_100a"}


def _candidates() -> list[Path]:
    env = os.environ.get("PILM_CUDA_LIB")
    out = [Path(env)] if env else []
    out.append(HERE / "libpilm_cuda.so")
    return out


def _load_lib():
    """Load and configure the library (bindings.py:28-57 analogue).  Raises when it is
    missing: there is no CPU fallback behind this module."""
    global _lib, _lib_path
    if _lib is not None:
        return _lib
    for c in _candidates():
        if c.exists():
            _lib = ctypes.CDLL(str(c))
            _lib_path = str(c)
            _configure(_lib)
            return _lib
    raise RuntimeError("libpilm_cuda.so not found: build it with `python -m pilm_b200.build` "
                       "or point PILM_CUDA_LIB at it")


def _configure(lib) -> None:
    lib.ecpu_version.restype = ctypes.c_char_p
    lib.ecpu_last_error.restype = ctypes.c_char_p
    lib.ecpu_config_default.restype = EcpuConfig
    lib.ecpu_init.argtypes = [ctypes.POINTER(EcpuConfig)]
    lib.ecpu_init.restype = _i32
    lib.ecpu_is_initialized.restype = _i32
    lib.ecpu_shutdown.argtypes = []
    lib.ecpu_shutdown.restype = None
    lib.ekernel_detect_isa.restype = _i32
    lib.ekernel_isa_name.argtypes = [_i32]
    lib.ekernel_isa_name.restype = ctypes.c_char_p
    lib.edevice_active.restype = ctypes.POINTER(EdeviceVtable)
    lib.edevice_get.argtypes = [_i32]
    lib.edevice_get.restype = ctypes.POINTER(EdeviceVtable)
    lib.ekernel_gemm.argtypes = [ctypes.POINTER(EkernelGemmDesc), _vp, _vp, _vp, _i32]
    for name in ("ekernel_linear_w8a32", "ekernel_linear_w8a16_bf16", "ekernel_linear_w4a16_bf16",
                 "ekernel_linear_w4a16g32_bf16", "ekernel_linear_w4a16g128_bf16",
                 "ekernel_linear_w4a16g128_bf16_kpairs", "ekernel_linear_w4a16_bf16_kpairs"):
        fn = getattr(lib, name)
        fn.argtypes = [ctypes.POINTER(EkernelLinearW8A32Desc), _vp, _vp, _vp, _vp, _i32]
        fn.restype = _i32
    lib.ekernel_linear_w8a16_bf16_argmax.argtypes = [ctypes.POINTER(EkernelLinearW8A32Desc), _vp, _vp, _vp,
                                                     ctypes.POINTER(_sz), ctypes.POINTER(ctypes.c_float), _i32]
    lib.ekernel_linear_w4a16g128_bf16_kpairs_deferred.argtypes = [ctypes.POINTER(EkernelLinearW8A32Desc), _vp, _vp,
                                                                  _vp, _vp, _vp, _sz, ctypes.POINTER(_i32)]
    lib.ekernel_linear_w4a16g128_bf16_kpairs_deferred.restype = _i32
    lib.ekernel_linear_w4a16g128_bf16_kpairs_argmax.argtypes = [ctypes.POINTER(EkernelLinearW8A32Desc), _vp, _vp,
                                                                _vp, _vp, _vp, ctypes.POINTER(_i32)]
    lib.ekernel_linear_w4a16g128_bf16_kpairs_argmax.restype = _i32
    lib.ekernel_verify_accept_greedy_keys.argtypes = [ctypes.POINTER(AcceptDesc)] + [_vp] * 8
    lib.ekernel_linear_w4a16g128_partials_bytes.argtypes = [_sz, _sz, _sz]
    lib.ekernel_linear_w4a16g128_partials_bytes.restype = _sz
    lib.ekernel_add_rmsnorm_bf16_splitk.argtypes = [_vp, _vp, _i32, _vp, _sz, _sz, ctypes.c_float, _i32, _vp]
    lib.ekernel_qk_norm_rope_kv_append_splitk.argtypes = [ctypes.POINTER(PagedAttnDesc), _vp, _i32] + [_vp] * 10
    lib.ekernel_linear_bf16.argtypes = [ctypes.POINTER(EkernelLinearW8A32Desc), _vp, _vp, _vp]
    lib.ekernel_linear_bf16.restype = _i32
    lib.ekernel_repack_w4_kpairs.argtypes = [_vp, _sz, _sz, _vp]
    lib.ekernel_repack_w4_kpairs.restype = _i32
    lib.ekernel_swiglu_bf16.argtypes = [_vp, _vp, _vp, _sz]
    lib.ekernel_swiglu_w4a16_bf16.argtypes = [ctypes.POINTER(EkernelW4A16SwiGLUDesc), _vp, _vp, _vp, _vp, _vp, _vp,
                                              _i32]
    lib.ekernel_rmsnorm_bf16.argtypes = [_vp, _vp, _vp, _sz, _sz, ctypes.c_float, _i32]
    lib.ekernel_set_stream.argtypes = [_vp]
    lib.ekernel_get_stream.restype = _vp
    lib.ekernel_launch_count.restype = ctypes.c_ulonglong
    lib.ekernel_alloc_count.restype = ctypes.c_ulonglong
    lib.ekernel_set_wait_limit.argtypes = [ctypes.c_longlong]
    lib.ekernel_embedding_bf16.argtypes = [_vp, _sz, _vp, _sz, _sz, _vp]
    lib.ekernel_add_rmsnorm_bf16.argtypes = [_vp, _vp, _vp, _sz, _sz, ctypes.c_float, _i32, _vp]
    lib.ekernel_silu_mul_bf16.argtypes = [_vp, _sz, _sz, _vp]
    lib.ekernel_mtp_fc_input_bf16.argtypes = [_vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp, _sz, _sz, ctypes.c_float, _i32,
                                              _vp]
    lib.ekernel_self_attention_bf16.argtypes = [_vp, _vp, _sz, _sz, _sz, _sz, _vp]
    lib.ekernel_embedding_f32.argtypes = [_vp, _sz, _vp, _sz, _sz, _vp]
    lib.ekernel_add_rmsnorm_f32.argtypes = [_vp, _vp, _vp, _sz, _sz, ctypes.c_float, _i32, _vp]
    lib.ekernel_qk_norm_rope_kv_append_f32.argtypes = [ctypes.POINTER(PagedAttnDesc)] + [_vp] * 11
    lib.ekernel_paged_attention_verify_f32.argtypes = [ctypes.POINTER(PagedAttnDesc)] + [_vp] * 8
    lib.ekernel_silu_mul_f32.argtypes = [_vp, _sz, _sz, _vp]
    lib.ekernel_qk_norm_rope_kv_append.argtypes = [ctypes.POINTER(PagedAttnDesc)] + [_vp] * 11
    lib.ekernel_paged_attention_verify.argtypes = [ctypes.POINTER(PagedAttnDesc)] + [_vp] * 8
    lib.ekernel_paged_attention_verify_noalloc.argtypes = [ctypes.POINTER(PagedAttnDesc)] + [_vp] * 8
    lib.ekernel_argmax_top2_f32.argtypes = [ctypes.POINTER(AcceptDesc), _vp, _vp, _vp, _vp]
    lib.ekernel_argmax_top2_bf16.argtypes = [ctypes.POINTER(AcceptDesc), _vp, _vp, _vp, _vp]
    lib.ekernel_verify_accept_greedy.argtypes = [ctypes.POINTER(AcceptDesc)] + [_vp] * 7
    lib.ekernel_verify_accept_rejection.argtypes = ([ctypes.POINTER(AcceptDesc)] + [_vp] * 4 +
                                                    [ctypes.c_float, ctypes.c_float] + [_vp] * 4)
    lib.ekernel_verify_accept_rejection_bf16.argtypes = lib.ekernel_verify_accept_rejection.argtypes


def lib():
    return _load_lib()


def last_error() -> str:
    e = _load_lib().ecpu_last_error()
    return e.decode() if e else ""


def check(rc: int, what: str) -> None:
    """ckernel.py:178-179 convention: a non-zero return code raises RuntimeError."""
    if rc != 0:
        raise RuntimeError(f"{what} failed: rc={rc}: {last_error()}")


def init(device_type: int = EDEV_CUDA, n_threads: int = 0, kv_cache_budget: int = 4 * 1024 ** 3):
    """bindings.py:298-308 analogue: ecpu_init with the CUDA device active."""
    L = _load_lib()
    if L.ecpu_is_initialized():
        return L
    cfg = L.ecpu_config_default()
    cfg.device_type = device_type
    cfg.n_threads = n_threads
    cfg.kv_cache_budget_bytes = kv_cache_budget
    rc = L.ecpu_init(ctypes.byref(cfg))
    if rc != 0:
        raise RuntimeError(f"ecpu_init failed ({rc}): {last_error() or 'unknown'}")
    return L


def version() -> str:
    return _load_lib().ecpu_version().decode()


def detect_isa() -> str:
    return ISA_NAMES.get(_load_lib().ekernel_detect_isa(), "unknown")


def library_path() -> str:
    _load_lib()
    return _lib_path


def available_kernel_symbols() -> dict[str, bool]:
    L = _load_lib()
    return {name: hasattr(L, name) for name in KERNEL_SYMBOLS}


def runtime_info() -> dict:
    return {
        "library_path": library_path(),
        "version": version(),
        "isa": detect_isa(),
        "device": "cuda",
        "sm": "sm_100a",
        "symbols": available_kernel_symbols(),
        "env_library_path": os.environ.get("PILM_CUDA_LIB"),
    }


def active_device_info():
    vt = _load_lib().edevice_active()
    if not vt:
        return None
    name = vt.contents.name.decode() if vt.contents.name else "unknown"
    return {"name": name, "id": vt.contents.id, "caps": vt.contents.caps}


def shutdown() -> None:
    _load_lib().ecpu_shutdown()


def set_stream(stream_ptr: int) -> None:
    """Route subsequent launches to a cudaStream_t (torch: stream.cuda_stream)."""
    global _stream
    if stream_ptr != _stream:
        _load_lib().ekernel_set_stream(_vp(stream_ptr))
        _stream = stream_ptr


def launch_count() -> int:
    return int(_load_lib().ekernel_launch_count())


def alloc_count() -> int:
    """Device allocations the library has made for its own use since it was loaded."""
    return int(_load_lib().ekernel_alloc_count())


def synchronize() -> None:
    check(_load_lib().ekernel_synchronize(), "ekernel_synchronize")


# ---- *_ptr wrappers with the reference's signatures (bindings.py:341-541) -------------

def gemm_f32_ptr(a_ptr, b_ptr, c_ptr, m, n, k, transpose_a=False, transpose_b=False, isa=None) -> int:
    d = EkernelGemmDesc(m, n, k, ECPU_PRECISION_F32, ECPU_PRECISION_F32, ECPU_PRECISION_F32, int(transpose_a),
                        int(transpose_b))
    return _load_lib().ekernel_gemm(ctypes.byref(d), a_ptr, b_ptr, c_ptr, 16 if isa is None else int(isa))


def _linear(name, a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa):
    d = EkernelLinearW8A32Desc(m, n, k)
    return getattr(_load_lib(), name)(ctypes.byref(d), a_ptr, w_ptr, scales_ptr, c_ptr, 16 if isa is None else int(isa))


def linear_w8a32_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa=None) -> int:
    return _linear("ekernel_linear_w8a32", a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa)


def linear_w8a16_bf16_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa=None) -> int:
    return _linear("ekernel_linear_w8a16_bf16", a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa)


def linear_w8a16_bf16_argmax_ptr(a_ptr, w_ptr, scales_ptr, m, n, k, isa=None) -> tuple[int, int, float]:
    d = EkernelLinearW8A32Desc(m, n, k)
    idx = ctypes.c_size_t(0)
    val = ctypes.c_float(0.0)
    rc = _load_lib().ekernel_linear_w8a16_bf16_argmax(ctypes.byref(d), a_ptr, w_ptr, scales_ptr, ctypes.byref(idx),
                                                      ctypes.byref(val), 16)
    return int(rc), int(idx.value), float(val.value)


def linear_w4a16_bf16_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa=None) -> int:
    return _linear("ekernel_linear_w4a16_bf16", a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa)


def linear_w4a16g32_bf16_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa=None) -> int:
    return _linear("ekernel_linear_w4a16g32_bf16", a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa)


def linear_w4a16g128_bf16_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa=None) -> int:
    return _linear("ekernel_linear_w4a16g128_bf16", a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa)


def linear_w4a16g128_bf16_kpairs_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa=None) -> int:
    return _linear("ekernel_linear_w4a16g128_bf16_kpairs", a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa)


def linear_w4a16_bf16_kpairs_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa=None) -> int:
    return _linear("ekernel_linear_w4a16_bf16_kpairs", a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, isa)


def linear_w4a16g128_bf16_kpairs_deferred_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, part_ptr,
                                              part_bytes) -> tuple[int, int]:
    """(rc, splits): splits > 0 means the result was left as split-K partial sums at part_ptr
    ([splits][m][n] fp32) and c_ptr was not written."""
    d = EkernelLinearW8A32Desc(m, n, k)
    sp = _i32(0)
    rc = _load_lib().ekernel_linear_w4a16g128_bf16_kpairs_deferred(ctypes.byref(d), a_ptr, w_ptr, scales_ptr, c_ptr,
                                                                   part_ptr, part_bytes, ctypes.byref(sp))
    return int(rc), int(sp.value)


def linear_w4a16g128_bf16_kpairs_argmax_ptr(a_ptr, w_ptr, scales_ptr, c_ptr, m, n, k, keys_ptr) -> tuple[int, int]:
    """(rc, fused): fused = 1 when the call also folded each output row's argmax into the
    uint64 keys at keys_ptr (which must be zero before the call)."""
    d = EkernelLinearW8A32Desc(m, n, k)
    f = _i32(0)
    rc = _load_lib().ekernel_linear_w4a16g128_bf16_kpairs_argmax(ctypes.byref(d), a_ptr, w_ptr, scales_ptr, c_ptr,
                                                                 keys_ptr, ctypes.byref(f))
    return int(rc), int(f.value)


def linear_w4a16g128_partials_bytes(m, n, k) -> int:
    return int(_load_lib().ekernel_linear_w4a16g128_partials_bytes(m, n, k))


def linear_bf16_ptr(a_ptr, w_ptr, c_ptr, m, n, k) -> int:
    d = EkernelLinearW8A32Desc(m, n, k)
    return int(_load_lib().ekernel_linear_bf16(ctypes.byref(d), a_ptr, w_ptr, c_ptr))


def repack_w4_kpairs_ptr(qweight_ptr, n, k, out_ptr) -> int:
    return int(_load_lib().ekernel_repack_w4_kpairs(qweight_ptr, n, k, out_ptr))


def swiglu_bf16_ptr(gate_ptr, up_ptr, out_ptr, n) -> int:
    return _load_lib().ekernel_swiglu_bf16(gate_ptr, up_ptr, out_ptr, n)


def swiglu_w4a16_bf16_ptr(x_ptr, gate_up_w_ptr, gate_up_scales_ptr, down_w_ptr, down_scales_ptr, c_ptr, m,
                          hidden_size, intermediate_size, gate_up_in_features, down_in_features, isa=None) -> int:
    d = EkernelW4A16SwiGLUDesc(m, hidden_size, intermediate_size, gate_up_in_features, down_in_features)
    return _load_lib().ekernel_swiglu_w4a16_bf16(ctypes.byref(d), x_ptr, gate_up_w_ptr, gate_up_scales_ptr,
                                                 down_w_ptr, down_scales_ptr, c_ptr, 16)


def rmsnorm_bf16_ptr(x_ptr, out_ptr, weight_ptr, rows, n, eps, add_one=False) -> int:
    return _load_lib().ekernel_rmsnorm_bf16(x_ptr, out_ptr, weight_ptr, rows, n, float(eps), 1 if add_one else 0)
