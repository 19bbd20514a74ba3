"""CPU tests of the C-ABI library: it loads, exports every function that
include/pilm_cuda.h declares, and rejects bad arguments before touching a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from pilm_b200 import bindings as abi

HEADER = Path(__file__).resolve().parents[1] / "include" / "pilm_cuda.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)
    keep = {n for n in names if n.startswith(("ecpu_", "ekernel_", "edevice_"))}
    return sorted(keep)


def test_library_exports_every_declared_function():
    lib = abi.lib()
    names = declared_functions()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_runtime_info_and_isa():
    info = abi.runtime_info()
    assert info["isa"] == "sm_100a"
    assert info["version"].startswith("0.1.0")
    assert all(info["symbols"].values())


def test_reference_symbol_surface_is_covered():
    """Every kernel symbol the reference binds on the verify path (bindings.py:9-26,
    minus the Qwen3.5-only recurrence and the experimental layouts) exists here."""
    needed = ["ekernel_gemm", "ekernel_linear_w8a32", "ekernel_linear_w8a16_bf16",
              "ekernel_linear_w8a16_bf16_argmax", "ekernel_linear_w4a16_bf16", "ekernel_linear_w4a16g32_bf16",
              "ekernel_linear_w4a16g128_bf16", "ekernel_swiglu_bf16", "ekernel_swiglu_w4a16_bf16",
              "ekernel_rmsnorm_bf16", "ecpu_init", "ecpu_shutdown", "ecpu_version", "ecpu_last_error",
              "ecpu_config_default", "ecpu_is_initialized", "ekernel_detect_isa", "ekernel_isa_name",
              "edevice_active"]
    lib = abi.lib()
    assert all(hasattr(lib, n) for n in needed)


def test_bad_arguments_rejected_without_gpu():
    lib = abi.lib()
    d = abi.EkernelLinearW8A32Desc(4, 8, 128)
    rc = lib.ekernel_linear_w4a16g128_bf16(ctypes.byref(d), None, None, None, None, 0)
    assert rc == -1 and "null" in abi.last_error()
    assert lib.ekernel_rmsnorm_bf16(None, None, None, 0, 0, ctypes.c_float(1e-6), 0) == -1
    desc = abi.PagedAttnDesc(1, 1, 1, 4, 2, 64, 16, 4, 4, 16, 512, 16, 64, 1e-6, 0, 0)
    assert lib.ekernel_paged_attention_verify(ctypes.byref(desc), *([None] * 8)) == -5  # head_dim 64 unsupported
    desc.head_dim = 128
    assert lib.ekernel_paged_attention_verify(ctypes.byref(desc), *([None] * 8)) == -1
    sw = abi.EkernelW4A16SwiGLUDesc(1, 8, 16, 8, 15)
    assert lib.ekernel_swiglu_w4a16_bf16(ctypes.byref(sw), 1, 1, 1, 1, 1, 1, 0) == -5  # down_in != intermediate


def test_device_registry_without_gpu():
    lib = abi.lib()
    cfg = lib.ecpu_config_default()
    assert cfg.device_type == abi.EDEV_CUDA
    host = lib.edevice_get(abi.EDEV_ECPU)
    assert host and host.contents.name.decode().startswith("ecpu")
    cuda = lib.edevice_get(abi.EDEV_CUDA)
    assert cuda and cuda.contents.name.decode().startswith("cuda")


def test_isa_name_table():
    lib = abi.lib()
    assert lib.ekernel_isa_name(16) == b"sm_100a"
    assert lib.ekernel_isa_name(1) == b"avx2"


def test_wrapper_output_buffers_are_checked_before_any_launch():
    """A caller-supplied output buffer is written through its raw pointer, so the wrappers
    accept only a contiguous tensor of the exact element count, dtype and device; anything
    else is refused on the host."""
    import torch

    from pilm_b200 import ckernel as ck

    cpu = torch.device("cpu")
    made = ck._out(None, (3, 4), torch.bfloat16, cpu)
    assert made.shape == (3, 4) and made.dtype == torch.bfloat16
    buf = torch.empty((5, 4), dtype=torch.bfloat16)
    assert ck._out(buf[1:4], (3, 4), torch.bfloat16, cpu).data_ptr() == buf[1].data_ptr()
    assert ck._out(buf[:3].view(12), (3, 4), torch.bfloat16, cpu).numel() == 12  # same bytes, other shape
    with pytest.raises(ValueError, match="12 elements"):
        ck._out(buf[:2], (3, 4), torch.bfloat16, cpu)                           # too small: would be overrun
    with pytest.raises(ValueError):
        ck._out(torch.empty((3, 4), dtype=torch.float32), (3, 4), torch.bfloat16, cpu)
    with pytest.raises(ValueError, match="not contiguous"):
        ck._out(torch.empty((4, 3), dtype=torch.bfloat16).t(), (3, 4), torch.bfloat16, cpu)
    with pytest.raises(ValueError):
        ck._out(torch.empty((3, 4), dtype=torch.bfloat16), (3, 4), torch.bfloat16, torch.device("meta"))
