"""The reference's own ctypes bindings (src/abi/bindings.py), unmodified, loaded against
libpilm_cuda.so through its PILM_ECPU_LIB switch (bindings.py:33-35): the drop-in check a
maintainer of the reference runs.  PILM_REF_BINDINGS names the reference's bindings.py; the
test is skipped when it is unset (the reference tree is not part of this repository).
No GPU is needed: only library loading, symbol configuration and the device registry run."""
import importlib.util
import os

import pytest

from pilm_b200 import bindings as abi

# kernels the reference binds that are not on the verify path: the experimental layouts
# (runtime_status.md:404-408) and the Qwen3.5 linear-attention recurrence
OFF_PATH = {"ekernel_linear_w8a16_bf16_i8b8", "ekernel_linear_w8a16_bf16_q8", "ekernel_linear_w4a16_bf16_q8",
            "ekernel_linear_w4a16_bf16_i4b8", "ekernel_linear_w4a16_bf16_b8", "ekernel_gated_delta_recurrent_f32"}


def test_reference_bindings_configure_against_this_library(monkeypatch):
    path = os.environ.get("PILM_REF_BINDINGS")
    if not path:
        pytest.skip("PILM_REF_BINDINGS (the reference's src/abi/bindings.py) is not set")
    lib_path = abi.library_path()
    monkeypatch.setenv("PILM_ECPU_LIB", lib_path)
    spec = importlib.util.spec_from_file_location("reference_bindings_under_test", path)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    info = ref.runtime_info()
    assert info["library_path"] == lib_path
    assert info["version"] == abi.version()
    missing = [n for n, ok in info["symbols"].items() if not ok and n not in OFF_PATH]
    assert not missing, missing
    # the reference's ISA_NAMES (bindings.py:302) has no entry for this library's ISA value
    # 16, so its detect_isa() reads "unknown"; this library's own name for it is sm_100a
    assert info["isa"] == "unknown" and abi.detect_isa() == "sm_100a"
    dev = ref.active_device_info()
    assert dev["id"] == abi.EDEV_CUDA and dev["name"].startswith("cuda")
