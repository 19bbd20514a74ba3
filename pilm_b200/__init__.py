"""pilm_b200: B200 (sm_100a) implementation of piLM's MTP speculative-verify path.

Drop-in for the Ecpu kernel library on the verify path: ``bindings`` mirrors
src/abi/bindings.py over ``libpilm_cuda.so`` (C ABI in include/pilm_cuda.h),
``ckernel`` mirrors src/runtime/ckernel.py for CUDA tensors, ``device`` provides
the CudaDevice that src/runtime/device/registry.py reserves, and ``qwen3`` /
``engine`` run the batched verify step.
"""
from . import bindings

__all__ = ["bindings"]
__version__ = "0.1.0"
