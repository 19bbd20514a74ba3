"""Helpers for the GPU parity tests: bf16 plumbing and the tolerance rules.

Tolerances: logits and bf16 outputs agree within a max
relative error of 1e-2, measured norm-wise as max|got - ref| / max|ref|; integer
outputs (page tables, slots, accept counts, argmax away from near-ties) are exact.
"""
from __future__ import annotations

import numpy as np
import torch

REL_TOL = 1e-2


def dev():
    return torch.device("cuda:0")


def bf16_from_bits(a: np.ndarray, device=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return t.to(device or dev())


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def f32_of_bits(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / scale)


def assert_bf16_close(got_bits, ref_bits, tol=REL_TOL, ulp_frac=None):
    g, r = f32_of_bits(got_bits), f32_of_bits(ref_bits)
    e = rel_err(g, r)
    assert e <= tol, f"relative error {e:.3g} > {tol}"
    if ulp_frac is not None:
        # fraction of elements within one bf16 ulp of the reference
        ulp = np.abs(r) * 2.0 ** -7 + 1e-30
        frac = float(np.mean(np.abs(g - r) <= ulp * 1.0001))
        assert frac >= ulp_frac, f"only {frac:.4f} of elements within 1 ulp"
    return e


def argmax_agrees(got_top1, ref_logits, tol=REL_TOL) -> bool:
    """Greedy ids must be identical except where the reference's top-2 margin is
    below the logit tolerance (then either of the tied ids is accepted)."""
    ref = torch.as_tensor(ref_logits, dtype=torch.float32)
    top = torch.topk(ref, 2, dim=-1)
    scale = float(ref.abs().max())
    for i, g in enumerate(got_top1):
        r1 = int(top.indices[i, 0])
        if int(g) == r1:
            continue
        margin = float(top.values[i, 0] - ref[i, int(g)])
        if margin > tol * scale:
            return False
    return True
