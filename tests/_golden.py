"""Loading helpers for the golden fixtures in tests/golden/ (made by make_golden.py)."""
from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle import model as om

GOLDEN = Path(__file__).resolve().parent / "golden"
MODEL_VARIANTS = ["qwen3_w4g128", "qwen35_w4g128", "qwen3_w4g128_gqa4", "qwen3_w8a32_f32"]


def load(name: str):
    return np.load(GOLDEN / name)


def model_config(z) -> tuple[om.Qwen3Config, int]:
    H, L, nh, nkv, hd, I, V, gated, gemma, bs, seed, f32 = [int(x) for x in z["config"]]
    cfg = om.Qwen3Config(hidden=H, layers=L, n_heads=nh, n_kv_heads=nkv, head_dim=hd, intermediate=I, vocab=V,
                         gated=bool(gated), gemma_norm=bool(gemma), quant=bytes(z["quant"]).decode(),
                         dtype="float32" if f32 else "bfloat16", block_size=bs)
    return cfg, seed


def num_seqs(z) -> int:
    return sum(1 for k in z.files if k.endswith(".prompt"))


def ilist(a) -> list[int]:
    return [int(x) for x in a]
