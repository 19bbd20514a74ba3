"""Quant-bundle loader: a pilm-quant-bundle-v1 directory, as the reference's
scripts/export_pilm_quant_bundle.py writes it, straight into device weights.

A bundle holds (export_pilm_quant_bundle.py:86-172):
  pilm_quant_manifest.json   format, the quantized linear source names, the residual exports
  config.json                the model config (text_config, runtime/loader/config_parser.py:81-125)
  linear_w4a16/<digest>-<name>.safetensors
                             one quantized linear each: qweight uint8 [N, ceil(K/2)] (even k in
                             the low nibble), scales fp32 [N, ceil(K/128)], in_features int32;
                             the file name is the reference's cache name (models/qwen3/weights.py:59-62)
  residual_bf16/*.safetensors
                             the unquantized tensors (embedding, norms) under their HF names

read_quant_bundle() returns the host tensors; load_quant_bundle() moves them to the device,
fuses q/k/v and gate/up like Qwen3Weights.from_checkpoint, and repacks the packed weights
into the k-pair nibble order the kernels read (W4Linear).  The reference's model is the
Qwen3.5 layout (a gated q_proj, GemmaRMSNorm); only full-attention layers and group-128
linears are on this path.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from .qwen3 import Qwen3Shape, Qwen3Weights, W4Linear

MANIFEST = "pilm_quant_manifest.json"
FORMAT = "pilm-quant-bundle-v1"
PREFIX = "model.language_model."
LINEARS = {"q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj", "v_proj": "self_attn.v_proj",
           "o_proj": "self_attn.o_proj", "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
NORMS = {"input_norm": "input_layernorm", "post_norm": "post_attention_layernorm", "q_norm": "self_attn.q_norm",
         "k_norm": "self_attn.k_norm"}


def cache_file_name(src: str) -> str:
    """The reference's cache file name of a source tensor (weights.py:59-62): the first 16
    hex digits of its SHA-1, then the name with '/' and '.' replaced by '_'."""
    digest = hashlib.sha1(src.encode("utf-8")).hexdigest()[:16]
    return f"{digest}-{src.replace('/', '_').replace('.', '_')}.safetensors"


def read_shape(bundle: Path, block_size: int = 16) -> Qwen3Shape:
    """Qwen3Shape from config.json, read the way the reference's config parser does
    (defaults of config_parser.py:86-117 for absent keys)."""
    raw = json.loads((bundle / "config.json").read_text(encoding="utf-8"))
    tc = raw.get("text_config", raw)
    rope = tc.get("rope_parameters", {})
    layers = int(tc.get("num_hidden_layers", 32))
    kinds = tc.get("layer_types") or ["full_attention"] * layers
    if any(k != "full_attention" for k in kinds):
        raise ValueError("the bundle has linear-attention layers; only full-attention layers are on this path")
    return Qwen3Shape(hidden=int(tc.get("hidden_size", 4096)), layers=layers,
                      n_heads=int(tc.get("num_attention_heads", 16)), n_kv_heads=int(tc.get("num_key_value_heads", 4)),
                      head_dim=int(tc.get("head_dim", 256)), intermediate=int(tc.get("intermediate_size", 12288)),
                      vocab=int(tc.get("vocab_size", 248320)), eps=float(tc.get("rms_norm_eps", 1e-6)),
                      rope_theta=float(rope.get("rope_theta", 10000.0)),
                      partial_rotary=float(rope.get("partial_rotary_factor", 1.0)), gated=True, gemma_norm=True,
                      block_size=block_size)


def read_quant_bundle(path) -> dict:
    """Host tensors of a bundle: {"shape", "linears": {src: (qweight, scales, in_features)},
    "residual": {name: tensor}}."""
    from safetensors.torch import load_file

    bundle = Path(path)
    manifest = json.loads((bundle / MANIFEST).read_text(encoding="utf-8"))
    if manifest.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} bundle: format {manifest.get('format')!r}")
    if manifest.get("missing_linear_cache"):
        raise ValueError(f"the bundle lacks {len(manifest['missing_linear_cache'])} quantized linears")
    shape = read_shape(bundle)
    linears = {}
    for src in manifest.get("quantized_linear_sources", []):
        payload = load_file(str(bundle / "linear_w4a16" / cache_file_name(src)))
        qw, s = payload["qweight"], payload["scales"]
        k = int(payload["in_features"].reshape(-1)[0]) if "in_features" in payload else 2 * qw.shape[1]
        if qw.dtype != torch.uint8 or s.dtype != torch.float32 or qw.shape[1] != (k + 1) // 2:
            raise ValueError(f"{src}: not a W4A16 linear cache")
        if s.dim() != 2 or s.shape[1] != (k + 127) // 128:
            raise ValueError(f"{src}: only group-128 scales are on this path (scales {tuple(s.shape)})")
        linears[src] = (qw, s, k)
    residual = {}
    for export in manifest.get("residual_exports", []):
        residual.update(load_file(str(bundle / export["file"])))
    return {"shape": shape, "linears": linears, "residual": residual}


def load_quant_bundle(path, device) -> Qwen3Weights:
    """The bundle's model as device weights for Qwen3Verifier."""
    host = read_quant_bundle(path)
    shape, lin, res = host["shape"], host["linears"], host["residual"]

    def w4(src: str) -> W4Linear:
        if src not in lin:
            raise KeyError(f"the bundle has no quantized linear {src!r}")
        qw, s, k = lin[src]
        return W4Linear(qw.to(device), s.to(device), k)

    def bf16(name: str) -> torch.Tensor:
        if name not in res:
            raise KeyError(f"the bundle has no residual tensor {name!r}")
        return res[name].to(device, torch.bfloat16).contiguous()

    layers = []
    for li in range(shape.layers):
        p = f"{PREFIX}layers.{li}."
        L = {"qkv": W4Linear.cat([w4(p + LINEARS[k] + ".weight") for k in ("q_proj", "k_proj", "v_proj")]),
             "o": w4(p + LINEARS["o_proj"] + ".weight"),
             "gate_up": W4Linear.cat([w4(p + LINEARS[k] + ".weight") for k in ("gate", "up")]),
             "down": w4(p + LINEARS["down"] + ".weight")}
        for k, v in NORMS.items():
            L[k] = bf16(p + v + ".weight")
        layers.append(L)
    return Qwen3Weights(shape, bf16(PREFIX + "embed_tokens.weight"), layers, bf16(PREFIX + "norm.weight"),
                        w4("lm_head.weight"))
