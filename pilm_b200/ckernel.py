"""torch-facing wrappers for libpilm_cuda (CUDA tensors).

Mirrors the reference's src/runtime/ckernel.py: same function names, argument
meaning, shape checks and error behaviour (``ValueError`` for bad tensors,
``RuntimeError(f"... failed: rc={rc}")`` for a non-zero return code), but the
tensors must live on a CUDA device instead of the CPU.  There is no CPU
fallback: a CPU tensor is rejected and a missing library raises on import of
the first call.

Also holds the verify-path wrappers (paged attention, acceptance) and on-device
versions of the reference weight quantizers (ckernel.py:70-161), used to build
large synthetic checkpoints directly in HBM.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import bindings as abi


def _stream() -> None:
    abi.set_stream(torch.cuda.current_stream().cuda_stream)


def _cuda(name: str, t: torch.Tensor, dtype: torch.dtype, ndim: Optional[int] = None) -> torch.Tensor:
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.ndim != ndim:
        raise ValueError(f"{name} must be {ndim}D, got shape={tuple(t.shape)}")
    return t.contiguous()


def _out(out: Optional[torch.Tensor], shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """The output buffer: a new one, or the caller's.  A caller's buffer must be a contiguous
    tensor of the given dtype and element count on the inputs' device: the kernels write
    through its raw pointer, so a smaller or strided buffer would be overrun."""
    shape = tuple(int(d) for d in shape)
    if out is None:
        return torch.empty(shape, dtype=dtype, device=device)
    numel = 1
    for d in shape:
        numel *= d
    if out.device != device or out.dtype != dtype or out.numel() != numel or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {dtype} tensor of {numel} elements {shape} on {device}, "
                         f"got {out.dtype} {tuple(out.shape)} on {out.device}"
                         + ("" if out.is_contiguous() else " (not contiguous)"))
    return out


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: rc={rc}: {abi.last_error()}")


# ---------------------------------------------------------------------------------------
# Reference-mirroring kernels (ckernel.py:24-679)
# ---------------------------------------------------------------------------------------

def gemm_f32(a: torch.Tensor, b: torch.Tensor, transpose_b: bool = False) -> torch.Tensor:
    a = _cuda("a", a, torch.float32, 2)
    b = _cuda("b", b, torch.float32, 2)
    m, k = a.shape
    n, kb = (b.shape if transpose_b else (b.shape[1], b.shape[0]))
    if kb != k:
        raise ValueError(f"incompatible GEMM shapes: a={tuple(a.shape)} b={tuple(b.shape)} transpose_b={transpose_b}")
    out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    _stream()
    _check(abi.gemm_f32_ptr(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k, False, transpose_b), "ekernel_gemm")
    return out


def linear_w8a32(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    x = _cuda("x", x, torch.float32, 2)
    qweight = _cuda("qweight", qweight, torch.int8, 2)
    scales = _cuda("scales", scales, torch.float32, 1)
    m, k = x.shape
    n, wk = qweight.shape
    if wk != k or scales.shape[0] != n:
        raise ValueError(f"incompatible W8A32 shapes: x={tuple(x.shape)} qweight={tuple(qweight.shape)} "
                         f"scales={tuple(scales.shape)}")
    out = _out(out, (m, n), torch.float32, x.device)
    _stream()
    _check(abi.linear_w8a32_ptr(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), out.data_ptr(), m, n, k),
           "ekernel_linear_w8a32")
    return out


def linear_w8a16_bf16(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    x = _cuda("x", x, torch.bfloat16, 2)
    qweight = _cuda("qweight", qweight, torch.int8, 2)
    scales = _cuda("scales", scales, torch.float32, 1)
    m, k = x.shape
    n, wk = qweight.shape
    if wk != k or scales.shape[0] != n:
        raise ValueError(f"incompatible W8A16 shapes: x={tuple(x.shape)} qweight={tuple(qweight.shape)} "
                         f"scales={tuple(scales.shape)}")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    _stream()
    _check(abi.linear_w8a16_bf16_ptr(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), out.data_ptr(), m, n, k),
           "ekernel_linear_w8a16_bf16")
    return out


def linear_w8a16_bf16_argmax(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor) -> int:
    x = _cuda("x", x, torch.bfloat16).reshape(1, -1)
    qweight = _cuda("qweight", qweight, torch.int8, 2)
    scales = _cuda("scales", scales, torch.float32, 1)
    _stream()
    rc, idx, _val = abi.linear_w8a16_bf16_argmax_ptr(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), 1,
                                                     qweight.shape[0], x.shape[1])
    _check(rc, "ekernel_linear_w8a16_bf16_argmax")
    return idx


def _w4_common(x, qweight, scales, in_features, scale_ndim, groups_of):
    x = _cuda("x", x, torch.bfloat16, 2)
    qweight = _cuda("qweight", qweight, torch.uint8, 2)
    scales = _cuda("scales", scales, torch.float32, scale_ndim)
    m, k = x.shape
    n, packed_k = qweight.shape
    if in_features is not None and int(in_features) != k:
        raise ValueError(f"in_features={in_features} does not match x K={k}")
    want = (n,) if groups_of is None else (n, (k + groups_of - 1) // groups_of)
    if packed_k != (k + 1) // 2 or tuple(scales.shape) != want:
        raise ValueError(f"incompatible W4A16 shapes: x={tuple(x.shape)} qweight={tuple(qweight.shape)} "
                         f"scales={tuple(scales.shape)}")
    return x, qweight, scales, m, n, k


def linear_w4a16_bf16(x, qweight, scales, in_features=None, out: Optional[torch.Tensor] = None,
                      kpairs: bool = False) -> torch.Tensor:
    """kpairs: qweight is in the k-pair nibble order (repack_w4_kpairs)."""
    x, qweight, scales, m, n, k = _w4_common(x, qweight, scales, in_features, 1, None)
    out = _out(out, (m, n), torch.bfloat16, x.device)
    _stream()
    fn = abi.linear_w4a16_bf16_kpairs_ptr if kpairs else abi.linear_w4a16_bf16_ptr
    _check(fn(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), out.data_ptr(), m, n, k),
           "ekernel_linear_w4a16_bf16" + ("_kpairs" if kpairs else ""))
    return out


def linear_bf16(x: torch.Tensor, weight: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """F.linear(x, weight) on bf16 tensors (BackendLinear, linear.py:170-183) through
    ekernel_linear_bf16: fp32 accumulation, one rounding to bf16."""
    x = _cuda("x", x, torch.bfloat16, 2)
    weight = _cuda("weight", weight, torch.bfloat16, 2)
    m, k = x.shape
    n, wk = weight.shape
    if wk != k:
        raise ValueError(f"incompatible bf16 linear shapes: x={tuple(x.shape)} weight={tuple(weight.shape)}")
    out = _out(out, (m, n), torch.bfloat16, x.device)
    _stream()
    _check(abi.linear_bf16_ptr(x.data_ptr(), weight.data_ptr(), out.data_ptr(), m, n, k), "ekernel_linear_bf16")
    return out


def repack_w4_kpairs(qweight: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Reference-packed int4 weights [N, K/2] -> the k-pair nibble order the kernels
    dequantize without byte permutes (ekernel_repack_w4_kpairs); out may be qweight."""
    qweight = _cuda("qweight", qweight, torch.uint8, 2)
    n, kb = qweight.shape
    out = _out(out, qweight.shape, qweight.dtype, qweight.device)
    _stream()
    _check(abi.repack_w4_kpairs_ptr(qweight.data_ptr(), n, 2 * kb, out.data_ptr()), "ekernel_repack_w4_kpairs")
    return out


def linear_w4a16g32_bf16(x, qweight, scales, in_features=None) -> torch.Tensor:
    x, qweight, scales, m, n, k = _w4_common(x, qweight, scales, in_features, 2, 32)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    _stream()
    _check(abi.linear_w4a16g32_bf16_ptr(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), out.data_ptr(), m, n,
                                        k), "ekernel_linear_w4a16g32_bf16")
    return out


def linear_w4a16g128_bf16(x, qweight, scales, in_features=None, out: Optional[torch.Tensor] = None,
                          kpairs: bool = False) -> torch.Tensor:
    """kpairs: qweight is in the k-pair nibble order (repack_w4_kpairs)."""
    x, qweight, scales, m, n, k = _w4_common(x, qweight, scales, in_features, 2, 128)
    out = _out(out, (m, n), torch.bfloat16, x.device)
    _stream()
    fn = abi.linear_w4a16g128_bf16_kpairs_ptr if kpairs else abi.linear_w4a16g128_bf16_ptr
    _check(fn(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(), out.data_ptr(), m, n, k),
           "ekernel_linear_w4a16g128_bf16" + ("_kpairs" if kpairs else ""))
    return out


def swiglu_bf16(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    gate = _cuda("gate", gate, torch.bfloat16)
    up = _cuda("up", up, torch.bfloat16)
    if tuple(gate.shape) != tuple(up.shape):
        raise ValueError(f"gate/up shapes differ: gate={tuple(gate.shape)} up={tuple(up.shape)}")
    out = torch.empty_like(gate)
    _stream()
    _check(abi.swiglu_bf16_ptr(gate.data_ptr(), up.data_ptr(), out.data_ptr(), gate.numel()), "ekernel_swiglu_bf16")
    return out


def swiglu_w4a16_bf16(x, gate_up_qweight, gate_up_scales, down_qweight, down_scales, intermediate_size,
                      gate_up_in_features=None, down_in_features=None) -> torch.Tensor:
    """Fused W4 SwiGLU MLP (ckernel.py:585-647); any M here (the reference: M=1)."""
    x = _cuda("x", x, torch.bfloat16, 2)
    gate_up_qweight = _cuda("gate_up_qweight", gate_up_qweight, torch.uint8, 2)
    down_qweight = _cuda("down_qweight", down_qweight, torch.uint8, 2)
    gate_up_scales = _cuda("gate_up_scales", gate_up_scales, torch.float32, 1)
    down_scales = _cuda("down_scales", down_scales, torch.float32, 1)
    m, k = x.shape
    inter = int(intermediate_size)
    gk = k if gate_up_in_features is None else int(gate_up_in_features)
    dk = inter if down_in_features is None else int(down_in_features)
    hidden = int(down_qweight.shape[0])
    if gk != k:
        raise ValueError(f"gate_up_in_features={gk} does not match x K={k}")
    if dk != inter:
        raise ValueError("down_in_features must equal intermediate_size")
    if tuple(gate_up_qweight.shape) != (2 * inter, (gk + 1) // 2):
        raise ValueError(f"gate_up_qweight shape must be {(2 * inter, (gk + 1) // 2)}, "
                         f"got {tuple(gate_up_qweight.shape)}")
    if down_qweight.shape[1] != (dk + 1) // 2:
        raise ValueError(f"down_qweight packed K does not match down_in_features={dk}")
    if gate_up_scales.shape[0] != 2 * inter or down_scales.shape[0] != hidden:
        raise ValueError("scale shapes do not match qweight rows")
    out = torch.empty((m, hidden), dtype=torch.bfloat16, device=x.device)
    _stream()
    _check(abi.swiglu_w4a16_bf16_ptr(x.data_ptr(), gate_up_qweight.data_ptr(), gate_up_scales.data_ptr(),
                                     down_qweight.data_ptr(), down_scales.data_ptr(), out.data_ptr(), m, hidden, inter,
                                     gk, dk), "ekernel_swiglu_w4a16_bf16")
    return out


def rmsnorm_bf16(x: torch.Tensor, weight: torch.Tensor, eps: float, add_one: bool = False) -> torch.Tensor:
    if x.device.type != "cuda" or x.dtype != torch.bfloat16:
        raise ValueError("x must be a CUDA torch.bfloat16 tensor")
    weight = _cuda("weight", weight, torch.bfloat16, 1)
    if x.shape[-1] != weight.shape[0]:
        raise ValueError(f"incompatible RMSNorm shapes: x={tuple(x.shape)} weight={tuple(weight.shape)}")
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    out = torch.empty_like(x2)
    _stream()
    _check(abi.rmsnorm_bf16_ptr(x2.data_ptr(), out.data_ptr(), weight.data_ptr(), x2.shape[0], x2.shape[1],
                                float(eps), bool(add_one)), "ekernel_rmsnorm_bf16")
    return out.reshape(x.shape)


# ---------------------------------------------------------------------------------------
# Verify-path kernels
# ---------------------------------------------------------------------------------------

def embedding_bf16(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    ids = _cuda("ids", ids, torch.int32, 1)
    table = _cuda("table", table, torch.bfloat16, 2)
    out = _out(out, (ids.shape[0], table.shape[1]), torch.bfloat16, ids.device)
    _stream()
    _check(abi.lib().ekernel_embedding_bf16(ids.data_ptr(), ids.shape[0], table.data_ptr(), table.shape[0],
                                            table.shape[1], out.data_ptr()), "ekernel_embedding_bf16")
    return out


def add_rmsnorm_bf16(residual: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor, eps: float,
                     add_one: bool, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """residual <- rne(residual + delta) (in place); returns the module-rounded RMSNorm."""
    if residual.device.type != "cuda" or residual.dtype != torch.bfloat16 or not residual.is_contiguous():
        raise ValueError("residual must be a contiguous CUDA bfloat16 tensor")
    rows, n = residual.shape
    out = _out(out, residual.shape, residual.dtype, residual.device)
    _stream()
    _check(abi.lib().ekernel_add_rmsnorm_bf16(residual.data_ptr(), delta.data_ptr() if delta is not None else None,
                                              weight.data_ptr(), rows, n, float(eps), int(add_one), out.data_ptr()),
           "ekernel_add_rmsnorm_bf16")
    return out


def add_rmsnorm_bf16_splitk(residual: torch.Tensor, partials: torch.Tensor, splits: int, weight: torch.Tensor,
                            eps: float, add_one: bool, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """add_rmsnorm_bf16 with the delta given as a deferred W4 linear's split-K partial sums
    (partials holds at least [splits, rows, n] fp32): bit-identical to passing the linear's
    bf16 output."""
    if residual.device.type != "cuda" or residual.dtype != torch.bfloat16 or not residual.is_contiguous():
        raise ValueError("residual must be a contiguous CUDA bfloat16 tensor")
    rows, n = residual.shape
    if partials.dtype != torch.float32 or partials.numel() < splits * rows * n:
        raise ValueError("partials must be fp32 with at least splits * rows * n elements")
    out = _out(out, residual.shape, residual.dtype, residual.device)
    _stream()
    _check(abi.lib().ekernel_add_rmsnorm_bf16_splitk(residual.data_ptr(), partials.data_ptr(), int(splits),
                                                     weight.data_ptr(), rows, n, float(eps), int(add_one),
                                                     out.data_ptr()),
           "ekernel_add_rmsnorm_bf16_splitk")
    return out


def mtp_fc_input_bf16(hidden: torch.Tensor, row_base: Optional[torch.Tensor], row_offset: Optional[torch.Tensor],
                      embed: torch.Tensor, tokens: torch.Tensor, w_embed_norm: torch.Tensor,
                      w_hidden_norm: torch.Tensor, eps: float, add_one: bool,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[norm(embed[tokens]) | norm(hidden[row_base + row_offset])] per sequence: the fc
    input of one MTP draft step (mtp.py:35-39)."""
    hidden = _cuda("hidden", hidden, torch.bfloat16, 2)
    embed = _cuda("embed", embed, torch.bfloat16, 2)
    tokens = _cuda("tokens", tokens, torch.int32, 1)
    B, H = tokens.shape[0], hidden.shape[1]
    out = _out(out, (B, 2 * H), torch.bfloat16, hidden.device)
    _stream()
    _check(abi.lib().ekernel_mtp_fc_input_bf16(hidden.data_ptr(), _p(row_base), _p(row_offset), embed.data_ptr(),
                                               tokens.data_ptr(), embed.shape[0], w_embed_norm.data_ptr(),
                                               w_hidden_norm.data_ptr(), B, H, float(eps), int(add_one),
                                               out.data_ptr()), "ekernel_mtp_fc_input_bf16")
    return out


def self_attention_bf16(v: torch.Tensor, gate: Optional[torch.Tensor], n_heads: int, n_kv_heads: int,
                        head_dim: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of each row over itself alone: V expanded over the GQA group (times
    sigmoid(gate) when gated)."""
    v = _cuda("v", v, torch.bfloat16, 2)
    rows = v.shape[0]
    out = _out(out, (rows, n_heads * head_dim), torch.bfloat16, v.device)
    _stream()
    _check(abi.lib().ekernel_self_attention_bf16(v.data_ptr(), _p(gate), rows, n_heads, n_kv_heads, head_dim,
                                                 out.data_ptr()), "ekernel_self_attention_bf16")
    return out


def silu_mul_bf16(gate_up: torch.Tensor, inter: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    gate_up = _cuda("gate_up", gate_up, torch.bfloat16, 2)
    rows = gate_up.shape[0]
    out = _out(out, (rows, inter), torch.bfloat16, gate_up.device)
    _stream()
    _check(abi.lib().ekernel_silu_mul_bf16(gate_up.data_ptr(), rows, inter, out.data_ptr()), "ekernel_silu_mul_bf16")
    return out


def attn_desc(*, num_seqs, total_q, max_q_len, n_heads, n_kv_heads, head_dim, block_size, num_blocks,
              max_blocks_per_seq, max_context, qkv_stride, rope_rows, rot_dim, eps, add_one, output_gate):
    return abi.PagedAttnDesc(num_seqs, total_q, max_q_len, n_heads, n_kv_heads, head_dim, block_size, num_blocks,
                             max_blocks_per_seq, max_context, qkv_stride, rope_rows, rot_dim, float(eps),
                             int(add_one), int(output_gate))


def _p(t: Optional[torch.Tensor]):
    return t.data_ptr() if t is not None else None


def qk_norm_rope_kv_append(desc, qkv, q_norm_w, k_norm_w, rope_cos, rope_sin, positions, slot_mapping, k_cache,
                           v_cache, q_out, gate_out=None) -> None:
    _stream()
    import ctypes
    _check(abi.lib().ekernel_qk_norm_rope_kv_append(ctypes.byref(desc), _p(qkv), _p(q_norm_w), _p(k_norm_w),
                                                    _p(rope_cos), _p(rope_sin), _p(positions), _p(slot_mapping),
                                                    _p(k_cache), _p(v_cache), _p(q_out), _p(gate_out)),
           "ekernel_qk_norm_rope_kv_append")


def qk_norm_rope_kv_append_splitk(desc, partials, splits, q_norm_w, k_norm_w, rope_cos, rope_sin, positions,
                                  slot_mapping, k_cache, v_cache, q_out, gate_out=None) -> None:
    """qk_norm_rope_kv_append with the fused projection given as a deferred W4 linear's
    split-K partial sums ([splits, total_q, qkv_stride] fp32): bit-identical results."""
    if partials.dtype != torch.float32 or partials.numel() < splits * desc.total_q * desc.qkv_stride:
        raise ValueError("partials must be fp32 with at least splits * total_q * qkv_stride elements")
    _stream()
    import ctypes
    _check(abi.lib().ekernel_qk_norm_rope_kv_append_splitk(ctypes.byref(desc), _p(partials), int(splits),
                                                           _p(q_norm_w), _p(k_norm_w), _p(rope_cos), _p(rope_sin),
                                                           _p(positions), _p(slot_mapping), _p(k_cache), _p(v_cache),
                                                           _p(q_out), _p(gate_out)),
           "ekernel_qk_norm_rope_kv_append_splitk")


def paged_attention_verify(desc, q, k_cache, v_cache, block_table, cu_q, context_lens, gate, out) -> None:
    _stream()
    import ctypes
    _check(abi.lib().ekernel_paged_attention_verify(ctypes.byref(desc), _p(q), _p(k_cache), _p(v_cache),
                                                    _p(block_table), _p(cu_q), _p(context_lens), _p(gate), _p(out)),
           "ekernel_paged_attention_verify")


# ---- fp32-activation path (the W8A32 configuration) --------------------------------------

def embedding_f32(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    ids = _cuda("ids", ids, torch.int32, 1)
    table = _cuda("table", table, torch.float32, 2)
    out = _out(out, (ids.shape[0], table.shape[1]), torch.float32, ids.device)
    _stream()
    _check(abi.lib().ekernel_embedding_f32(ids.data_ptr(), ids.shape[0], table.data_ptr(), table.shape[0],
                                           table.shape[1], out.data_ptr()), "ekernel_embedding_f32")
    return out


def add_rmsnorm_f32(residual: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor, eps: float,
                    add_one: bool, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if residual.device.type != "cuda" or residual.dtype != torch.float32 or not residual.is_contiguous():
        raise ValueError("residual must be a contiguous CUDA float32 tensor")
    rows, n = residual.shape
    out = _out(out, residual.shape, residual.dtype, residual.device)
    _stream()
    _check(abi.lib().ekernel_add_rmsnorm_f32(residual.data_ptr(), _p(delta), weight.data_ptr(), rows, n, float(eps),
                                             int(add_one), out.data_ptr()), "ekernel_add_rmsnorm_f32")
    return out


def qk_norm_rope_kv_append_f32(desc, qkv, q_norm_w, k_norm_w, rope_cos, rope_sin, positions, slot_mapping, k_cache,
                               v_cache, q_out, gate_out=None) -> None:
    import ctypes
    _stream()
    _check(abi.lib().ekernel_qk_norm_rope_kv_append_f32(ctypes.byref(desc), _p(qkv), _p(q_norm_w), _p(k_norm_w),
                                                        _p(rope_cos), _p(rope_sin), _p(positions), _p(slot_mapping),
                                                        _p(k_cache), _p(v_cache), _p(q_out), _p(gate_out)),
           "ekernel_qk_norm_rope_kv_append_f32")


def paged_attention_verify_f32(desc, q, k_cache, v_cache, block_table, cu_q, context_lens, gate, out) -> None:
    import ctypes
    _stream()
    _check(abi.lib().ekernel_paged_attention_verify_f32(ctypes.byref(desc), _p(q), _p(k_cache), _p(v_cache),
                                                        _p(block_table), _p(cu_q), _p(context_lens), _p(gate),
                                                        _p(out)), "ekernel_paged_attention_verify_f32")


def silu_mul_f32(gate_up: torch.Tensor, inter: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    gate_up = _cuda("gate_up", gate_up, torch.float32, 2)
    rows = gate_up.shape[0]
    out = _out(out, (rows, inter), torch.float32, gate_up.device)
    _stream()
    _check(abi.lib().ekernel_silu_mul_f32(gate_up.data_ptr(), rows, inter, out.data_ptr()), "ekernel_silu_mul_f32")
    return out


def argmax_top2(logits: torch.Tensor, top1: torch.Tensor, top1_val=None, margin=None) -> None:
    import ctypes
    rows, vocab = logits.shape
    d = abi.AcceptDesc(0, rows, vocab)
    _stream()
    if logits.dtype == torch.float32:
        rc = abi.lib().ekernel_argmax_top2_f32(ctypes.byref(d), logits.data_ptr(), _p(top1), _p(top1_val), _p(margin))
    elif logits.dtype == torch.bfloat16:
        rc = abi.lib().ekernel_argmax_top2_bf16(ctypes.byref(d), logits.data_ptr(), _p(top1), _p(top1_val), _p(margin))
    else:
        raise ValueError("logits must be float32 or bfloat16")
    _check(rc, "ekernel_argmax_top2")


def verify_accept_greedy(num_seqs, verify_ids, top1, cu_q, accept_counts, next_tokens, context_lens,
                         slot_mapping=None) -> None:
    import ctypes
    d = abi.AcceptDesc(num_seqs, verify_ids.shape[0], 0)
    _stream()
    _check(abi.lib().ekernel_verify_accept_greedy(ctypes.byref(d), _p(verify_ids), _p(top1), _p(cu_q),
                                                  _p(accept_counts), _p(next_tokens), _p(context_lens),
                                                  _p(slot_mapping)), "ekernel_verify_accept_greedy")


def verify_accept_greedy_keys(num_seqs, verify_ids, row_keys, cu_q, accept_counts, next_tokens, context_lens,
                              slot_mapping=None, top1=None) -> None:
    """Greedy acceptance from the row argmax keys of a fused LM head
    (linear_w4a16g128_bf16_kpairs_argmax); the keys are reset to 0, top1 (optional) gets
    the decoded row argmaxes."""
    import ctypes
    if row_keys.dtype != torch.int64 or row_keys.numel() < verify_ids.shape[0]:
        raise ValueError("row_keys must be int64 (uint64 bits) with one entry per verify row")
    d = abi.AcceptDesc(num_seqs, verify_ids.shape[0], 0)
    _stream()
    _check(abi.lib().ekernel_verify_accept_greedy_keys(ctypes.byref(d), _p(verify_ids), _p(row_keys), _p(cu_q),
                                                       _p(accept_counts), _p(next_tokens), _p(context_lens),
                                                       _p(slot_mapping), _p(top1)), "ekernel_verify_accept_greedy_keys")


def verify_accept_rejection(num_seqs, logits, verify_ids, cu_q, uniforms, temperature, top_p, accept_counts,
                            next_tokens, context_lens, slot_mapping=None) -> None:
    """Rejection-sampling acceptance over fp32 or bf16 logits [total_q, vocab] with
    uniforms [total_q, 2] fp32 (accept test, sample) per row."""
    import ctypes
    if logits.dtype == torch.bfloat16:
        logits = _cuda("logits", logits, torch.bfloat16, 2)
        fn, name = abi.lib().ekernel_verify_accept_rejection_bf16, "ekernel_verify_accept_rejection_bf16"
    else:
        logits = _cuda("logits", logits, torch.float32, 2)
        fn, name = abi.lib().ekernel_verify_accept_rejection, "ekernel_verify_accept_rejection"
    uniforms = _cuda("uniforms", uniforms, torch.float32, 2)
    if uniforms.shape != (logits.shape[0], 2):
        raise ValueError(f"uniforms must be [{logits.shape[0]}, 2], got {tuple(uniforms.shape)}")
    d = abi.AcceptDesc(num_seqs, logits.shape[0], logits.shape[1])
    _stream()
    _check(fn(ctypes.byref(d), logits.data_ptr(), _p(verify_ids), _p(cu_q), _p(uniforms), float(temperature),
              float(top_p), _p(accept_counts), _p(next_tokens), _p(context_lens), _p(slot_mapping)), name)


# ---------------------------------------------------------------------------------------
# On-device quantizers (same formats as ckernel.py:70-161)
#
# torch on CUDA turns `tensor / python_scalar` into a multiply by the reciprocal,
# which rounds differently from the reference's CPU division; the divisors below are
# device tensors so every quotient is a correctly rounded division, bit-identical to
# the reference quantizer.
# ---------------------------------------------------------------------------------------

def _c(v: float, like: torch.Tensor) -> torch.Tensor:
    return torch.full((), v, dtype=torch.float32, device=like.device)

def _pack_i4(q: torch.Tensor) -> torch.Tensor:
    if q.shape[1] % 2:
        q = torch.nn.functional.pad(q, (0, 1))
    lo = torch.bitwise_and(q[:, 0::2], 0x0F).to(torch.uint8)
    hi = torch.bitwise_left_shift(torch.bitwise_and(q[:, 1::2], 0x0F), 4).to(torch.uint8)
    return torch.bitwise_or(lo, hi).contiguous()


def quantize_weight_i4_grouped(w: torch.Tensor, group_size: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_weight_i4_grouped_chunked (ckernel.py:124-161) on any device."""
    w = w.to(torch.float32)
    rows, cols = w.shape
    groups = (cols + group_size - 1) // group_size
    wp = torch.nn.functional.pad(w, (0, groups * group_size - cols)) if cols % group_size else w
    g = wp.reshape(rows, groups, group_size)
    s = torch.clamp(g.abs().amax(dim=2) / _c(7.0, g), min=1e-8)
    q = torch.round(g / s.unsqueeze(2)).clamp(-7, 7).to(torch.int16).reshape(rows, groups * group_size)[:, :cols]
    return _pack_i4(q), s.contiguous()


def quantize_weight_i4_per_row(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_weight_i4_per_row_chunked (ckernel.py:98-121) on any device."""
    w = w.to(torch.float32)
    s = torch.clamp(w.abs().amax(dim=1) / _c(7.0, w), min=1e-8)
    q = torch.round(w / s.unsqueeze(1)).clamp(-7, 7).to(torch.int16)
    return _pack_i4(q), s.contiguous()


def quantize_weight_i8_per_row(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """quantize_weight_i8_per_row (ckernel.py:70-75) on any device."""
    w = w.to(torch.float32)
    s = torch.clamp(w.abs().amax(dim=1) / _c(127.0, w), min=1e-8)
    return torch.round(w / s.unsqueeze(1)).clamp(-127, 127).to(torch.int8).contiguous(), s.contiguous()
