"""Qwen3 verify forward on the B200 kernels.

The batched counterpart of the reference's Qwen3Model.forward
(src/models/qwen3/model.py:95-127) for the MTP verify step: all sequences' verify
rows ([last, d1..dn] per sequence) go through one pass of every layer.  Per layer:

    h   = RMSNorm(residual)                      add_rmsnorm   (layers.py:94-119)
    qkv = W4 linear(h, [q_proj; k_proj; v_proj]) linear_w4a16g128 (linear.py:298-340)
    q,k = QK-RMSNorm + RoPE, K/V -> page slots   qk_norm_rope_kv_append (attention.py:79-97)
    a   = paged attention (+ sigmoid gate)       paged_attention_verify (attention.py:98-139)
    o   = W4 linear(a, o_proj)
    h   = RMSNorm(residual += o)                 add_rmsnorm
    gu  = W4 linear(h, [gate; up])               one fused weight [2I, H]
    m   = W4 linear(rne(rne(silu(g)) * u), down) silu_mul + linear (layers.py:192-193)
    residual += m                                (fused into the next layer's add_rmsnorm)

Weights are device-resident; q/k/v and gate/up are concatenated row-wise at load,
which leaves every output element identical to the separate reference linears
(each output row is an independent dot product).  KV pages use the reference
layout [num_blocks, 16, n_kv, head_dim] per layer (physical_kv.py:30-33).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import bindings as abi
from . import ckernel as ck


@dataclass
class Qwen3Shape:
    hidden: int
    layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    partial_rotary: float = 1.0
    gated: bool = False        # Qwen3.5 gated attention (q_proj 2x wide)
    gemma_norm: bool = False   # x * (w + 1) norms
    block_size: int = 16

    @property
    def q_rows(self) -> int:
        return self.n_heads * self.head_dim * (2 if self.gated else 1)

    @property
    def qkv_rows(self) -> int:
        return self.q_rows + 2 * self.n_kv_heads * self.head_dim

    @property
    def rot_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)


QWEN3_8B = Qwen3Shape(hidden=4096, layers=36, n_heads=32, n_kv_heads=8, head_dim=128, intermediate=12288,
                      vocab=151936)
QWEN3_1_7B = Qwen3Shape(hidden=2048, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=6144,
                        vocab=151936)
QWEN3_0_6B = Qwen3Shape(hidden=1024, layers=28, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=3072,
                        vocab=151936)


class W4Linear:
    """Device-resident W4A16 group-128 linear: the reference's scales (fp32 [N, ceil(K/128)])
    and packed weights (uint8 [N, ceil(K/2)]), the latter held in the k-pair nibble order
    (ekernel_repack_w4_kpairs) that the kernels dequantize without byte permutes.  Rows are
    independent, so repacked linears concatenate like reference-packed ones."""

    def __init__(self, qweight: torch.Tensor, scales: torch.Tensor, in_features: int, kpairs: bool = False):
        qweight = qweight.contiguous()
        self.qweight = qweight if kpairs else ck.repack_w4_kpairs(qweight)
        self.scales = scales.contiguous()
        self.in_features = int(in_features)
        self.out_features = int(qweight.shape[0])

    @classmethod
    def cat(cls, parts: list["W4Linear"]) -> "W4Linear":
        return cls(torch.cat([p.qweight for p in parts]), torch.cat([p.scales for p in parts]), parts[0].in_features,
                   kpairs=True)

    @property
    def nbytes(self) -> int:
        return self.qweight.numel() + self.scales.numel() * 4

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        m = x.shape[0]
        if out is None:
            out = torch.empty((m, self.out_features), dtype=torch.bfloat16, device=x.device)
        ck._stream()  # launch on the caller's current stream (graph capture included)
        rc = abi.linear_w4a16g128_bf16_kpairs_ptr(x.data_ptr(), self.qweight.data_ptr(), self.scales.data_ptr(),
                                                  out.data_ptr(), m, self.out_features, self.in_features)
        if rc != 0:
            raise RuntimeError(f"ekernel_linear_w4a16g128_bf16_kpairs failed: rc={rc}: {abi.last_error()}")
        return out

    def deferred(self, x: torch.Tensor, out: torch.Tensor, partials: torch.Tensor) -> int:
        """The linear, leaving its result as split-K partial sums in partials when its GEMM
        runs the split schedule and they fit (returns the split count; out is not written),
        else writing out (returns 0).  A consumer that sums the partials itself saves the
        GEMM's combine pass."""
        ck._stream()
        rc, sp = abi.linear_w4a16g128_bf16_kpairs_deferred_ptr(
            x.data_ptr(), self.qweight.data_ptr(), self.scales.data_ptr(), out.data_ptr(), x.shape[0],
            self.out_features, self.in_features, partials.data_ptr(), partials.numel() * partials.element_size())
        if rc != 0:
            raise RuntimeError(f"ekernel_linear_w4a16g128_bf16_kpairs_deferred failed: rc={rc}: {abi.last_error()}")
        return sp

    def with_argmax(self, x: torch.Tensor, out: torch.Tensor, row_keys: torch.Tensor) -> bool:
        """The linear (out written as usual) that, on its stream-K schedule, also folds each
        output row's argmax into row_keys (int64 holding uint64 keys, zero before the call);
        returns whether it did (else the caller takes the argmax from out)."""
        ck._stream()
        rc, fused = abi.linear_w4a16g128_bf16_kpairs_argmax_ptr(
            x.data_ptr(), self.qweight.data_ptr(), self.scales.data_ptr(), out.data_ptr(), x.shape[0],
            self.out_features, self.in_features, row_keys.data_ptr())
        if rc != 0:
            raise RuntimeError(f"ekernel_linear_w4a16g128_bf16_kpairs_argmax failed: rc={rc}: {abi.last_error()}")
        return bool(fused)

    def partials_bytes(self, max_rows: int) -> int:
        """Most bytes of partials a deferred call of up to max_rows rows leaves.  The split
        count is fixed within each 128-row band of M, so the band ends bound it."""
        return max(abi.linear_w4a16g128_partials_bytes(min(max_rows, 128 * t), self.out_features, self.in_features)
                   for t in range(1, (max_rows + 127) // 128 + 1))


class Qwen3Weights:
    def __init__(self, shape: Qwen3Shape, embed: torch.Tensor, layers: list[dict], final_norm: torch.Tensor,
                 lm_head: W4Linear):
        self.shape = shape
        self.embed = embed
        self.layers = layers
        self.final_norm = final_norm
        self.lm_head = lm_head

    @property
    def linear_bytes(self) -> int:
        n = self.lm_head.nbytes
        for L in self.layers:
            n += sum(L[k].nbytes for k in ("qkv", "o", "gate_up", "down"))
        return n

    @classmethod
    def from_checkpoint(cls, shape: Qwen3Shape, ck_tensors: dict[str, torch.Tensor], device) -> "Qwen3Weights":
        """Quantize a bf16 checkpoint dict (oracle.model.make_checkpoint naming) on the
        device with the reference quantizer (group 128) and fuse q/k/v and gate/up."""
        def q(name):
            w = ck_tensors[name].to(device)
            qw, s = ck.quantize_weight_i4_grouped(w, 128)
            return W4Linear(qw, s, w.shape[1])

        layers = []
        for li in range(shape.layers):
            p = f"l{li}."
            layers.append({
                "qkv": W4Linear.cat([q(p + "q_proj"), q(p + "k_proj"), q(p + "v_proj")]),
                "o": q(p + "o_proj"),
                "gate_up": W4Linear.cat([q(p + "gate"), q(p + "up")]),
                "down": q(p + "down"),
                "input_norm": ck_tensors[p + "input_norm"].to(device, torch.bfloat16).contiguous(),
                "post_norm": ck_tensors[p + "post_norm"].to(device, torch.bfloat16).contiguous(),
                "q_norm": ck_tensors[p + "q_norm"].to(device, torch.bfloat16).contiguous(),
                "k_norm": ck_tensors[p + "k_norm"].to(device, torch.bfloat16).contiguous(),
            })
        embed = ck_tensors["embed"].to(device, torch.bfloat16).contiguous()
        qw, s = ck.quantize_weight_i4_grouped(embed, 128)
        return cls(shape, embed, layers, ck_tensors["final_norm"].to(device, torch.bfloat16).contiguous(),
                   W4Linear(qw, s, shape.hidden))

    @classmethod
    def synthetic(cls, shape: Qwen3Shape, seed: int, device) -> "Qwen3Weights":
        """Seeded random-init model generated and quantized on the device: N(0, 0.02)
        weights rounded to bf16 (the checkpoint dtype), then group-128 int4; norm
        weights ones (plain) or zeros (Gemma); tied LM head."""
        g = torch.Generator(device=device).manual_seed(seed)

        def lin(n, k):
            w = (torch.randn((n, k), generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)
            qw, s = ck.quantize_weight_i4_grouped(w, 128)
            del w
            return W4Linear(qw, s, k)

        H, I = shape.hidden, shape.intermediate
        init = torch.zeros if shape.gemma_norm else torch.ones
        embed = (torch.randn((shape.vocab, H), generator=g, device=device, dtype=torch.float32) * 0.02).to(
            torch.bfloat16)
        layers = []
        for _ in range(shape.layers):
            layers.append({
                "qkv": lin(shape.qkv_rows, H),
                "o": lin(H, shape.n_heads * shape.head_dim),
                "gate_up": lin(2 * I, H),
                "down": lin(H, I),
                "input_norm": init(H, dtype=torch.bfloat16, device=device),
                "post_norm": init(H, dtype=torch.bfloat16, device=device),
                "q_norm": init(shape.head_dim, dtype=torch.bfloat16, device=device),
                "k_norm": init(shape.head_dim, dtype=torch.bfloat16, device=device),
            })
        qw, s = ck.quantize_weight_i4_grouped(embed, 128)
        return cls(shape, embed, layers, init(H, dtype=torch.bfloat16, device=device), W4Linear(qw, s, H))


def rope_tables(shape: Qwen3Shape, max_pos: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_pos, rot_dim/2] fp32, computed on the host exactly like the reference
    (_rope_inv_freq / _rope_cos_sin, layers.py:50-80) and uploaded."""
    n_freq = shape.rot_dim // 2
    inv_freq = 1.0 / (shape.rope_theta ** (torch.arange(0, n_freq, dtype=torch.float32) / n_freq))
    pos = torch.arange(max_pos, dtype=torch.long).to(torch.float32)
    freqs = pos.unsqueeze(1) * inv_freq.unsqueeze(0)
    return torch.cos(freqs).contiguous().to(device), torch.sin(freqs).contiguous().to(device)


class PagedKVCache:
    """Device-resident paged KV: per layer K and V [num_blocks, block_size, n_kv, hd] bf16."""

    def __init__(self, shape: Qwen3Shape, num_blocks: int, device, fill: Optional[str] = None, seed: int = 0,
                 dtype: torch.dtype = torch.bfloat16):
        """dtype: bf16, or fp32 for the fp32-activation (W8A32) model (zero-filled only)."""
        self.num_blocks = num_blocks
        self.block_size = shape.block_size
        self.dtype = dtype
        dims = (num_blocks, shape.block_size, shape.n_kv_heads, shape.head_dim)
        self.k = []
        self.v = []
        if dtype == torch.float32:
            for _ in range(shape.layers):
                self.k.append(torch.zeros(dims, dtype=torch.float32, device=device))
                self.v.append(torch.zeros(dims, dtype=torch.float32, device=device))
            return
        g = torch.Generator(device=device).manual_seed(seed) if fill == "random" else None
        for _ in range(shape.layers):
            if fill == "random":
                self.k.append(torch.randn(dims, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16))
                self.v.append((torch.randn(dims, generator=g, device=device, dtype=torch.float32) * 0.02).to(
                    torch.bfloat16))
            else:
                self.k.append(torch.zeros(dims, dtype=torch.bfloat16, device=device))
                self.v.append(torch.zeros(dims, dtype=torch.bfloat16, device=device))

    @property
    def bytes_per_token(self) -> int:
        return len(self.k) * 2 * self.k[0].shape[2] * self.k[0].shape[3] * self.k[0].element_size()


@dataclass
class VerifyBatch:
    """Device metadata of one verify (or prefill-chunk) pass over B sequences."""
    ids: torch.Tensor           # [T] int32 token ids of the rows
    positions: torch.Tensor     # [T] int32
    slots: torch.Tensor         # [T] int32 page * block_size + offset
    block_table: torch.Tensor   # [B, max_blocks] int32
    cu_q: torch.Tensor          # [B+1] int32 row offsets
    context_lens: torch.Tensor  # [B] int32 keys per sequence incl. these rows
    max_q_len: int
    max_context: int

    @property
    def num_seqs(self) -> int:
        return self.cu_q.shape[0] - 1

    @property
    def total_q(self) -> int:
        return self.ids.shape[0]


def attention_slices(cu_q, context_lens, group: int, max_slices: int = 1024):
    """Cut a pass's query rows into sequences the whole-page attention kernel takes (at
    most 16 rows, q_len x group, per KV head): each sequence's rows become slices of
    16 // group positions, each a sequence of its own with the same page-table row, its
    rows in place, and a context ending at the slice's last row (the kernel's causal rule
    for rows at the end of a context, which is the reference's triangular mask).
    Returns (sequence of each slice, cu_q of the slices, their contexts, positions per
    slice) as numpy arrays, or None when the slices would exceed max_slices."""
    span = 16 // group
    cu = np.asarray(cu_q, np.int64)
    ctx = np.asarray(context_lens, np.int64)
    ql = cu[1:] - cu[:-1]
    ns = (ql + span - 1) // span
    total = int(ns.sum())
    if total > max_slices:
        return None
    seq = np.repeat(np.arange(len(ql)), ns)
    k = np.arange(total) - np.repeat(np.cumsum(ns) - ns, ns)  # slice index within its sequence
    n = np.minimum(span, ql[seq] - k * span)                  # rows in the slice
    ends = ctx[seq] - ql[seq] + k * span + n                  # context through the slice's last row
    return seq, np.concatenate([[0], np.cumsum(n)]), ends, span


class Qwen3Verifier:
    """Runs the batched verify forward, the LM head and the acceptance kernels."""

    def __init__(self, weights: Qwen3Weights, kv: PagedKVCache, max_rows: int, max_pos: int, device):
        self.w = weights
        self.shape = weights.shape
        self.kv = kv
        self.device = device
        self.max_rows = max_rows
        s = self.shape
        self.cos, self.sin = rope_tables(s, max_pos, device)
        self.max_pos = max_pos
        bf = dict(dtype=torch.bfloat16, device=device)
        self.residual = torch.empty((max_rows, s.hidden), **bf)
        self.h = torch.empty((max_rows, s.hidden), **bf)
        self.qkv = torch.empty((max_rows, s.qkv_rows), **bf)
        self.q = torch.empty((max_rows, s.n_heads * s.head_dim), **bf)
        self.gate = torch.empty((max_rows, s.n_heads * s.head_dim), **bf) if s.gated else None
        self.attn = torch.empty((max_rows, s.n_heads * s.head_dim), **bf)
        self.o = torch.empty((max_rows, s.hidden), **bf)
        self.gu = torch.empty((max_rows, 2 * s.intermediate), **bf)
        self.act = torch.empty((max_rows, s.intermediate), **bf)
        self.mlp = torch.empty((max_rows, s.hidden), **bf)
        self.logits = torch.empty((max_rows, s.vocab), **bf)
        i32 = dict(dtype=torch.int32, device=device)
        self.top1 = torch.empty((max_rows,), **i32)
        self.margin = torch.empty((max_rows,), dtype=torch.float32, device=device)
        # fuse_lm_argmax: greedy verification with the row argmax folded into the LM-head
        # GEMM (its stream-K schedule) and the accept kernel decoding and re-zeroing these
        # keys, instead of a separate row top-2 pass over the logits.  Off by default: on
        # the Qwen3-8B bench step the fused form measured 0.03 ms slower (the extra work in
        # the GEMM's tile write-out delays its MMA pipeline by more than the 15 us top-2 pass
        # costs).  Other LM-head shapes take row_top2 either way.
        self.fuse_lm_argmax = False
        self.row_keys = torch.zeros((max_rows,), dtype=torch.int64, device=device)
        # Split-K partials of the q/k/v, o and down projections, summed by the kernel that
        # consumes them (QK-norm/RoPE/KV-append, residual add + RMSNorm) instead of a
        # separate combine pass; the results are bit-identical either way.  One buffer:
        # each projection's partials are consumed before the next projection runs.
        self.defer_splitk = True
        need = 0
        for L in weights.layers:
            for k in ("qkv", "o", "down"):
                if isinstance(L.get(k), W4Linear):
                    need = max(need, L[k].partials_bytes(max_rows))
            break  # every layer has the same shapes
        need = min(need, 256 << 20)  # calls whose partials exceed this write bf16 and combine
        self.part = torch.empty((need + 3) // 4, dtype=torch.float32, device=device) if need else None
        # optional CUDA-event timing of the attention and linear launches (bench.py)
        self.op_timing = False
        # passes of more than 16 query rows per KV head: run on the per-head kernel (False),
        # or cut into 16-row slices for the whole-page kernel (True).  The slices re-read
        # their sequence's pages once per slice; on B200 that is slower at 1K-8K contexts
        # (q_len 5, GQA 4: 415 vs 320 us at 1K) and a few percent faster at 32K.
        self.slice_attention = False
        self.op_events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self._launches_before = None
        self._last_step_launches = None

    def _ev(self, name: str):
        if not self.op_timing:
            return None
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        self.op_events.append((name, a, b))
        return b

    def collect_op_times(self) -> dict:
        """Average ms per launch for 'attention'; per-step sums for the linears."""
        torch.cuda.synchronize()
        tot: dict[str, float] = {}
        cnt: dict[str, int] = {}
        for name, a, b in self.op_events:
            tot[name] = tot.get(name, 0.0) + a.elapsed_time(b)
            cnt[name] = cnt.get(name, 0) + 1
        steps = max(1, cnt.get("lm_head", 1))
        out = {}
        if "attention" in tot:
            out["attention"] = tot["attention"] / cnt["attention"]
            out["attention_total"] = tot["attention"] / steps
        lin = [k for k in tot if k.startswith("linear_")]
        for k in lin:
            out[k] = tot[k] / steps
        if lin:
            out["linear_total"] = sum(tot[k] for k in lin) / steps + tot.get("lm_head", 0.0) / steps
        if "lm_head" in tot:
            out["lm_head"] = tot["lm_head"] / steps
        self.op_events.clear()
        return out

    def launches_per_step(self) -> int:
        return int(self._last_step_launches or 0)

    def _desc(self, b: VerifyBatch):
        s = self.shape
        return ck.attn_desc(num_seqs=b.num_seqs, total_q=b.total_q, max_q_len=b.max_q_len, n_heads=s.n_heads,
                            n_kv_heads=s.n_kv_heads, head_dim=s.head_dim, block_size=s.block_size,
                            num_blocks=self.kv.num_blocks, max_blocks_per_seq=b.block_table.shape[1],
                            max_context=b.max_context, qkv_stride=s.qkv_rows, rope_rows=self.max_pos,
                            rot_dim=s.rot_dim, eps=s.eps, add_one=s.gemma_norm, output_gate=s.gated)

    def _attention_view(self, b: VerifyBatch):
        """Attention metadata for passes with more than 16 query rows per KV head, cut by
        attention_slices() for the whole-page kernel.  None (the per-head kernel takes the
        pass as it is) when the pass fits the page kernel already, when slicing is off, or
        while a CUDA graph is being captured: the slices are cut from the host copy of
        cu_q, which a replay with other row counts would not update."""
        s = self.shape
        gsz = s.n_heads // s.n_kv_heads
        if (not self.slice_attention or b.max_q_len * gsz <= 16 or gsz > 16
                or torch.cuda.is_current_stream_capturing()):
            return None
        cut = attention_slices(b.cu_q.cpu().numpy(), b.context_lens.cpu().numpy(), gsz)
        if cut is None:
            return None
        seq, cu_v, ctx_v, span = cut
        i32 = dict(dtype=torch.int32, device=self.device)
        table_v = b.block_table.index_select(0, torch.tensor(seq, dtype=torch.int64, device=self.device)).contiguous()
        vb = VerifyBatch(ids=b.ids, positions=b.positions, slots=b.slots, block_table=table_v,
                         cu_q=torch.tensor(cu_v, **i32), context_lens=torch.tensor(ctx_v, **i32), max_q_len=span,
                         max_context=int(ctx_v.max()))
        return self._desc(vb), vb

    def forward(self, b: VerifyBatch) -> torch.Tensor:
        """Post-final-norm hidden states [T, H] (Qwen3Model.forward, return_last_hidden)."""
        s = self.shape
        T = b.total_q
        if T > self.max_rows:
            raise ValueError(f"{T} rows exceed max_rows={self.max_rows}")
        desc = self._desc(b)
        view = self._attention_view(b)
        adesc, ab = view if view is not None else (desc, b)
        res, h = self.residual[:T], self.h[:T]
        ck.embedding_bf16(b.ids, self.w.embed, out=res)
        part = self.part if self.defer_splitk else None

        def linear(lin, x, out) -> int:  # split count of partials left in part, else 0 (out written)
            if part is None:
                lin(x, out=out)
                return 0
            return lin.deferred(x, out, part)

        def add_norm(delta, sp, w):
            if sp:
                ck.add_rmsnorm_bf16_splitk(res, part, sp, w, s.eps, s.gemma_norm, out=h)
            else:
                ck.add_rmsnorm_bf16(res, delta, w, s.eps, s.gemma_norm, out=h)

        delta, delta_sp = None, 0
        for li, L in enumerate(self.w.layers):
            add_norm(delta, delta_sp, L["input_norm"])
            e = self._ev("linear_qkv")
            sp = linear(L["qkv"], h, self.qkv[:T])
            if e is not None:
                e.record()
            gate = self.gate[:T] if s.gated else None
            if sp:
                ck.qk_norm_rope_kv_append_splitk(desc, part, sp, L["q_norm"], L["k_norm"], self.cos, self.sin,
                                                 b.positions, b.slots, self.kv.k[li], self.kv.v[li], self.q[:T], gate)
            else:
                ck.qk_norm_rope_kv_append(desc, self.qkv[:T], L["q_norm"], L["k_norm"], self.cos, self.sin,
                                          b.positions, b.slots, self.kv.k[li], self.kv.v[li], self.q[:T], gate)
            e = self._ev("attention")
            ck.paged_attention_verify(adesc, self.q[:T], self.kv.k[li], self.kv.v[li], ab.block_table, ab.cu_q,
                                      ab.context_lens, self.gate[:T] if s.gated else None, self.attn[:T])
            if e is not None:
                e.record()
            e = self._ev("linear_o")
            sp = linear(L["o"], self.attn[:T], self.o[:T])
            if e is not None:
                e.record()
            add_norm(self.o[:T], sp, L["post_norm"])
            e = self._ev("linear_gate_up")
            L["gate_up"](h, out=self.gu[:T])
            if e is not None:
                e.record()
            ck.silu_mul_bf16(self.gu[:T], s.intermediate, out=self.act[:T])
            e = self._ev("linear_down")
            delta_sp = linear(L["down"], self.act[:T], self.mlp[:T])
            if e is not None:
                e.record()
            delta = self.mlp[:T]
        add_norm(delta, delta_sp, self.w.final_norm)
        return h

    def time_attention(self, b: VerifyBatch, reps: int = 2) -> float:
        """Average ms per paged-attention call (kernel + merge): every layer's attention over
        the batch, captured once as a graph and replayed reps times between two CUDA events,
        so the figure is device time, free of host launch overhead."""
        s = self.shape
        T = b.total_q
        desc = self._desc(b)
        gate = self.gate[:T] if s.gated else None

        def body():
            for li in range(s.layers):
                ck.paged_attention_verify(desc, self.q[:T], self.kv.k[li], self.kv.v[li], b.block_table, b.cu_q,
                                          b.context_lens, gate, self.attn[:T])
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            body()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / (reps * s.layers)

    def time_linears(self, T: int, reps: int = 5) -> dict:
        """ms per verify step spent in the W4 linears (all layers + LM head at T rows),
        replayed from a captured graph of just those launches."""
        def body():
            for L in self.w.layers:
                L["qkv"](self.h[:T], out=self.qkv[:T])
                L["o"](self.attn[:T], out=self.o[:T])
                L["gate_up"](self.h[:T], out=self.gu[:T])
                L["down"](self.act[:T], out=self.mlp[:T])
            self.w.lm_head(self.h[:T], out=self.logits[:T])
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            body()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return {"linear_total": e0.elapsed_time(e1) / reps}

    def lm_head(self, hidden: torch.Tensor) -> torch.Tensor:
        T = hidden.shape[0]
        e = self._ev("lm_head")
        out = self.w.lm_head(hidden, out=self.logits[:T])
        if e is not None:
            e.record()
        return out

    def verify_greedy(self, b: VerifyBatch, accept_counts: torch.Tensor, next_tokens: torch.Tensor,
                      context_lens: torch.Tensor, slots: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Verify forward + LM head + row argmax + greedy accept and rollback, all on the
        stream; returns the logits buffer view (bf16)."""
        n0 = abi.launch_count()
        h = self.forward(b)
        self.hidden_out = h  # normed hidden states of the rows (the MTP drafter's input)
        T = b.total_q
        fused = False
        if self.fuse_lm_argmax and isinstance(self.w.lm_head, W4Linear):
            e = self._ev("lm_head")
            fused = self.w.lm_head.with_argmax(h, self.logits[:T], self.row_keys[:T])
            if e is not None:
                e.record()
            logits = self.logits[:T]
        else:
            logits = self.lm_head(h)
        if fused:
            ck.verify_accept_greedy_keys(b.num_seqs, b.ids, self.row_keys[:T], b.cu_q, accept_counts, next_tokens,
                                         context_lens, slots, top1=self.top1[:T])
        else:
            ck.argmax_top2(logits, self.top1[:T], None, self.margin[:T])
            ck.verify_accept_greedy(b.num_seqs, b.ids, self.top1[:T], b.cu_q, accept_counts, next_tokens,
                                    context_lens, slots)
        self._last_step_launches = abi.launch_count() - n0
        return logits

    def verify_sampled(self, b: VerifyBatch, uniforms: torch.Tensor, temperature: float, top_p: float,
                       accept_counts: torch.Tensor, next_tokens: torch.Tensor, context_lens: torch.Tensor,
                       slots: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Verify forward + LM head + rejection-sampling accept and rollback (temperature,
        top-p nucleus, uniforms [total_q, 2] per row), all on the stream; returns the logits
        buffer view.  The reference verifies greedily only (engine.py:373-379)."""
        n0 = abi.launch_count()
        h = self.forward(b)
        self.hidden_out = h
        logits = self.lm_head(h)
        ck.verify_accept_rejection(b.num_seqs, logits, b.ids, b.cu_q, uniforms, temperature, top_p, accept_counts,
                                   next_tokens, context_lens, slots)
        self._last_step_launches = abi.launch_count() - n0
        return logits


class VerifyGraph:
    """The whole verify step (forward, LM head, argmax, accept + rollback) captured as
    one CUDA graph for a fixed (sequences, rows, rows-per-sequence bound).

    Inputs live in static device buffers; ``load`` copies a batch's metadata into them
    (page tables are zero-padded to the captured width) and ``replay`` runs the graph.
    The attention split count is fixed at capture from ``max_context`` (a capacity), so
    any batch whose contexts stay within it can be replayed."""

    def __init__(self, verifier: "Qwen3Verifier", num_seqs: int, total_q: int, max_q_len: int, max_pages: int,
                 max_context: int, drafter=None, draft_k: int = 0, sampling: Optional[tuple[float, float]] = None):
        """drafter (pilm_b200.mtp.MTPDrafter) and draft_k > 0 add the next step's MTP drafts
        to the graph: k draft steps from the row that produced each sequence's next token,
        written to ``drafts`` [k, num_seqs].  sampling = (temperature, top_p) verifies by
        rejection sampling with the per-row uniforms ``load`` copies in, instead of greedily."""
        dev = verifier.device
        i32 = dict(dtype=torch.int32, device=dev)
        self.v = verifier
        self.drafter = drafter if draft_k > 0 else None
        self.draft_k = draft_k if self.drafter is not None else 0
        # the step's results as rows of one tensor, read back with a single copy:
        # accept counts, next tokens, then the k drafts
        self.results = torch.zeros((2 + self.draft_k, num_seqs), **i32)
        self.acc, self.next = self.results[0], self.results[1]
        self.drafts = self.results[2:] if self.draft_k else torch.zeros((1, num_seqs), **i32)
        self.batch = VerifyBatch(ids=torch.zeros(total_q, **i32), positions=torch.zeros(total_q, **i32),
                                 slots=torch.full((total_q,), -1, **i32),
                                 block_table=torch.zeros((num_seqs, max_pages), **i32),
                                 cu_q=torch.zeros(num_seqs + 1, **i32), context_lens=torch.zeros(num_seqs, **i32),
                                 max_q_len=max_q_len, max_context=max_context)
        self.ctx_out = torch.zeros(num_seqs, **i32)
        self.sampling = sampling
        self.uniforms = torch.zeros((total_q, 2), dtype=torch.float32, device=dev) if sampling else None
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.launches = 0

    def load(self, b: VerifyBatch, uniforms: Optional[torch.Tensor] = None) -> None:
        s = self.batch
        if b.total_q != s.total_q or b.num_seqs != s.num_seqs:
            raise ValueError("batch shape differs from the captured graph")
        if self.sampling:
            if uniforms is None or tuple(uniforms.shape) != (s.total_q, 2):
                raise ValueError("a sampling graph needs uniforms [total_q, 2] per step")
            self.uniforms.copy_(uniforms, non_blocking=True)
        s.ids.copy_(b.ids, non_blocking=True)
        s.positions.copy_(b.positions, non_blocking=True)
        s.slots.copy_(b.slots, non_blocking=True)
        s.cu_q.copy_(b.cu_q, non_blocking=True)
        s.context_lens.copy_(b.context_lens, non_blocking=True)
        w = b.block_table.shape[1]
        s.block_table[:, :w].copy_(b.block_table, non_blocking=True)
        if w < s.block_table.shape[1]:
            s.block_table[:, w:].zero_()

    def _body(self) -> None:
        self.ctx_out.copy_(self.batch.context_lens)
        if self.sampling:
            self.v.verify_sampled(self.batch, self.uniforms, self.sampling[0], self.sampling[1], self.acc, self.next,
                                  self.ctx_out)
        else:
            self.v.verify_greedy(self.batch, self.acc, self.next, self.ctx_out)
        if self.drafter is not None:
            self.drafter.draft(self.v.hidden_out, self.batch.cu_q, self.acc, self.next, self.draft_k, self.drafts)

    def capture(self) -> None:
        """One eager run (sizes the library's scratch memory, which must not grow
        while capturing), then the capture."""
        side = torch.cuda.Stream(device=self.v.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self._body()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        n0 = abi.launch_count()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._body()
        self.launches = abi.launch_count() - n0
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()


def attention_bytes(shape: Qwen3Shape, context_lens: list[int], q_lens: list[int]) -> int:
    """Algorithmic HBM bytes of one layer's paged attention: every key/value of each
    sequence once, the queries and outputs, and the appended K/V rows."""
    kv = sum(context_lens) * shape.n_kv_heads * shape.head_dim * 2 * 2
    rows = sum(q_lens)
    qo = rows * shape.n_heads * shape.head_dim * 2 * 2
    app = rows * shape.n_kv_heads * shape.head_dim * 2 * 2
    return kv + qo + app


# ---------------------------------------------------------------------------------------
# fp32-activation model: the W8A32 configuration
# ---------------------------------------------------------------------------------------

class W8Linear:
    """Device-resident W8A32 linear (QuantizedW8A32Linear, linear.py:188-233): int8
    [N, K] with per-row fp32 scales, fp32 activations in and out."""

    def __init__(self, qweight: torch.Tensor, scales: torch.Tensor):
        self.qweight = qweight.contiguous()
        self.scales = scales.contiguous()
        self.in_features = int(qweight.shape[1])
        self.out_features = int(qweight.shape[0])

    @classmethod
    def quantize(cls, w: torch.Tensor) -> "W8Linear":
        qw, s = ck.quantize_weight_i8_per_row(w)
        return cls(qw, s)

    @classmethod
    def cat(cls, parts: list["W8Linear"]) -> "W8Linear":
        return cls(torch.cat([p.qweight for p in parts]), torch.cat([p.scales for p in parts]))

    @property
    def nbytes(self) -> int:
        return self.qweight.numel() + self.scales.numel() * 4

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return ck.linear_w8a32(x, self.qweight, self.scales, out=out)


class Qwen3WeightsF32(Qwen3Weights):
    """fp32 model with W8A32 linears; q/k/v and gate/up fused row-wise (rows are
    independent, per-row scales), tied LM head."""

    @classmethod
    def from_checkpoint(cls, shape: Qwen3Shape, ck_tensors: dict[str, torch.Tensor], device) -> "Qwen3WeightsF32":
        def q(name):
            return W8Linear.quantize(ck_tensors[name].to(device))

        def f(name):
            return ck_tensors[name].to(device, torch.float32).contiguous()

        layers = []
        for li in range(shape.layers):
            p = f"l{li}."
            layers.append({
                "qkv": W8Linear.cat([q(p + "q_proj"), q(p + "k_proj"), q(p + "v_proj")]),
                "o": q(p + "o_proj"),
                "gate_up": W8Linear.cat([q(p + "gate"), q(p + "up")]),
                "down": q(p + "down"),
                "input_norm": f(p + "input_norm"), "post_norm": f(p + "post_norm"),
                "q_norm": f(p + "q_norm"), "k_norm": f(p + "k_norm"),
            })
        return cls(shape, f("embed"), layers, f("final_norm"), W8Linear.quantize(ck_tensors["embed"].to(device)))

    @classmethod
    def synthetic(cls, shape: Qwen3Shape, seed: int, device) -> "Qwen3WeightsF32":
        """Seeded random-init fp32 model quantized on the device: N(0, 0.02) weights,
        int8 per-row (the W8A32 format), fp32 norms of ones (zeros for Gemma norms), fp32
        embedding and the tied LM head quantized from it."""
        g = torch.Generator(device=device).manual_seed(seed)

        def lin(n, k):
            w = torch.randn((n, k), generator=g, device=device, dtype=torch.float32) * 0.02
            return W8Linear.quantize(w)

        H, I = shape.hidden, shape.intermediate
        init = torch.zeros if shape.gemma_norm else torch.ones
        f = dict(dtype=torch.float32, device=device)
        embed = torch.randn((shape.vocab, H), generator=g, **f) * 0.02
        layers = []
        for _ in range(shape.layers):
            layers.append({
                "qkv": lin(shape.qkv_rows, H), "o": lin(H, shape.n_heads * shape.head_dim),
                "gate_up": lin(2 * I, H), "down": lin(H, I),
                "input_norm": init(H, **f), "post_norm": init(H, **f),
                "q_norm": init(shape.head_dim, **f), "k_norm": init(shape.head_dim, **f),
            })
        return cls(shape, embed, layers, init(H, **f), W8Linear.quantize(embed))


class Qwen3VerifierF32(Qwen3Verifier):
    """The verify forward with fp32 activations and KV (model dtype float32, W8A32):
    the same structure as Qwen3Verifier with the fp32 kernels; fp32 logits."""

    def __init__(self, weights: Qwen3WeightsF32, kv: PagedKVCache, max_rows: int, max_pos: int, device):
        if kv.dtype != torch.float32:
            raise ValueError("the fp32 verifier needs an fp32 KV cache")
        super().__init__(weights, kv, max_rows, max_pos, device)
        s = self.shape
        f = dict(dtype=torch.float32, device=device)
        self.residual = torch.empty((max_rows, s.hidden), **f)
        self.h = torch.empty((max_rows, s.hidden), **f)
        self.qkv = torch.empty((max_rows, s.qkv_rows), **f)
        self.q = torch.empty((max_rows, s.n_heads * s.head_dim), **f)
        self.gate = torch.empty((max_rows, s.n_heads * s.head_dim), **f) if s.gated else None
        self.attn = torch.empty((max_rows, s.n_heads * s.head_dim), **f)
        self.o = torch.empty((max_rows, s.hidden), **f)
        self.gu = torch.empty((max_rows, 2 * s.intermediate), **f)
        self.act = torch.empty((max_rows, s.intermediate), **f)
        self.mlp = torch.empty((max_rows, s.hidden), **f)
        self.logits = torch.empty((max_rows, s.vocab), **f)

    def forward(self, b: VerifyBatch) -> torch.Tensor:
        s = self.shape
        T = b.total_q
        if T > self.max_rows:
            raise ValueError(f"{T} rows exceed max_rows={self.max_rows}")
        desc = self._desc(b)
        res, h = self.residual[:T], self.h[:T]
        ck.embedding_f32(b.ids, self.w.embed, out=res)
        delta = None
        gate = self.gate[:T] if s.gated else None
        for li, L in enumerate(self.w.layers):
            ck.add_rmsnorm_f32(res, delta, L["input_norm"], s.eps, s.gemma_norm, out=h)
            L["qkv"](h, out=self.qkv[:T])
            ck.qk_norm_rope_kv_append_f32(desc, self.qkv[:T], L["q_norm"], L["k_norm"], self.cos, self.sin,
                                          b.positions, b.slots, self.kv.k[li], self.kv.v[li], self.q[:T], gate)
            ck.paged_attention_verify_f32(desc, self.q[:T], self.kv.k[li], self.kv.v[li], b.block_table, b.cu_q,
                                          b.context_lens, gate, self.attn[:T])
            L["o"](self.attn[:T], out=self.o[:T])
            ck.add_rmsnorm_f32(res, self.o[:T], L["post_norm"], s.eps, s.gemma_norm, out=h)
            L["gate_up"](h, out=self.gu[:T])
            ck.silu_mul_f32(self.gu[:T], s.intermediate, out=self.act[:T])
            L["down"](self.act[:T], out=self.mlp[:T])
            delta = self.mlp[:T]
        ck.add_rmsnorm_f32(res, delta, self.w.final_norm, s.eps, s.gemma_norm, out=h)
        return h
