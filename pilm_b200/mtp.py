"""The MTP draft module on the GPU: Qwen3MTPDraft (src/models/qwen3/mtp.py:15-82).

One draft step, batched over B sequences, everything on the device:

    f   = [norm_e(embed[token]) | norm_h(state)]        ekernel_mtp_fc_input_bf16  (mtp.py:35-39)
    x   = fc(f)                                         bf16 or W4 per-row linear, 2H -> H
    a   = input_norm(x)                                 ekernel_add_rmsnorm_bf16 (no add)
    att = expand(v_proj(a)) [* sigmoid(gate_proj(a))]   ekernel_self_attention_bf16
    x   = x + o_proj(att); m = post_norm(x)             ekernel_add_rmsnorm_bf16
    x   = x + down(silu(gate(m)) * up(m))               fused gate/up, ekernel_silu_mul_bf16
    out = final_norm(x)                                 the next step's state (mtp.py:80)
    token = argmax(lm_head(out))                        the model's LM head, ekernel_argmax_top2

The block is TransformerBlock called without a KV cache, so attention sees the token alone
and reduces to V expanded over the GQA group (times the output gate when gated): no Q, K,
norms or RoPE are computed.  The linears use the reference's W4A16 option for the draft
module (PILM_MTP_QUANTIZE=w4a16: per-row int4, mtp.py:85-94, linear.py:291-296), each
ekernel_linear_w4a16_bf16_kpairs, or the reference's default bf16 layers (F.linear), each
ekernel_linear_bf16.  The first step reads the verify row that produced the next
token directly from the verify output (row cu_q[b] + accepted[b]), as the reference engine
passes that row's hidden state (engine.py:527-557); later steps read the previous step's
output.  Buffers are preallocated, so draft() allocates nothing and can be captured in a
CUDA graph together with the verify step.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ckernel as ck
from .qwen3 import Qwen3Shape, Qwen3Weights

NORMS = ("pre_fc_norm_embedding", "pre_fc_norm_hidden", "input_norm", "post_norm", "final_norm")


class W4RowLinear:
    """Device-resident W4A16 linear with per-row scales (scales fp32 [N]); the packed
    weights (uint8 [N, ceil(K/2)]) are held in the k-pair nibble order
    (ekernel_repack_w4_kpairs).  Rows are independent: repacked rows concatenate and
    select like reference-packed ones."""

    def __init__(self, qweight: torch.Tensor, scales: torch.Tensor, in_features: int, kpairs: bool = False):
        qweight = qweight.contiguous()
        self.qweight = qweight if kpairs else ck.repack_w4_kpairs(qweight)
        self.scales = scales.contiguous()
        self.in_features = int(in_features)
        self.out_features = int(qweight.shape[0])

    @classmethod
    def quantize(cls, w: torch.Tensor) -> "W4RowLinear":
        qw, s = ck.quantize_weight_i4_per_row(w)
        return cls(qw, s, w.shape[1])

    @classmethod
    def cat(cls, parts: list["W4RowLinear"]) -> "W4RowLinear":
        return cls(torch.cat([p.qweight for p in parts]), torch.cat([p.scales for p in parts]), parts[0].in_features,
                   kpairs=True)

    def rows(self, index: torch.Tensor) -> "W4RowLinear":
        """The linear restricted to some output rows (rows are independent)."""
        return W4RowLinear(self.qweight.index_select(0, index), self.scales.index_select(0, index), self.in_features,
                           kpairs=True)

    @property
    def nbytes(self) -> int:
        return self.qweight.numel() + self.scales.numel() * 4

    def __call__(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        return ck.linear_w4a16_bf16(x, self.qweight, self.scales, out=out, kpairs=True)


class BF16Linear:
    """Device-resident bf16 linear (weight [N, K]): the reference's default BackendLinear
    (F.linear, linear.py:170-183), through ekernel_linear_bf16."""

    def __init__(self, weight: torch.Tensor):
        self.weight = weight.to(torch.bfloat16).contiguous()
        self.in_features = int(weight.shape[1])
        self.out_features = int(weight.shape[0])

    @classmethod
    def cat(cls, parts: list["BF16Linear"]) -> "BF16Linear":
        return cls(torch.cat([p.weight for p in parts]))

    def rows(self, index: torch.Tensor) -> "BF16Linear":
        return BF16Linear(self.weight.index_select(0, index))

    @property
    def nbytes(self) -> int:
        return self.weight.numel() * 2

    def __call__(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        return ck.linear_bf16(x, self.weight, out=out)


LINEAR_MODES = {"bf16": lambda w: BF16Linear(w), "w4a16": lambda w: W4RowLinear.quantize(w)}


class MTPWeights:
    """The draft module's weights.  linears: "bf16" is the reference's default (plain bf16
    BackendLinear layers, mtp.py:21 and 137); "w4a16" is its PILM_MTP_QUANTIZE=w4a16 option
    (per-row int4, mtp.py:85-94, linear.py:291-296)."""

    def __init__(self, shape: Qwen3Shape, fc, gate_proj, v_proj, o_proj, gate_up, down,
                 norms: dict[str, torch.Tensor], linears: str = "bf16"):
        self.linears = linears
        self.shape = shape
        self.fc, self.gate_proj, self.v_proj, self.o_proj = fc, gate_proj, v_proj, o_proj
        self.gate_up, self.down = gate_up, down
        self.norms = norms

    @property
    def linear_bytes(self) -> int:
        lins = [self.fc, self.v_proj, self.o_proj, self.gate_up, self.down]
        if self.gate_proj is not None:
            lins.append(self.gate_proj)
        return sum(l.nbytes for l in lins)

    @classmethod
    def from_checkpoint(cls, shape: Qwen3Shape, ck_tensors: dict[str, torch.Tensor], device,
                        linears: str = "bf16") -> "MTPWeights":
        """A bf16 draft-module checkpoint (oracle.model.make_mtp_checkpoint naming) on the
        device, its linears kept in bf16 or quantized with the reference's per-row int4
        quantizer (linears="w4a16").  Of the (gated) q_proj only the gate half of each head
        is kept: [q_h | gate_h] per head (attention.py:81-83)."""
        make = LINEAR_MODES[linears]

        def q(name):
            return make(ck_tensors[name].to(device))

        gate_proj = None
        if shape.gated:
            hd = shape.head_dim
            idx = torch.cat([torch.arange(h * 2 * hd + hd, h * 2 * hd + 2 * hd) for h in range(shape.n_heads)])
            gate_proj = q("q_proj").rows(idx.to(device))
        norms = {n: ck_tensors[n].to(device, torch.bfloat16).contiguous() for n in NORMS}
        gu = q("gate"), q("up")
        return cls(shape, q("fc"), gate_proj, q("v_proj"), q("o_proj"), type(gu[0]).cat(list(gu)), q("down"), norms,
                   linears)

    @classmethod
    def synthetic(cls, shape: Qwen3Shape, seed: int, device, linears: str = "bf16") -> "MTPWeights":
        """Seeded random-init draft module generated on the device: N(0, 0.02) weights
        rounded to bf16, kept in bf16 or quantized per row to int4 (linears="w4a16"); norm
        weights ones (plain) or zeros (Gemma)."""
        g = torch.Generator(device=device).manual_seed(seed)
        H, I, hd = shape.hidden, shape.intermediate, shape.head_dim
        make = LINEAR_MODES[linears]

        def q(n, k):
            w = (torch.randn((n, k), generator=g, device=device) * 0.02).to(torch.bfloat16)
            return make(w)

        mk = torch.zeros if shape.gemma_norm else torch.ones
        norms = {n: mk(H, dtype=torch.bfloat16, device=device) for n in NORMS}
        gate_proj = q(shape.n_heads * hd, H) if shape.gated else None
        return cls(shape, q(H, 2 * H), gate_proj, q(shape.n_kv_heads * hd, H), q(H, shape.n_heads * hd),
                   q(2 * I, H), q(H, I), norms, linears)


class MTPDrafter:
    """k draft steps for up to max_seqs sequences, sharing the model's embedding and LM head."""

    def __init__(self, weights: MTPWeights, model: Qwen3Weights, max_seqs: int, device):
        self.w = weights
        self.model = model
        s = weights.shape
        self.max_seqs = max_seqs
        bf = dict(dtype=torch.bfloat16, device=device)
        B, H = max_seqs, s.hidden
        self.fc_in = torch.empty((B, 2 * H), **bf)
        self.x = torch.empty((B, H), **bf)
        self.a = torch.empty((B, H), **bf)
        self.v = torch.empty((B, s.n_kv_heads * s.head_dim), **bf)
        self.g = torch.empty((B, s.n_heads * s.head_dim), **bf) if s.gated else None
        self.att = torch.empty((B, s.n_heads * s.head_dim), **bf)
        self.o = torch.empty((B, H), **bf)
        self.m = torch.empty((B, H), **bf)
        self.gu = torch.empty((B, 2 * s.intermediate), **bf)
        self.act = torch.empty((B, s.intermediate), **bf)
        self.dn = torch.empty((B, H), **bf)
        self.state = [torch.empty((B, H), **bf), torch.empty((B, H), **bf)]
        self.logits = torch.empty((B, s.vocab), **bf)

    def step(self, hidden: torch.Tensor, row_base: Optional[torch.Tensor], row_offset: Optional[torch.Tensor],
             tokens: torch.Tensor, out_state: torch.Tensor, out_tokens: torch.Tensor) -> None:
        """One draft step for B = tokens.shape[0] sequences (Qwen3MTPDraft.hidden plus the
        LM-head argmax, mtp.py:68-81)."""
        s, w = self.w.shape, self.w
        B = tokens.shape[0]
        n = w.norms
        ck.mtp_fc_input_bf16(hidden, row_base, row_offset, self.model.embed, tokens, n["pre_fc_norm_embedding"],
                             n["pre_fc_norm_hidden"], s.eps, s.gemma_norm, out=self.fc_in[:B])
        x = w.fc(self.fc_in[:B], self.x[:B])
        a = ck.add_rmsnorm_bf16(x, None, n["input_norm"], s.eps, s.gemma_norm, out=self.a[:B])
        v = w.v_proj(a, self.v[:B])
        g = w.gate_proj(a, self.g[:B]) if w.gate_proj is not None else None
        att = ck.self_attention_bf16(v, g, s.n_heads, s.n_kv_heads, s.head_dim, out=self.att[:B])
        o = w.o_proj(att, self.o[:B])
        m = ck.add_rmsnorm_bf16(x, o, n["post_norm"], s.eps, s.gemma_norm, out=self.m[:B])
        gu = w.gate_up(m, self.gu[:B])
        act = ck.silu_mul_bf16(gu, s.intermediate, out=self.act[:B])
        dn = w.down(act, self.dn[:B])
        ck.add_rmsnorm_bf16(x, dn, n["final_norm"], s.eps, s.gemma_norm, out=out_state)
        logits = self.model.lm_head(out_state, out=self.logits[:B])
        ck.argmax_top2(logits, out_tokens)

    def draft(self, hidden: torch.Tensor, row_base: Optional[torch.Tensor], row_offset: Optional[torch.Tensor],
              first_tokens: torch.Tensor, k: int, out_tokens: torch.Tensor) -> torch.Tensor:
        """Qwen3MTPDraft.draft_tokens (mtp.py:56-82) for every sequence at once.

        hidden      normed hidden states; sequence b's row is row_base[b] + row_offset[b]
                    (or b when row_base is None): after a verify step, the verify output
                    with row_base = cu_q and row_offset = the accept counts
        first_tokens int32 [B]: the token each sequence continues from (the verify's next token)
        out_tokens  int32 [k, B]: draft j of sequence b lands in out_tokens[j, b]
        Returns the last step's hidden states [B, H]."""
        B = first_tokens.shape[0]
        if B > self.max_seqs:
            raise ValueError(f"{B} sequences exceed the drafter's max_seqs={self.max_seqs}")
        tok, src, rb, ro = first_tokens, hidden, row_base, row_offset
        out = None
        for j in range(k):
            out = self.state[j % 2][:B]
            self.step(src, rb, ro, tok, out, out_tokens[j])
            tok, src, rb, ro = out_tokens[j], out, None, None
        return out
