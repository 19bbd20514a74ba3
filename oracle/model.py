"""TEST INFRASTRUCTURE -- the parity oracle's model layer, not the product.

A CPU restatement of piLM's Qwen3 verify forward and MTP acceptance logic:

* decoder block / model   -- src/models/qwen3/model.py:43-127
* full attention          -- src/models/qwen3/attention.py:68-141
* RMSNorm / GemmaRMSNorm  -- src/models/base/layers.py:83-119
* partial NeoX RoPE       -- src/models/base/layers.py:50-176
* SwiGLU                  -- src/models/base/layers.py:185-193
* greedy accept + cap     -- src/engine.py:391-408, 479-503, 551-570

Floating-point ops run in torch (the reference's own arithmetic for these
modules) in the same order and dtype as the reference, so the oracle is
bit-identical to the reference modules; the quantized linears run through the
pinned C restatement in ``oracle_kernels.c``.  Two architecture switches cover
both the reference's Qwen3.5-style full attention (``gated=True``,
``gemma_norm=True``: sigmoid output gate on a 2x-wide q_proj and x*(w+1) norms)
and plain Qwen3 (both False), the documented deviation used for the
BASELINE configs.

Rejection sampling has no reference implementation: ``rejection_accept`` is a
restatement of standard speculative sampling (Leviathan et al. 2023; Chen et
al. 2023) for a one-hot (greedy) draft distribution -- parity unpinned
against reference code.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import kernels as K


@dataclass
class Qwen3Config:
    hidden: int = 256
    layers: int = 2
    n_heads: int = 4
    n_kv_heads: int = 2
    head_dim: int = 128
    intermediate: int = 512
    vocab: int = 1024
    eps: float = 1e-6
    rope_theta: float = 1e6
    partial_rotary: float = 1.0
    gated: bool = False          # Qwen3.5 gated q_proj (attention.py:61,81-83,139)
    gemma_norm: bool = False     # x*(w+1) norms (layers.py:101-119)
    quant: str = "w4g128"        # w4g128 | w4g32 | w4row | w8a32 | w8a16
    dtype: str = "bfloat16"      # activation / KV dtype: bfloat16 or float32
    block_size: int = 16

    @property
    def q_rows(self) -> int:
        return self.n_heads * self.head_dim * (2 if self.gated else 1)

    @property
    def kv_rows(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def torch_dtype(self) -> torch.dtype:
        return torch.bfloat16 if self.dtype == "bfloat16" else torch.float32


LINEAR_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate", "up", "down")


def linear_shapes(cfg: Qwen3Config) -> dict[str, tuple[int, int]]:
    H, I = cfg.hidden, cfg.intermediate
    return {
        "q_proj": (cfg.q_rows, H), "k_proj": (cfg.kv_rows, H), "v_proj": (cfg.kv_rows, H),
        "o_proj": (H, cfg.n_heads * cfg.head_dim), "gate": (I, H), "up": (I, H), "down": (H, I),
    }


def make_checkpoint(cfg: Qwen3Config, seed: int) -> dict[str, torch.Tensor]:
    """Seeded synthetic checkpoint: N(0, 0.02) weights stored as bf16 (the reference
    loader quantizes from the checkpoint tensor cast to fp32, weights.py:461-645).
    Norm weights are zeros for Gemma norms (effective scale 1) and ones otherwise.
    The LM head is tied to the embedding."""
    g = torch.Generator().manual_seed(seed)
    ck: dict[str, torch.Tensor] = {}

    def rnd(shape):
        return (torch.randn(shape, generator=g, dtype=torch.float32) * 0.02).to(torch.bfloat16)

    ck["embed"] = rnd((cfg.vocab, cfg.hidden))
    shapes = linear_shapes(cfg)
    norm_init = torch.zeros if cfg.gemma_norm else torch.ones
    for li in range(cfg.layers):
        for name in LINEAR_NAMES:
            ck[f"l{li}.{name}"] = rnd(shapes[name])
        ck[f"l{li}.input_norm"] = norm_init(cfg.hidden, dtype=torch.bfloat16)
        ck[f"l{li}.post_norm"] = norm_init(cfg.hidden, dtype=torch.bfloat16)
        ck[f"l{li}.q_norm"] = norm_init(cfg.head_dim, dtype=torch.bfloat16)
        ck[f"l{li}.k_norm"] = norm_init(cfg.head_dim, dtype=torch.bfloat16)
    ck["final_norm"] = norm_init(cfg.hidden, dtype=torch.bfloat16)
    return ck


def quantize_linear(w_bf16: torch.Tensor, quant: str) -> dict[str, np.ndarray]:
    """Pack one linear the way the reference loader does (ckernel.py:70-161)."""
    w = w_bf16.to(torch.float32).numpy()
    if quant == "w4g128":
        qw, s = K.quantize_i4_grouped(w, 128)
    elif quant == "w4g32":
        qw, s = K.quantize_i4_grouped(w, 32)
    elif quant == "w4row":
        qw, s = K.quantize_i4_per_row(w)
    elif quant in ("w8a32", "w8a16"):
        qw, s = K.quantize_i8_per_row(w)
    else:
        raise ValueError(quant)
    return {"qweight": qw, "scales": s, "in_features": np.int32(w.shape[1])}


def quantize_checkpoint(cfg: Qwen3Config, ck: dict[str, torch.Tensor]) -> dict[str, dict[str, np.ndarray]]:
    q = {}
    for li in range(cfg.layers):
        for name in LINEAR_NAMES:
            q[f"l{li}.{name}"] = quantize_linear(ck[f"l{li}.{name}"], cfg.quant)
    q["lm_head"] = quantize_linear(ck["embed"], cfg.quant)
    return q


# ---------------------------------------------------------------------------------------
# torch <-> numpy bf16 plumbing
# ---------------------------------------------------------------------------------------

def _to_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def qlinear(x: torch.Tensor, lin: dict[str, np.ndarray], quant: str) -> torch.Tensor:
    """QuantizedW4A16Linear / QuantizedW8A32Linear.forward (linear.py:188-340)."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    if quant == "w8a32" and x2.dtype == torch.float32:
        out = torch.from_numpy(K.linear_w8a32(x2.numpy(), lin["qweight"], lin["scales"]))
    elif quant in ("w8a32", "w8a16"):
        out = _from_bits(K.linear_w8a16_bf16(_to_bits(x2), lin["qweight"], lin["scales"]))
    elif quant == "w4row":
        out = _from_bits(K.linear_w4a16_bf16(_to_bits(x2), lin["qweight"], lin["scales"]))
    elif quant in ("w4g128", "w4g32"):
        grp = 128 if quant == "w4g128" else 32
        out = _from_bits(K.linear_w4a16g_bf16(_to_bits(x2), lin["qweight"], lin["scales"], grp))
    else:
        raise ValueError(quant)
    return out.reshape(*shape[:-1], out.shape[-1])


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, gemma: bool) -> torch.Tensor:
    """RMSNorm.forward / GemmaRMSNorm.forward torch path (layers.py:94-98, 115-119)."""
    orig = x.dtype
    x32 = x.to(torch.float32)
    var = x32.pow(2).mean(-1, keepdim=True)
    x32 = x32 * torch.rsqrt(var + eps)
    if gemma:
        return (w + 1.0) * x32.to(orig)
    return w * x32.to(orig)


def rope_tables(cfg: Qwen3Config, max_pos: int) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin for positions [0, max_pos): _rope_inv_freq and _rope_cos_sin
    (layers.py:50-80), fp32; rows = positions, cols = rot_dim/2 frequencies."""
    rot_dim = int(cfg.head_dim * cfg.partial_rotary)
    n_freq = rot_dim // 2
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, n_freq, dtype=torch.float32) / n_freq))
    pos = torch.arange(max_pos, dtype=torch.long).to(torch.float32)
    freqs = pos.unsqueeze(1) * inv_freq.unsqueeze(0)
    return torch.cos(freqs), torch.sin(freqs)


def apply_rope(q: torch.Tensor, k: torch.Tensor, positions: torch.Tensor, cfg: Qwen3Config):
    """apply_rope (layers.py:122-176): half-split pairs (i, i+n_freq) on the first
    rot_dim dims, fp32 math, cast back."""
    rot_dim = int(cfg.head_dim * cfg.partial_rotary)
    n_freq = rot_dim // 2
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, n_freq, dtype=torch.float32) / n_freq))
    pos = positions.to(torch.float32).reshape(-1)
    freqs = pos.unsqueeze(1) * inv_freq.unsqueeze(0)
    cos, sin = torch.cos(freqs), torch.sin(freqs)
    out = []
    for t in (q, k):
        r = t[..., :rot_dim].to(torch.float32)
        a, b = r[..., :n_freq], r[..., n_freq:]
        c, s = cos.unsqueeze(1), sin.unsqueeze(1)
        rr = torch.cat([a * c - b * s, a * s + b * c], dim=-1)
        out.append(torch.cat([rr.to(t.dtype), t[..., rot_dim:]], dim=-1))
    return out[0], out[1]


def attention_from_proj(c: Qwen3Config, qp: torch.Tensor, kp: torch.Tensor, vp: torch.Tensor,
                        q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, positions: torch.Tensor,
                        kv_k: torch.Tensor, kv_v: torch.Tensor, block_ids: list[int], is_decode: bool) -> torch.Tensor:
    """FullAttention.forward after the projections (attention.py:79-139) for one
    sequence's rows, with the engine's block/slot choice (engine.py:428-434): the
    rows never cross a page.  Writes K/V into the paged caches and returns the
    (gated) attention output [seq, n_heads*hd] before o_proj."""
    seq = qp.shape[0]
    if c.gated:
        qg = qp.view(seq, c.n_heads, c.head_dim * 2)
        qs, gate = torch.chunk(qg, 2, dim=-1)
        gate = gate.reshape(seq, -1)
    else:
        qs, gate = qp.view(seq, c.n_heads, c.head_dim), None
    qs = rms_norm(qs, q_norm_w, c.eps, c.gemma_norm)
    ks = rms_norm(kp.view(seq, c.n_kv_heads, c.head_dim), k_norm_w, c.eps, c.gemma_norm)
    vs = vp.view(seq, c.n_kv_heads, c.head_dim)
    qs, ks = apply_rope(qs, ks, positions, c)

    bs = c.block_size
    start = int(positions[0])
    block_id = block_ids[start // bs]
    slot = start % bs
    kv_k[block_id, slot:slot + seq] = ks
    kv_v[block_id, slot:slot + seq] = vs
    return attend(c, qs, gate, kv_k, kv_v, block_ids, int(positions[-1]) + 1, not is_decode or seq > 1)


def attend(c: Qwen3Config, qs: torch.Tensor, gate, kv_k: torch.Tensor, kv_v: torch.Tensor, block_ids: list[int],
           cache_len: int, masked: bool) -> torch.Tensor:
    """The attention of FullAttention.forward once K/V are in the cache (attention.py:
    99-139): the sequence's pages gathered up to cache_len, GQA expansion, bf16 scores
    times the scale, the triangular mask over the last rows when masked, fp32 softmax,
    bf16 P V, times sigmoid(gate).  qs: post-RoPE queries [seq, n_heads, hd]."""
    seq = qs.shape[0]
    bs = c.block_size
    needed = (cache_len + bs - 1) // bs
    full_k = torch.cat([kv_k[b] for b in block_ids[:needed]], dim=0)[:cache_len]
    full_v = torch.cat([kv_v[b] for b in block_ids[:needed]], dim=0)[:cache_len]

    rep = c.n_heads // c.n_kv_heads
    if rep > 1:
        full_k = full_k.unsqueeze(2).expand(-1, -1, rep, -1).reshape(full_k.shape[0], c.n_heads, c.head_dim)
        full_v = full_v.unsqueeze(2).expand(-1, -1, rep, -1).reshape(full_v.shape[0], c.n_heads, c.head_dim)
    qt, kt, vt = qs.transpose(0, 1), full_k.transpose(0, 1), full_v.transpose(0, 1)
    scores = torch.bmm(qt, kt.transpose(1, 2)) * (1.0 / math.sqrt(c.head_dim))
    if masked:
        kv_len = full_k.shape[0]
        mask = torch.triu(torch.ones(seq, kv_len, dtype=torch.bool), diagonal=kv_len - seq + 1)
        scores = scores.masked_fill(mask.unsqueeze(0), float("-inf"))
    attn = torch.softmax(scores.to(torch.float32), dim=-1).to(vt.dtype)
    out = torch.bmm(attn, vt).transpose(0, 1).reshape(seq, -1)
    if gate is not None:
        out = out * torch.sigmoid(gate)
    return out


class OracleModel:
    """Qwen3Model (model.py:76-127) over a paged KV cache, one sequence per call
    (the reference runs one forward per request, engine.py:416-472)."""

    def __init__(self, cfg: Qwen3Config, ck: dict[str, torch.Tensor], q: dict | None = None):
        self.cfg = cfg
        self.ck = ck
        self.q = q if q is not None else quantize_checkpoint(cfg, ck)
        dt = cfg.torch_dtype
        self.embed = ck["embed"].to(dt)
        self.norms = {k: v.to(dt) for k, v in ck.items() if k.endswith("norm")}

    def new_kv(self, num_blocks: int) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
        """PhysicalKVCache layout (physical_kv.py:30-33): [blocks, block_size, n_kv, hd]."""
        c = self.cfg
        shape = (num_blocks, c.block_size, c.n_kv_heads, c.head_dim)
        return ([torch.zeros(shape, dtype=c.torch_dtype) for _ in range(c.layers)],
                [torch.zeros(shape, dtype=c.torch_dtype) for _ in range(c.layers)])

    def attention(self, li: int, x: torch.Tensor, positions: torch.Tensor, kv_k: torch.Tensor,
                  kv_v: torch.Tensor, block_ids: list[int], is_decode: bool) -> torch.Tensor:
        """FullAttention.forward (attention.py:68-141): projections, then
        attention_from_proj, then o_proj."""
        c = self.cfg
        qp = qlinear(x, self.q[f"l{li}.q_proj"], c.quant)
        kp = qlinear(x, self.q[f"l{li}.k_proj"], c.quant)
        vp = qlinear(x, self.q[f"l{li}.v_proj"], c.quant)
        out = attention_from_proj(c, qp, kp, vp, self.norms[f"l{li}.q_norm"], self.norms[f"l{li}.k_norm"],
                                  positions, kv_k, kv_v, block_ids, is_decode)
        return qlinear(out, self.q[f"l{li}.o_proj"], c.quant)

    def mlp(self, li: int, x: torch.Tensor) -> torch.Tensor:
        """SwiGLU.forward (layers.py:192-193): down(silu(gate(x)) * up(x))."""
        c = self.cfg
        g = qlinear(x, self.q[f"l{li}.gate"], c.quant)
        u = qlinear(x, self.q[f"l{li}.up"], c.quant)
        return qlinear(torch.nn.functional.silu(g) * u, self.q[f"l{li}.down"], c.quant)

    def forward(self, token_ids, positions, kv_k, kv_v, block_ids, is_decode=True) -> torch.Tensor:
        """Qwen3Model.forward with return_last_hidden=True (model.py:95-127):
        returns the post-final-norm hidden states [seq, H]."""
        c = self.cfg
        ids = torch.as_tensor(token_ids, dtype=torch.long)
        pos = torch.as_tensor(positions, dtype=torch.long)
        x = self.embed[ids]
        for li in range(c.layers):
            r = x
            h = rms_norm(x, self.norms[f"l{li}.input_norm"], c.eps, c.gemma_norm)
            x = r + self.attention(li, h, pos, kv_k[li], kv_v[li], block_ids, is_decode)
            r = x
            h = rms_norm(x, self.norms[f"l{li}.post_norm"], c.eps, c.gemma_norm)
            x = r + self.mlp(li, h)
        return rms_norm(x, self.norms["final_norm"], c.eps, c.gemma_norm)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """engine.py:480: lm_head(model_out).to(float32)."""
        return qlinear(hidden, self.q["lm_head"], self.cfg.quant).to(torch.float32)

    def replay_chunks(self, prompts: list[list[int]], chunks, kv_k, kv_v, block_tables: list[list[int]]) -> None:
        """Prefill several sequences following a recorded scheduler chunk list
        (rows: sequence, start position, token count), as engine.py:416-472 runs them."""
        for b, start, n in chunks:
            b, start, n = int(b), int(start), int(n)
            self.forward(prompts[b][start:start + n], list(range(start, start + n)), kv_k, kv_v,
                         block_tables[b], is_decode=False)

    def prefill(self, prompt: list[int], kv_k, kv_v, block_ids: list[int]) -> torch.Tensor:
        """Chunked prefill the way the scheduler splits it: chunks end at page
        boundaries (scheduler.py:85-86, 134-135).  Returns the last chunk's hidden."""
        bs = self.cfg.block_size
        pos = 0
        h = None
        while pos < len(prompt):
            n = min(len(prompt) - pos, bs - pos % bs)
            h = self.forward(prompt[pos:pos + n], list(range(pos, pos + n)), kv_k, kv_v, block_ids, is_decode=False)
            pos += n
        return h


# ---------------------------------------------------------------------------------------
# MTP draft module (mtp.py:15-82)
# ---------------------------------------------------------------------------------------

MTP_LINEARS = ("fc", "q_proj", "k_proj", "v_proj", "o_proj", "gate", "up", "down")
MTP_NORMS = ("pre_fc_norm_embedding", "pre_fc_norm_hidden", "input_norm", "post_norm", "q_norm", "k_norm",
             "final_norm")


def make_mtp_checkpoint(cfg: Qwen3Config, seed: int) -> dict[str, torch.Tensor]:
    """Seeded synthetic Qwen3MTPDraft weights (mtp.py:15-23): fc [H, 2H] and one transformer
    block shaped like the model's, N(0, 0.02) in bf16; norm weights as make_checkpoint.
    Drawn from a separate stream (seed + 7919) so the model's own weights are unchanged."""
    g = torch.Generator().manual_seed(seed + 7919)

    def rnd(shape):
        return (torch.randn(shape, generator=g, dtype=torch.float32) * 0.02).to(torch.bfloat16)

    shapes = linear_shapes(cfg)
    ck = {"fc": rnd((cfg.hidden, 2 * cfg.hidden))}
    for name in LINEAR_NAMES:
        ck[name] = rnd(shapes[name])
    norm_init = torch.zeros if cfg.gemma_norm else torch.ones
    for name in MTP_NORMS:
        ck[name] = norm_init(cfg.head_dim if name in ("q_norm", "k_norm") else cfg.hidden, dtype=torch.bfloat16)
    return ck


def quantize_mtp(ck: dict[str, torch.Tensor]) -> dict[str, dict[str, np.ndarray]]:
    """The reference's W4A16 option for the draft module (mtp.py:85-94, PILM_MTP_QUANTIZE=
    w4a16): every bias-free linear becomes QuantizedW4A16Linear.from_linear, per-row scales
    (linear.py:291-296)."""
    return {name: quantize_linear(ck[name], "w4row") for name in MTP_LINEARS}


class OracleMTP:
    """Qwen3MTPDraft.hidden / draft_tokens (mtp.py:25-82) with W4 per-row linears, sharing
    the model's embedding and LM head.  The block is TransformerBlock (model.py:43-73)
    called without a KV cache, so its attention sees only the token itself
    (attention.py:113-116): the softmax over one key is exactly 1, the output is that
    token's V expanded over the GQA group (attention.py:118-121, 134-136), times
    sigmoid(gate) when the q projection is gated (attention.py:139).  Q, K, their norms and
    RoPE cannot change it and are not computed."""

    def __init__(self, cfg: Qwen3Config, ck: dict[str, torch.Tensor], model: OracleModel,
                 q: dict | None = None, linears: str = "w4row"):
        """linears: "w4row" (the PILM_MTP_QUANTIZE=w4a16 option) or "bf16" (the reference's
        default: BackendLinear, i.e. F.linear on the bf16 weights, linear.py:170-183)."""
        self.cfg = cfg
        self.linears = linears
        if linears == "w4row":
            self.q = q if q is not None else quantize_mtp(ck)
        elif linears == "bf16":
            self.w = {name: ck[name].to(torch.bfloat16) for name in MTP_LINEARS}
        else:
            raise ValueError(f"unknown draft-module linears {linears!r}")
        self.norms = {k: ck[k] for k in MTP_NORMS}
        self.model = model

    def _lin(self, x: torch.Tensor, name: str) -> torch.Tensor:
        if self.linears == "bf16":
            return torch.nn.functional.linear(x, self.w[name])
        return qlinear(x, self.q[name], "w4row")

    def hidden(self, hidden: torch.Tensor, token_embedding: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        h = rms_norm(hidden.reshape(1, -1), self.norms["pre_fc_norm_hidden"], c.eps, c.gemma_norm)
        e = rms_norm(token_embedding.reshape(1, -1), self.norms["pre_fc_norm_embedding"], c.eps, c.gemma_norm)
        x = self._lin(torch.cat([e, h], dim=-1), "fc")
        r = x
        a = rms_norm(x, self.norms["input_norm"], c.eps, c.gemma_norm)
        v = self._lin(a, "v_proj")
        rep = c.n_heads // c.n_kv_heads
        out = v.view(1, c.n_kv_heads, 1, c.head_dim).expand(1, c.n_kv_heads, rep, c.head_dim)
        out = out.reshape(1, c.n_heads * c.head_dim)
        if c.gated:
            qg = self._lin(a, "q_proj").view(1, c.n_heads, 2 * c.head_dim)
            gate = qg[..., c.head_dim:].reshape(1, -1)
            out = out * torch.sigmoid(gate)
        x = r + self._lin(out, "o_proj")
        r = x
        m = rms_norm(x, self.norms["post_norm"], c.eps, c.gemma_norm)
        g = self._lin(m, "gate")
        u = self._lin(m, "up")
        x = r + self._lin(torch.nn.functional.silu(g) * u, "down")
        return rms_norm(x, self.norms["final_norm"], c.eps, c.gemma_norm)

    def draft_tokens(self, hidden: torch.Tensor, first_token_id: int, num_tokens: int):
        """k sequential drafts from the verify row's normed hidden state and the token it
        produced; returns (drafts, the last draft step's hidden)."""
        drafts = []
        token_id = int(first_token_id)
        state = hidden.reshape(1, -1)
        last = state
        for _ in range(max(0, int(num_tokens))):
            last = self.hidden(state, self.model.embed[token_id])
            token_id = int(torch.argmax(self.model.logits(last)[-1]).item())
            drafts.append(token_id)
            state = last
        return drafts, last[-1]


# ---------------------------------------------------------------------------------------
# Speculative verify bookkeeping (engine.py)
# ---------------------------------------------------------------------------------------

def draft_limit(num_computed: int, block_size: int, remaining_output: int, n_pending: int) -> int:
    """engine.py:399-401: drafts never cross the current page."""
    block_remaining = block_size - (num_computed % block_size)
    return max(0, min(remaining_output, block_remaining - 1, n_pending))


def greedy_accept(logits: torch.Tensor, drafts: list[int]) -> tuple[int, int]:
    """engine.py:483-503 and :551-557: count leading drafts equal to the row argmax
    (torch.argmax: first maximum); the next token is the argmax of the first
    mismatching row, or of the bonus row when every draft matched.
    Returns (accepted_count, next_token)."""
    acc = 0
    for i, d in enumerate(drafts):
        if int(torch.argmax(logits[i])) != int(d):
            break
        acc += 1
    return acc, int(torch.argmax(logits[acc]))


def top2_margin(logits: torch.Tensor) -> torch.Tensor:
    """Per-row gap between the two largest logits (used to excuse near-tie argmax flips)."""
    t = torch.topk(logits.to(torch.float32), 2, dim=-1).values
    return t[..., 0] - t[..., 1]


def nucleus_probs(logits: torch.Tensor, temperature: float, top_p: float) -> torch.Tensor:
    """Target distribution for rejection sampling: softmax(logits / T) restricted to
    the nucleus {j : mass of tokens with strictly larger probability < top_p}, renormalised.
    Ties at the nucleus edge are all kept (no index-order dependence)."""
    z = logits.to(torch.float64) / temperature
    p = torch.softmax(z, dim=-1)
    order = torch.argsort(p, descending=True, stable=True)
    ps = p[order]
    # mass strictly above each sorted entry, with equal values grouped together
    csum = torch.cumsum(ps, 0) - ps
    uniq, inv = torch.unique_consecutive(ps, return_inverse=True)
    first = torch.zeros(len(uniq), dtype=torch.long)
    first.scatter_reduce_(0, inv, torch.arange(len(ps)), reduce="amin", include_self=False)
    above = csum[first][inv]
    keep_sorted = above < top_p
    keep = torch.zeros_like(keep_sorted)
    keep[order] = keep_sorted
    q = torch.where(keep, p, torch.zeros_like(p))
    return q / q.sum()


def sample_from(probs: torch.Tensor, u: float) -> int:
    """Inverse-CDF sample in token-index order: smallest j with cumsum(probs)[j] > u."""
    c = torch.cumsum(probs, 0)
    j = int(torch.searchsorted(c, torch.tensor(u, dtype=c.dtype), right=True))
    nz = torch.nonzero(probs > 0).reshape(-1)
    return int(min(j, int(nz[-1]))) if len(nz) else 0


def rejection_accept(logits: torch.Tensor, drafts: list[int], u_accept: list[float], u_sample: list[float],
                     temperature: float, top_p: float) -> tuple[int, int]:
    """Speculative sampling with a greedy (one-hot) draft: accept draft i iff
    u_accept[i] < p_i(d_i); on the first rejection sample from p_i with d_i removed
    (the residual max(0, p - q) renormalised); after all accepted sample the bonus
    token from p_n.  Returns (accepted_count, next_token)."""
    for i, d in enumerate(drafts):
        p = nucleus_probs(logits[i], temperature, top_p)
        if u_accept[i] < float(p[d]):
            continue
        r = p.clone()
        r[d] = 0.0
        s = r.sum()
        r = r / s if s > 0 else p
        return i, sample_from(r, u_sample[i])
    n = len(drafts)
    return n, sample_from(nucleus_probs(logits[n], temperature, top_p), u_sample[n])
