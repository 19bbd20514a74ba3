"""Generate the golden fixtures in tests/golden/ from the UNMODIFIED piLM reference.

Run where the reference sources exist (not on the GPU box):

    make -C oracle ref            # reference C library -> oracle/_ref/libecpu.so
    python tests/golden/make_golden.py

What runs is the reference's own code: its ctypes bindings + C kernels for the
quantized linears (runtime/ckernel.py -> src/ecpu), its quantizers, its torch
Qwen3Model / FullAttention / RMSNorm modules, and its Scheduler /
KVCacheManager / BlockPool for page tables.  The harness only drives them the
way src/engine.py:391-570 does and records inputs and outputs.

Plain Qwen3 (no output gate, x*w norms) is obtained WITHOUT editing reference
code: the gate half of the reference's 2x-wide q_proj output is filled with
+inf so that sigmoid(gate) == 1.0 exactly, and GemmaRMSNorm modules are
swapped for the reference's own RMSNorm class.

Outputs (small, committed):
  kernels.npz      per-kernel inputs/outputs of the reference C library, including
                   the reference quantizers' packed weights and scales
  model_<v>.npz    verify-step traces for model variants v (see VARIANTS)
  paging.npz       block-pool allocation trace of the reference scheduler
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
# the reference's src/ tree: PILM_REF_SRC, else a reference checkout beside this repository
REF_SRC = Path(os.environ.get("PILM_REF_SRC") or Path(__file__).resolve().parents[3] / "reference" / "src")
OUT = Path(__file__).resolve().parent

os.environ["PILM_ECPU_LIB"] = str(REPO / "oracle" / "_ref" / "libecpu.so")
sys.path.insert(0, str(REPO))
sys.path.insert(1, str(REF_SRC))

import torch.nn as nn  # noqa: E402

from runtime import ckernel as ref_ck  # noqa: E402  (reference)
from runtime.loader.config_parser import ModelConfig, RopeConfig, TextConfig  # noqa: E402
from runtime.scheduler import KVCacheManager, Request, Scheduler  # noqa: E402
from runtime.kvcache import PhysicalKVCache  # noqa: E402
from models.qwen3.model import Qwen3Model  # noqa: E402
from models.base.layers import RMSNorm  # noqa: E402
from models.base.linear import BackendLinear, QuantizedW4A16Linear, QuantizedW8A32Linear  # noqa: E402
from models.qwen3.mtp import Qwen3MTPDraft, _quantize_mtp_linears  # noqa: E402

from oracle import model as om  # noqa: E402  (only for the seeded checkpoint recipe)

torch.set_num_threads(4)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


# ------------------------------------------------------------------------------------------
# 1. kernels: reference C library through the reference torch wrappers
# ------------------------------------------------------------------------------------------

def kernel_goldens() -> dict[str, np.ndarray]:
    g = torch.Generator().manual_seed(1234)
    out: dict[str, np.ndarray] = {}
    shapes = [(1, 64, 256), (3, 96, 384), (4, 40, 512), (8, 128, 256), (2, 33, 130), (5, 17, 200)]
    for i, (M, N, K) in enumerate(shapes):
        x = torch.randn((M, K), generator=g).to(torch.bfloat16)
        xf = torch.randn((M, K), generator=g)
        w = (torch.randn((N, K), generator=g) * 0.02).to(torch.bfloat16).to(torch.float32)
        out[f"s{i}.shape"] = np.array([M, N, K], np.int64)
        out[f"s{i}.x"] = bits(x)
        out[f"s{i}.xf"] = xf.numpy().copy()
        out[f"s{i}.w"] = w.numpy().copy()
        for grp in (32, 128):
            qw, s = ref_ck.quantize_weight_i4_grouped_chunked(w, group_size=grp)
            fn = ref_ck.linear_w4a16g128_bf16 if grp == 128 else ref_ck.linear_w4a16g32_bf16
            out[f"s{i}.w4g{grp}.qw"] = qw.numpy().copy()
            out[f"s{i}.w4g{grp}.s"] = s.numpy().copy()
            out[f"s{i}.w4g{grp}.y"] = bits(fn(x, qw, s, K))
        qw, s = ref_ck.quantize_weight_i4_per_row_chunked(w)
        out[f"s{i}.w4row.qw"] = qw.numpy().copy()
        out[f"s{i}.w4row.s"] = s.numpy().copy()
        out[f"s{i}.w4row.y"] = bits(ref_ck.linear_w4a16_bf16(x, qw, s, K))
        q8, s8 = ref_ck.quantize_weight_i8_per_row(w)
        out[f"s{i}.w8.qw"] = q8.numpy().copy()
        out[f"s{i}.w8.s"] = s8.numpy().copy()
        out[f"s{i}.w8a16.y"] = bits(ref_ck.linear_w8a16_bf16(x, q8, s8))
        out[f"s{i}.w8a32.y"] = ref_ck.linear_w8a32(xf, q8, s8).numpy().copy()
        nw = (torch.randn((K,), generator=g) * 0.1).to(torch.bfloat16)
        out[f"s{i}.norm.w"] = bits(nw)
        for add_one in (0, 1):
            out[f"s{i}.norm{add_one}.y"] = bits(ref_ck.rmsnorm_bf16(x, nw, 1e-6, add_one=bool(add_one)))
    # swiglu activation and the fused M=1 W4 MLP
    gt = (torch.randn((3, 300), generator=g) * 3).to(torch.bfloat16)
    ut = torch.randn((3, 300), generator=g).to(torch.bfloat16)
    out["swiglu.g"], out["swiglu.u"] = bits(gt), bits(ut)
    out["swiglu.y"] = bits(ref_ck.swiglu_bf16(gt, ut))
    H, I, Kh = 128, 192, 256
    x1 = torch.randn((1, Kh), generator=g).to(torch.bfloat16)
    wg = (torch.randn((2 * I, Kh), generator=g) * 0.02)
    wd = (torch.randn((H, I), generator=g) * 0.02)
    gq, gs = ref_ck.quantize_weight_i4_per_row_chunked(wg)
    dq, ds = ref_ck.quantize_weight_i4_per_row_chunked(wd)
    out["mlp.x"] = bits(x1)
    out["mlp.gu_qw"], out["mlp.gu_s"] = gq.numpy().copy(), gs.numpy().copy()
    out["mlp.d_qw"], out["mlp.d_s"] = dq.numpy().copy(), ds.numpy().copy()
    out["mlp.dims"] = np.array([H, I, Kh], np.int64)
    out["mlp.y"] = bits(ref_ck.swiglu_w4a16_bf16(x1, gq, gs, dq, ds, I, Kh, I))
    return out


# ------------------------------------------------------------------------------------------
# 2. model verify traces
# ------------------------------------------------------------------------------------------

VARIANTS = {
    # name: (oracle config kwargs)
    "qwen3_w4g128": dict(gated=False, gemma_norm=False, quant="w4g128", n_heads=4, n_kv_heads=2),
    "qwen35_w4g128": dict(gated=True, gemma_norm=True, quant="w4g128", n_heads=4, n_kv_heads=2),
    "qwen3_w4g128_gqa4": dict(gated=False, gemma_norm=False, quant="w4g128", n_heads=8, n_kv_heads=2),
    "qwen3_w8a32_f32": dict(gated=False, gemma_norm=False, quant="w8a32", dtype="float32", n_heads=4, n_kv_heads=2),
}


class _GateFreeQ(nn.Module):
    """Harness shim (not reference code): wraps a quantized q_proj producing
    [seq, n_heads*hd] and appends a +inf gate half per head so the reference's
    FullAttention (attention.py:81-83,139) multiplies by sigmoid(+inf) == 1.0."""

    def __init__(self, inner: nn.Module, n_heads: int, head_dim: int):
        super().__init__()
        self.inner, self.n_heads, self.head_dim = inner, n_heads, head_dim

    def forward(self, x):
        q = self.inner(x)
        seq = q.shape[0]
        q = q.view(seq, self.n_heads, self.head_dim)
        gate = torch.full_like(q, float("inf"))
        return torch.cat([q, gate], dim=-1).reshape(seq, -1)


def build_reference_model(cfg: om.Qwen3Config, ck: dict[str, torch.Tensor]) -> Qwen3Model:
    tc = TextConfig(hidden_size=cfg.hidden, num_hidden_layers=cfg.layers, num_attention_heads=cfg.n_heads,
                    num_key_value_heads=cfg.n_kv_heads, head_dim=cfg.head_dim,
                    intermediate_size=cfg.intermediate, vocab_size=cfg.vocab, rms_norm_eps=cfg.eps,
                    dtype=cfg.dtype, layer_types=["full_attention"] * cfg.layers,
                    rope=RopeConfig(rope_theta=cfg.rope_theta, partial_rotary_factor=cfg.partial_rotary))
    mc = ModelConfig(architectures=["Qwen3ForCausalLM"], text_config=tc, dtype=cfg.dtype)
    model = Qwen3Model(mc)
    dt = cfg.torch_dtype

    def quantized(w_bf16: torch.Tensor) -> nn.Module:
        w = w_bf16.to(torch.float32)
        if cfg.quant == "w4g128":
            qw, s = ref_ck.quantize_weight_i4_grouped_chunked(w, group_size=128)
            return QuantizedW4A16Linear(qw, s, w.shape[1])
        if cfg.quant == "w8a32":
            qw, s = ref_ck.quantize_weight_i8_per_row(w)
            return QuantizedW8A32Linear(qw, s)
        raise ValueError(cfg.quant)

    model.embed_tokens.weight = nn.Parameter(ck["embed"].to(dt), requires_grad=False)
    for li, layer in enumerate(model.layers):
        at = layer.self_attn
        if cfg.gated:
            at.q_proj = quantized(ck[f"l{li}.q_proj"])
        else:
            at.q_proj = _GateFreeQ(quantized(ck[f"l{li}.q_proj"]), cfg.n_heads, cfg.head_dim)
        at.k_proj = quantized(ck[f"l{li}.k_proj"])
        at.v_proj = quantized(ck[f"l{li}.v_proj"])
        at.o_proj = quantized(ck[f"l{li}.o_proj"])
        layer.mlp.gate = quantized(ck[f"l{li}.gate"])
        layer.mlp.up = quantized(ck[f"l{li}.up"])
        layer.mlp.down = quantized(ck[f"l{li}.down"])
        pairs = [(layer, "input_layernorm", f"l{li}.input_norm"), (layer, "post_attention_layernorm", f"l{li}.post_norm"),
                 (at, "q_norm", f"l{li}.q_norm"), (at, "k_norm", f"l{li}.k_norm")]
        for mod, attr, key in pairs:
            _set_norm(mod, attr, ck[key].to(dt), cfg)
    _set_norm(model, "norm", ck["final_norm"].to(dt), cfg)
    model.lm_head = quantized(ck["embed"])
    model.eval()
    return model


def build_reference_mtp(cfg: om.Qwen3Config, mck: dict[str, torch.Tensor], mc, quantize: bool = True) -> Qwen3MTPDraft:
    """The reference draft module (mtp.py:15-23) with the seeded weights: quantized by the
    reference's own W4A16 option (_quantize_mtp_linears, mtp.py:85-94, PILM_MTP_QUANTIZE=
    w4a16), or with its default bf16 BackendLinear layers (quantize=False, mtp.py:137).
    Plain Qwen3 uses the same harness shims as the main model (+inf gate half, RMSNorm for
    GemmaRMSNorm)."""
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        mtp = Qwen3MTPDraft(mc)
    finally:
        torch.set_default_dtype(prev)

    def lin(w: torch.Tensor) -> BackendLinear:
        m = BackendLinear(w.shape[1], w.shape[0], bias=False)
        m.weight = nn.Parameter(w.clone(), requires_grad=False)
        return m

    blk = mtp.layers[0]
    at = blk.self_attn
    mtp.fc = lin(mck["fc"])
    at.q_proj = lin(mck["q_proj"])
    at.k_proj = lin(mck["k_proj"])
    at.v_proj = lin(mck["v_proj"])
    at.o_proj = lin(mck["o_proj"])
    blk.mlp.gate = lin(mck["gate"])
    blk.mlp.up = lin(mck["up"])
    blk.mlp.down = lin(mck["down"])
    if quantize:
        mtp.quantized_linear_modules = _quantize_mtp_linears(mtp)
    if not cfg.gated:
        at.q_proj = _GateFreeQ(at.q_proj, cfg.n_heads, cfg.head_dim)
    pairs = [(mtp, "pre_fc_norm_embedding", "pre_fc_norm_embedding"), (mtp, "pre_fc_norm_hidden", "pre_fc_norm_hidden"),
             (blk, "input_layernorm", "input_norm"), (blk, "post_attention_layernorm", "post_norm"),
             (at, "q_norm", "q_norm"), (at, "k_norm", "k_norm"), (mtp, "norm", "final_norm")]
    for mod, attr, key in pairs:
        _set_norm(mod, attr, mck[key], cfg)
    mtp.eval()
    return mtp


def _set_norm(mod: nn.Module, attr: str, w: torch.Tensor, cfg: om.Qwen3Config) -> None:
    if not cfg.gemma_norm:
        setattr(mod, attr, RMSNorm(w.shape[0], cfg.eps))
    getattr(mod, attr).weight = nn.Parameter(w.clone(), requires_grad=False)


def greedy_accept_engine(logits: torch.Tensor, drafts: list[int]) -> tuple[int, int]:
    """The accept/bonus rule of engine.py:483-503 and :551-557, written out."""
    acc = 0
    for i, d in enumerate(drafts):
        if int(torch.argmax(logits[i]).item()) != int(d):
            return acc, int(torch.argmax(logits[i]).item())
        acc += 1
    return acc, int(torch.argmax(logits[len(drafts)]).item())


def run_forward(model, kv, token_ids, positions, block_ids, is_decode):
    start = positions[0]
    bs = kv.block_size
    with torch.no_grad():
        h, _, _ = model(input_ids=torch.tensor(token_ids, dtype=torch.long),
                        positions=torch.tensor(positions, dtype=torch.long),
                        kv_caches_k=kv.k_cache, kv_caches_v=kv.v_cache,
                        block_id=block_ids[start // bs], slot_offset=start % bs, is_decode=is_decode,
                        block_ids=block_ids, logits_last_only=False, return_last_hidden=True)
    return h


def model_trace(name: str, kwargs: dict, seed: int) -> dict[str, np.ndarray]:
    cfg = om.Qwen3Config(**kwargs)
    ck = om.make_checkpoint(cfg, seed)
    model = build_reference_model(cfg, ck)
    mtp = mtp_bf16 = None
    if cfg.quant == "w4g128":  # the draft module (bf16 activations): W4A16 option and bf16 default
        mck = om.make_mtp_checkpoint(cfg, seed)
        mtp = build_reference_mtp(cfg, mck, model.config)
        mtp_bf16 = build_reference_mtp(cfg, mck, model.config, quantize=False)
    rng = np.random.default_rng(seed)
    prompts = [list(rng.integers(0, cfg.vocab, size=n)) for n in (21, 27, 13, 31)]
    k = 3
    num_blocks = 32
    mgr = KVCacheManager(num_blocks, cfg.block_size, enable_caching=False)
    sched = Scheduler(mgr, max_num_batched_tokens=cfg.block_size)
    kv = PhysicalKVCache(cfg.layers, num_blocks, cfg.block_size, cfg.n_kv_heads, cfg.head_dim, dtype=cfg.torch_dtype)
    for t in (kv.k_cache + kv.v_cache):
        t.zero_()
    reqs = []
    for i, p in enumerate(prompts):
        r = Request(req_id=i + 1, prompt_token_ids=[int(t) for t in p], max_new_tokens=64, eos_token_id=-1)
        sched.add_request(r)
        reqs.append(r)
    # prefill through the reference scheduler (chunks of <= block_size tokens)
    last_hidden = {}
    chunks = []
    while any(r.num_computed_tokens < r.num_prompt_tokens for r in reqs):
        out = sched.schedule()
        for sr in out.scheduled:
            r = next(r for r in reqs if r.req_id == sr.req_id)
            ids = r.all_token_ids[sr.positions[0]:sr.positions[0] + sr.num_tokens]
            chunks.append([reqs.index(r), sr.positions[0], sr.num_tokens])
            last_hidden[r.req_id] = run_forward(model, kv, ids, sr.positions, sr.block_ids, not sr.is_prefill)
    # the first generated token (greedy) becomes the verify row 0 ("last token")
    first_tokens = []
    for r in reqs:
        lg = model.lm_head(last_hidden[r.req_id][-1:]).to(torch.float32)
        first_tokens.append(int(torch.argmax(lg[0])))
        r.append_output_token_ids([first_tokens[-1]], cfg.block_size)
    # drafts (capped at the page boundary like engine.py:399-401): sequence 0 gets its
    # own greedy continuation (all accepted), sequence 1 the continuation with the 2nd
    # draft corrupted (1 accepted), sequence 2 random drafts, sequence 3 sits on the
    # last slot of a page so its cap is 0 (a plain one-row decode).
    kv_snap = ([t.clone() for t in kv.k_cache], [t.clone() for t in kv.v_cache])
    drafts_all = []
    for bi, r in enumerate(reqs):
        n_comp = r.num_computed_tokens
        cap = om.draft_limit(n_comp, cfg.block_size, 64, k)
        d = [int(x) for x in rng.integers(0, cfg.vocab, size=cap)]
        if bi < 2:
            for j in range(cap):
                # rows 0..j of the verify depend only on tokens 0..j: re-run to extend
                ids = [first_tokens[bi]] + d[:j]
                pos = list(range(n_comp, n_comp + 1 + j))
                blocks = list(r.block_ids)
                need = (n_comp + 1 + j + cfg.block_size - 1) // cfg.block_size
                if need > len(blocks):
                    break
                h = run_forward(model, kv, ids, pos, blocks, True)
                d[j] = int(torch.argmax(model.lm_head(h[-1:]).to(torch.float32)[0]))
            if bi == 1 and cap >= 2:
                d[1] = (d[1] + 1) % cfg.vocab
        drafts_all.append(d)
    for t, s in zip(kv.k_cache + kv.v_cache, kv_snap[0] + kv_snap[1]):
        t.copy_(s)
    # KV cache content after prefill: the verify step's input state
    kv_in = {}
    for li in range(cfg.layers):
        for nm, t in (("k", kv.k_cache[li]), ("v", kv.v_cache[li])):
            kv_in[f"kv.{nm}{li}"] = bits(t) if t.dtype == torch.bfloat16 else t.numpy().copy()
    # verify step: append drafts, schedule, forward k+1 rows, lm_head, accept, roll back
    for r, d in zip(reqs, drafts_all):
        r._all_token_ids.extend(d)
        r._update_block_hashes(cfg.block_size)
    out = sched.schedule()
    res: dict[str, np.ndarray] = {}
    cfgv = [cfg.hidden, cfg.layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab,
            int(cfg.gated), int(cfg.gemma_norm), cfg.block_size, seed, int(cfg.dtype == "float32")]
    res["config"] = np.array(cfgv, np.int64)
    res["quant"] = np.array(list(cfg.quant.encode()), np.uint8)
    res["prefill_chunks"] = np.array(chunks, np.int64)
    for bi, r in enumerate(reqs):
        res[f"b{bi}.prompt"] = np.array(prompts[bi], np.int64)
        res[f"b{bi}.first_token"] = np.array([first_tokens[bi]], np.int64)
        res[f"b{bi}.drafts"] = np.array(drafts_all[bi], np.int64)
    for bi, r in enumerate(reqs):
        sr = next(s for s in out.scheduled if s.req_id == r.req_id)
        ids = r.all_token_ids[sr.positions[0]:sr.positions[0] + sr.num_tokens]
        res[f"b{bi}.block_ids"] = np.array(sr.block_ids, np.int64)
        res[f"b{bi}.positions"] = np.array(sr.positions, np.int64)
        res[f"b{bi}.verify_ids"] = np.array(ids, np.int64)
        res[f"b{bi}.slots"] = np.array([sr.block_ids[p // cfg.block_size] * cfg.block_size + p % cfg.block_size
                                        for p in sr.positions], np.int64)
        h = run_forward(model, kv, ids, sr.positions, sr.block_ids, True)
        logits = model.lm_head(h).to(torch.float32)
        acc, nxt = greedy_accept_engine(logits, drafts_all[bi])
        start = sr.positions[0]
        res[f"b{bi}.hidden"] = bits(h) if h.dtype == torch.bfloat16 else h.numpy().copy()
        res[f"b{bi}.logits"] = logits.numpy().copy()
        res[f"b{bi}.accept"] = np.array([acc, nxt], np.int64)
        res[f"b{bi}.num_computed_after"] = np.array([start + 1 + acc], np.int64)
        if mtp is not None:
            # the next cycle's drafts (engine.py:527-536 after a reject, :548-557 after a full
            # accept): from the normed hidden of the row that produced the next token
            with torch.no_grad():
                d_next, h_last = mtp.draft_tokens(h[acc], nxt, start + acc + 1, model.embed_tokens, model.lm_head,
                                                  num_tokens=3)
            res[f"b{bi}.mtp_drafts"] = np.array(d_next, np.int64)
            res[f"b{bi}.mtp_last_hidden"] = bits(h_last.reshape(1, -1))
            with torch.no_grad():
                d_next, h_last = mtp_bf16.draft_tokens(h[acc], nxt, start + acc + 1, model.embed_tokens,
                                                       model.lm_head, num_tokens=3)
            res[f"b{bi}.mtp_drafts_bf16"] = np.array(d_next, np.int64)
            res[f"b{bi}.mtp_last_hidden_bf16"] = bits(h_last.reshape(1, -1))
        if acc < len(drafts_all[bi]):
            # reference reject path (engine.py:505-525): re-run the accepted prefix
            hp = run_forward(model, kv, ids[:1 + acc], sr.positions[:1 + acc], sr.block_ids, True)
            res[f"b{bi}.recompute_hidden_last"] = (bits(hp[-1:]) if hp.dtype == torch.bfloat16
                                                   else hp[-1:].numpy().copy())
    res.update(kv_in)
    # checksum of the quantized weights so CPU tests catch seeded-RNG drift
    q = om.quantize_checkpoint(cfg, ck)
    hsh = hashlib.sha256()
    for key in sorted(q):
        hsh.update(q[key]["qweight"].tobytes())
        hsh.update(q[key]["scales"].tobytes())
    res["qweights_sha256"] = np.frombuffer(hsh.digest(), np.uint8).copy()
    if mtp is not None:
        hsh = hashlib.sha256()
        mq = om.quantize_mtp(om.make_mtp_checkpoint(cfg, seed))
        for key in sorted(mq):
            hsh.update(mq[key]["qweight"].tobytes())
            hsh.update(mq[key]["scales"].tobytes())
        res["mtp_qweights_sha256"] = np.frombuffer(hsh.digest(), np.uint8).copy()
    return res


# ------------------------------------------------------------------------------------------
# 3. paging: reference block pool trace
# ------------------------------------------------------------------------------------------

def paging_trace() -> dict[str, np.ndarray]:
    """Three requests through the reference Scheduler with a small pool, including a
    preemption and frees; records block_ids after every schedule() call."""
    rng = np.random.default_rng(7)
    mgr = KVCacheManager(12, 16, enable_caching=False)
    sched = Scheduler(mgr, max_num_batched_tokens=16, max_num_seqs=8)
    lens = [37, 20, 50]
    reqs = [Request(req_id=i + 1, prompt_token_ids=[int(t) for t in rng.integers(0, 1000, n)], max_new_tokens=6,
                    eos_token_id=-1) for i, n in enumerate(lens)]
    for r in reqs:
        sched.add_request(r)
    rows = []
    for step in range(40):
        out = sched.schedule()
        if out.is_empty:
            break
        gen = {}
        for sr in out.scheduled:
            rows.append([step, sr.req_id, sr.num_tokens, sr.positions[0], int(sr.is_prefill)] +
                        (list(sr.block_ids) + [-1] * 8)[:8])
            r = next(x for x in reqs if x.req_id == sr.req_id)
            if not sr.is_prefill_chunk and r.num_computed_tokens >= r.num_prompt_tokens:
                gen[sr.req_id] = [int(rng.integers(0, 1000))]
        for pid in out.preempted:
            rows.append([step, -pid, 0, 0, 0] + [-1] * 8)
        sched.update_from_output(out, gen)
    return {"rows": np.array(rows, np.int64), "pool": np.array([12, 16], np.int64),
            "lens": np.array(lens, np.int64)}


# ------------------------------------------------------------------------------------------
# 4. a quant bundle in the reference's export format (scripts/export_pilm_quant_bundle.py)
# ------------------------------------------------------------------------------------------

BUNDLE_VARIANT = "qwen35_w4g128"


def quant_bundle(name: str, kwargs: dict, seed: int, out_dir: Path) -> None:
    """The seeded checkpoint of a model variant as a pilm-quant-bundle-v1 directory: every
    linear (LM head included: the w4a16-all policy) quantized by the reference's group-128
    quantizer and written by the reference's own cache writer under its cache file name
    (models/qwen3/weights.py:59-62, 252-266); the embedding and norms as bf16 residual
    tensors; the HF source names of weights.py:20-44; a config.json the reference's
    config parser reads (runtime/loader/config_parser.py:81-125)."""
    import json
    import shutil

    from safetensors.torch import save_file

    from models.qwen3.weights import _quant_cache_path, _save_quantized_linear_cache

    cfg = om.Qwen3Config(**kwargs)
    ck = om.make_checkpoint(cfg, seed)
    if out_dir.exists():
        shutil.rmtree(out_dir)
    (out_dir / "linear_w4a16").mkdir(parents=True)
    (out_dir / "residual_bf16").mkdir()
    pre = "model.language_model."
    hf_lin = {"q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj", "v_proj": "self_attn.v_proj",
              "o_proj": "self_attn.o_proj", "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
    hf_norm = {"input_norm": "input_layernorm", "post_norm": "post_attention_layernorm",
               "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm"}
    quantized = {}
    for li in range(cfg.layers):
        for k, v in hf_lin.items():
            quantized[f"{pre}layers.{li}.{v}.weight"] = ck[f"l{li}.{k}"]
    quantized["lm_head.weight"] = ck["embed"]  # tied LM head, quantized like any linear
    for src, w in sorted(quantized.items()):
        qw, s = ref_ck.quantize_weight_i4_grouped_chunked(w.to(torch.float32), group_size=128)
        _save_quantized_linear_cache(_quant_cache_path(out_dir / "linear_w4a16", src), qw, s, w.shape[1])
    residual = {f"{pre}embed_tokens.weight": ck["embed"], f"{pre}norm.weight": ck["final_norm"]}
    for li in range(cfg.layers):
        for k, v in hf_norm.items():
            residual[f"{pre}layers.{li}.{v}.weight"] = ck[f"l{li}.{k}"]
    rel = "residual_bf16/residual-0001.safetensors"
    save_file({k: v.contiguous() for k, v in residual.items()}, str(out_dir / rel))
    text = {"hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.n_heads,
            "num_key_value_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim,
            "intermediate_size": cfg.intermediate, "vocab_size": cfg.vocab, "rms_norm_eps": cfg.eps,
            "layer_types": ["full_attention"] * cfg.layers, "tie_word_embeddings": True,
            "rope_parameters": {"rope_type": "default", "rope_theta": cfg.rope_theta,
                                "partial_rotary_factor": cfg.partial_rotary}}
    (out_dir / "config.json").write_text(json.dumps({"model_type": "qwen3_5", "text_config": text,
                                                     "tie_word_embeddings": True}, indent=2))
    manifest = {"format": "pilm-quant-bundle-v1", "quantize": "w4a16-all", "small_files": ["config.json"],
                "quantized_linear_tensors": len(quantized), "residual_bf16_tensors": len(residual),
                "mtp_bf16_tensors": 0, "quantized_linear_sources": sorted(quantized),
                "residual_sources": sorted(residual), "mtp_sources": [], "missing_linear_cache": [],
                "residual_exports": [{"file": rel, "tensors": len(residual)}], "mtp_exports": []}
    (out_dir / "pilm_quant_manifest.json").write_text(json.dumps(manifest, indent=2))
    _check_bundle_with_reference(out_dir, cfg, quantized)


def _check_bundle_with_reference(out_dir: Path, cfg: om.Qwen3Config, quantized: dict) -> None:
    """Read the bundle back through the reference's own loader code: its config parser,
    manifest reader and bundle weight map, and every linear cache file by name with the
    shapes and dtypes its cache loader accepts (weights.py:200-249)."""
    from safetensors.torch import load_file

    from models.qwen3.weights import _bundle_weight_map, _load_quant_bundle_manifest, _quant_cache_path
    from runtime.loader.config_parser import parse_config

    mc = parse_config(str(out_dir))
    tc = mc.text_config
    assert (tc.hidden_size, tc.num_hidden_layers, tc.num_attention_heads, tc.num_key_value_heads, tc.head_dim,
            tc.intermediate_size, tc.vocab_size) == (cfg.hidden, cfg.layers, cfg.n_heads, cfg.n_kv_heads,
                                                     cfg.head_dim, cfg.intermediate, cfg.vocab)
    manifest = _load_quant_bundle_manifest(out_dir)
    wmap = _bundle_weight_map(out_dir, manifest)
    assert all(wmap[k] == "__pilm_linear_cache__" for k in quantized)
    for src, w in quantized.items():
        payload = load_file(str(_quant_cache_path(out_dir / "linear_w4a16", src)))
        n, k = w.shape
        assert tuple(payload["qweight"].shape) == (n, (k + 1) // 2) and payload["qweight"].dtype == torch.uint8
        assert tuple(payload["scales"].shape) == (n, (k + 127) // 128) and payload["scales"].dtype == torch.float32
        assert int(payload["in_features"].reshape(-1)[0]) == k


def main() -> None:
    np.savez_compressed(OUT / "kernels.npz", **kernel_goldens())
    for i, (name, kw) in enumerate(VARIANTS.items()):
        np.savez_compressed(OUT / f"model_{name}.npz", **model_trace(name, kw, seed=100 + i))
    np.savez_compressed(OUT / "paging.npz", **paging_trace())
    names = list(VARIANTS)
    quant_bundle(BUNDLE_VARIANT, VARIANTS[BUNDLE_VARIANT], 100 + names.index(BUNDLE_VARIANT),
                 OUT / f"bundle_{BUNDLE_VARIANT}")
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
