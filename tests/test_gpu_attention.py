"""GPU parity of the fused QK-norm/RoPE/KV-append prologue and the paged verify
attention against the oracle restatement of FullAttention (attention.py:79-139)."""
import numpy as np
import pytest
import torch

from oracle import model as om
from pilm_b200 import bindings as abi
from pilm_b200 import ckernel as ck
from tests._gpu import REL_TOL, bits_of, dev, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    abi.init()
    yield


def run_case(nh, nkv, ctxs, qlens, gated=False, gemma=False, seed=0, num_blocks=None, partial=1.0, poison=False):
    g = torch.Generator().manual_seed(seed)
    cfg = om.Qwen3Config(n_heads=nh, n_kv_heads=nkv, gated=gated, gemma_norm=gemma, partial_rotary=partial)
    hd, bs = 128, 16
    B = len(ctxs)
    pages = [(c + bs - 1) // bs for c in ctxs]
    nb = num_blocks or (sum(pages) + 8)
    perm = torch.randperm(nb - 1, generator=g)[: sum(pages)] + 1
    tables, off = [], 0
    for p in pages:
        tables.append([int(x) for x in perm[off:off + p]])
        off += p
    maxp = max(pages)
    kc = torch.randn((nb, bs, nkv, hd), generator=g).to(torch.bfloat16)
    vc = (torch.randn((nb, bs, nkv, hd), generator=g) * 0.5).to(torch.bfloat16)
    qrows = cfg.q_rows
    T = sum(qlens)
    qkv = (torch.randn((T, qrows + 2 * nkv * hd), generator=g) * 2).to(torch.bfloat16)
    qn = (torch.randn(hd, generator=g) * 0.1 + (0 if gemma else 1)).to(torch.bfloat16)
    kn = (torch.randn(hd, generator=g) * 0.1 + (0 if gemma else 1)).to(torch.bfloat16)
    positions, slots, cu = [], [], [0]
    for b in range(B):
        st = ctxs[b] - qlens[b]
        assert st % bs + qlens[b] <= bs, "verify rows never cross a page (engine.py:399-401)"
        for j in range(qlens[b]):
            p = st + j
            positions.append(p)
            slots.append(tables[b][p // bs] * bs + p % bs)
        cu.append(cu[-1] + qlens[b])
    # oracle, one sequence at a time on a copy of the caches
    kc_ref, vc_ref = kc.clone(), vc.clone()
    outs = []
    for b in range(B):
        rows = slice(cu[b], cu[b + 1])
        x = qkv[rows]
        qp, kp, vp = x[:, :qrows], x[:, qrows:qrows + nkv * hd], x[:, qrows + nkv * hd:]
        outs.append(om.attention_from_proj(cfg, qp, kp, vp, qn, kn, torch.tensor(positions[rows]), kc_ref, vc_ref,
                                           tables[b], True))
    ref = torch.cat(outs)
    # GPU
    max_pos = max(ctxs) + 1
    cos, sin = om.rope_tables(cfg, max_pos)
    d = dev()
    bt = torch.tensor([t + [0] * (maxp - len(t)) for t in tables], dtype=torch.int32, device=d)
    desc = ck.attn_desc(num_seqs=B, total_q=T, max_q_len=max(qlens), n_heads=nh, n_kv_heads=nkv, head_dim=hd,
                        block_size=bs, num_blocks=nb, max_blocks_per_seq=maxp, max_context=max(ctxs),
                        qkv_stride=qkv.shape[1], rope_rows=max_pos, rot_dim=int(hd * partial), eps=1e-6,
                        add_one=gemma, output_gate=gated)
    kc_d, vc_d = kc.to(d), vc.to(d)
    if poison:  # the slots past each context in its last page hold NaN on the device
        for b in range(B):
            if ctxs[b] % bs:
                kc_d[tables[b][-1], ctxs[b] % bs:] = float("nan")
                vc_d[tables[b][-1], ctxs[b] % bs:] = float("nan")
    q_out = torch.empty((T, nh * hd), dtype=torch.bfloat16, device=d)
    gate = torch.empty((T, nh * hd), dtype=torch.bfloat16, device=d) if gated else None
    out = torch.empty((T, nh * hd), dtype=torch.bfloat16, device=d)
    i32 = dict(dtype=torch.int32, device=d)
    ck.qk_norm_rope_kv_append(desc, qkv.to(d), qn.to(d), kn.to(d), cos.to(d), sin.to(d),
                              torch.tensor(positions, **i32), torch.tensor(slots, **i32), kc_d, vc_d, q_out, gate)
    ck.paged_attention_verify(desc, q_out, kc_d, vc_d, bt, torch.tensor(cu, **i32),
                              torch.tensor(ctxs, **i32), gate, out)
    torch.cuda.synchronize()
    # appended K/V: V is copied exactly; K within one bf16 rounding of the oracle
    sl = torch.tensor(slots)
    kv_ref_k = kc_ref.view(-1, nkv, hd)[sl].float()
    kv_got_k = kc_d.view(-1, nkv, hd)[sl.to(d)].float().cpu()
    assert rel_err(kv_got_k.numpy(), kv_ref_k.numpy()) <= REL_TOL
    assert torch.equal(vc_d.view(-1, nkv, hd)[sl.to(d)].cpu(), vc_ref.view(-1, nkv, hd)[sl])
    e = rel_err(out.float().cpu().numpy(), ref.float().numpy())
    assert e <= REL_TOL, e
    return e


def test_verify_rows_gqa4_k2():
    run_case(8, 2, ctxs=[40, 99, 16, 131], qlens=[3, 3, 1, 3])


def test_verify_rows_gqa2_k3_gated_gemma():
    run_case(4, 2, ctxs=[21, 64, 300], qlens=[4, 2, 4], gated=True, gemma=True, seed=1)


def test_long_context_split_kv():
    run_case(8, 2, ctxs=[2051, 4100], qlens=[3, 2], seed=2)


def test_prefill_chunk_rows_two_mtiles():
    # 16-token chunk with 4 query heads per KV head: 64 rows -> 2 row chunks of 32
    run_case(8, 2, ctxs=[16, 45], qlens=[16, 13], seed=3)


def test_partial_rotary():
    run_case(4, 2, ctxs=[34, 51], qlens=[2, 3], seed=4, partial=0.25)


def test_qwen3_8b_head_layout():
    run_case(32, 8, ctxs=[531, 1000], qlens=[3, 3], seed=5)


def test_many_ragged_sequences_nan_past_context():
    """40 sequences of ragged lengths: the whole-page kernel's per-SM page ranges start and
    end inside sequences, so many rows are combined from several CTAs' partials.  The slots
    past each context in its last page are NaN: keys past the context never reach the output."""
    import random
    rnd = random.Random(7)
    ctxs, qlens = [], []
    for _ in range(40):
        q = rnd.randint(1, 3)
        st = 16 * rnd.randint(0, 40) + rnd.randint(0, 16 - q)
        ctxs.append(st + q)
        qlens.append(q)
    run_case(32, 8, ctxs=ctxs, qlens=qlens, seed=8, poison=True)


def test_rows_17_to_32_per_kv_head_qwen3_8b_heads():
    """17 to 32 query rows per KV head (q_len 5 to 8 with 4 query heads per KV head, mixed with
    shorter passes in the same call): beyond the whole-page kernel's one 16-row tile.  40
    ragged sequences; the slots past each context in its last page are NaN."""
    import random
    rnd = random.Random(17)
    ctxs, qlens = [], []
    for _ in range(40):
        q = rnd.choice([1, 3, 5, 6, 8])
        st = 16 * rnd.randint(0, 40) + rnd.randint(0, 16 - q)
        ctxs.append(st + q)
        qlens.append(q)
    run_case(32, 8, ctxs=ctxs, qlens=qlens, seed=18, poison=True)


def test_rows_17_to_32_per_kv_head_two_kv_heads():
    """The same range of rows per KV head with two KV heads (8 query heads)."""
    run_case(8, 2, ctxs=[40, 112, 16, 136, 704], qlens=[5, 8, 1, 6, 7], seed=19, poison=True)


def test_rows_17_to_32_per_kv_head_gated_gemma():
    """Gated attention with Gemma norms, 2 query heads per KV head and q_len up to 16 (32 rows
    per KV head)."""
    run_case(16, 8, ctxs=[30, 77, 496, 16], qlens=[12, 9, 16, 16], gated=True, gemma=True, seed=20)


def prefill_case(nh, nkv, qlens, prefixes, gated=False, seed=0):
    """Prompt chunks (q_len positions after a cached prefix) straight into the attention
    entry point: post-RoPE queries against paged caches whose slots past each context
    hold NaN, against the oracle's attention (attention.py:99-139) per sequence."""
    g = torch.Generator().manual_seed(seed)
    cfg = om.Qwen3Config(n_heads=nh, n_kv_heads=nkv, gated=gated)
    hd, bs = 128, 16
    ctxs = [q + p for q, p in zip(qlens, prefixes)]
    B = len(ctxs)
    pages = [(c + bs - 1) // bs for c in ctxs]
    nb = sum(pages) + 4
    perm = torch.randperm(nb - 1, generator=g)[: sum(pages)] + 1
    tables, off = [], 0
    for p in pages:
        tables.append([int(x) for x in perm[off:off + p]])
        off += p
    maxp = max(pages)
    kc = torch.randn((nb, bs, nkv, hd), generator=g).to(torch.bfloat16)
    vc = (torch.randn((nb, bs, nkv, hd), generator=g) * 0.5).to(torch.bfloat16)
    T = sum(qlens)
    q = torch.randn((T, nh, hd), generator=g).to(torch.bfloat16)
    gate = torch.randn((T, nh * hd), generator=g).to(torch.bfloat16) if gated else None
    cu = [0]
    for n in qlens:
        cu.append(cu[-1] + n)
    ref = torch.cat([om.attend(cfg, q[cu[b]:cu[b + 1]], gate[cu[b]:cu[b + 1]] if gated else None, kc, vc,
                               tables[b], ctxs[b], True) for b in range(B)])
    d = dev()
    kc_d, vc_d = kc.to(d), vc.to(d)
    for b in range(B):
        if ctxs[b] % bs:
            kc_d[tables[b][-1], ctxs[b] % bs:] = float("nan")
            vc_d[tables[b][-1], ctxs[b] % bs:] = float("nan")
    i32 = dict(dtype=torch.int32, device=d)
    bt = torch.tensor([t + [0] * (maxp - len(t)) for t in tables], **i32)
    desc = ck.attn_desc(num_seqs=B, total_q=T, max_q_len=max(qlens), n_heads=nh, n_kv_heads=nkv, head_dim=hd,
                        block_size=bs, num_blocks=nb, max_blocks_per_seq=maxp, max_context=max(ctxs),
                        qkv_stride=nh * hd, rope_rows=0, rot_dim=hd, eps=1e-6, add_one=0, output_gate=gated)
    out = torch.empty((T, nh * hd), dtype=torch.bfloat16, device=d)
    ck.paged_attention_verify(desc, q.view(T, nh * hd).to(d), kc_d, vc_d, bt, torch.tensor(cu, **i32),
                              torch.tensor(ctxs, **i32), gate.to(d) if gated else None, out)
    torch.cuda.synchronize()
    e = rel_err(out.float().cpu().numpy(), ref.float().numpy())
    assert e <= REL_TOL, e
    return e


def test_prefill_chunks_qwen3_8b_heads():
    """Six chunks of up to 512 positions with GQA 4 (up to 2048 rows per KV head, 64
    row chunks of the per-head kernel); ragged chunk ends and prefixes put the last page
    of most sequences part-full (NaN past the context)."""
    prefill_case(32, 8, qlens=[300, 257, 130, 512, 96, 200], prefixes=[0, 37, 1000, 5, 0, 16], seed=11)


def test_prefill_chunks_gated_gqa2():
    prefill_case(16, 8, qlens=[512, 301, 450, 128], prefixes=[64, 0, 211, 3], gated=True, seed=12)


def test_prefill_single_chunk_long_prefix():
    """One 200-position chunk after a 700-token prefix: few row chunks, so the keys are
    split across CTAs and merged."""
    prefill_case(32, 8, qlens=[200], prefixes=[700], seed=13)
