"""Split-K partials summed by their consumer instead of the GEMM's combine pass.

ekernel_linear_w4a16g128_bf16_kpairs_deferred leaves a split-schedule GEMM's fp32
partials in a caller's buffer; ekernel_add_rmsnorm_bf16_splitk and
ekernel_qk_norm_rope_kv_append_splitk sum them in split order and round to bf16, which
is what the combine pass writes.  Every result must therefore be bit-identical to the
linear + combine + consumer path:
  * the partials' layout: summed on the host in split order they give the linear's output;
  * residual add + RMSNorm at the o/down shape of Qwen3-8B (M = 96);
  * QK-norm + RoPE + KV append at the fused q/k/v shape, plain and gated;
  * the whole verify forward of a two-layer Qwen3-1.7B-shaped model, plain and gated
    (prefill of 102 rows, then a verify step), with deferral on and off: K/V caches,
    logits and accept results equal.
"""
import numpy as np
import pytest
import torch

from oracle import kernels as ok
from pilm_b200 import bindings as abi
from pilm_b200 import ckernel as ck
from pilm_b200.engine import MTPVerifyEngine
from pilm_b200.qwen3 import PagedKVCache, Qwen3Shape, Qwen3Verifier, Qwen3Weights, W4Linear, rope_tables
from tests._gpu import dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    abi.init()
    yield


def _w4(N, K, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    qw, s = ok.quantize_i4_grouped(w, 128)
    return W4Linear(torch.from_numpy(qw).to(dev()), torch.from_numpy(s).to(dev()), K)


def _x(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn((M, K), generator=g).to(torch.bfloat16).to(dev())


def _deferred(lin, x):
    M = x.shape[0]
    need = lin.partials_bytes(M)
    assert need > 0, "this shape should run the split schedule"
    part = torch.empty(need // 4, dtype=torch.float32, device=dev())
    out = torch.full((M, lin.out_features), 7.0, dtype=torch.bfloat16, device=dev())
    sp = lin.deferred(x, out, part)
    assert sp > 1 and sp * M * lin.out_features * 4 == need
    assert bool((out == 7.0).all()), "a deferred call must not write its bf16 output"
    return part, sp


def test_partials_sum_to_the_linear_output():
    M, K, N = 96, 4096, 4096
    lin, x = _w4(N, K, 1), _x(M, K, 2)
    y = lin(x)
    part, sp = _deferred(lin, x)
    p = part[:sp * M * N].view(sp, M, N).cpu()
    acc = torch.zeros((M, N), dtype=torch.float32)
    for s in range(sp):  # fp32 adds in split order, as the combine pass does
        acc = acc + p[s]
    assert torch.equal(acc.to(torch.bfloat16), y.cpu())


@pytest.mark.parametrize("K,N", [(4096, 4096), (12288, 4096)])  # o and down of Qwen3-8B
def test_add_rmsnorm_from_partials_is_bit_identical(K, N):
    M = 96
    lin, x = _w4(N, K, K), _x(M, K, 3)
    g = torch.Generator().manual_seed(4)
    res0 = torch.randn((M, N), generator=g).to(torch.bfloat16).to(dev())
    w = (1 + 0.1 * torch.randn((N,), generator=g)).to(torch.bfloat16).to(dev())
    for add_one in (False, True):
        ra = res0.clone()
        ha = ck.add_rmsnorm_bf16(ra, lin(x), w, 1e-6, add_one)
        part, sp = _deferred(lin, x)
        rb = res0.clone()
        hb = ck.add_rmsnorm_bf16_splitk(rb, part, sp, w, 1e-6, add_one)
        assert torch.equal(ra, rb) and torch.equal(ha, hb)


# (8, 2, True, 40, 4096) runs 7 splits: the prologue adds them in two batches of loads
@pytest.mark.parametrize("nh,nkv,gated,M,K", [(32, 8, False, 96, 4096), (8, 2, True, 48, 1024),
                                              (8, 2, True, 40, 4096)])
def test_qk_prologue_from_partials_is_bit_identical(nh, nkv, gated, M, K):
    hd = 128
    N = nh * hd * (2 if gated else 1) + 2 * nkv * hd
    lin, x = _w4(N, K, N), _x(M, K, 5)
    shape = Qwen3Shape(hidden=K, layers=1, n_heads=nh, n_kv_heads=nkv, head_dim=hd, intermediate=256, vocab=256,
                       gated=gated)
    cos, sin = rope_tables(shape, 4096, dev())
    nb = (M + 15) // 16 + 2
    g = torch.Generator().manual_seed(6)
    qn = (1 + 0.1 * torch.randn((hd,), generator=g)).to(torch.bfloat16).to(dev())
    kn = (1 + 0.1 * torch.randn((hd,), generator=g)).to(torch.bfloat16).to(dev())
    pos = torch.arange(1000, 1000 + M, dtype=torch.int32, device=dev())
    slots = torch.arange(16, 16 + M, dtype=torch.int32, device=dev())
    slots[3] = -1  # a rejected row: not written
    desc = ck.attn_desc(num_seqs=1, total_q=M, max_q_len=M, n_heads=nh, n_kv_heads=nkv, head_dim=hd,
                        block_size=16, num_blocks=nb, max_blocks_per_seq=nb, max_context=1000 + M, qkv_stride=N,
                        rope_rows=4096, rot_dim=hd, eps=1e-6, add_one=False, output_gate=gated)
    outs = []
    for deferred in (False, True):
        kc = torch.zeros((nb, 16, nkv, hd), dtype=torch.bfloat16, device=dev())
        vc = torch.zeros_like(kc)
        q = torch.empty((M, nh * hd), dtype=torch.bfloat16, device=dev())
        gate = torch.empty((M, nh * hd), dtype=torch.bfloat16, device=dev()) if gated else None
        if deferred:
            part, sp = _deferred(lin, x)
            ck.qk_norm_rope_kv_append_splitk(desc, part, sp, qn, kn, cos, sin, pos, slots, kc, vc, q, gate)
        else:
            ck.qk_norm_rope_kv_append(desc, lin(x), qn, kn, cos, sin, pos, slots, kc, vc, q, gate)
        outs.append([t.cpu() for t in (q, kc, vc) + ((gate,) if gated else ())])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("gated", [False, True])
def test_verify_forward_with_and_without_deferral_is_identical(gated):
    """Two Qwen3-1.7B-shaped layers (synthetic weights): a 102-row prefill pass runs q/k/v, o
    and down on the split schedule, so all three consumers take partials; then a verify
    step.  K/V caches, first tokens, logits and accept results are equal either way."""
    shape = Qwen3Shape(hidden=2048, layers=2, n_heads=16, n_kv_heads=8, head_dim=128, intermediate=6144,
                       vocab=4096, gated=gated, gemma_norm=gated)
    w = Qwen3Weights.synthetic(shape, 11, dev())
    rng = np.random.default_rng(8)
    prompts = [[int(t) for t in rng.integers(0, shape.vocab, n)] for n in (40, 29, 33)]
    drafts = [[int(t) for t in rng.integers(0, shape.vocab, 2)] for _ in prompts]
    runs = []
    for defer in (False, True):
        kv = PagedKVCache(w.shape, 32, dev())
        ver = Qwen3Verifier(w, kv, max_rows=128, max_pos=256, device=dev())
        assert ver.part is not None
        ver.defer_splitk = defer
        eng = MTPVerifyEngine(ver, num_blocks=32, max_model_len=256, max_num_batched_tokens=128,
                              page_aligned_chunks=False)
        sids = [eng.add_request(p, max_new_tokens=8) for p in prompts]
        first = eng.prefill()
        res = eng.verify_step({sid: d for sid, d in zip(sids, drafts)})
        rows = sum(1 + len(r.drafts) for r in res)
        runs.append((sorted(first.items()), sorted((r.seq_id, r.accepted, r.next_token) for r in res),
                     ver.logits[:rows].cpu(), [t.cpu() for t in kv.k], [t.cpu() for t in kv.v]))
    a, b = runs
    assert a[0] == b[0] and a[1] == b[1]
    assert torch.equal(a[2], b[2])
    for x, y in zip(a[3] + a[4], b[3] + b[4]):
        assert torch.equal(x, y)
