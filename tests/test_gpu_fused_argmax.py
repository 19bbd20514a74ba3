"""The LM head with the row argmax folded into its GEMM, and greedy acceptance from those keys.

ekernel_linear_w4a16g128_bf16_kpairs_argmax folds each output row's argmax into a uint64
key per row (stream-K schedule); ekernel_verify_accept_greedy_keys decodes the keys,
resets them and accepts.  Checked against the separate path (row_top2 over the bf16
logits, then ekernel_verify_accept_greedy) and against torch's first-max argmax:
  * at a stream-K shape (19000 vocabulary rows, M = 96), with a tie planted at each row's
    maximum (a duplicated weight row scaled up), so the smaller index must win;
  * the accept results, next tokens, context rollback and slot invalidation are the same,
    the keys are zero afterwards and a second call agrees;
  * a verify step of a two-layer model with a 32768-word vocabulary, fused and not (the
    model's default is the separate path, which measured faster on the bench step).
"""
import numpy as np
import pytest
import torch

from oracle import kernels as ok
from pilm_b200 import bindings as abi
from pilm_b200 import ckernel as ck
from pilm_b200.engine import MTPVerifyEngine
from pilm_b200.qwen3 import PagedKVCache, Qwen3Shape, Qwen3Verifier, Qwen3Weights, W4Linear
from tests._gpu import dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    abi.init()
    yield


def _lm_head(N, K, seed, tie=(4321, 17001)):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[tie[0]] *= 8.0       # a row whose outputs are large ...
    w[tie[1]] = w[tie[0]]  # ... and its duplicate at a larger index: equal outputs
    qw, s = ok.quantize_i4_grouped(w, 128)
    return W4Linear(torch.from_numpy(qw).to(dev()), torch.from_numpy(s).to(dev()), K)


def test_fused_argmax_matches_first_max_argmax_with_ties():
    N, K, M = 19000, 512, 96
    lin = _lm_head(N, K, 3)
    g = torch.Generator().manual_seed(4)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16).to(dev())
    keys = torch.zeros(M, dtype=torch.int64, device=dev())
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev())
    assert lin.with_argmax(x, out, keys)  # 149 tiles: the stream-K schedule
    k = keys.cpu().numpy().view(np.uint64)
    got = (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64)
    want = torch.argmax(out.float().cpu(), dim=-1).numpy()  # first maximal index
    assert np.array_equal(got, want)
    top1 = torch.empty(M, dtype=torch.int32, device=dev())
    ck.argmax_top2(out, top1)
    assert np.array_equal(got, top1.cpu().numpy())
    # the planted tie decides rows whose maximum is the large row: the smaller index wins
    o = out.float().cpu()
    tied = (o[:, 4321] == o[:, 17001]) & (o[:, 4321] == o.max(dim=-1).values)
    assert int(tied.sum()) > 0 and bool((torch.from_numpy(got)[tied] == 4321).all())


def test_accept_from_keys_equals_accept_from_top1():
    N, K = 19000, 512
    B, q = 32, 3
    M = B * q
    lin = _lm_head(N, K, 5)
    g = torch.Generator().manual_seed(6)
    x = torch.randn((M, K), generator=g).to(torch.bfloat16).to(dev())
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev())
    keys = torch.zeros(M, dtype=torch.int64, device=dev())
    lin(x, out=out)
    top1 = torch.empty(M, dtype=torch.int32, device=dev())
    ck.argmax_top2(out, top1)
    ids = torch.randint(0, N, (M,), generator=g, dtype=torch.int32)
    t1 = top1.cpu()
    for b in range(0, B, 2):  # every other sequence's drafts match, so acceptance happens
        for j in range(q - 1):
            ids[b * q + j + 1] = t1[b * q + j]
    ids = ids.to(dev())
    i32 = dict(dtype=torch.int32, device=dev())
    cu = torch.arange(0, M + 1, q, **i32)
    runs = []
    for fused in (False, True, True):
        acc, nxt = torch.empty(B, **i32), torch.empty(B, **i32)
        ctx = torch.full((B,), 1000, **i32)
        slots = torch.arange(M, **i32)
        if fused:
            assert lin.with_argmax(x, out, keys)
            dec = torch.full((M,), -7, **i32)
            ck.verify_accept_greedy_keys(B, ids, keys, cu, acc, nxt, ctx, slots, top1=dec)
            assert torch.equal(dec.cpu(), t1)
            assert int(keys.abs().sum()) == 0  # reset for the next step
        else:
            ck.verify_accept_greedy(B, ids, top1, cu, acc, nxt, ctx, slots)
        runs.append([t.cpu() for t in (acc, nxt, ctx, slots)])
    for a, b in zip(runs[0], runs[1]):
        assert torch.equal(a, b)
    for a, b in zip(runs[1], runs[2]):
        assert torch.equal(a, b)
    assert int(runs[0][0][::2].min()) == q - 1


def test_verify_step_fused_and_separate_agree():
    shape = Qwen3Shape(hidden=1024, layers=2, n_heads=8, n_kv_heads=4, head_dim=128, intermediate=3072,
                       vocab=32768)
    w = Qwen3Weights.synthetic(shape, 12, dev())
    rng = np.random.default_rng(9)
    prompts = [[int(t) for t in rng.integers(0, shape.vocab, n)] for n in (20, 35, 17, 40, 22, 31, 26, 18)]
    drafts = [[int(t) for t in rng.integers(0, shape.vocab, 2)] for _ in prompts]
    runs = []
    for fuse in (False, True):
        kv = PagedKVCache(w.shape, 64, dev())
        ver = Qwen3Verifier(w, kv, max_rows=128, max_pos=256, device=dev())
        ver.fuse_lm_argmax = fuse
        eng = MTPVerifyEngine(ver, num_blocks=64, max_model_len=256, max_num_batched_tokens=128,
                              page_aligned_chunks=False)
        sids = [eng.add_request(p, max_new_tokens=8) for p in prompts]
        eng.prefill()
        out = []
        for step in range(2):
            res = eng.verify_step({sid: d for sid, d in zip(sids, drafts)} if step == 0 else {})
            rows = sum(1 + len(r.drafts) for r in res)
            out.append((sorted((r.seq_id, r.accepted, r.next_token) for r in res), ver.top1[:rows].cpu(),
                        ver.logits[:rows].cpu()))
        assert int(ver.row_keys.abs().sum()) == 0
        runs.append(out)
    for (ra, ta, la), (rb, tb, lb) in zip(*runs):
        assert ra == rb and torch.equal(ta, tb) and torch.equal(la, lb)
