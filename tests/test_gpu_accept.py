"""GPU acceptance kernels: row top-2, greedy accept + rollback, rejection sampling
against the oracle restatement with identical uniforms."""
import numpy as np
import pytest
import torch

from oracle import model as om
from pilm_b200 import bindings as abi
from pilm_b200 import ckernel as ck
from tests._gpu import dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    abi.init()
    yield


def test_top2_matches_torch_first_max():
    g = torch.Generator().manual_seed(0)
    x = torch.randn((37, 151936), generator=g)
    x[3, 1000] = x[3, 2000] = 50.0  # tie -> first index
    top1 = torch.empty(37, dtype=torch.int32, device=dev())
    margin = torch.empty(37, dtype=torch.float32, device=dev())
    ck.argmax_top2(x.to(dev()), top1, None, margin)
    assert top1.cpu().tolist() == torch.argmax(x, -1).tolist()
    t = torch.topk(x, 2, -1).values
    assert torch.allclose(margin.cpu(), t[:, 0] - t[:, 1])
    xb = x.to(torch.bfloat16)
    ck.argmax_top2(xb.to(dev()), top1, None, None)
    assert top1.cpu().tolist() == torch.argmax(xb.float(), -1).tolist()


@pytest.mark.parametrize("V", [1, 3, 7, 9, 1001, 32003])
def test_top2_ragged_vocab_unaligned_rows(V):
    """Vocabularies that leave rows off 16-byte boundaries: the scalar head and tail and
    the vector middle agree with torch's first-max argmax, ties across the three included."""
    g = torch.Generator().manual_seed(V)
    x = torch.randn((6, V), generator=g)
    if V >= 3:
        x[1, 0] = x[1, V - 1] = 40.0       # head vs tail
        x[2, V // 2] = x[2, V - 1] = 41.0  # middle vs tail
        x[3, 1] = x[3, V // 2] = 42.0      # head vs middle
    x[4, V - 1] = 43.0
    t = torch.topk(x, min(2, V), -1).values
    for dt in (torch.float32, torch.bfloat16):
        xd = x.to(dt)
        top1 = torch.empty(6, dtype=torch.int32, device=dev())
        margin = torch.empty(6, dtype=torch.float32, device=dev())
        ck.argmax_top2(xd.to(dev()), top1, None, margin)
        assert top1.cpu().tolist() == torch.argmax(xd.float(), -1).tolist()
        if dt == torch.float32 and V >= 2:
            assert torch.allclose(margin.cpu(), t[:, 0] - t[:, 1])


def test_greedy_accept_and_rollback():
    # 4 sequences: full accept, partial, immediate reject, no drafts
    cu = [0, 4, 8, 11, 12]
    ids = [5, 10, 11, 12, 6, 20, 21, 22, 7, 30, 31, 8]
    top1 = [10, 11, 12, 99, 20, 77, 0, 0, 1, 2, 3, 44]
    ctx = [104, 36, 23, 50]
    i32 = dict(dtype=torch.int32, device=dev())
    acc = torch.empty(4, **i32)
    nxt = torch.empty(4, **i32)
    c = torch.tensor(ctx, **i32)
    slots = torch.arange(12, **i32)
    ck.verify_accept_greedy(4, torch.tensor(ids, **i32), torch.tensor(top1, **i32), torch.tensor(cu, **i32), acc,
                            nxt, c, slots)
    assert acc.cpu().tolist() == [3, 1, 0, 0]
    assert nxt.cpu().tolist() == [99, 77, 1, 44]
    assert c.cpu().tolist() == [104, 34, 21, 50]
    s = slots.cpu().tolist()
    assert s[:4] == [0, 1, 2, 3] and s[4:8] == [4, 5, -1, -1] and s[8:11] == [8, -1, -1] and s[11] == 11


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_rejection_sampling_decisions_match_oracle(seed):
    g = torch.Generator().manual_seed(seed)
    B, k, V = 6, 3, 5000
    logits = torch.randn((B * (k + 1), V), generator=g) * 4
    uni = torch.rand((B * (k + 1), 2), generator=g)
    ids = torch.randint(0, V, (B * (k + 1),), generator=g)
    # make some drafts the argmax so that acceptance happens
    for r in range(0, B * (k + 1), 2):
        if (r + 1) % (k + 1):
            ids[r + 1] = torch.argmax(logits[r])
    cu = list(range(0, B * (k + 1) + 1, k + 1))
    i32 = dict(dtype=torch.int32, device=dev())
    acc = torch.empty(B, **i32)
    nxt = torch.empty(B, **i32)
    ctx = torch.full((B,), 100, **i32)
    ck.verify_accept_rejection(B, logits.to(dev()), ids.to(torch.int32).to(dev()), torch.tensor(cu, **i32),
                               uni.to(dev()), 0.8, 0.95, acc, nxt, ctx)
    for b in range(B):
        rows = slice(cu[b], cu[b + 1])
        drafts = ids[rows][1:].tolist()
        a, t = om.rejection_accept(logits[rows], drafts, uni[rows, 0].tolist(), uni[rows, 1].tolist(), 0.8, 0.95)
        assert int(acc[b]) == a
        assert int(nxt[b]) == t
        assert int(ctx[b]) == 100 - (k + 1) + 1 + a


@pytest.mark.parametrize("seed", [3, 4])
def test_rejection_sampling_bf16_logits_vocab_151936(seed):
    """The LM head's bf16 logits at the Qwen3 vocabulary, ragged rows per sequence (q_len 1
    to 4, config 3's k = 3), T = 0.8 and top-p 0.95: accept counts, next tokens and the
    rollback equal the oracle restatement's given the same uniforms (parity unpinned: the
    reference has no rejection sampling).  Half the drafts are their row's argmax so that
    acceptance happens; logits scaled so the nucleus is a few hundred tokens."""
    g = torch.Generator().manual_seed(seed)
    qlens = [1, 2, 3, 4, 4, 3, 2, 4, 4, 1, 4, 3]
    B, V, T, P = len(qlens), 151936, 0.8, 0.95
    cu = [0]
    for n in qlens:
        cu.append(cu[-1] + n)
    R = cu[-1]
    logits = (torch.randn((R, V), generator=g) * 6).to(torch.bfloat16)
    uni = torch.rand((R, 2), generator=g)
    ids = torch.randint(0, V, (R,), generator=g)
    am = torch.argmax(logits.float(), -1)
    for b in range(0, B, 2):
        for j in range(qlens[b] - 1):
            ids[cu[b] + j + 1] = am[cu[b] + j]
    i32 = dict(dtype=torch.int32, device=dev())
    acc, nxt = torch.empty(B, **i32), torch.empty(B, **i32)
    ctx = torch.full((B,), 1000, **i32)
    slots = torch.arange(R, **i32)
    ids_d, cu_d, uni_d = ids.to(torch.int32).to(dev()), torch.tensor(cu, **i32), uni.to(dev())
    ck.verify_accept_rejection(B, logits.to(dev()), ids_d, cu_d, uni_d, T, P, acc, nxt, ctx, slots)
    # the fp32 entry point on the same values gives the same decisions
    acc2, nxt2 = torch.empty(B, **i32), torch.empty(B, **i32)
    ctx2 = torch.full((B,), 1000, **i32)
    ck.verify_accept_rejection(B, logits.float().to(dev()), ids_d, cu_d, uni_d, T, P, acc2, nxt2, ctx2)
    assert acc.tolist() == acc2.tolist() and nxt.tolist() == nxt2.tolist()
    accepted = 0
    for b in range(B):
        rows = slice(cu[b], cu[b + 1])
        drafts = ids[rows][1:].tolist()
        a, t = om.rejection_accept(logits[rows].float(), drafts, uni[rows, 0].tolist(), uni[rows, 1].tolist(), T, P)
        assert (int(acc[b]), int(nxt[b])) == (a, t), b
        assert int(ctx[b]) == 1000 - qlens[b] + 1 + a
        s = slots.cpu().tolist()[rows]
        assert s[:1 + a] == list(range(cu[b], cu[b] + 1 + a)) and all(v == -1 for v in s[1 + a:])
        accepted += a
    assert accepted > 0
