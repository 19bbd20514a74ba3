"""GPU parity at the shapes of the Qwen3-8B verify step the benchmark times (32 query /
8 KV heads, M = 96 verify rows, vocabulary 151936), against the oracle.

* Paged attention (attention.py:68-141) over 8K and 32K contexts with ragged lengths,
  so that the whole-page kernel's per-SM page ranges cut every sequence into pieces
  that are merged in the kernel's second pass.
* The W4A16 g128 tensor-core GEMM (kernels.c:1089-1157) on the two projections that run
  the stream-K schedule, gate/up (4096 -> 24576) and the LM head (4096 -> 151936), in
  the model's k-pair weight layout.  Output rows are independent, so the oracle checks
  a sample: every tile that a CTA's range boundary cuts (its pieces are summed in the
  kernel), rows from all four lane quadrants of each, and two whole tiles.
* Row top-2 over bf16 logits and greedy acceptance (engine.py:479-503) at V = 151936.
"""
import numpy as np
import pytest
import torch

from oracle import kernels as ok
from oracle import model as om
from pilm_b200 import bindings as abi
from pilm_b200 import ckernel as ck
from tests._gpu import assert_bf16_close, bf16_from_bits, bits_of, dev
from tests.test_gpu_attention import run_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    abi.init()
    yield


def _ragged_contexts(n, pages_lo, pages_hi, q, seed):
    """Contexts that end q rows into a page (the verify rows never cross a page)."""
    rng = np.random.default_rng(seed)
    return [int(16 * p + q) for p in rng.integers(pages_lo, pages_hi, n)]


def test_attention_qwen3_8b_heads_8k_ragged():
    """Twelve sequences of 7K-9K keys, k = 2 (three verify rows each, twelve rows per KV
    head): about 34 pages per SM, so every sequence is cut into many pieces."""
    run_case(32, 8, ctxs=_ragged_contexts(12, 440, 570, 3, seed=21), qlens=[3] * 12, seed=21, poison=True)


def test_attention_qwen3_8b_heads_32k():
    """Three sequences of about 32K keys, mixed verify lengths (k = 2 and k = 3)."""
    ctxs = [16 * 2048 + 3, 16 * 2040 + 4, 16 * 1990 + 1]
    run_case(32, 8, ctxs=ctxs, qlens=[3, 4, 1], seed=22, poison=True)


def test_attention_qwen3_8b_heads_8k_q5():
    """Twenty sequences of 7K-9K keys at k = 4 (five verify rows each, twenty rows per KV
    head, more than the whole-page kernel's one 16-row tile)."""
    run_case(32, 8, ctxs=_ragged_contexts(20, 440, 570, 5, seed=23), qlens=[5] * 20, seed=23, poison=True)


def _cut_tiles(N, K, sms):
    """Tiles that a stream-K range boundary [c U / P, ...) cuts, for P = sms CTAs."""
    tiles, G = (N + 127) // 128, K // 128
    U = tiles * G
    cut = set()
    for c in range(1, sms):
        w = c * U // sms
        if w % G:
            cut.add(w // G)
    return sorted(cut), tiles


@pytest.mark.parametrize("N", [24576, 151936])
def test_w4_gemm_stream_k_bench_shapes_m96(N):
    K, M = 4096, 96
    sms = torch.cuda.get_device_properties(dev()).multi_processor_count
    cut, tiles = _cut_tiles(N, K, sms)
    assert tiles >= sms and len(cut) > 0.8 * (sms - 1)  # the stream-K schedule, nearly every boundary mid-tile
    rows = []
    for t in cut + [0, tiles - 1]:
        rows += [t * 128 + r for r in (0, 31, 32, 63, 64, 95, 96, 127)]
    rows += list(range(128, 256))  # one whole tile
    rows = np.array(sorted(set(r for r in rows if r < N)), dtype=np.int64)
    rng = np.random.default_rng(N)
    nib = lambda: (rng.integers(-7, 8, (N, K // 2)) & 0xF).astype(np.uint8)  # int4 in [-7, 7] (ckernel.py:98-161)
    qw = nib() | (nib() << 4)
    s = (rng.random((N, K // 128), dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    ref = ok.linear_w4a16g_bf16(x, qw[rows], s[rows], 128)
    qk = ck.repack_w4_kpairs(torch.from_numpy(qw).to(dev()))
    sd = torch.from_numpy(s).to(dev())
    xd = bf16_from_bits(x)
    rows_d = torch.from_numpy(rows).to(dev())
    for _ in range(2):  # the per-tile arrival counters reset themselves between calls
        y = ck.linear_w4a16g128_bf16(xd, qk, sd, kpairs=True)
        assert_bf16_close(bits_of(y.index_select(1, rows_d)), ref, ulp_frac=0.99)


def test_top2_and_greedy_accept_vocab_151936():
    """32 sequences x 3 verify rows of bf16 logits: the GPU's row argmax is torch's
    first-max argmax, and the accept counts and next tokens equal the engine rule's.
    Every other sequence's drafts are made the row argmaxes, so acceptance happens."""
    B, k, V = 32, 2, 151936
    g = torch.Generator().manual_seed(5)
    logits = (torch.randn((B * (k + 1), V), generator=g) * 3).to(torch.bfloat16)
    ids = torch.randint(0, V, (B * (k + 1),), generator=g)
    am = torch.argmax(logits.float(), -1)
    for b in range(0, B, 2):
        for j in range(k):
            ids[b * (k + 1) + j + 1] = am[b * (k + 1) + j]
    i32 = dict(dtype=torch.int32, device=dev())
    top1 = torch.empty(B * (k + 1), **i32)
    ck.argmax_top2(logits.to(dev()), top1)
    assert top1.cpu().tolist() == am.tolist()
    cu = torch.arange(0, B * (k + 1) + 1, k + 1, **i32)
    acc, nxt = torch.empty(B, **i32), torch.empty(B, **i32)
    ctx = torch.full((B,), 8195, **i32)
    ck.verify_accept_greedy(B, ids.to(torch.int32).to(dev()), top1, cu, acc, nxt, ctx)
    for b in range(B):
        rows = slice(b * (k + 1), (b + 1) * (k + 1))
        a, t = om.greedy_accept(logits[rows].float(), ids[rows][1:].tolist())
        assert (int(acc[b]), int(nxt[b])) == (a, t)
        assert int(ctx[b]) == 8195 - (k + 1) + 1 + a
    assert int(acc.cpu()[::2].min()) == k
