"""Rejection-sampling verification through the engine (MTPVerifyEngine with temperature
> 0): the captured verify step draws two uniforms per row, and every sequence's accept
count and next token equal the CPU restatement's (oracle/model.py rejection_accept) on
that step's logits and uniforms; the token lists and computed counts roll back as in the
greedy path.  Parity unpinned: the reference verifies greedily only (engine.py:373-379)."""
import numpy as np
import pytest
import torch

from oracle import model as om
from pilm_b200 import bindings
from pilm_b200.engine import MTPVerifyEngine
from pilm_b200.qwen3 import PagedKVCache, Qwen3Shape, Qwen3Verifier, Qwen3Weights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    bindings.init()
    dev = torch.device("cuda:0")
    cfg = om.Qwen3Config(hidden=256, layers=2, n_heads=8, n_kv_heads=2, intermediate=512, vocab=4096)
    ckpt = om.make_checkpoint(cfg, seed=11)
    shape = Qwen3Shape(hidden=cfg.hidden, layers=cfg.layers, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
                       head_dim=cfg.head_dim, intermediate=cfg.intermediate, vocab=cfg.vocab)
    return dev, shape, Qwen3Weights.from_checkpoint(shape, ckpt, dev)


def _engine(model, **kw):
    dev, shape, w = model
    ver = Qwen3Verifier(w, PagedKVCache(shape, 64, dev), max_rows=64, max_pos=512, device=dev)
    return MTPVerifyEngine(ver, num_blocks=64, max_model_len=512, **kw)


def _prompts(vocab):
    rng = np.random.default_rng(5)
    return [[int(t) for t in rng.integers(0, vocab, n)] for n in (19, 7, 30, 13)]


def _check_step(eng, drafts, T, P):
    """One verify step; returns the total accepted drafts."""
    before = {s.seq_id: (list(s.tokens), s.num_computed) for s in eng.sched.running}
    res = eng.verify_step(drafts)
    torch.cuda.synchronize()
    uni = eng.last_uniforms
    logits = eng.v.logits[:uni.shape[0]].float().cpu()
    row, total = 0, 0
    for r in res:
        n = 1 + len(r.drafts)
        a, t = om.rejection_accept(logits[row:row + n], r.drafts, uni[row:row + n, 0].tolist(),
                                   uni[row:row + n, 1].tolist(), T, P)
        assert (r.accepted, r.next_token) == (a, t), (r, a, t)
        toks, comp = before[r.seq_id]
        s = eng.sched.seqs[r.seq_id]
        assert s.tokens == toks + r.drafts[:a] + [t]
        assert s.num_computed == comp + 1 + a
        row += n
        total += a
    return total


def test_sampled_verify_steps_match_restatement(model):
    """Config 3's T = 0.8, top-p 0.95 with random drafts (the sample-from-residual path)."""
    T, P = 0.8, 0.95
    eng = _engine(model, temperature=T, top_p=P, sample_seed=3)
    vocab = model[1].vocab
    for p in _prompts(vocab):
        eng.add_request(p, 64)
    eng.prefill()
    g = torch.Generator().manual_seed(9)
    for _ in range(4):
        drafts = {s.seq_id: torch.randint(0, vocab, (3,), generator=g).tolist() for s in eng.sched.running}
        _check_step(eng, drafts, T, P)
    assert len(eng.graphs) >= 1  # the sampled step ran from a captured graph


def test_sampled_verify_accepts_likely_drafts(model):
    """At a low temperature the greedy continuation is nearly certain: drafts taken from a
    greedy engine's next tokens are accepted, and each decision still equals the
    restatement's."""
    greedy = _engine(model)
    vocab = model[1].vocab
    prompts = _prompts(vocab)
    for p in prompts:
        greedy.add_request(p, 64)
    greedy.prefill()
    cont = {s.seq_id: [] for s in greedy.sched.running}
    for _ in range(3):
        for r in greedy.verify_step({}):
            cont[r.seq_id].append(r.next_token)
    T, P = 0.05, 0.9
    eng = _engine(model, temperature=T, top_p=P, sample_seed=4)
    for p in prompts:
        eng.add_request(p, 64)
    eng.prefill()  # the same greedy first token as the greedy engine's
    drafts = {sid: cont[sid][:2] for sid in cont}
    assert _check_step(eng, drafts, T, P) > 0
