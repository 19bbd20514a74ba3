"""bench.greedy_rollout on the host, with a stand-in greedy model: drafts taken from the
model's own continuation are all accepted (up to the page-boundary cap), the sequences
advance by k + 1 tokens per step, and the tokens they end up with equal a plain
one-token-per-step run of the same model.  The stand-in's greedy token depends only on
(token, position), like a deterministic model whose rows do not depend on the batch."""
import bench
from pilm_b200.engine import MTPVerifyEngine

V = 1000


def _top1(tok: int, pos: int) -> int:
    return (tok * 31 + pos * 7 + 3) % V


class _FakeVerifier:
    device = "cpu"

    def verify_greedy(self, b, acc, nxt, ctx):
        """The greedy accept rule (engine.py:479-503) over _top1 of every verify row."""
        ids, pos, cu = b.ids.tolist(), b.positions.tolist(), b.cu_q.tolist()
        top = [_top1(t, p) for t, p in zip(ids, pos)]
        for i in range(len(cu) - 1):
            q0, n = cu[i], cu[i + 1] - cu[i]
            a = 0
            while a < n - 1 and top[q0 + a] == ids[q0 + a + 1]:
                a += 1
            acc[i] = a
            nxt[i] = top[q0 + a]
            ctx[i] = ctx[i] - n + 1 + a


def _engine(prompts):
    eng = MTPVerifyEngine(_FakeVerifier(), num_blocks=400, pin_memory=False, max_model_len=1024,
                          use_graphs=False)
    for p in prompts:
        sid = eng.add_request(list(p), max_new_tokens=400)
        eng.admit_prefilled(sid)
    for s in eng.sched.running:  # the first generated token, pending
        t = _top1(s.tokens[-1], len(s.tokens) - 1)
        s.tokens.append(t)
        s.outputs.append(t)
    return eng


def test_rollout_drafts_are_accepted_and_match_plain_decoding():
    prompts = [range(5, 5 + n) for n in (40, 61, 77)]
    k, steps = 2, 12
    eng = _engine(prompts)
    before = {s.seq_id: (list(s.tokens), s.num_computed, len(s.pages)) for s in eng.sched.running}
    drafts = bench.greedy_rollout(eng, steps * (k + 1) + 2, k)
    for s in eng.sched.running:  # rewound to where it started, pages kept
        toks, nc, npg = before[s.seq_id]
        assert s.tokens == toks and s.num_computed == nc and len(s.pages) >= npg
    att = acc = 0
    for _ in range(steps):
        d = drafts()
        for r in eng.verify_step(d):
            assert r.accepted == len(r.drafts)
            att += len(r.drafts)
            acc += r.accepted
    assert acc == att and att > steps * len(prompts)  # most steps verify k drafts

    ref = _engine(prompts)
    total = max(len(s.tokens) for s in eng.sched.running)
    while min(len(s.tokens) for s in ref.sched.running) < total:
        ref.verify_step({})
    for s, r in zip(eng.sched.running, ref.sched.running):
        assert s.tokens == r.tokens[:len(s.tokens)]
        assert s.num_computed == len(s.tokens) - 1


def test_rollout_leaves_engine_stats_consistent():
    eng = _engine([range(3, 50)])
    drafts = bench.greedy_rollout(eng, 9, 2)
    n0 = len(eng.sched.running[0].tokens)
    res = eng.verify_step(drafts())
    assert res[0].accepted == len(res[0].drafts)
    assert len(eng.sched.running[0].tokens) == n0 + 1 + res[0].accepted
