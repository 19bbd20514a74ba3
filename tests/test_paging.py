"""Host paging logic against the reference scheduler's page-table trace."""
import numpy as np

from pilm_b200.engine import draft_limit
from pilm_b200.paging import PagePool, PageTableManager, Sequence, VerifyScheduler
from tests import _golden as G


def test_page_tables_match_reference_scheduler_trace():
    """Replays the request mix of make_golden.paging_trace through VerifyScheduler:
    every scheduled chunk (sequence, size, start, prefill flag, page table) and every
    preemption equals the reference Scheduler/KVCacheManager/BlockPool output."""
    z = G.load("paging.npz")
    nblocks, bs = [int(x) for x in z["pool"]]
    rng = np.random.default_rng(7)
    mgr = PageTableManager(nblocks, bs)
    sched = VerifyScheduler(mgr, max_num_batched_tokens=16, max_num_seqs=8)
    seqs = [Sequence(i + 1, [int(t) for t in rng.integers(0, 1000, int(n))], 6, -1) for i, n in enumerate(z["lens"])]
    for s in seqs:
        sched.add(s)
    rows = []
    for step in range(40):
        out = sched.schedule()
        if out.is_empty:
            break
        gen = {}
        for c in out.scheduled:
            rows.append([step, c.seq_id, c.num_tokens, c.positions[0], int(c.is_prefill)] + (c.pages + [-1] * 8)[:8])
            s = sched.seqs[c.seq_id]
            if not c.is_prefill_chunk and s.num_computed >= len(s.prompt):
                gen[c.seq_id] = [int(rng.integers(0, 1000))]
        for pid in out.preempted:
            rows.append([step, -pid, 0, 0, 0] + [-1] * 8)
        sched.update(out, gen)
    assert np.array_equal(np.array(rows, np.int64), z["rows"])


def test_pool_free_order_is_lifo_for_unhashed_pages():
    p = PagePool(6)
    a = p.take(3)
    assert a == [1, 2, 3]
    p.release([1, 2])
    assert p.take(2) == [2, 1]


def test_verify_rows_never_cross_a_page():
    mgr = PageTableManager(64, 16)
    for computed in range(0, 64):
        for k in range(0, 5):
            n = draft_limit(computed, 16, 100, k)
            assert (computed % 16) + 1 + n <= 16
    s = Sequence(0, list(range(31)))
    s.num_computed = 31
    assert mgr.allocate(s, 1) == [1, 2]


def test_prefill_schedule_and_verify_pages_match_reference_engine():
    """With the reference engine's one-page token budget (engine.py:218) the prefill
    chunk schedule and the page tables of the verify step equal the reference's."""
    for v in G.MODEL_VARIANTS:
        z = G.load(f"model_{v}.npz")
        mgr = PageTableManager(32, 16)
        sch = VerifyScheduler(mgr, max_num_batched_tokens=16, max_num_seqs=1 << 20, max_model_len=256,
                              max_pages_per_seq=16)
        seqs = [Sequence(b, G.ilist(z[f"b{b}.prompt"]), 64) for b in range(G.num_seqs(z))]
        for s in seqs:
            sch.add(s)
        chunks = []
        while sch.waiting or any(s.is_prefill for s in sch.running):
            for c in sch.schedule().scheduled:
                chunks.append([c.seq_id, c.positions[0], c.num_tokens])
        assert chunks == z["prefill_chunks"].tolist()
        for s in seqs:
            s.tokens.append(int(z[f"b{s.seq_id}.first_token"][0]))
            d = G.ilist(z[f"b{s.seq_id}.drafts"])
            assert len(d) == draft_limit(s.num_computed, 16, 64, 3)
            s.tokens.extend(d)
            mgr.allocate(s, 1 + len(d), 16)
            assert s.pages == G.ilist(z[f"b{s.seq_id}.block_ids"])
            slots = [s.slot(p, 16) for p in range(s.num_computed, s.num_computed + 1 + len(d))]
            assert slots == G.ilist(z[f"b{s.seq_id}.slots"])


def test_host_verify_batch_matches_list_build_across_growth_preemption_and_finish():
    """The engine's per-step host metadata (incrementally extended page rows, pinned
    staging buffers) equals a from-scratch build of the same batch, step after step,
    while pages are appended, a sequence is preempted and re-allocated (its page list
    released and rebuilt) and another finishes."""
    import random

    from pilm_b200.engine import MTPVerifyEngine

    class _NoDevice:
        device = "cpu"

    eng = MTPVerifyEngine(_NoDevice(), num_blocks=4000, pin_memory=False, max_model_len=4096)
    rnd = random.Random(1)
    seqs = []
    for i in range(5):
        s = Sequence(i, list(range(100 + 37 * i)), 64)
        eng.pages.allocate(s, s.num_tokens, eng.max_pages)
        s.num_computed = s.num_tokens - 1
        seqs.append(s)

    def scratch_build(seqs, starts, counts):
        bs = eng.block_size
        maxp = max(len(s.pages) for s in seqs)
        ids, pos, slots, table, cu, ctx = [], [], [], [], [0], []
        for s, st, n in zip(seqs, starts, counts):
            ids += s.tokens[st:st + n]
            pos += list(range(st, st + n))
            slots += [s.pages[p // bs] * bs + p % bs for p in range(st, st + n)]
            table.append(s.pages + [0] * (maxp - len(s.pages)))
            cu.append(cu[-1] + n)
            ctx.append(st + n)
        return [ids, pos, slots, table, cu, ctx]

    for step in range(30):
        starts, counts = [], []
        for s in seqs:
            n = rnd.randint(1, 3)
            s.tokens.extend(rnd.randint(0, 999) for _ in range(n - 1))
            assert eng.pages.allocate(s, n, eng.max_pages) is not None
            starts.append(s.num_computed)
            counts.append(n)
        b = eng.build_batch(seqs, starts, counts, on_device=False)
        got = [b.ids.tolist(), b.positions.tolist(), b.slots.tolist(), b.block_table.tolist(), b.cu_q.tolist(),
               b.context_lens.tolist()]
        assert got == scratch_build(seqs, starts, counts), f"step {step}"
        assert b.max_context == max(b.context_lens.tolist()) and b.max_q_len == max(counts)
        for s, st, n in zip(seqs, starts, counts):
            s.num_computed = st + n
            del s.tokens[s.num_computed:]
            s.tokens.append(rnd.randint(0, 999))
        if step == 10:  # preemption: the page list is released, then rebuilt from new pages
            victim = seqs[2]
            eng.pages.free(victim)
            eng.pages.allocate(victim, victim.num_computed + 1, eng.max_pages)
        if step == 20:  # a finished sequence leaves the batch
            eng.pages.free(seqs[4])
            seqs.pop(4)


def test_cross_page_chunks_take_the_whole_budget():
    """page_aligned_chunks=False: a 300-token prompt under a 128-token budget runs in
    chunks of 128, 128 and 44 tokens; each chunk's page table covers its last token, and
    the pages are the same ones the page-aligned schedule allocates for one sequence."""
    def run(aligned):
        mgr = PageTableManager(64, 16)
        sch = VerifyScheduler(mgr, max_num_batched_tokens=128, max_num_seqs=4, max_model_len=1024,
                              page_aligned_chunks=aligned)
        s = Sequence(0, list(range(300)), 8)
        sch.add(s)
        chunks = []
        while sch.waiting or any(q.is_prefill for q in sch.running):
            for c in sch.schedule().scheduled:
                assert len(c.pages) * 16 >= c.positions[-1] + 1
                assert c.positions == list(range(c.positions[0], c.positions[0] + c.num_tokens))
                chunks.append((c.positions[0], c.num_tokens, c.is_prefill_chunk))
        return chunks, list(s.pages)

    chunks, pages = run(False)
    assert chunks == [(0, 128, True), (128, 128, True), (256, 44, False)]
    aligned_chunks, aligned_pages = run(True)
    assert all(n <= 16 - p % 16 for p, n, _ in aligned_chunks)
    assert pages == aligned_pages and len(pages) == 19


def test_attention_slices_cover_every_row_once_with_its_causal_context():
    """attention_slices: every query row of the pass lands in exactly one slice, in place
    and in order; a slice has at most 16 // group rows, all of one sequence; and the
    slice's context ends at its last row, so row r of a sequence with context c and q_len
    rows sees the keys up to position c - q_len + r, as under the reference's mask."""
    from pilm_b200.qwen3 import attention_slices
    rng = np.random.default_rng(4)
    for group in (1, 2, 4, 8, 16):
        ql = rng.integers(1, 70, 9)
        ctx = ql + rng.integers(0, 300, 9)
        cu = np.concatenate([[0], np.cumsum(ql)])
        seq, cu_v, ctx_v, span = attention_slices(cu, ctx, group)
        assert span == 16 // group and cu_v[0] == 0 and cu_v[-1] == cu[-1]
        n = np.diff(cu_v)
        assert (n >= 1).all() and (n <= span).all() and (np.diff(seq) >= 0).all()
        for i, b in enumerate(seq):
            rows = np.arange(cu_v[i], cu_v[i + 1])
            assert (rows >= cu[b]).all() and (rows < cu[b + 1]).all()
            # the slice's last row is row (rows[-1] - cu[b]) of its sequence
            assert ctx_v[i] == ctx[b] - ql[b] + (rows[-1] - cu[b]) + 1
    assert attention_slices(np.arange(0, 2049 * 4, 4), np.full(2049, 100), 4) is None
