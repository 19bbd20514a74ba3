"""Batched MTP speculative-verify engine on the B200 kernels.

The reference runs one request per forward (src/engine.py:416-472); this engine
verifies many sequences per step with the same per-sequence rules:

* drafts appended per step are capped at
  min(remaining output, tokens left in the current page - 1, pending drafts)
  (engine.py:399-401), so verify rows never cross a page;
* the verify rows are [last token, d1..dn] at positions num_computed..;
* greedy acceptance counts leading drafts equal to the row argmax; the next
  token is the argmax of the first mismatching row or of the bonus row
  (engine.py:479-503, 551-557);
* on rejection the sequence is rolled back to start + 1 + accepted tokens
  (engine.py:505-510).  The page table is unchanged (no page boundary is ever
  crossed).  The reference then re-runs the accepted prefix to refresh state;
  for full-attention Qwen3 the verify pass already wrote identical K/V for those
  rows and the accepted row's hidden state equals the re-run's (bit-identical in
  bf16, checked against the reference), so no re-run is done here.

Prefill runs through the same forward in page-aligned chunks of at most one
page per sequence per pass (engine.py:218 uses 16-token chunks), or can be
skipped for synthetic benchmarks whose KV pages are filled directly.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import ckernel as ck
from .paging import PageTableManager, Sequence, Status, VerifyScheduler
from .qwen3 import Qwen3Verifier, VerifyBatch, VerifyGraph


def draft_limit(num_computed: int, block_size: int, remaining_output: int, n_pending: int) -> int:
    """engine.py:399-401."""
    block_remaining = block_size - (num_computed % block_size)
    return max(0, min(remaining_output, block_remaining - 1, n_pending))


@dataclass
class StepResult:
    seq_id: int
    drafts: list[int]
    accepted: int
    next_token: int


class MTPVerifyEngine:
    def __init__(self, verifier: Qwen3Verifier, num_blocks: int, block_size: int = 16, max_model_len: int = 65536,
                 max_pages_per_seq: Optional[int] = None, pin_memory: bool = True,
                 max_num_batched_tokens: int = 1 << 30, use_graphs: bool = True, drafter=None, draft_k: int = 0,
                 page_aligned_chunks: bool = True, temperature: float = 0.0, top_p: float = 1.0,
                 sample_seed: int = 0):
        """max_num_batched_tokens is the scheduler's per-pass token budget; the reference
        engine uses one page (16, engine.py:218), which also fixes its page order.
        page_aligned_chunks=False lets a prefill pass run past page boundaries (a long
        prompt in budget-sized passes; the verifier's max_rows must cover the budget);
        the default keeps the reference's one-page chunks and page order.
        use_graphs replays each verify-step shape (sequences, rows) from a captured CUDA
        graph instead of launching ~15 kernels per layer from Python.
        drafter (pilm_b200.mtp.MTPDrafter) with draft_k > 0 drafts each sequence's next
        tokens on the GPU right after its verify step (in the same graph); verify_step()
        without explicit drafts then uses them, as the reference's speculative loop does
        with pending_mtp_draft_ids (engine.py:380-408, 527-557).
        temperature > 0 verifies by rejection sampling from the top-p nucleus of
        softmax(logits / temperature) instead of greedily (the reference is greedy-only,
        engine.py:373-379): each step draws two uniforms per verify row, (accept test,
        sample), from a generator seeded with sample_seed, so a run is reproducible and
        the same uniforms can be fed to a CPU restatement (``last_uniforms``)."""
        self.v = verifier
        self.device = verifier.device
        self.block_size = block_size
        self.pages = PageTableManager(num_blocks, block_size)
        mp = max_pages_per_seq or (max_model_len + block_size - 1) // block_size
        self.max_pages = mp
        self.sched = VerifyScheduler(self.pages, max_num_batched_tokens=max_num_batched_tokens, max_num_seqs=1 << 20,
                                     max_model_len=max_model_len, max_pages_per_seq=mp,
                                     page_aligned_chunks=page_aligned_chunks)
        self._next_id = 0
        self.max_model_len = max_model_len
        self.use_graphs = use_graphs
        self.graphs: dict[tuple[int, int, int], VerifyGraph] = {}
        self.pin = pin_memory and torch.cuda.is_available()
        self.stats = {"attempts": 0, "accepts": 0, "rejects": 0, "steps": 0, "verified_rows": 0}
        # host side of the verify step: per-sequence page rows kept as int32 arrays and
        # extended in place (page lists only grow until they are released), and pinned
        # staging buffers reused every step
        self._page_rows: dict[int, tuple[int, np.ndarray, int]] = {}
        self._staging: dict[str, torch.Tensor] = {}
        self.drafter = drafter if draft_k > 0 else None
        self.draft_k = draft_k if self.drafter is not None else 0
        if self.drafter is not None and not use_graphs:
            raise ValueError("the GPU drafter runs inside the captured verify step (use_graphs=True)")
        self.pending: dict[int, list[int]] = {}  # next step's drafts per sequence (from the drafter)
        if temperature < 0 or not 0 < top_p <= 1:
            raise ValueError("temperature must be >= 0 and top_p in (0, 1]")
        self.sampling = (float(temperature), float(top_p)) if temperature > 0 else None
        self._rng = torch.Generator().manual_seed(sample_seed)
        self.last_uniforms: Optional[torch.Tensor] = None  # [total_q, 2] of the latest sampled step
        self._uniforms_staged: Optional[torch.Tensor] = None

    # ---- admission -------------------------------------------------------------------
    def add_request(self, prompt: list[int], max_new_tokens: int = 256, eos_token_id: int = -1) -> int:
        sid = self._next_id
        self._next_id += 1
        self.sched.add(Sequence(sid, list(prompt), max_new_tokens, eos_token_id))
        return sid

    def admit_prefilled(self, sid: int) -> None:
        """Benchmark admission: take the pages of the whole prompt and mark it computed,
        assuming its K/V are already in the pool (synthetic KV)."""
        seq = self.sched.seqs[sid]
        self.sched.waiting.remove(seq)
        if self.pages.allocate(seq, seq.num_tokens, self.max_pages) is None:
            raise RuntimeError("KV pool exhausted")
        seq.num_computed = seq.num_tokens
        seq.status = Status.RUNNING
        self.sched.running.append(seq)

    # ---- batch construction ------------------------------------------------------------
    def _tensor(self, data, dtype=torch.int32) -> torch.Tensor:
        t = torch.tensor(data, dtype=dtype, pin_memory=self.pin)
        return t.to(self.device, non_blocking=True)

    def _page_row(self, s: Sequence) -> np.ndarray:
        """The sequence's page list as int32, zero-padded to max_pages; rebuilt only after
        the list was released, otherwise extended by the pages appended since."""
        n = len(s.pages)
        c = self._page_rows.get(s.seq_id)
        if c is None or c[0] != s.page_gen or c[2] > n or c[1].shape[0] < n:
            arr = np.zeros(max(self.max_pages, n), dtype=np.int32)
            arr[:n] = s.pages
            self._page_rows[s.seq_id] = (s.page_gen, arr, n)
            return arr
        gen, arr, m = c
        if m < n:
            arr[m:n] = s.pages[m:n]
            self._page_rows[s.seq_id] = (gen, arr, n)
        return arr

    def _stage(self, name: str, shape: tuple[int, ...]) -> torch.Tensor:
        """A pinned int32 host buffer of at least this shape (a view of it)."""
        numel = int(np.prod(shape))
        t = self._staging.get(name)
        if t is None or t.numel() < numel:
            t = torch.empty(max(numel, 1), dtype=torch.int32, pin_memory=self.pin)
            self._staging[name] = t
        return t[:numel].view(shape)

    def build_batch(self, seqs: list[Sequence], starts: list[int], counts: list[int],
                    on_device: bool = True) -> VerifyBatch:
        if not on_device:
            return self._build_host_batch(seqs, starts, counts)
        ids, pos, slots, cu = [], [], [], [0]
        bs = self.block_size
        maxp = max(1, max(len(s.pages) for s in seqs))
        table = []
        ctx = []
        for s, st, n in zip(seqs, starts, counts):
            ids.extend(s.tokens[st:st + n])
            pos.extend(range(st, st + n))
            slots.extend(s.pages[p // bs] * bs + p % bs for p in range(st, st + n))
            cu.append(cu[-1] + n)
            table.append(s.pages + [0] * (maxp - len(s.pages)))
            ctx.append(st + n)
        mk = self._tensor if on_device else (lambda d: torch.tensor(d, dtype=torch.int32, pin_memory=self.pin))
        return VerifyBatch(ids=mk(ids), positions=mk(pos), slots=mk(slots), block_table=mk(table), cu_q=mk(cu),
                           context_lens=mk(ctx), max_q_len=max(counts), max_context=max(ctx))

    def _build_host_batch(self, seqs: list[Sequence], starts: list[int], counts: list[int]) -> VerifyBatch:
        """The verify step's metadata in pinned host buffers (copied to the graph's device
        buffers by VerifyGraph.load).  The buffers are rewritten by the next step, which
        starts only after this step's results were read back, so after its copies."""
        bs = self.block_size
        B = len(seqs)
        T = int(sum(counts))
        maxp = max(1, max(len(s.pages) for s in seqs))
        ids, pos, slots = self._stage("ids", (T,)), self._stage("pos", (T,)), self._stage("slots", (T,))
        cu, ctx = self._stage("cu", (B + 1,)), self._stage("ctx", (B,))
        table = self._stage("table", (B, maxp))
        ids_n, pos_n, slots_n = ids.numpy(), pos.numpy(), slots.numpy()
        cu_n, ctx_n, table_n = cu.numpy(), ctx.numpy(), table.numpy()
        cnt = np.asarray(counts, dtype=np.int32)
        st = np.asarray(starts, dtype=np.int32)
        cu_n[0] = 0
        np.cumsum(cnt, out=cu_n[1:])
        np.add(st, cnt, out=ctx_n)
        for i, s in enumerate(seqs):
            table_n[i] = self._page_row(s)[:maxp]
        ids_n[:] = np.fromiter(itertools.chain.from_iterable(s.tokens[a:a + n] for s, a, n in zip(seqs, starts, counts)),
                               dtype=np.int32, count=T)
        # row r of sequence b sits at position starts[b] + (r - cu[b])
        seq_of_row = np.repeat(np.arange(B), cnt)
        p = np.arange(T, dtype=np.int32) + np.repeat(st - cu_n[:-1], cnt)
        pos_n[:] = p
        slots_n[:] = table_n[seq_of_row, p // bs] * bs + p % bs
        return VerifyBatch(ids=ids, positions=pos, slots=slots, block_table=table, cu_q=cu, context_lens=ctx,
                           max_q_len=max(counts), max_context=int(ctx_n.max()))

    def graph_for(self, b: VerifyBatch) -> VerifyGraph:
        """Captured verify step for this batch shape; captured on first use (the capture
        runs the step once eagerly on the loaded batch, which the replay then repeats
        with identical results: K/V writes and the rollback are idempotent)."""
        key = (b.num_seqs, b.total_q, b.max_q_len)
        g = self.graphs.get(key)
        if g is None:
            g = VerifyGraph(self.v, b.num_seqs, b.total_q, b.max_q_len, self.max_pages, self.max_model_len,
                            self.drafter, self.draft_k, self.sampling)
            g.load(b, self._uniforms_staged)
            g.capture()
            self.graphs[key] = g
        else:
            g.load(b, self._uniforms_staged)
        return g

    def _draw_uniforms(self, rows: int) -> None:
        """This step's uniforms [rows, 2] (accept test, sample) from the engine's generator,
        in a pinned staging buffer (the graph copies them in with the batch)."""
        self._uniforms_staged = None
        if self.sampling is None:
            return
        u = torch.rand((rows, 2), generator=self._rng)
        self.last_uniforms = u
        st = self._staging.get("uniforms")
        if st is None or st.numel() < 2 * rows:
            st = torch.empty(max(2 * rows, 1024), dtype=torch.float32, pin_memory=self.pin)
            self._staging["uniforms"] = st
        st = st[:2 * rows].view(rows, 2)
        st.copy_(u)
        self._uniforms_staged = st

    # ---- prefill ----------------------------------------------------------------------
    def prefill(self) -> dict[int, int]:
        """Run every waiting prompt through the model in page-aligned chunks and take
        the greedy first token of each.  First tokens are appended only after every
        prompt is done, so no decode rows are mixed into the prefill passes.
        Returns {seq_id: first_token}."""
        first = {}
        while self.sched.waiting or any(s.is_prefill for s in self.sched.running):
            out = self.sched.schedule()
            if out.is_empty:
                raise RuntimeError("prefill could not be scheduled (KV pool too small?)")
            seqs = [self.sched.seqs[c.seq_id] for c in out.scheduled]
            starts = [c.positions[0] for c in out.scheduled]
            counts = [c.num_tokens for c in out.scheduled]
            b = self.build_batch(seqs, starts, counts)
            h = self.v.forward(b)
            done = [i for i, c in enumerate(out.scheduled) if not c.is_prefill_chunk]
            if done:
                ends = [sum(counts[:i + 1]) - 1 for i in done]
                rows = torch.tensor(ends, device=self.device)
                logits = self.v.lm_head(h.index_select(0, rows).contiguous())
                top = torch.argmax(logits.float(), dim=-1).tolist()
                for j, i in enumerate(done):
                    first[out.scheduled[i].seq_id] = int(top[j])
        for sid, t in first.items():
            s = self.sched.seqs[sid]
            s.tokens.append(t)
            s.outputs.append(t)
        return first

    # ---- the verify step --------------------------------------------------------------
    def verify_step(self, drafts: Optional[dict[int, list[int]]] = None) -> list[StepResult]:
        """One MTP verify step over every running sequence in decode state.  Without
        explicit drafts each sequence verifies the drafts the GPU drafter produced in its
        previous step (none before its first step)."""
        if drafts is None:
            drafts = self.pending
        seqs, starts, counts, used = [], [], [], []
        for s in list(self.sched.running):
            if s.num_uncomputed != 1 or s.is_prefill:
                continue
            d = drafts.get(s.seq_id, [])
            remaining = s.max_new_tokens - len(s.outputs)
            n = draft_limit(s.num_computed, self.block_size, remaining, len(d))
            d = [int(t) for t in d[:n]]
            s.tokens.extend(d)
            if self.pages.allocate(s, 1 + n, self.max_pages) is None:
                del s.tokens[len(s.tokens) - n:]
                continue
            seqs.append(s)
            starts.append(s.num_computed)
            counts.append(1 + n)
            used.append(d)
        if not seqs:
            return []
        B = len(seqs)
        new_drafts = None
        self._draw_uniforms(int(sum(counts)))
        if self.use_graphs:
            b = self.build_batch(seqs, starts, counts, on_device=False)
            g = self.graph_for(b)
            g.replay()
            new_drafts = g.drafts if self.draft_k else None
            res = g.results.to("cpu").tolist()  # accept counts, next tokens, drafts: one copy
        else:
            b = self.build_batch(seqs, starts, counts)
            acc = torch.empty(B, dtype=torch.int32, device=self.device)
            nxt = torch.empty(B, dtype=torch.int32, device=self.device)
            ctx = b.context_lens.clone()
            if self.sampling:
                self.v.verify_sampled(b, self._uniforms_staged.to(self.device), self.sampling[0], self.sampling[1],
                                      acc, nxt, ctx)
            else:
                self.v.verify_greedy(b, acc, nxt, ctx)
            res = torch.stack([acc, nxt]).to("cpu").tolist()
        if new_drafts is not None:
            self.pending = {s.seq_id: [int(res[2 + j][i]) for j in range(self.draft_k)] for i, s in enumerate(seqs)}
        out = []
        for i, s in enumerate(seqs):
            a, t = int(res[0][i]), int(res[1][i])
            st, d = starts[i], used[i]
            accepted = d[:a]
            del s.tokens[st + 1:]
            s.tokens.extend(accepted)
            s.outputs.extend(accepted)
            s.num_computed = st + 1 + a
            s.tokens.append(t)
            s.outputs.append(t)
            self.stats["attempts"] += min(len(d), a + 1)
            self.stats["accepts"] += a
            self.stats["rejects"] += 1 if a < len(d) else 0
            out.append(StepResult(s.seq_id, d, a, t))
        self.stats["steps"] += 1
        self.stats["verified_rows"] += b.total_q
        finished = [s for s in seqs if self.sched._check_stop(s)]
        for s in finished:
            self.sched.running.remove(s)
            self.pages.free(s)
            self._page_rows.pop(s.seq_id, None)
            self.pending.pop(s.seq_id, None)
        return out
