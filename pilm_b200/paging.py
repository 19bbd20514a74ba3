"""Host-side paging for the verify path: page pool, per-request page tables,
scheduling of verify rows.

Behaviour follows the reference scheduler package (src/runtime/scheduler/):
page ids handed out must be identical to the reference's for the same request
sequence, because page tables and slot mappings are compared bit for bit.
The decisions that fix those ids:

* pool: page 0 is reserved as the null page; free pages are taken from the
  front of an LRU list; freed pages without a prefix hash go to the FRONT in
  reverse order of the free call, hashed pages to the BACK
  (block_pool.py:27-30, 39-80; block.py:55-117);
* a request needs ceil((num_computed + new) / page) pages; missing pages are
  taken when scheduled (kv_cache_manager.py:42-94);
* a chunk never crosses a page boundary and the scheduler's token budget is
  shared in running-then-waiting FCFS order; on a failed allocation the newest
  running request is preempted (RECOMPUTE: pages freed, progress reset, put at
  the front of the waiting queue) (scheduler.py:70-211).

The implementation is this module's own: an OrderedDict free list and plain
lists instead of the reference's linked-list objects.  Prefix caching (hash
chains) is not needed by the verify path and is not implemented here.
"""
from __future__ import annotations

from collections import OrderedDict, deque
from dataclasses import dataclass, field
from typing import Optional

DEFAULT_BLOCK_SIZE = 16


class PagePool:
    def __init__(self, num_blocks: int, block_size: int = DEFAULT_BLOCK_SIZE):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.ref = [0] * num_blocks
        self._free: OrderedDict[int, None] = OrderedDict((i, None) for i in range(num_blocks))
        self.null_block = None
        if num_blocks > 0:
            self.null_block, _ = self._free.popitem(last=False)

    @property
    def num_free(self) -> int:
        return len(self._free)

    def take(self, n: int) -> list[int]:
        if n > len(self._free):
            return []
        out = []
        for _ in range(n):
            b, _ = self._free.popitem(last=False)
            self.ref[b] = 1
            out.append(b)
        return out

    def release(self, pages: list[int]) -> None:
        """Decrement reference counts; pages reaching zero rejoin the free list at the
        front, the last released page first (no prefix hashes are kept)."""
        for b in pages:
            if b == self.null_block or b < 0 or b >= self.num_blocks:
                continue
            self.ref[b] -= 1
            if self.ref[b] <= 0:
                self.ref[b] = 0
                self._free[b] = None
                self._free.move_to_end(b, last=False)


class Status:
    WAITING = 1
    RUNNING = 2
    PREEMPTED = 3
    FINISHED_STOPPED = 4
    FINISHED_LENGTH_CAPPED = 5
    FINISHED_ABORTED = 6


@dataclass
class Sequence:
    """One request's token stream and page table (request.py:33-61)."""
    seq_id: int
    prompt: list[int]
    max_new_tokens: int = 256
    eos_token_id: int = -1
    tokens: list[int] = field(default_factory=list)
    outputs: list[int] = field(default_factory=list)
    num_computed: int = 0
    pages: list[int] = field(default_factory=list)
    status: int = Status.WAITING
    pending_drafts: list[int] = field(default_factory=list)
    page_gen: int = 0  # bumped whenever the page list is released (pages only grow between)

    def __post_init__(self):
        if not self.tokens:
            self.tokens = list(self.prompt)

    @property
    def num_tokens(self) -> int:
        return len(self.tokens)

    @property
    def num_uncomputed(self) -> int:
        return self.num_tokens - self.num_computed

    @property
    def is_prefill(self) -> bool:
        return self.num_computed < len(self.prompt)

    def slot(self, pos: int, block_size: int) -> int:
        return self.pages[pos // block_size] * block_size + pos % block_size


class PageTableManager:
    """allocate_slots / free_request_blocks (kv_cache_manager.py:42-113) without caching."""

    def __init__(self, num_blocks: int, block_size: int = DEFAULT_BLOCK_SIZE):
        self.block_size = block_size
        self.pool = PagePool(num_blocks, block_size)

    def allocate(self, seq: Sequence, num_new: int, max_pages: int = 512) -> Optional[list[int]]:
        need = (seq.num_computed + num_new + self.block_size - 1) // self.block_size - len(seq.pages)
        if need + len(seq.pages) > max_pages:
            return None
        if need > self.pool.num_free:
            return None
        new = self.pool.take(need) if need > 0 else []
        if need > 0 and len(new) < need:
            self.pool.release(new)
            return None
        seq.pages.extend(new)
        return new

    def free(self, seq: Sequence) -> None:
        self.pool.release(list(seq.pages))
        seq.pages = []
        seq.page_gen += 1


@dataclass
class ScheduledChunk:
    seq_id: int
    num_tokens: int
    pages: list[int]
    positions: list[int]
    is_prefill: bool
    is_prefill_chunk: bool = False


@dataclass
class ScheduleResult:
    scheduled: list[ScheduledChunk] = field(default_factory=list)
    preempted: list[int] = field(default_factory=list)
    finished: list[int] = field(default_factory=list)

    @property
    def is_empty(self) -> bool:
        return not self.scheduled


class VerifyScheduler:
    """FCFS continuous batching with page-aligned chunks (scheduler.py:70-235).

    page_aligned_chunks=False lifts the reference's rule that a pass ends each sequence's
    chunk at its current page boundary (the reference's attention writes a pass's K/V
    inside one page); chunks then take the whole token budget, so a long prompt runs in a
    few large passes instead of one per page.  Page ids stay in allocation order per
    sequence, but with several sequences they interleave differently from the
    reference's."""

    def __init__(self, pages: PageTableManager, max_num_batched_tokens: int = 2048, max_num_seqs: int = 128,
                 max_model_len: int = 8192, max_pages_per_seq: int = 512, page_aligned_chunks: bool = True):
        self.page_aligned_chunks = page_aligned_chunks
        self.pages = pages
        self.block_size = pages.block_size
        self.max_num_batched_tokens = max_num_batched_tokens
        self.max_num_seqs = max_num_seqs
        self.max_model_len = max_model_len
        self.max_pages_per_seq = max_pages_per_seq
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []
        self.seqs: dict[int, Sequence] = {}

    def add(self, seq: Sequence) -> None:
        seq.status = Status.WAITING
        self.waiting.append(seq)
        self.seqs[seq.seq_id] = seq

    def _cap(self, seq: Sequence, num_new: int, budget: int, computed: int) -> int:
        num_new = min(num_new, budget, self.max_model_len - computed - 1)
        if not self.page_aligned_chunks:
            return num_new
        return min(num_new, self.block_size - (computed % self.block_size))

    def schedule(self) -> ScheduleResult:
        out = ScheduleResult()
        budget = self.max_num_batched_tokens
        i = 0
        while i < len(self.running) and budget > 0:
            seq = self.running[i]
            if seq.num_uncomputed <= 0:
                i += 1
                continue
            n = self._cap(seq, seq.num_uncomputed, budget, seq.num_computed)
            if n <= 0:
                i += 1
                continue
            if self.pages.allocate(seq, n, self.max_pages_per_seq) is None:
                self._preempt_for(seq, out)
                break
            is_chunk = seq.is_prefill and n < seq.num_uncomputed
            out.scheduled.append(ScheduledChunk(seq.seq_id, n, list(seq.pages),
                                                list(range(seq.num_computed, seq.num_computed + n)),
                                                seq.is_prefill, is_chunk))
            budget -= n
            seq.num_computed += n
            i += 1
        while self.waiting and len(self.running) < self.max_num_seqs and budget > 0:
            seq = self.waiting[0]
            n_left = seq.num_tokens
            if n_left <= 0:
                self.waiting.popleft()
                seq.status = Status.FINISHED_STOPPED
                out.finished.append(seq.seq_id)
                continue
            n = self._cap(seq, n_left, budget, 0)
            if n <= 0:
                break
            if self.pages.allocate(seq, n, self.max_pages_per_seq) is None:
                if not self._preempt_one(out):
                    break
                head = self.waiting[0] if self.waiting else None
                if head is None or head.status == Status.PREEMPTED:
                    break
                continue
            self.waiting.popleft()
            self.running.append(seq)
            seq.status = Status.RUNNING
            seq.num_computed = 0
            is_chunk = n < seq.num_tokens
            out.scheduled.append(ScheduledChunk(seq.seq_id, n, list(seq.pages), list(range(0, n)), True, is_chunk))
            budget -= n
            seq.num_computed += n
        return out

    def _preempt_for(self, seq: Sequence, out: ScheduleResult) -> bool:
        if len(self.running) <= 1:
            return False
        return self._preempt_one(out, exclude=seq)

    def _preempt_one(self, out: ScheduleResult, exclude: Optional[Sequence] = None) -> bool:
        victim = next((s for s in reversed(self.running) if s is not exclude), None)
        if victim is None:
            return False
        self.running.remove(victim)
        self.pages.free(victim)
        victim.num_computed = 0
        victim.status = Status.PREEMPTED
        self.waiting.appendleft(victim)
        out.preempted.append(victim.seq_id)
        return True

    def update(self, out: ScheduleResult, generated: dict[int, list[int]]) -> None:
        """update_from_output (scheduler.py:213-235) with release of finished requests."""
        finished = []
        for seq in self.running:
            new = generated.get(seq.seq_id, [])
            if new:
                seq.outputs.extend(new)
                seq.tokens.extend(new)
            if self._check_stop(seq):
                finished.append(seq)
        for seq in finished:
            self.running.remove(seq)
            self.pages.free(seq)

    def _check_stop(self, seq: Sequence) -> bool:
        if not seq.outputs:
            return False
        last = seq.outputs[-1]
        if seq.eos_token_id >= 0 and last == seq.eos_token_id:
            seq.status = Status.FINISHED_STOPPED
            return True
        if seq.num_tokens >= self.max_model_len or len(seq.outputs) >= seq.max_new_tokens:
            seq.status = Status.FINISHED_LENGTH_CAPPED
            return True
        return False
