"""Continuous-batching scheduler: prefill-first, then batched decode.

Policy parity with ``braidinfer/engine/scheduler.py:42-113``: admit waiting
sequences for prefill up to ``max_num_seqs`` / ``max_num_batched_tokens``,
otherwise decode every running sequence; on page exhaustion preempt the most
recently admitted sequence and re-queue it; stop/EOS tokens are not appended;
finish on stop, EOS, ``max_tokens``.  Differences: pages are allocated on
demand (a page when a sequence crosses a page boundary) instead of reserving
``len + max_tokens`` up front; before preempting, unreferenced chunk KV is
evicted; preemption and finish free only the sequence's private pages (chunk
pages are refcounted); multi-token stop strings are matched on token
suffixes.
"""
from __future__ import annotations

from collections import deque
from typing import List, Tuple

from ..errors import OutOfPagesError
from .page_manager import PageManager
from .sequence import Sequence, SequenceStatus


class Scheduler:
    def __init__(self, config, page_manager: PageManager, eos_ids: List[int]):
        self.max_num_seqs = config.max_num_seqs
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.max_model_len = config.max_model_len
        self.page_manager = page_manager
        self.eos_ids = set(int(e) for e in eos_ids if e is not None and e >= 0)
        self.eos = min(self.eos_ids) if self.eos_ids else -1
        self.waiting: deque[Sequence] = deque()
        self.running: List[Sequence] = []
        self.num_preemptions = 0

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, seq: Sequence) -> None:
        self.page_manager.acquire_segments(seq)
        self.waiting.append(seq)

    def abort(self, seq: Sequence) -> None:
        if seq in self.running:
            self.running.remove(seq)
        elif seq in self.waiting:
            self.waiting.remove(seq)
        seq.status = SequenceStatus.FINISHED
        seq.finish_reason = "abort"
        self.page_manager.deallocate(seq)

    def _preempt(self, seq: Sequence) -> None:
        self.running.remove(seq)
        seq.status = SequenceStatus.WAITING
        self.page_manager.free_private(seq)
        self.waiting.appendleft(seq)
        self.num_preemptions += 1

    def schedule(self) -> Tuple[List[Sequence], bool]:
        pm = self.page_manager
        batch: List[Sequence] = []
        ntok = 0
        while self.waiting and len(self.running) + len(batch) < self.max_num_seqs:
            seq = self.waiting[0]
            new = max(seq.num_tokens - seq.num_cached_tokens, 0)
            if batch and ntok + new > self.max_num_batched_tokens:
                break
            if not pm.ensure_capacity(seq, seq.num_tokens):
                if batch or self.running:
                    break
                raise OutOfPagesError(
                    f"sequence {seq.seq_id} needs {pm.pages_for(seq.num_tokens)} pages; "
                    f"pool has {pm.num_free_pages} free and nothing to preempt")
            self.waiting.popleft()
            seq.status = SequenceStatus.RUNNING
            batch.append(seq)
            ntok += new
        if batch:
            self.running.extend(batch)
            return batch, True
        if not self.running:
            return [], False
        scheduled: List[Sequence] = []
        for seq in list(self.running):
            if seq not in self.running:
                continue  # preempted below
            while not pm.ensure_capacity(seq, seq.num_tokens):
                victim = self.running[-1]
                self._preempt(victim)
                if victim is seq:
                    break
            else:
                scheduled.append(seq)
        return scheduled, False

    def _stop_suffix(self, seq: Sequence) -> int:
        comp = seq.completion_token_ids
        for st in seq.stop_sequences:
            if st and len(comp) >= len(st) and comp[-len(st):] == st:
                return len(st)
        return 0

    def postprocess(self, seqs: List[Sequence], token_ids: List[int]) -> List[Sequence]:
        finished = []
        for seq, tok in zip(seqs, token_ids):
            seq.num_cached_tokens = seq.num_tokens
            if getattr(seq, "flush_pending", False):
                # the retained sequence's last token now has KV; finish it
                seq.flush_pending = False
                self._finish(seq, finished)
                continue
            tok = int(tok)
            is_stop = (not seq.ignore_eos and tok in self.eos_ids) or tok in seq.stop_token_ids
            if not is_stop:
                seq.append_token(tok)
            reason = None
            if is_stop:
                reason = "stop"
            else:
                n = self._stop_suffix(seq)
                if n:
                    del seq.token_ids[-n:]
                    seq.num_cached_tokens = min(seq.num_cached_tokens, seq.num_tokens)
                    reason = "stop"
                elif seq.num_completion_tokens >= seq.max_tokens:
                    reason = "length"
                elif seq.pos_base + seq.num_tokens >= self.max_model_len:
                    reason = "length"
            if reason is None:
                continue
            seq.finish_reason = reason
            if seq.retain_output_cache and seq.num_cached_tokens < seq.num_tokens:
                # one more forward writes the last token's KV before retention
                seq.flush_pending = True
                continue
            self._finish(seq, finished)
        self.page_manager.update_sequence_lengths(seqs)
        return finished

    def _finish(self, seq: Sequence, finished: List[Sequence]) -> None:
        seq.status = SequenceStatus.FINISHED
        self.running.remove(seq)
        if seq.retain_output_cache:
            self.page_manager.release_segments(seq)
        else:
            self.page_manager.deallocate(seq)
        finished.append(seq)
