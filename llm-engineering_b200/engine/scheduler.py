"""Continuous-batching scheduler (interface and policy of serving/engine/scheduler.py:12-458).

Policy, which the slot mappings depend on and which therefore matches the reference:
every running sequence decodes first (one budget token each); waiting sequences are then
admitted first-come-first-served for whole-history prefill while the token budget, the
concurrency limit and the free blocks allow, stopping at the first one that does not
fit. When reserving a block for a generated token runs out of blocks, the most recently
admitted other running sequence is preempted (blocks freed, put back at the head of the
waiting queue) and re-prefilled later.

With ``enable_chunked_prefill`` (not in the reference, off by default) a prefill may be
cut to the step's remaining budget (and to ``max_prefill_chunk`` tokens when set): after
the decodes, sequences whose prefill is under way continue first (in admission order),
then waiting sequences are admitted as before, the last one taking whatever budget is
left. A sequence decodes once all of its history
is in the pool; preemption drops the progress and the sequence is re-prefilled later.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass

from .block import BlockPool, BlockTable, blocks_needed
from .config import EngineConfiguration
from .request import Request
from .sequence import FinishReason, SequenceState

_NO_BLOCKS = "Not enough free blocks available"


@dataclass(frozen=True)
class SchedulerOutput:
    decode_sequences: tuple[SequenceState, ...]
    prefill_sequences: tuple[SequenceState, ...]
    num_batched_tokens: int
    # (first position, query tokens) of each prefill, aligned with prefill_sequences; empty
    # when every prefill covers its whole history (the reference's policy).
    prefill_chunks: tuple[tuple[int, int], ...] = ()


class Scheduler:
    """Owns the request queues, the block pool and the block table of one replica."""

    def __init__(self, configuration: EngineConfiguration) -> None:
        self.configuration = configuration
        self.block_pool = BlockPool(num_blocks=configuration.num_blocks)
        self.block_table = BlockTable(pool=self.block_pool, block_size=configuration.block_size)
        self._waiting: deque[SequenceState] = deque()
        self._running: list[SequenceState] = []
        # identities of the running sequences: membership checks in O(1) (the list keeps
        # the admission order that preemption and the step's execution order follow)
        self._running_ids: set[int] = set()
        self._finished: list[SequenceState] = []
        self._ids: set[str] = set()
        self._num_preemptions = 0
        # chunked prefill: positions of each admitted sequence already in the pool, for the
        # sequences whose prefill is not finished
        self._prefilled: dict[str, int] = {}

    # ------------------------------------------------------------------ views
    @property
    def waiting_sequences(self) -> tuple[SequenceState, ...]:
        return tuple(self._waiting)

    @property
    def running_sequences(self) -> tuple[SequenceState, ...]:
        return tuple(self._running)

    @property
    def finished_sequences(self) -> tuple[SequenceState, ...]:
        return tuple(self._finished)

    @property
    def num_preemptions(self) -> int:
        return self._num_preemptions

    @property
    def has_unfinished_requests(self) -> bool:
        return bool(self._waiting or self._running)

    # ------------------------------------------------------------------ requests
    def submit(self, request: Request) -> SequenceState:
        if request.request_id in self._ids:
            raise ValueError(f"request_id {request.request_id!r} has already been submitted.")
        cfg = self.configuration
        n = len(request.prompt_token_ids)
        longest = n + request.max_new_tokens - 1  # the last token never needs a KV slot
        if not cfg.enable_chunked_prefill:
            if n > cfg.max_batched_tokens:
                raise ValueError("Prompt length exceeds max_batched_tokens and cannot be "
                                 "prefilled without chunked prefill.")
            if longest > cfg.max_batched_tokens:
                raise ValueError("Maximum non-terminal sequence length exceeds "
                                 "max_batched_tokens and cannot be re-prefilled without "
                                 "chunked prefill.")
        if blocks_needed(longest, cfg.block_size) > cfg.num_blocks:
            raise ValueError("Maximum non-terminal sequence length requires more KV-cache "
                             "blocks than the scheduler owns.")
        seq = SequenceState(request=request)
        self._waiting.append(seq)
        self._ids.add(request.request_id)
        return seq

    def cancel(self, request_id: str) -> bool:
        for seq in self._waiting:
            if seq.request.request_id == request_id:
                self._waiting.remove(seq)
                seq.mark_finished(FinishReason.CANCELLED)
                self._finished.append(seq)
                return True
        for seq in self._running:
            if seq.request.request_id == request_id:
                self._release(seq)
                seq.mark_finished(FinishReason.CANCELLED)
                self._finished.append(seq)
                return True
        return False

    # ------------------------------------------------------------------ scheduling
    def _fits(self, seq: SequenceState) -> bool:
        if len(self._running) >= self.configuration.max_sequences:
            return False
        need = blocks_needed(seq.current_length, self.configuration.block_size)
        return need <= self.block_pool.num_free_blocks

    def _admit(self, seq: SequenceState) -> None:
        if not self._waiting or self._waiting[0] is not seq:
            raise RuntimeError("Admission violated waiting-queue ordering.")
        self.block_table.allocate_for_request(seq.request.request_id, seq.current_length)
        self._waiting.popleft()
        seq.mark_running()
        self._running.append(seq)
        self._running_ids.add(id(seq))

    def schedule(self) -> SchedulerOutput:
        if self.configuration.enable_chunked_prefill:
            return self._schedule_chunked()
        budget = self.configuration.max_batched_tokens
        decode = tuple(self._running)
        budget -= len(decode)
        prefill: list[SequenceState] = []
        while self._waiting and budget > 0:
            head = self._waiting[0]
            need = head.current_length
            if need > budget or not self._fits(head):
                break
            self._admit(head)
            prefill.append(head)
            budget -= need
        tokens = len(decode) + sum(s.current_length for s in prefill)
        return SchedulerOutput(decode_sequences=decode, prefill_sequences=tuple(prefill),
                               num_batched_tokens=tokens)

    def _schedule_chunked(self) -> SchedulerOutput:
        budget = self.configuration.max_batched_tokens
        cap = self.configuration.max_prefill_chunk or budget
        decode = tuple(s for s in self._running if s.request.request_id not in self._prefilled)
        budget -= len(decode)
        prefill: list[SequenceState] = []
        chunks: list[tuple[int, int]] = []
        for seq in self._running:  # prefills under way, in admission order
            if budget <= 0:
                break
            done = self._prefilled.get(seq.request.request_id)
            if done is None:
                continue
            n = min(seq.current_length - done, budget, cap)
            prefill.append(seq)
            chunks.append((done, n))
            budget -= n
        while self._waiting and budget > 0:
            head = self._waiting[0]
            if not self._fits(head):
                break
            self._admit(head)
            self._prefilled[head.request.request_id] = 0
            n = min(head.current_length, budget, cap)
            prefill.append(head)
            chunks.append((0, n))
            budget -= n
        tokens = len(decode) + sum(n for _, n in chunks)
        return SchedulerOutput(decode_sequences=decode, prefill_sequences=tuple(prefill),
                               num_batched_tokens=tokens, prefill_chunks=tuple(chunks))

    def complete_prefill_chunk(self, sequence: SequenceState, num_tokens: int) -> bool:
        """Record that ``num_tokens`` more positions of ``sequence`` are in the pool; True
        when its whole history is (the step's logits then give its next token)."""
        rid = sequence.request.request_id
        if rid not in self._prefilled:
            raise RuntimeError("The sequence has no prefill under way.")
        done = self._prefilled[rid] + num_tokens
        if done > sequence.current_length:
            raise RuntimeError("Prefill chunk runs past the sequence's history.")
        if done == sequence.current_length:
            del self._prefilled[rid]
            return True
        self._prefilled[rid] = done
        return False

    def reserve_generated_token(self, sequence: SequenceState) -> None:
        if sequence.is_finished:
            raise RuntimeError("Cannot reserve KV-cache storage for a finished sequence.")
        if id(sequence) not in self._running_ids:
            raise RuntimeError(
                "Cannot reserve KV-cache storage for a sequence that is not running.")
        rid = sequence.request.request_id
        try:
            self.block_table.append_token(rid, sequence.current_length)
            return
        except RuntimeError as err:
            if _NO_BLOCKS not in str(err):
                raise
        victim = next((s for s in reversed(self._running) if s is not sequence), None)
        if victim is None:
            raise RuntimeError(
                "Not enough KV-cache capacity and no eligible preemption victim exists.")
        self._preempt(victim)
        self.block_table.append_token(rid, sequence.current_length)

    def finish_sequence(self, sequence: SequenceState, reason: FinishReason) -> None:
        if sequence.is_finished:
            raise RuntimeError("Cannot finish a sequence that is already finished.")
        if id(sequence) not in self._running_ids:
            raise RuntimeError("Cannot finish a sequence that is not running.")
        self._release(sequence)
        sequence.mark_finished(reason)
        self._finished.append(sequence)

    # ------------------------------------------------------------------ internals
    def _release(self, seq: SequenceState) -> None:
        self.block_table.free_request(seq.request.request_id)
        self._prefilled.pop(seq.request.request_id, None)
        self._running = [s for s in self._running if s is not seq]
        self._running_ids.discard(id(seq))

    def _preempt(self, seq: SequenceState) -> None:
        if seq.is_finished:
            raise RuntimeError("Cannot preempt a finished sequence.")
        if id(seq) not in self._running_ids:
            raise RuntimeError("Cannot preempt a sequence that is not running.")
        self._release(seq)
        seq.mark_preempted()
        self._waiting.appendleft(seq)
        self._num_preemptions += 1
