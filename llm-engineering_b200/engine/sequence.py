"""Per-request mutable state of the engine.

Interface kept from the reference (serving/engine/sequence.py:8-119): the status and
finish-reason values, ``request``, ``generated_token_ids``, ``current_length``,
``all_token_ids``, ``append_token`` and the ``mark_*`` transitions with their error types
and messages, because the scheduler, the engine loop and callers match on them.

The representation is this package's own. A sequence keeps its whole token history
(prompt, then generated tokens) in one growing int64 buffer, so the runner takes any
position range of it as an array view (``token_slice``) without rebuilding the history
each step, and each lifecycle change checks the status against a fixed set of states it
may start from.
"""

from __future__ import annotations

from enum import StrEnum

import numpy as np

from .request import Request


class SequenceStatus(StrEnum):
    WAITING = "waiting"
    RUNNING = "running"
    PREEMPTED = "preempted"
    FINISHED = "finished"


class FinishReason(StrEnum):
    EOS = "eos"
    LENGTH = "length"
    CANCELLED = "cancelled"


# statuses from which mark_running / mark_preempted may move a sequence
_RUNNABLE_FROM = frozenset({SequenceStatus.WAITING, SequenceStatus.PREEMPTED})
_PREEMPTIBLE_FROM = frozenset({SequenceStatus.RUNNING})


class SequenceState:
    """Token history and lifecycle of one request."""

    __slots__ = ("request", "_buf", "_prompt_len", "_len", "status", "finish_reason",
                 "admissions")

    def __init__(self, request: Request, generated_token_ids=(),
                 status: SequenceStatus = SequenceStatus.WAITING,
                 finish_reason: FinishReason | None = None) -> None:
        self.request = request
        prompt = np.asarray(request.prompt_token_ids, dtype=np.int64)
        gen = np.asarray(list(generated_token_ids), dtype=np.int64)
        self._prompt_len = int(prompt.size)
        self._len = self._prompt_len + int(gen.size)
        cap = max(16, 1 << (self._len + request.max_new_tokens).bit_length())
        self._buf = np.empty(cap, dtype=np.int64)
        self._buf[:self._prompt_len] = prompt
        self._buf[self._prompt_len:self._len] = gen
        self.status = SequenceStatus(status)
        self.finish_reason = None if finish_reason is None else FinishReason(finish_reason)
        # Times the sequence was admitted to run: its block table is only ever appended to
        # between two admissions (a preemption frees it, the next admission allocates anew).
        self.admissions = 0

    # ------------------------------------------------------------------ token history
    @property
    def current_length(self) -> int:
        return self._len

    @property
    def num_generated_tokens(self) -> int:
        return self._len - self._prompt_len

    @property
    def generated_token_ids(self) -> tuple[int, ...]:
        """Generated tokens, oldest first (a snapshot; append through ``append_token``)."""
        return tuple(self._buf[self._prompt_len:self._len].tolist())

    @property
    def all_token_ids(self) -> tuple[int, ...]:
        return tuple(self._buf[:self._len].tolist())

    def token_slice(self, start: int, stop: int) -> np.ndarray:
        """Token ids of positions [start, stop) as an int64 array view of the history."""
        if not 0 <= start <= stop <= self._len:
            raise IndexError(f"positions [{start}, {stop}) outside the history of {self._len}")
        return self._buf[start:stop]

    def append_token(self, token_id: int) -> None:
        if self.is_finished:
            raise ValueError("Cannot append a token to a finished sequence.")
        if self._len == self._buf.size:
            grown = np.empty(2 * self._buf.size, dtype=np.int64)
            grown[:self._len] = self._buf[:self._len]
            self._buf = grown
        self._buf[self._len] = int(token_id)
        self._len += 1

    def discard_generated(self) -> None:
        """Drop every generated token (the history goes back to the prompt)."""
        self._len = self._prompt_len

    # ------------------------------------------------------------------ lifecycle
    @property
    def is_finished(self) -> bool:
        return self.finish_reason is not None

    def mark_running(self) -> None:
        if self.status not in _RUNNABLE_FROM:
            raise RuntimeError("Only a waiting or preempted sequence can be marked running.")
        self.status = SequenceStatus.RUNNING
        self.admissions += 1

    def mark_preempted(self) -> None:
        if self.status not in _PREEMPTIBLE_FROM:
            raise RuntimeError("Only a running sequence can be preempted.")
        self.status = SequenceStatus.PREEMPTED

    def mark_finished(self, reason: FinishReason) -> None:
        if self.is_finished:
            raise ValueError("Cannot finish an already finished sequence.")
        self.status = SequenceStatus.FINISHED
        self.finish_reason = FinishReason(reason)

    def __repr__(self) -> str:
        return (f"SequenceState(request={self.request.request_id!r}, status={self.status.value}, "
                f"length={self._len}, generated={self.num_generated_tokens})")
