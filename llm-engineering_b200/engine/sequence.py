"""Per-request mutable state (interface of serving/engine/sequence.py:8-119)."""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import StrEnum

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


@dataclass
class SequenceState:
    """Prompt plus generated tokens of one request and its lifecycle status."""

    request: Request
    generated_token_ids: list[int] = field(default_factory=list)
    status: SequenceStatus = SequenceStatus.WAITING
    finish_reason: FinishReason | None = None

    @property
    def num_generated_tokens(self) -> int:
        return len(self.generated_token_ids)

    @property
    def current_length(self) -> int:
        return len(self.request.prompt_token_ids) + len(self.generated_token_ids)

    @property
    def all_token_ids(self) -> tuple[int, ...]:
        return self.request.prompt_token_ids + tuple(self.generated_token_ids)

    @property
    def is_finished(self) -> bool:
        return self.finish_reason is not None

    def append_token(self, token_id: int) -> None:
        if self.is_finished:
            raise ValueError("Cannot append a token to a finished sequence.")
        self.generated_token_ids.append(token_id)

    def mark_running(self) -> None:
        if self.status not in (SequenceStatus.WAITING, SequenceStatus.PREEMPTED):
            raise RuntimeError("Only a waiting or preempted sequence can be marked running.")
        self.status = SequenceStatus.RUNNING

    def mark_preempted(self) -> None:
        if self.status != SequenceStatus.RUNNING:
            raise RuntimeError("Only a running sequence can be preempted.")
        self.status = SequenceStatus.PREEMPTED

    def mark_finished(self, reason: FinishReason) -> None:
        if self.is_finished:
            raise ValueError("Cannot finish an already finished sequence.")
        self.status = SequenceStatus.FINISHED
        self.finish_reason = reason
