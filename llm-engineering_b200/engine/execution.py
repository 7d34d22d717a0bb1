"""Scheduled work descriptors (interface of serving/engine/execution.py:9-47).

``ModelExecution`` keeps the reference's fields — the sequence, its phase and the
physical slot of every logical position of the current history — and may also carry the
sequence's block list, from which the slots follow as ``block * block_size + pos %
block_size`` (serving/engine/block.py:370-405). The runner reads the blocks when they are
present, so this engine never materialises the per-token slot tuple unless a caller asks
for ``slot_ids``.
"""

from __future__ import annotations

from enum import StrEnum

import numpy as np

from .sequence import SequenceState


class ExecutionPhase(StrEnum):
    PREFILL = "prefill"
    DECODE = "decode"


class ModelExecution:
    """One sequence's share of an engine step."""

    __slots__ = ("sequence", "phase", "_slot_ids", "block_ids", "block_size", "query_length",
                 "length")

    def __init__(
        self,
        sequence: SequenceState,
        phase: ExecutionPhase,
        slot_ids: tuple[int, ...] | None = None,
        *,
        block_ids: tuple[int, ...] | None = None,
        block_size: int | None = None,
        query_length: int | None = None,
        length: int | None = None,
    ) -> None:
        self.sequence = sequence
        self.phase = ExecutionPhase(phase)
        self.block_ids = block_ids
        self.block_size = block_size
        # History covered by this step: the whole sequence, or the positions up to the end
        # of a prefill chunk.
        if length is None:
            length = sequence.current_length
        if not 1 <= length <= sequence.current_length:
            raise ValueError("length must be within 1..current_length.")
        self.length = length
        if slot_ids is None and (block_ids is None or not block_size):
            raise ValueError("ModelExecution needs slot_ids or block_ids with block_size.")
        if slot_ids is not None:
            slot_ids = tuple(slot_ids)
            if len(slot_ids) != length:
                raise ValueError("slot_ids length must equal the sequence current length.")
            if any(s < 0 for s in slot_ids):
                raise ValueError("slot_ids must not contain negative values.")
        elif block_size * len(block_ids) < length:
            raise ValueError("block_ids do not cover the sequence current length.")
        self._slot_ids = slot_ids
        # Query tokens contributed this step. Prefill: the whole history (the reference's
        # recompute prefill) unless a chunk is given (the last ``query_length`` positions of
        # ``length``); decode: the newest token.
        if query_length is None:
            query_length = length if self.phase is ExecutionPhase.PREFILL else 1
        if not 1 <= query_length <= length:
            raise ValueError("query_length must be within 1..current_length.")
        if self.phase is ExecutionPhase.DECODE and query_length != 1:
            raise ValueError("decode executions contribute exactly one query token.")
        self.query_length = query_length

    @property
    def slot_ids(self) -> tuple[int, ...]:
        if self._slot_ids is None:
            pos = np.arange(self.length, dtype=np.int64)
            blocks = np.asarray(self.block_ids, dtype=np.int64)
            slots = blocks[pos // self.block_size] * self.block_size + pos % self.block_size
            self._slot_ids = tuple(slots.tolist())
        return self._slot_ids

    def __repr__(self) -> str:
        return (f"ModelExecution(request={self.sequence.request.request_id!r}, "
                f"phase={self.phase.value}, length={self.sequence.current_length})")
