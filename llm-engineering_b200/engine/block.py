"""KV block bookkeeping (interface of serving/engine/block.py:38-456).

Allocation order is part of the contract, because slot mappings must match the
reference bit for bit: free blocks leave from the head of a FIFO queue and a block
whose last reference is released rejoins at its tail.
"""

from __future__ import annotations

from collections import deque
from collections.abc import Iterable
from dataclasses import dataclass


def blocks_needed(num_tokens: int, block_size: int) -> int:
    """ceil(num_tokens / block_size) (serving/engine/block.py:53-75)."""
    if num_tokens < 0:
        raise ValueError("num_tokens must not be negative.")
    if block_size <= 0:
        raise ValueError("block_size must be greater than zero.")
    return -(-num_tokens // block_size)


@dataclass
class Block:
    block_id: int
    ref_count: int = 0


class BlockPool:
    """Fixed set of physical blocks with reference counts and a FIFO free queue."""

    def __init__(self, num_blocks: int) -> None:
        if num_blocks <= 0:
            raise ValueError("num_blocks must be greater than zero.")
        self.num_blocks = num_blocks
        self._refs = [0] * num_blocks
        self._free = deque(range(num_blocks))

    @property
    def num_free_blocks(self) -> int:
        return len(self._free)

    @property
    def num_allocated_blocks(self) -> int:
        return self.num_blocks - len(self._free)

    @property
    def utilization(self) -> float:
        return self.num_allocated_blocks / self.num_blocks

    def block(self, block_id: int) -> Block:
        self._check(block_id)
        return Block(block_id=block_id, ref_count=self._refs[block_id])

    def allocate(self, num_blocks: int) -> tuple[int, ...]:
        if num_blocks <= 0:
            raise ValueError("num_blocks must be greater than zero.")
        if num_blocks > len(self._free):
            raise RuntimeError("Not enough free blocks available.")
        taken = tuple(self._free.popleft() for _ in range(num_blocks))
        for b in taken:
            self._refs[b] = 1
        return taken

    def increment_ref_count(self, block_id: int) -> None:
        self._check(block_id)
        if self._refs[block_id] == 0:
            raise ValueError("Cannot increment the reference count of a free block.")
        self._refs[block_id] += 1

    def free(self, block_id: int) -> None:
        self._check(block_id)
        if self._refs[block_id] == 0:
            raise ValueError("Cannot free a block that is already free.")
        self._refs[block_id] -= 1
        if self._refs[block_id] == 0:
            self._free.append(block_id)

    def free_many(self, block_ids: Iterable[int]) -> None:
        for b in block_ids:
            self.free(b)

    def _check(self, block_id: int) -> None:
        if block_id < 0 or block_id >= self.num_blocks:
            raise ValueError(f"Invalid block_id: {block_id!r}.")


class BlockTable:
    """Request id -> ordered list of physical blocks."""

    def __init__(self, pool: BlockPool, block_size: int) -> None:
        if block_size <= 0:
            raise ValueError("block_size must be greater than zero.")
        self.pool = pool
        self.block_size = block_size
        self._tables: dict[str, list[int]] = {}

    def allocate_for_request(self, request_id: str, num_tokens: int) -> tuple[int, ...]:
        if request_id in self._tables:
            raise ValueError(f"request_id {request_id!r} already has a block table.")
        if num_tokens <= 0:
            raise ValueError("num_tokens must be greater than zero.")
        blocks = self.pool.allocate(blocks_needed(num_tokens, self.block_size))
        self._tables[request_id] = list(blocks)
        return blocks

    def blocks_for_request(self, request_id: str) -> tuple[int, ...]:
        return tuple(self._table(request_id))

    def free_request(self, request_id: str) -> None:
        self.pool.free_many(self._table(request_id))
        del self._tables[request_id]

    def append_token(self, request_id: str, token_position: int) -> None:
        table = self._table(request_id)
        if token_position < 0:
            raise ValueError("token_position must not be negative.")
        logical = token_position // self.block_size
        if logical < len(table):
            return
        if logical > len(table):
            raise ValueError("token_position skips one or more logical blocks.")
        table.append(self.pool.allocate(1)[0])

    def slot_for_position(self, request_id: str, token_position: int) -> int:
        table = self._table(request_id)
        if token_position < 0:
            raise ValueError("token_position must not be negative.")
        logical = token_position // self.block_size
        if logical >= len(table):
            raise ValueError(f"No physical block exists for token position: {token_position!r}")
        return table[logical] * self.block_size + token_position % self.block_size

    def fragmentation_slots(self, request_id: str, num_tokens: int) -> int:
        table = self._table(request_id)
        if num_tokens <= 0:
            raise ValueError("num_tokens must be greater than zero.")
        if blocks_needed(num_tokens, self.block_size) != len(table):
            raise ValueError("num_tokens is inconsistent with the allocated blocks.")
        return len(table) * self.block_size - num_tokens

    def _table(self, request_id: str) -> list[int]:
        try:
            return self._tables[request_id]
        except KeyError:
            raise ValueError(f"Unknown request_id: {request_id!r}.") from None
