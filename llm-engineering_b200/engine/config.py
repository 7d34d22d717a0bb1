"""Engine configuration (interface of serving/engine/config.py:6-60)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class EngineConfiguration:
    """Runtime limits of one engine replica.

    Same fields, defaults and validation errors as the reference's
    ``EngineConfiguration`` (serving/engine/config.py:6-60), so configurations move
    between the two engines unchanged, plus ``enable_chunked_prefill`` (off by default,
    which keeps the reference's policy): prompts longer than ``max_batched_tokens`` are
    then admitted and prefilled over several steps in chunks that fit the step's budget;
    ``max_prefill_chunk`` (chunked prefill only; None = no limit) caps the tokens one
    prefill contributes to a step, so that a step's prefill budget is shared by several
    prompts (e.g. 4 slices of 512 tokens).
    """

    device: str = "cpu"
    max_sequences: int = 8
    eos_token_id: int = 0
    block_size: int = 16
    num_blocks: int = 256
    max_batched_tokens: int = 2_048
    seed: int = 0
    enable_chunked_prefill: bool = False
    max_prefill_chunk: int | None = None

    def __post_init__(self) -> None:
        if not self.device.strip():
            raise ValueError("device must not be empty.")
        positive = (
            ("max_sequences", self.max_sequences),
            ("block_size", self.block_size),
            ("num_blocks", self.num_blocks),
            ("max_batched_tokens", self.max_batched_tokens),
        )
        if self.max_sequences <= 0:
            raise ValueError("max_sequences must be greater than zero.")
        if self.eos_token_id < 0:
            raise ValueError("eos_token_id must not be negative.")
        for name, value in positive[1:]:
            if value <= 0:
                raise ValueError(f"{name} must be greater than zero.")
        if self.max_batched_tokens < self.max_sequences:
            raise ValueError(
                "max_batched_tokens must be greater than or equal to max_sequences."
            )
        if self.seed < 0:
            raise ValueError("seed must not be negative.")
        if self.max_prefill_chunk is not None:
            if self.max_prefill_chunk <= 0:
                raise ValueError("max_prefill_chunk must be greater than zero.")
            if not self.enable_chunked_prefill:
                raise ValueError("max_prefill_chunk requires enable_chunked_prefill.")
