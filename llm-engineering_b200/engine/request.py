"""Generation requests (interface of serving/engine/request.py:8-45)."""

from __future__ import annotations

from dataclasses import dataclass, field

from .sampling import SamplingParameters


@dataclass(frozen=True)
class Request:
    """An immutable generation request: prompt ids, token budget and sampling settings."""

    request_id: str
    prompt_token_ids: tuple[int, ...]
    max_new_tokens: int
    ignore_eos: bool = False
    arrival_time: float = 0.0
    sampling_parameters: SamplingParameters = field(default_factory=SamplingParameters)

    def __post_init__(self) -> None:
        if not self.request_id.strip():
            raise ValueError("request_id must not be empty.")
        if not self.prompt_token_ids:
            raise ValueError("prompt_token_ids must not be empty.")
        if self.max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be greater than zero.")
