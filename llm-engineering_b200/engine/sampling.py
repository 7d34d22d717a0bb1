"""Token selection (interface and order of serving/engine/sampling.py:1-181).

Non-greedy sampling applies temperature, then top-k, then top-p over what is left, then
a softmax and an inverse-CDF draw from a seeded generator, exactly in the reference's
order so seeded runs select the same tokens. ``greedy_batch`` is this engine's batched
form of the greedy rule (one argmax launch and one device-to-host copy per step instead
of one ``.item()`` per sequence); it returns the same ids as per-row ``argmax``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class SamplingParameters:
    temperature: float = 1.0
    top_k: int | None = None
    top_p: float | None = None
    greedy: bool = True

    def __post_init__(self) -> None:
        if self.temperature <= 0:
            raise ValueError("temperature must be greater than zero.")
        if self.top_k is not None and self.top_k <= 0:
            raise ValueError("top_k must be greater than zero.")
        if self.top_p is not None and not 0 < self.top_p <= 1:
            raise ValueError("top_p must be greater than zero and at most one.")


class Sampler:
    """Selects one token per sequence from vocabulary logits."""

    def __init__(self, generator: torch.Generator) -> None:
        self._generator = generator

    def sample_token(self, logits: torch.Tensor, parameters: SamplingParameters) -> int:
        if parameters.greedy:
            return int(torch.argmax(logits).item())
        scores = logits / parameters.temperature
        if parameters.top_k is not None:
            keep = min(parameters.top_k, scores.numel())
            idx = torch.topk(scores, k=keep).indices
            masked = torch.full_like(scores, float("-inf"))
            masked[idx] = scores[idx]
            scores = masked
        if parameters.top_p is not None and parameters.top_p != 1.0:
            order = torch.sort(scores, descending=True)
            cdf = torch.cumsum(torch.softmax(order.values, dim=-1), dim=-1)
            hits = torch.nonzero(cdf >= parameters.top_p, as_tuple=False)
            cut = int(hits[0].item()) if hits.numel() > 0 else scores.numel() - 1
            scores = scores.clone()
            scores[order.indices[cut + 1:]] = float("-inf")
        probs = torch.softmax(scores, dim=-1)
        cdf = torch.cumsum(probs, dim=-1)
        cdf = cdf / cdf[-1]
        draw = torch.rand((), generator=self._generator, device=logits.device)
        return int(torch.searchsorted(cdf, draw, right=True).item())

    @staticmethod
    def greedy_batch(logits: torch.Tensor) -> list[int]:
        """Argmax of every row with a single device-to-host transfer."""
        return torch.argmax(logits, dim=-1).tolist()
