"""CPU restatement of the reference's packed paged model runner — TEST INFRASTRUCTURE ONLY.

Follows ``PagedModelRunner.forward`` (serving/engine/paged_model_runner.py:44-91):
BatchLayout (batch_layout.py) -> packed input/position ids (packed_inputs.py:28-78) ->
dense additive block-diagonal mask (attention_mask.py:9-120) -> one HF forward with a
cache adapter that, per layer and per execution, scatters the new K/V rows (prefill: all
slots, decode: the last, paged_kv_cache.py:51-58), gathers the whole history and
concatenates all histories (hf_batched_paged_cache.py:52-148) -> logits of each
execution's last query row (paged_model_runner.py:85-91). The model must use an
attention implementation that accepts the explicit 4-D mask ("sdpa" or "eager").
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
from transformers.cache_utils import Cache

from . import paged


def _phase(ex) -> str:
    return getattr(ex.phase, "value", ex.phase)


def _length(ex) -> int:
    return getattr(ex, "length", None) or ex.sequence.current_length


class _GatheringCache(Cache):
    """hf_batched_paged_cache.py:52-148 restated over ``paged.scatter`` / ``paged.gather``."""

    def __init__(self, kc, vc, phases, slot_histories, layout):
        super().__init__(layers=[])
        self.kc, self.vc = kc, vc
        self.phases, self.slots, self.layout = phases, slot_histories, layout

    def update(self, key_states, value_states, layer_idx, *args, **kwargs):
        hk, hv = [], []
        for i, phase in enumerate(self.phases):
            a = self.layout["query_offsets"][i]
            b = a + self.layout["query_lengths"][i]
            k = key_states[0, :, a:b, :].transpose(0, 1)
            v = value_states[0, :, a:b, :].transpose(0, 1)
            write = self.slots[i] if phase == paged.PREFILL else self.slots[i][-1:]
            paged.scatter(self.kc, self.vc, layer_idx, write, k, v)
            gk, gv = paged.gather(self.kc, self.vc, layer_idx, self.slots[i])
            hk.append(gk)
            hv.append(gv)
        return (torch.cat(hk, 0).transpose(0, 1).unsqueeze(0),
                torch.cat(hv, 0).transpose(0, 1).unsqueeze(0))


class ReferencePackedRunner:
    """One packed forward per step with gather-then-dense attention (the reference path)."""

    def __init__(self, model, key_cache: torch.Tensor, value_cache: torch.Tensor,
                 block_size: int) -> None:
        self.model = model.eval()
        self.kc, self.vc, self.block_size = key_cache, value_cache, block_size
        self.calls: list[torch.Tensor] = []

    def forward(self, executions: Sequence) -> torch.Tensor:
        if not executions:
            raise ValueError("At least one execution is required.")
        phases = [_phase(ex) for ex in executions]
        lengths = [_length(ex) for ex in executions]
        layout = paged.batch_layout(phases, lengths)
        slot_histories = []
        for ex, n in zip(executions, lengths, strict=True):
            blocks = getattr(ex, "block_ids", None)
            if blocks is not None:
                slot_histories.append(paged.history_slots(blocks, n, self.block_size).tolist())
            else:
                slot_histories.append(list(ex.slot_ids))
        histories = [ex.sequence.all_token_ids[:n] for ex, n in zip(executions, lengths, strict=True)]
        input_ids = torch.from_numpy(paged.packed_input_ids(phases, histories))
        position_ids = torch.from_numpy(paged.packed_positions(phases, lengths))
        mask = paged.additive_mask(paged.attention_mask(phases, lengths), self.model.dtype)
        cache = _GatheringCache(self.kc, self.vc, phases, slot_histories, layout)
        dev = self.kc.device
        with torch.inference_mode():
            out = self.model(input_ids=input_ids.unsqueeze(0).to(dev),
                             position_ids=position_ids.unsqueeze(0).to(dev),
                             attention_mask=mask.to(dev), past_key_values=cache, use_cache=True)
        idx = torch.tensor(layout["logit_indices"], dtype=torch.long, device=dev)
        logits = out.logits[0].index_select(0, idx)
        self.calls.append(logits)
        return logits


def token_history_array(seq) -> np.ndarray:
    return np.asarray(seq.all_token_ids, dtype=np.int64)
