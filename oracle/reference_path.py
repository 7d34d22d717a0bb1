"""The reference's own CPU algorithm for one packed decode layer, restated for timing.

Test infrastructure only (see ``oracle/__init__.py``): ``bench.py --impl reference``
times this on the host cores as the reference arm. It follows, per layer,
  * ``HFBatchedPagedCache.update`` (serving/engine/hf_batched_paged_cache.py:52-148): for
    every execution, slice its packed K/V, ``PagedKVCache.update_and_gather``
    (serving/engine/paged_kv_cache.py:23-70: decode writes the last slot) ->
    ``PagedKVStorage.scatter`` / ``gather`` (serving/engine/paged_kv_storage.py:76-174,
    slot tuples turned into long tensors on every call), then ``torch.cat`` of all
    histories;
  * ``build_attention_mask`` + ``semantic_to_additive_attention_mask``
    (serving/engine/attention_mask.py:9-120): dense (Tq, Tk) block-diagonal mask;
  * HF ``sdpa_attention_forward`` (transformers/integrations/sdpa_attention.py:40-104):
    with an explicit mask it expands KV heads (repeat_kv) and calls torch SDPA.
The pool is fp32, as in the reference's CPU configuration.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import paged


class DecodeLayer:
    """One decode step of one attention layer over a whole batch, reference-style."""

    def __init__(self, workload: dict, hq: int, hkv: int, head_dim: int, block_size: int):
        self.hq, self.hkv, self.d, self.bs = hq, hkv, head_dim, block_size
        self.kc = workload["kc"].float()
        self.vc = workload["vc"].float()
        self.q = workload["q"].float()
        self.new_k = workload["new_k"].float()
        self.new_v = workload["new_v"].float()
        ctx = workload["ctx"]
        tables = workload["tables"]
        # ModelExecution.slot_ids: tuples of the whole history (engine.py:121-127).
        self.slot_ids = [
            tuple(paged.history_slots(tables[i][tables[i] >= 0], int(c), block_size).tolist())
            for i, c in enumerate(ctx)
        ]
        self.ctx = [int(c) for c in ctx]
        self.scale = head_dim ** -0.5

    def step(self) -> torch.Tensor:
        layer = 0
        hist_k, hist_v = [], []
        for i, slots in enumerate(self.slot_ids):
            # decode: write the newest token's K/V to the last slot, gather everything
            paged.scatter(self.kc, self.vc, layer, slots[-1:], self.new_k[i:i + 1],
                          self.new_v[i:i + 1])
            k, v = paged.gather(self.kc, self.vc, layer, slots)
            hist_k.append(k)
            hist_v.append(v)
        k_all = torch.cat(hist_k, 0).transpose(0, 1).unsqueeze(0)  # (1, HKV, Tk, D)
        v_all = torch.cat(hist_v, 0).transpose(0, 1).unsqueeze(0)
        phases = [paged.DECODE] * len(self.ctx)
        mask = paged.additive_mask(paged.attention_mask(phases, self.ctx))
        group = self.hq // self.hkv
        k_rep = k_all.repeat_interleave(group, dim=1)
        v_rep = v_all.repeat_interleave(group, dim=1)
        q = self.q.transpose(0, 1).unsqueeze(0)  # (1, HQ, Tq, D)
        out = F.scaled_dot_product_attention(q, k_rep, v_rep, attn_mask=mask, scale=self.scale)
        return out.transpose(1, 2)[0]

