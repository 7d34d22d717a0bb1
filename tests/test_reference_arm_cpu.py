"""The reference arm's CPU port against the reference's own code (CPU).

``bench.py --impl reference`` times ``oracle/reference_path.DecodeLayer``, a restatement
of one packed decode layer of the reference: HFBatchedPagedCache.update (scatter of each
newest row, gather of every history, concatenation), build_attention_mask +
semantic_to_additive_attention_mask, and HF sdpa_attention_forward. The reference
itself cannot run on the GPU box, so this test pins the port here: on a small decode batch
it must return what the reference's own functions return, imported from its checkout
(serving/engine/hf_batched_paged_cache.py:52-148, attention_mask.py:9-120,
transformers/integrations/sdpa_attention.py:40-104), and leave the same pool.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import paged as ref
from oracle import reference_path


def _workload(seed, n, hq, hkv, d, bs):
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 300, size=n).astype(np.int32)
    nblk = (ctx + bs - 1) // bs
    num_blocks = int(nblk.sum()) + 4
    perm = rng.permutation(num_blocks)
    tables = np.full((n, int(nblk.max())), -1, dtype=np.int32)
    used = 0
    for i, b in enumerate(nblk):
        tables[i, :b] = perm[used:used + b]
        used += b
    g = torch.Generator().manual_seed(seed)
    return {"ctx": ctx, "tables": tables,
            "kc": torch.randn(1, num_blocks * bs, hkv, d, generator=g),
            "vc": torch.randn(1, num_blocks * bs, hkv, d, generator=g),
            "q": torch.randn(n, hq, d, generator=g),
            "new_k": torch.randn(n, hkv, d, generator=g),
            "new_v": torch.randn(n, hkv, d, generator=g)}


def test_reference_arm_port_matches_reference_decode_layer(reference_engine):
    import importlib

    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    r = reference_engine
    hf_cache = importlib.import_module("serving.engine.hf_batched_paged_cache")
    mask_mod = importlib.import_module("serving.engine.attention_mask")
    layout_mod = importlib.import_module("serving.engine.batch_layout")
    hq, hkv, d, bs = 12, 2, 128, 16
    w = _workload(5, 24, hq, hkv, d, bs)

    port = reference_path.DecodeLayer(dict(w, kc=w["kc"].clone(), vc=w["vc"].clone()),
                                      hq, hkv, d, bs)
    got = port.step()

    storage = r["paged_kv_storage"].PagedKVStorage(
        num_layers=1, num_blocks=w["kc"].shape[1] // bs, block_size=bs, num_kv_heads=hkv,
        head_dim=d, dtype=torch.float32, device=torch.device("cpu"))
    storage.key_cache.copy_(w["kc"])
    storage.value_cache.copy_(w["vc"])
    executions = []
    for i, c in enumerate(w["ctx"].tolist()):
        # a history of c tokens: c - 1 prompt tokens and one generated (c == 1: the prompt)
        prompt, gen = (tuple(range(1, c)), [7]) if c > 1 else ((1,), [])
        req = r["request"].Request(request_id=f"s{i}", prompt_token_ids=prompt, max_new_tokens=4)
        seq = r["sequence"].SequenceState(request=req, generated_token_ids=gen)
        slots = ref.history_slots(w["tables"][i][w["tables"][i] >= 0], c, bs)
        executions.append(r["execution"].ModelExecution(
            sequence=seq, phase=r["execution"].ExecutionPhase.DECODE,
            slot_ids=tuple(int(s) for s in slots)))
    layout = layout_mod.BatchLayout(executions=tuple(executions))
    cache = hf_cache.HFBatchedPagedCache(paged_cache=r["paged_kv_cache"].PagedKVCache(storage),
                                         layout=layout)
    k_all, v_all = cache.update(w["new_k"].transpose(0, 1).unsqueeze(0),
                                w["new_v"].transpose(0, 1).unsqueeze(0), 0)
    mask = mask_mod.semantic_to_additive_attention_mask(
        mask_mod.build_attention_mask(layout, device=torch.device("cpu")), dtype=torch.float32)

    class _Attn(torch.nn.Module):
        num_key_value_groups = hq // hkv
        is_causal = True

    want, _ = sdpa_attention_forward(_Attn(), w["q"].transpose(0, 1).unsqueeze(0), k_all, v_all,
                                     mask, scaling=d ** -0.5)
    torch.testing.assert_close(got, want[0], rtol=1e-5, atol=1e-5)
    assert torch.equal(port.kc[0], storage.key_cache[0])
    assert torch.equal(port.vc[0], storage.value_cache[0])
