"""The CPU oracle against fixtures produced by the reference itself (tests/golden/).

This is what makes the oracle trustworthy as the checker of the CUDA kernels: its
scatter/gather, batch layout, positions, written slots, dense mask and packed attention
must reproduce the reference's outputs exactly (integers) or to fp32 rounding (attention).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import paged as ref

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_storage_roundtrip_matches_reference():
    z = np.load(GOLDEN / "storage_roundtrip.npz")
    kc = torch.zeros(3, 32, 2, 8)
    vc = torch.zeros(3, 32, 2, 8)
    i = 0
    while f"w{i}_slots" in z:
        ref.scatter(kc, vc, int(z[f"w{i}_layer"]), z[f"w{i}_slots"].tolist(),
                    torch.from_numpy(z[f"w{i}_keys"]), torch.from_numpy(z[f"w{i}_values"]))
        i += 1
    assert torch.equal(kc, torch.from_numpy(z["key_cache"]))
    assert torch.equal(vc, torch.from_numpy(z["value_cache"]))
    i = 0
    while f"r{i}_slots" in z:
        k, v = ref.gather(kc, vc, int(z[f"r{i}_layer"]), z[f"r{i}_slots"].tolist())
        assert torch.equal(k, torch.from_numpy(z[f"r{i}_keys"]))
        assert torch.equal(v, torch.from_numpy(z[f"r{i}_values"]))
        i += 1


def test_storage_errors_match_reference_messages():
    kc = torch.zeros(2, 8, 1, 2)
    with pytest.raises(ValueError, match="layer_index must be within"):
        ref.scatter(kc, kc.clone(), 2, [0], torch.zeros(1, 1, 2), torch.zeros(1, 1, 2))
    with pytest.raises(ValueError, match="slot_ids must be within"):
        ref.gather(kc, kc.clone(), 0, [8])


@pytest.mark.parametrize("case", json.loads((GOLDEN / "layouts.json").read_text()),
                         ids=lambda c: c["name"])
def test_layout_positions_slots_mask_match_reference(case):
    execs = case["executions"]
    phases = [e["phase"] for e in execs]
    lengths = [len(e["prompt"]) + len(e["generated"]) for e in execs]
    lay = ref.batch_layout(phases, lengths)
    for key in ("query_lengths", "key_lengths", "query_offsets", "key_offsets", "logit_indices"):
        assert list(lay[key]) == case[key], key
    assert lay["total_query_tokens"] == case["total_query_tokens"]
    assert lay["total_key_tokens"] == case["total_key_tokens"]
    assert ref.packed_positions(phases, lengths).tolist() == case["position_ids"]
    hist = [e["prompt"] + e["generated"] for e in execs]
    assert ref.packed_input_ids(phases, hist).tolist() == case["input_ids"]
    written = ref.write_slots(phases, [e["slot_ids"] for e in execs]).tolist()
    assert written == [s for w in case["written_slots"] for s in w]
    if case["mask"] is not None:
        mask = ref.attention_mask(phases, lengths)
        assert mask.to(torch.int8).tolist() == case["mask"]


def test_history_slots_match_reference_slot_ids():
    for case in json.loads((GOLDEN / "layouts.json").read_text()):
        for e in case["executions"]:
            slots = e["slot_ids"]
            length = len(slots)
            bs = 4
            blocks = [s // bs for s in slots[::bs]]
            assert ref.history_slots(blocks, length, bs).tolist() == slots
            assert [ref.slot_for_position(blocks, p, bs) for p in range(length)] == slots


def test_packed_attention_matches_reference_sdpa_path():
    z = np.load(GOLDEN / "attention_packed.npz")
    hq, hkv, d, bs, layer = (int(z[k]) for k in ("hq", "hkv", "d", "block_size", "layer"))
    phases = [str(p) for p in z["phases"]]
    lengths = z["lengths"].tolist()
    slot_ids = z["slot_ids"].tolist()
    hist, o = [], 0
    for n in lengths:
        hist.append(slot_ids[o:o + n])
        o += n
    kc = torch.from_numpy(z["pool_k_before"]).clone()
    vc = torch.from_numpy(z["pool_v_before"]).clone()
    q = torch.from_numpy(z["q"])[0].transpose(0, 1)          # (Tq, HQ, D)
    k_new = torch.from_numpy(z["k_new"])[0].transpose(0, 1)  # (Tq, HKV, D)
    v_new = torch.from_numpy(z["v_new"])[0].transpose(0, 1)
    lay = ref.batch_layout(phases, lengths)
    # the write half: PagedKVCache semantics per execution
    for i, p in enumerate(phases):
        a = lay["query_offsets"][i]
        b = a + lay["query_lengths"][i]
        slots = hist[i] if p == ref.PREFILL else hist[i][-1:]
        ref.scatter(kc, vc, layer, slots, k_new[a:b], v_new[a:b])
    assert torch.equal(kc, torch.from_numpy(z["pool_k_after"]))
    assert torch.equal(vc, torch.from_numpy(z["pool_v_after"]))
    # the attention half: dense block-diagonal path and the per-sequence forms
    ks, vs = zip(*(ref.gather(kc, vc, layer, h) for h in hist))
    k_all, v_all = torch.cat(ks), torch.cat(vs)
    mask = ref.additive_mask(ref.attention_mask(phases, lengths))
    expect = torch.from_numpy(z["out"])[0]                    # (Tq, HQ, D)
    dense = ref.dense_packed_attention(q, k_all, v_all, mask, d ** -0.5)
    torch.testing.assert_close(dense, expect, rtol=1e-5, atol=1e-5)
    tables = [[s // bs for s in h[::bs]] for h in hist]
    dec = [i for i, p in enumerate(phases) if p == ref.DECODE]
    pre = [i for i, p in enumerate(phases) if p == ref.PREFILL]
    rows_dec = [lay["query_offsets"][i] for i in dec]
    out_dec = ref.decode_attention(q[rows_dec], kc, vc, layer, [tables[i] for i in dec],
                                   [lengths[i] for i in dec], bs, d ** -0.5)
    torch.testing.assert_close(out_dec, expect[rows_dec], rtol=1e-5, atol=1e-5)
    cu = [0]
    rows_pre = []
    for i in pre:
        a = lay["query_offsets"][i]
        rows_pre += list(range(a, a + lay["query_lengths"][i]))
        cu.append(cu[-1] + lay["query_lengths"][i])
    out_pre = ref.prefill_attention(q[rows_pre], kc, vc, layer, [tables[i] for i in pre], cu,
                                    [lengths[i] for i in pre], bs, d ** -0.5)
    torch.testing.assert_close(out_pre, expect[rows_pre], rtol=1e-5, atol=1e-5)
