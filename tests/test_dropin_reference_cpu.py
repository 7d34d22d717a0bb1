"""The drop-in under the reference's own engine (CPU).

The reference's ``Engine``, ``Scheduler``, ``BlockPool``, ``PagedKVStorage`` and
``PagedKVCache`` (imported from the reference checkout, serving/engine/*.py) drive
``B200PagedModelRunner`` exactly as they drive the reference's ``PagedModelRunner``
(serving/engine/engine.py:106-133,176; paged_kv_cache.py:23-70;
paged_model_runner.py:31-91): the runner receives the reference's ``ModelExecution``
objects (whole-history ``slot_ids``) and the reference's ``PagedKVCache``.

The CUDA kernels cannot run here, so the runner's kernel module is monkeypatched with the
oracle-backed CPU stand-in of tests/test_runner_cpu.py (in this file only; the product
runner always calls the CUDA ops, whose GPU half of this check is
tests/test_runner_gpu.py::test_reference_style_executions_reproduce_config1_tokens).
Checked:

* configuration 1 (random-init Qwen2.5-0.5B shape, fp32, 8 requests x 32 greedy tokens)
  reproduces the reference engine's golden tokens token for token;
* the reference's ``PagedKVStorage.gather`` reads, from the pool the runner filled, the
  K/V history of every request that the reference's own runner leaves in its pool.
"""

from __future__ import annotations

import copy
import json
from pathlib import Path

import pytest
import torch

from llm_engineering_b200 import runner as runner_mod
from llm_engineering_b200.runner import B200PagedModelRunner
from test_runner_cpu import CpuKernels

GOLDEN = Path(__file__).resolve().parent / "golden"


class Recording:
    """Forwards to a runner and keeps the last slot_ids of every request."""

    def __init__(self, inner):
        self.inner = inner
        self.slots: dict[str, tuple[int, ...]] = {}

    def forward(self, executions):
        for ex in executions:
            self.slots[ex.sequence.request.request_id] = tuple(ex.slot_ids)
        return self.inner.forward(executions)


def c1_model():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=151936, hidden_size=896, intermediate_size=4864,
                      num_hidden_layers=24, num_attention_heads=14, num_key_value_heads=2,
                      rope_theta=1_000_000.0, tie_word_embeddings=True,
                      max_position_embeddings=32768, attn_implementation="sdpa")
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def _run(ref, runner_factory, golden):
    cfg = ref["config"].EngineConfiguration(device="cpu", block_size=16, num_blocks=2048,
                                            max_sequences=8, max_batched_tokens=2048, seed=0)
    storage = ref["paged_kv_storage"].PagedKVStorage(
        num_layers=24, num_blocks=2048, block_size=16, num_kv_heads=2, head_dim=64,
        dtype=torch.float32, device=torch.device("cpu"))
    cache = ref["paged_kv_cache"].PagedKVCache(storage)
    runner = Recording(runner_factory(cache))
    engine = ref["engine"].Engine(configuration=cfg, model_runner=runner)
    for r in golden["requests"]:
        engine.submit(ref["request"].Request(request_id=r["request_id"],
                                             prompt_token_ids=tuple(r["prompt"]),
                                             max_new_tokens=32, ignore_eos=True))
    engine.run_until_complete()
    tokens = {s.request.request_id: list(s.generated_token_ids)
              for s in engine.finished_sequences}
    return tokens, storage, runner.slots


def test_reference_engine_drives_b200_runner_config1(reference_engine, monkeypatch):
    monkeypatch.setattr(runner_mod, "_ops", CpuKernels())
    golden = json.loads((GOLDEN / "greedy_c1.json").read_text())
    model = c1_model()
    ref = reference_engine

    ours_tokens, ours_storage, ours_slots = _run(
        ref, lambda cache: B200PagedModelRunner(copy.deepcopy(model), torch.device("cpu"), cache),
        golden)
    for rid, want in golden["generated"].items():
        assert ours_tokens[rid] == want, (rid, ours_tokens[rid], want)

    theirs_tokens, theirs_storage, theirs_slots = _run(
        ref, lambda cache: ref["paged_model_runner"].PagedModelRunner(
            copy.deepcopy(model), torch.device("cpu"), cache), golden)
    assert theirs_tokens == ours_tokens
    assert theirs_slots == ours_slots
    # The reference's gather over each request's history at its last step (every slot of
    # it written by then) reads, from the pool this runner filled, what the reference's
    # own runner left in its pool.
    for rid, slots in ours_slots.items():
        for layer in (0, 11, 23):
            k1, v1 = ours_storage.gather(layer_index=layer, slot_ids=slots)
            k2, v2 = theirs_storage.gather(layer_index=layer, slot_ids=slots)
            torch.testing.assert_close(k1, k2, rtol=1e-4, atol=1e-4)
            torch.testing.assert_close(v1, v2, rtol=1e-4, atol=1e-4)


def test_reference_runner_interface_errors(reference_engine, monkeypatch):
    """The reference's empty-batch error, raised by the drop-in with the same message."""
    monkeypatch.setattr(runner_mod, "_ops", CpuKernels())
    ref = reference_engine
    storage = ref["paged_kv_storage"].PagedKVStorage(
        num_layers=24, num_blocks=8, block_size=16, num_kv_heads=2, head_dim=64,
        dtype=torch.float32, device=torch.device("cpu"))
    runner = B200PagedModelRunner(c1_model(), torch.device("cpu"),
                                  ref["paged_kv_cache"].PagedKVCache(storage))
    with pytest.raises(ValueError, match="At least one execution is required."):
        runner.forward([])
