"""CPU parity of the engine bookkeeping with traces recorded from the reference engine.

tests/golden/engine_trace_*.json were produced by running the reference Engine,
Scheduler and BlockPool (tests/golden/make_golden.py) with a deterministic stand-in model.
Replaying the same requests through this package's engine must give the same executions
at every step — request order, phase, length, block list, last slot and a checksum of the
whole-history slot ids — the same preemption count and the same finished tokens.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from llm_engineering_b200 import engine as eng

GOLDEN = Path(__file__).resolve().parent / "golden"


class HashRunner:
    """The stand-in model used when the traces were recorded."""

    def __init__(self, vocab: int, eos: int | None = None, eos_every: int = 0):
        self.vocab, self.eos, self.eos_every = vocab, eos, eos_every
        self.calls: list = []

    def forward(self, executions):
        logits = torch.full((len(executions), self.vocab), -1.0)
        for i, ex in enumerate(executions):
            seq = ex.sequence
            h = int(hashlib.sha256(f"{seq.request.request_id}:{seq.current_length}".encode())
                    .hexdigest()[:8], 16)
            tok = h % self.vocab
            if self.eos is not None and self.eos_every and h % self.eos_every == 0:
                tok = self.eos
            logits[i, tok] = 1.0
        self.calls.append(executions)
        return logits


def slot_checksum(slots) -> str:
    return hashlib.sha256(np.asarray(slots, dtype=np.int64).tobytes()).hexdigest()[:16]


@pytest.mark.parametrize("name", ["c1", "churn"])
def test_engine_replays_reference_trace(name):
    trace = json.loads((GOLDEN / f"engine_trace_{name}.json").read_text())
    c = trace["config"]
    cfg = eng.EngineConfiguration(block_size=c["block_size"], num_blocks=c["num_blocks"],
                                  max_sequences=c["max_sequences"],
                                  max_batched_tokens=c["max_batched_tokens"],
                                  eos_token_id=c["eos_token_id"])
    eos = 0 if trace["eos_every"] else None
    runner = HashRunner(trace["vocab"], eos, trace["eos_every"])
    engine = eng.Engine(configuration=cfg, model_runner=runner)
    for r in trace["requests"]:
        engine.submit(eng.Request(request_id=r["request_id"],
                                  prompt_token_ids=tuple(r["prompt"]),
                                  max_new_tokens=r["max_new_tokens"],
                                  ignore_eos=r["ignore_eos"]))
    for step_no, expected in enumerate(trace["steps"]):
        assert engine.has_unfinished_requests
        n = len(runner.calls)
        engine.step()
        got = []
        if len(runner.calls) > n:
            for ex in runner.calls[-1]:
                slots = ex.slot_ids
                got.append({
                    "request_id": ex.sequence.request.request_id,
                    "phase": ex.phase.value,
                    "length": len(slots),
                    "blocks": list(ex.block_ids),
                    "last_slot": slots[-1],
                    "slot_sha": slot_checksum(slots),
                })
        assert got == expected["executions"], f"step {step_no}"
        assert engine.scheduler.num_preemptions == expected["preemptions"], f"step {step_no}"
    assert not engine.has_unfinished_requests
    finished = [{"request_id": s.request.request_id, "tokens": list(s.generated_token_ids),
                 "finish_reason": s.finish_reason.value} for s in engine.finished_sequences]
    assert finished == trace["finished"]
    if name == "churn":
        assert trace["num_preemptions"] > 0  # the trace does exercise recompute preemption


def test_submit_rejections_match_reference_messages():
    cfg = eng.EngineConfiguration(block_size=4, num_blocks=4, max_sequences=2,
                                  max_batched_tokens=16)
    s = eng.Scheduler(cfg)
    with pytest.raises(ValueError, match="without chunked prefill"):
        s.submit(eng.Request("a", tuple(range(17)), 1))
    with pytest.raises(ValueError, match="re-prefilled without chunked prefill"):
        s.submit(eng.Request("b", tuple(range(10)), 8))
    cfg2 = eng.EngineConfiguration(block_size=4, num_blocks=2, max_sequences=2,
                                   max_batched_tokens=64)
    with pytest.raises(ValueError, match="more KV-cache blocks"):
        eng.Scheduler(cfg2).submit(eng.Request("c", tuple(range(9)), 1))
    s.submit(eng.Request("d", (1, 2), 2))
    with pytest.raises(ValueError, match="already been submitted"):
        s.submit(eng.Request("d", (1, 2), 2))


def test_block_pool_fifo_order_and_errors():
    pool = eng.BlockPool(4)
    assert pool.allocate(2) == (0, 1)
    pool.free(0)
    assert pool.allocate(3) == (2, 3, 0)
    with pytest.raises(RuntimeError, match="Not enough free blocks available"):
        pool.allocate(1)
    with pytest.raises(ValueError, match="Invalid block_id"):
        pool.free(7)
    table = eng.BlockTable(eng.BlockPool(8), block_size=4)
    table.allocate_for_request("r", 5)
    assert table.slot_for_position("r", 4) == 1 * 4 + 0
    with pytest.raises(ValueError, match="No physical block exists"):
        table.slot_for_position("r", 8)
    with pytest.raises(ValueError, match="skips one or more logical blocks"):
        table.append_token("r", 12)


# ------------------------------------------------------------------ chunked prefill
def _run(cfg, requests, runner):
    engine = eng.Engine(configuration=cfg, model_runner=runner)
    for r in requests:
        engine.submit(r)
    engine.run_until_complete()
    return engine, {s.request.request_id: list(s.generated_token_ids)
                    for s in engine.finished_sequences}


def test_chunked_prefill_admits_long_prompts_and_splits_them_to_the_budget():
    cfg = eng.EngineConfiguration(block_size=4, num_blocks=64, max_sequences=4,
                                  max_batched_tokens=16, enable_chunked_prefill=True)
    s = eng.Scheduler(cfg)
    s.submit(eng.Request("long", tuple(range(40)), 3))  # refused without chunked prefill
    s.submit(eng.Request("short", tuple(range(5)), 2))
    out = s.schedule()
    assert [q.request.request_id for q in out.prefill_sequences] == ["long"]
    assert out.prefill_chunks == ((0, 16),) and out.num_batched_tokens == 16
    long_seq = out.prefill_sequences[0]
    assert s.complete_prefill_chunk(long_seq, 16) is False
    out = s.schedule()  # the prefill under way continues before new admissions
    assert out.prefill_chunks == ((16, 16),) and not out.decode_sequences
    assert s.complete_prefill_chunk(long_seq, 16) is False
    out = s.schedule()  # 8 tokens finish "long", the other 8 start "short"
    assert [q.request.request_id for q in out.prefill_sequences] == ["long", "short"]
    assert out.prefill_chunks == ((32, 8), (0, 5)) and out.num_batched_tokens == 13
    assert s.complete_prefill_chunk(out.prefill_sequences[0], 8) is True
    with pytest.raises(RuntimeError, match="past the sequence's history"):
        s.complete_prefill_chunk(out.prefill_sequences[1], 6)


def test_prefill_chunk_cap_shares_the_budget_between_prompts():
    """max_prefill_chunk = 4 with a 14-token budget and one decode: three prompts each get a
    4-token slice in one step (13 tokens), and the slices continue in admission order."""
    cfg = eng.EngineConfiguration(block_size=4, num_blocks=64, max_sequences=8,
                                  max_batched_tokens=14, enable_chunked_prefill=True,
                                  max_prefill_chunk=4)
    s = eng.Scheduler(cfg)
    s.submit(eng.Request("d", (1, 2), 4))
    out = s.schedule()
    assert out.prefill_chunks == ((0, 2),)
    assert s.complete_prefill_chunk(out.prefill_sequences[0], 2) is True
    s.reserve_generated_token(out.prefill_sequences[0])
    out.prefill_sequences[0].append_token(9)
    for rid, n in (("a", 10), ("b", 6), ("c", 9), ("e", 3)):
        s.submit(eng.Request(rid, tuple(range(n)), 2))
    out = s.schedule()
    assert [q.request.request_id for q in out.decode_sequences] == ["d"]
    assert [q.request.request_id for q in out.prefill_sequences] == ["a", "b", "c", "e"]
    assert out.prefill_chunks == ((0, 4), (0, 4), (0, 4), (0, 1))
    assert out.num_batched_tokens == 14
    for q, (_, n) in zip(out.prefill_sequences, out.prefill_chunks):
        s.complete_prefill_chunk(q, n)
    out = s.schedule()
    assert out.prefill_chunks == ((4, 4), (4, 2), (4, 4), (1, 2))
    with pytest.raises(ValueError, match="requires enable_chunked_prefill"):
        eng.EngineConfiguration(max_prefill_chunk=4)
    with pytest.raises(ValueError, match="max_prefill_chunk must be greater than zero"):
        eng.EngineConfiguration(enable_chunked_prefill=True, max_prefill_chunk=0)


def test_chunked_prefill_gives_the_tokens_of_whole_prefill():
    """The stand-in model's token depends on (request, history length) only, so every
    request must finish with the same tokens whether its prompt was prefilled whole or in
    chunks; chunked runs also go through preemption (few blocks)."""
    rng = np.random.default_rng(5)
    requests = [eng.Request(request_id=f"r{i}",
                            prompt_token_ids=tuple(int(x) for x in rng.integers(1, 50, size=n)),
                            max_new_tokens=m, ignore_eos=True)
                for i, (n, m) in enumerate([(30, 5), (7, 9), (45, 3), (12, 12), (3, 20)])]
    whole = eng.EngineConfiguration(block_size=4, num_blocks=200, max_sequences=4,
                                    max_batched_tokens=64)
    _, expect = _run(whole, requests, HashRunner(vocab=50))
    for budget, blocks in ((16, 200), (9, 40), (16, 20)):
        cfg = eng.EngineConfiguration(block_size=4, num_blocks=blocks, max_sequences=4,
                                      max_batched_tokens=budget, enable_chunked_prefill=True)
        runner = HashRunner(vocab=50)
        engine, got = _run(cfg, requests, runner)
        assert got == expect, (budget, blocks)
        for step in runner.calls:
            assert sum(ex.query_length for ex in step) <= budget
            for ex in step:
                assert ex.length - ex.query_length >= 0 and ex.length <= ex.sequence.current_length
        if blocks == 20:
            assert engine.scheduler.num_preemptions > 0
