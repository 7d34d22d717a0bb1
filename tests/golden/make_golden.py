"""Generate the golden fixtures by running the reference engine itself.

Run where the reference project is checked out (it is imported from the path given;
nothing at test time reads it):

    python tests/golden/make_golden.py --reference PATH [--skip-greedy]

(``LLM_ENGINEERING_REFERENCE`` may give the path instead of ``--reference``.)

Fixtures written next to this script:
  storage_roundtrip.npz  PagedKVStorage.scatter/gather on non-contiguous slots, 3 layers
  layouts.json           BatchLayout / build_packed_inputs / build_attention_mask /
                         PagedKVCache write slots for several mixed decode+prefill batches
  engine_trace_*.json    Engine + Scheduler + BlockPool traces (stub model): per step, every
                         execution's request, phase, length, block table, slot-id checksum
  attention_packed.npz   the reference's packed attention path (HFBatchedPagedCache.update +
                         dense mask + HF sdpa_attention_forward), fp32, mixed batch
  greedy_c1.json         greedy tokens of the reference engine (PagedModelRunner, fp32 CPU)
                         on random-init Qwen2.5-0.5B-shaped weights, 8 requests x 32 tokens
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import random
import sys
from pathlib import Path

import numpy as np
import torch


def _reference_root() -> Path:
    ap = argparse.ArgumentParser(add_help=False)
    ap.add_argument("--reference")
    known, _ = ap.parse_known_args()
    root = known.reference or os.environ.get("LLM_ENGINEERING_REFERENCE")
    if not root:
        sys.exit("make_golden.py: pass --reference PATH (the reference project's checkout) "
                 "or set LLM_ENGINEERING_REFERENCE")
    return Path(root)


REF = _reference_root()
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(REF))

from serving.engine.attention_mask import (  # noqa: E402
    build_attention_mask,
    semantic_to_additive_attention_mask,
)
from serving.engine.batch_layout import BatchLayout  # noqa: E402
from serving.engine.config import EngineConfiguration  # noqa: E402
from serving.engine.engine import Engine  # noqa: E402
from serving.engine.execution import ExecutionPhase, ModelExecution  # noqa: E402
from serving.engine.hf_batched_paged_cache import HFBatchedPagedCache  # noqa: E402
from serving.engine.packed_inputs import build_packed_inputs  # noqa: E402
from serving.engine.paged_kv_cache import PagedKVCache  # noqa: E402
from serving.engine.paged_kv_storage import PagedKVStorage  # noqa: E402
from serving.engine.request import Request  # noqa: E402
from serving.engine.sequence import SequenceState  # noqa: E402


def slot_checksum(slots) -> str:
    return hashlib.sha256(np.asarray(slots, dtype=np.int64).tobytes()).hexdigest()[:16]


# --------------------------------------------------------------------- storage
def make_storage_roundtrip() -> None:
    torch.manual_seed(100)
    st = PagedKVStorage(num_layers=3, num_blocks=8, block_size=4, num_kv_heads=2, head_dim=8,
                        dtype=torch.float32, device=torch.device("cpu"))
    st.key_cache.zero_()
    st.value_cache.zero_()
    writes = [
        (0, (3, 17, 5, 30, 12)),
        (2, (0, 31, 16, 1)),
        (1, (9, 8, 7)),
        (0, (17, 4)),  # overwrite one slot of the first write
    ]
    arrays = {}
    for i, (layer, slots) in enumerate(writes):
        k = torch.randn(len(slots), 2, 8)
        v = torch.randn(len(slots), 2, 8)
        st.scatter(layer_index=layer, slot_ids=slots, keys=k, values=v)
        arrays[f"w{i}_layer"] = np.array(layer)
        arrays[f"w{i}_slots"] = np.array(slots)
        arrays[f"w{i}_keys"] = k.numpy()
        arrays[f"w{i}_values"] = v.numpy()
    reads = [(0, (30, 3, 4, 17, 5, 12)), (2, (1, 0, 16, 31)), (1, (7, 8, 9, 10))]
    for i, (layer, slots) in enumerate(reads):
        k, v = st.gather(layer_index=layer, slot_ids=slots)
        arrays[f"r{i}_layer"] = np.array(layer)
        arrays[f"r{i}_slots"] = np.array(slots)
        arrays[f"r{i}_keys"] = k.numpy()
        arrays[f"r{i}_values"] = v.numpy()
    arrays["key_cache"] = st.key_cache.numpy()
    arrays["value_cache"] = st.value_cache.numpy()
    np.savez_compressed(OUT / "storage_roundtrip.npz", **arrays)


# --------------------------------------------------------------------- layouts
def execution(rid, prompt, generated, phase, slots) -> ModelExecution:
    req = Request(request_id=rid, prompt_token_ids=tuple(prompt), max_new_tokens=64)
    seq = SequenceState(request=req, generated_token_ids=list(generated))
    return ModelExecution(sequence=seq, phase=phase, slot_ids=tuple(slots))


class RecordingStorage(PagedKVStorage):
    """Reference storage that remembers which slots each scatter wrote."""

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.written: list[tuple[int, ...]] = []

    def scatter(self, layer_index, slot_ids, keys, values):
        self.written.append(tuple(slot_ids))
        super().scatter(layer_index, slot_ids, keys, values)


def layout_case(name, specs, block_size=4):
    """specs: (rid, prompt, generated, phase, slot list)."""
    execs = tuple(execution(*s) for s in specs)
    lay = BatchLayout(executions=execs)
    packed = build_packed_inputs(lay, device=torch.device("cpu"))
    mask = build_attention_mask(lay, device=torch.device("cpu"))
    st = RecordingStorage(num_layers=1, num_blocks=64, block_size=block_size, num_kv_heads=1,
                          head_dim=2, dtype=torch.float32, device=torch.device("cpu"))
    cache = HFBatchedPagedCache(paged_cache=PagedKVCache(st), layout=lay)
    kv = torch.zeros(1, 1, lay.total_query_tokens, 2)
    cache.update(kv, kv.clone(), 0)
    return {
        "name": name,
        "executions": [
            {"request_id": s[0], "prompt": list(s[1]), "generated": list(s[2]),
             "phase": s[3].value, "slot_ids": list(s[4])}
            for s in specs
        ],
        "query_lengths": list(lay.query_lengths),
        "key_lengths": list(lay.key_lengths),
        "query_offsets": list(lay.query_offsets),
        "key_offsets": list(lay.key_offsets),
        "logit_indices": list(lay.logit_indices),
        "total_query_tokens": lay.total_query_tokens,
        "total_key_tokens": lay.total_key_tokens,
        "input_ids": packed.input_ids.tolist(),
        "position_ids": packed.position_ids.tolist(),
        "written_slots": [list(w) for w in st.written],
        "mask": mask.to(torch.int8).tolist() if mask.numel() <= 4096 else None,
    }


def make_layouts() -> None:
    D, P = ExecutionPhase.DECODE, ExecutionPhase.PREFILL
    rng = random.Random(7)
    cases = [
        # decode + prefill, the reference's own shape (test_paged_model_runner.py:273-312)
        layout_case("decode_then_prefill",
                    [("a", (1, 2, 3), (4,), D, (0, 1, 2, 3)),
                     ("b", (5, 6), (), P, (8, 9))]),
        layout_case("three_prefills_noncontiguous",
                    [("a", (9, 8, 7, 6, 5), (), P, (12, 13, 14, 15, 40)),
                     ("b", (1,), (), P, (4,)),
                     ("c", (3, 3, 3), (), P, (20, 21, 22))]),
        layout_case("decodes_only",
                    [("a", (1,), (2, 3, 4, 5), D, (60, 61, 62, 63, 0)),
                     ("b", (7, 7), (8,), D, (16, 17, 18))]),
    ]
    # a larger random mixed batch with block tables drawn from a shuffled pool
    specs = []
    pool = list(range(64))
    rng.shuffle(pool)
    used = 0
    for i in range(6):
        plen = rng.randint(1, 20)
        phase = D if i < 4 else P
        gen = [rng.randint(0, 999) for _ in range(rng.randint(1, 6))] if phase is D else []
        length = plen + len(gen)
        nb = (length + 3) // 4
        blocks = pool[used:used + nb]
        used += nb
        slots = tuple(blocks[p // 4] * 4 + p % 4 for p in range(length))
        specs.append((f"r{i}", tuple(rng.randint(0, 999) for _ in range(plen)), tuple(gen), phase,
                      slots))
    cases.append(layout_case("random_mixed", specs))
    (OUT / "layouts.json").write_text(json.dumps(cases, indent=1))


# --------------------------------------------------------------------- engine traces
class HashRunner:
    """Deterministic stand-in model: the next token is a hash of (request, length)."""

    def __init__(self, vocab: int, eos: int | None = None, eos_every: int = 0):
        self.vocab = vocab
        self.calls: list = []
        self.eos = eos
        self.eos_every = eos_every

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


def run_trace(name, cfg, requests, vocab=1000, eos=None, eos_every=0):
    runner = HashRunner(vocab, eos, eos_every)
    eng = Engine(configuration=cfg, model_runner=runner)
    for r in requests:
        eng.submit(r)
    steps = []
    while eng.has_unfinished_requests:
        n_calls = len(runner.calls)
        eng.step()
        step = {"preemptions": eng.scheduler.num_preemptions, "executions": []}
        if len(runner.calls) > n_calls:
            for ex in runner.calls[-1]:
                rid = ex.sequence.request.request_id
                step["executions"].append({
                    "request_id": rid,
                    "phase": ex.phase.value,
                    "length": len(ex.slot_ids),
                    # logical block list = the block of the first slot of each block
                    "blocks": [s // cfg.block_size for s in ex.slot_ids[::cfg.block_size]],
                    "last_slot": ex.slot_ids[-1],
                    "slot_sha": slot_checksum(ex.slot_ids),
                })
        steps.append(step)
    finished = [
        {"request_id": s.request.request_id, "tokens": list(s.generated_token_ids),
         "finish_reason": s.finish_reason.value}
        for s in eng.finished_sequences
    ]
    data = {
        "name": name,
        "config": {"block_size": cfg.block_size, "num_blocks": cfg.num_blocks,
                   "max_sequences": cfg.max_sequences,
                   "max_batched_tokens": cfg.max_batched_tokens, "eos_token_id": cfg.eos_token_id},
        "vocab": vocab, "eos_every": eos_every,
        "requests": [{"request_id": r.request_id, "prompt": list(r.prompt_token_ids),
                      "max_new_tokens": r.max_new_tokens, "ignore_eos": r.ignore_eos}
                     for r in requests],
        "steps": steps,
        "finished": finished,
        "num_preemptions": eng.scheduler.num_preemptions,
    }
    (OUT / f"engine_trace_{name}.json").write_text(json.dumps(data))


def c1_requests(vocab=151936, seed=0):
    rng = random.Random(seed)
    reqs = []
    for i in range(8):
        n = rng.randint(16, 128)
        reqs.append(Request(request_id=f"req-{i}",
                            prompt_token_ids=tuple(rng.randrange(vocab) for _ in range(n)),
                            max_new_tokens=32, ignore_eos=True))
    return reqs


def make_traces() -> None:
    cfg = EngineConfiguration(block_size=16, num_blocks=2048, max_sequences=8,
                              max_batched_tokens=2048)
    run_trace("c1", cfg, c1_requests(vocab=1000), vocab=1000)
    # churn: a pool small enough to force recompute preemption and block reuse
    rng = random.Random(3)
    reqs = [Request(request_id=f"c{i}", prompt_token_ids=tuple(rng.randrange(500)
                                                               for _ in range(rng.randint(5, 40))),
                    max_new_tokens=rng.randint(10, 40), ignore_eos=False) for i in range(10)]
    cfg2 = EngineConfiguration(block_size=4, num_blocks=40, max_sequences=6,
                               max_batched_tokens=160, eos_token_id=0)
    run_trace("churn", cfg2, reqs, vocab=500, eos=0, eos_every=23)


# --------------------------------------------------------------------- attention
def make_attention() -> None:
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    torch.manual_seed(5)
    hq, hkv, d, bs = 6, 2, 16, 4
    st = PagedKVStorage(num_layers=2, num_blocks=32, block_size=bs, num_kv_heads=hkv, head_dim=d,
                        dtype=torch.float32, device=torch.device("cpu"))
    st.key_cache.normal_()
    st.value_cache.normal_()
    pool_k0, pool_v0 = st.key_cache.clone(), st.value_cache.clone()
    D, P = ExecutionPhase.DECODE, ExecutionPhase.PREFILL
    perm = torch.randperm(32).tolist()

    def slots_for(blocks, n):
        return tuple(blocks[p // bs] * bs + p % bs for p in range(n))

    specs = [
        ("d0", tuple(range(9)), (3,), D, slots_for(perm[0:3], 10)),
        ("d1", tuple(range(4)), (1, 2, 3, 4), D, slots_for(perm[3:5], 8)),
        ("p0", tuple(range(7)), (), P, slots_for(perm[5:7], 7)),
        ("p1", tuple(range(13)), (), P, slots_for(perm[7:11], 13)),
    ]
    execs = tuple(execution(*s) for s in specs)
    lay = BatchLayout(executions=execs)
    cache = HFBatchedPagedCache(paged_cache=PagedKVCache(st), layout=lay)
    tq = lay.total_query_tokens
    q = torch.randn(1, hq, tq, d)
    k_new = torch.randn(1, hkv, tq, d)
    v_new = torch.randn(1, hkv, tq, d)
    layer = 1
    k_all, v_all = cache.update(k_new, v_new, layer)
    mask = semantic_to_additive_attention_mask(
        build_attention_mask(lay, device=torch.device("cpu")), dtype=torch.float32)

    class Mod(torch.nn.Module):
        num_key_value_groups = hq // hkv
        is_causal = True

    out, _ = sdpa_attention_forward(Mod(), q, k_all, v_all, mask, scaling=d ** -0.5)
    np.savez_compressed(
        OUT / "attention_packed.npz",
        hq=hq, hkv=hkv, d=d, block_size=bs, layer=layer,
        pool_k_before=pool_k0.numpy(), pool_v_before=pool_v0.numpy(),
        pool_k_after=st.key_cache.numpy(), pool_v_after=st.value_cache.numpy(),
        phases=np.array([s[3].value for s in specs]),
        lengths=np.array([len(s[4]) for s in specs]),
        slot_ids=np.concatenate([np.array(s[4]) for s in specs]),
        q=q.numpy(), k_new=k_new.numpy(), v_new=v_new.numpy(),
        out=out.numpy(),  # (1, Tq, HQ, D)
    )


# --------------------------------------------------------------------- greedy c1
def c1_model():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=151936, hidden_size=896, intermediate_size=4864,
                      num_hidden_layers=24, num_attention_heads=14, num_key_value_heads=2,
                      rope_theta=1_000_000.0, tie_word_embeddings=True,
                      max_position_embeddings=32768, attn_implementation="sdpa")
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg).eval()
    return model


def make_greedy_c1() -> None:
    from serving.engine.paged_model_runner import PagedModelRunner

    torch.set_num_threads(8)
    model = c1_model()
    probe = float(sum(p.double().sum() for p in model.parameters()))
    st = PagedKVStorage(num_layers=24, num_blocks=2048, block_size=16, num_kv_heads=2,
                        head_dim=64, dtype=torch.float32, device=torch.device("cpu"))
    runner = PagedModelRunner(model=model, device=torch.device("cpu"), paged_cache=PagedKVCache(st))
    margins: dict[str, list[float]] = {}
    orig_forward = runner.forward

    def forward(executions):
        logits = orig_forward(executions)
        top = torch.topk(logits.float(), 2, dim=-1).values
        for i, ex in enumerate(executions):
            margins.setdefault(ex.sequence.request.request_id, []).append(
                float(top[i, 0] - top[i, 1]))
        return logits

    runner.forward = forward
    cfg = EngineConfiguration(block_size=16, num_blocks=2048, max_sequences=8,
                              max_batched_tokens=2048, seed=0)
    eng = Engine(configuration=cfg, model_runner=runner)
    reqs = c1_requests()
    for r in reqs:
        eng.submit(r)
    eng.run_until_complete()
    out = {
        "model": "random-init Qwen2.5-0.5B architecture (torch.manual_seed(0), fp32)",
        "param_sum": probe,
        "requests": [{"request_id": r.request_id, "prompt": list(r.prompt_token_ids)}
                     for r in reqs],
        "generated": {s.request.request_id: list(s.generated_token_ids)
                      for s in eng.finished_sequences},
        "top2_margins": margins,
    }
    (OUT / "greedy_c1.json").write_text(json.dumps(out))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", help="the reference project's checkout")
    ap.add_argument("--skip-greedy", action="store_true")
    args = ap.parse_args()
    make_storage_roundtrip()
    make_layouts()
    make_traces()
    make_attention()
    if not args.skip_greedy:
        make_greedy_c1()
    for f in sorted(OUT.iterdir()):
        if f.suffix in (".json", ".npz"):
            print(f"{f.name}: {f.stat().st_size} bytes")


if __name__ == "__main__":
    main()
