"""End-to-end parity of the CUDA path through the engine and the ModelRunner drop-in.

* Greedy tokens, fp32: the reference engine's configuration-1 run (random-init
  Qwen2.5-0.5B architecture from torch.manual_seed(0), 8 requests, 32 greedy tokens each,
  block 16, pool 2048) recorded by tests/golden/make_golden.py must be reproduced token
  for token by this package's engine + B200PagedModelRunner on the GPU.
* Logits, bf16: 2-layer models with the Qwen2.5-1.5B attention shape (12/2 heads,
  head_dim 128) and the Qwen2.5-0.5B one (14/2 heads, head_dim 64) against the reference-style packed runner (gather + dense mask + SDPA)
  run in fp32 on the same weights. The bf16 error budget is that of the reference path
  itself: the same packed runner run in bf16 on the GPU sets it, and this package's logits
  must stay within 1.5x of its max-abs error (and never above 0.1); top-1 agreement on
  every row where the fp32 margin exceeds 5e-2.
"""

from __future__ import annotations

import copy
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from llm_engineering_b200 import engine as eng
from llm_engineering_b200.runner import B200PagedModelRunner
from llm_engineering_b200.storage import PagedKVStorage
from oracle.runner import ReferencePackedRunner

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def c1_model():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=151936, hidden_size=896, intermediate_size=4864,
                      num_hidden_layers=24, num_attention_heads=14, num_key_value_heads=2,
                      rope_theta=1_000_000.0, tie_word_embeddings=True,
                      max_position_embeddings=32768, attn_implementation="sdpa")
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def test_greedy_tokens_match_reference_engine_config1_fp32():
    golden = json.loads((GOLDEN / "greedy_c1.json").read_text())
    torch.backends.cuda.matmul.allow_tf32 = False
    model = c1_model()
    param_sum = float(sum(p.double().sum() for p in model.parameters()).item())
    assert abs(param_sum - golden["param_sum"]) < 1e-6 * abs(golden["param_sum"]) + 1e-3, \
        "random-init weights differ from the ones the golden tokens were generated with"
    dev = torch.device("cuda")
    model = model.to(dev)
    storage = PagedKVStorage(num_layers=24, num_blocks=2048, block_size=16, num_kv_heads=2,
                             head_dim=64, dtype=torch.float32, device=dev)
    runner = B200PagedModelRunner(model, dev, storage)
    cfg = eng.EngineConfiguration(device="cuda", block_size=16, num_blocks=2048, max_sequences=8,
                                  max_batched_tokens=2048, seed=0)
    engine = eng.Engine(configuration=cfg, model_runner=runner)
    for r in golden["requests"]:
        engine.submit(eng.Request(request_id=r["request_id"], prompt_token_ids=tuple(r["prompt"]),
                                  max_new_tokens=32, ignore_eos=True))
    engine.run_until_complete()
    assert runner.device_error() == 0
    got = {s.request.request_id: list(s.generated_token_ids) for s in engine.finished_sequences}
    for rid, want in golden["generated"].items():
        assert got[rid] == want, (rid, got[rid], want)


def test_chunked_prefill_engine_reproduces_reference_tokens_fp32():
    """The configuration-1 run again, with chunked prefill and a 48-token step budget (the
    prompts, 16..128 tokens, mostly span several steps and share them with decodes): the
    tokens must still be the reference engine's."""
    golden = json.loads((GOLDEN / "greedy_c1.json").read_text())
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda")
    model = c1_model().to(dev)
    storage = PagedKVStorage(num_layers=24, num_blocks=2048, block_size=16, num_kv_heads=2,
                             head_dim=64, dtype=torch.float32, device=dev)
    runner = B200PagedModelRunner(model, dev, storage)
    cfg = eng.EngineConfiguration(device="cuda", block_size=16, num_blocks=2048, max_sequences=8,
                                  max_batched_tokens=48, seed=0, enable_chunked_prefill=True)
    engine = eng.Engine(configuration=cfg, model_runner=runner)
    for r in golden["requests"]:
        engine.submit(eng.Request(request_id=r["request_id"], prompt_token_ids=tuple(r["prompt"]),
                                  max_new_tokens=32, ignore_eos=True))
    engine.run_until_complete()
    assert runner.device_error() == 0
    got = {s.request.request_id: list(s.generated_token_ids) for s in engine.finished_sequences}
    for rid, want in golden["generated"].items():
        assert got[rid] == want, (rid, got[rid], want)


def small_1p5b_attention_model(seed=0, hidden=1536, heads=12):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=1000, hidden_size=hidden, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=heads, num_key_value_heads=2,
                      rope_theta=1_000_000.0, max_position_embeddings=4096,
                      attn_implementation="sdpa")
    torch.manual_seed(seed)
    return Qwen2ForCausalLM(cfg).eval()


@pytest.mark.parametrize("hidden,heads", [(1536, 12), (896, 14)])
def test_bf16_runner_logits_match_reference_path(hidden, heads):
    dev = torch.device("cuda")
    base = small_1p5b_attention_model(hidden=hidden, heads=heads)
    d = hidden // heads  # 128 (Qwen2.5-1.5B shape) or 64 (Qwen2.5-0.5B shape)
    ref_model = copy.deepcopy(base).float()
    ours_model = copy.deepcopy(base).to(dev, torch.bfloat16)
    bs, blocks = 16, 256
    storage = PagedKVStorage(2, blocks, bs, 2, d, torch.bfloat16, dev)
    runner = B200PagedModelRunner(ours_model, dev, storage)
    kr = torch.zeros(2, blocks * bs, 2, d)
    vr = torch.zeros(2, blocks * bs, 2, d)
    reference = ReferencePackedRunner(ref_model, kr, vr, bs)
    # the reference path itself in bf16 (GPU): its distance from fp32 is the bf16 budget
    kb = torch.zeros(2, blocks * bs, 2, d, dtype=torch.bfloat16, device=dev)
    reference_bf16 = ReferencePackedRunner(copy.deepcopy(base).to(dev, torch.bfloat16), kb,
                                           torch.zeros_like(kb), bs)
    rng = np.random.default_rng(9)
    requests = [eng.Request(request_id=f"r{i}",
                            prompt_token_ids=tuple(int(x) for x in rng.integers(0, 1000, size=n)),
                            max_new_tokens=5, ignore_eos=True)
                for i, n in enumerate([40, 17, 250, 129, 64, 3])]
    cfg = eng.EngineConfiguration(block_size=bs, num_blocks=blocks, max_sequences=6,
                                  max_batched_tokens=1024)

    class Both:
        """Runs both runners on every step; the engine follows the reference's tokens."""

        def __init__(self):
            self.max_err = 0.0
            self.budget = 0.0
            self.checked = 0

        def forward(self, executions):
            want = reference.forward(executions)
            got = ours.forward(executions).float().cpu()
            torch_bf16 = reference_bf16.forward(executions).float().cpu()
            self.max_err = max(self.max_err, (got - want).abs().max().item())
            self.budget = max(self.budget, (torch_bf16 - want).abs().max().item())
            top2 = torch.topk(want, 2, dim=-1).values
            confident = (top2[:, 0] - top2[:, 1]) > 5e-2
            agree = got.argmax(-1) == want.argmax(-1)
            assert bool((agree | ~confident).all())
            self.checked += len(executions)
            return want

    ours = runner
    both = Both()
    engine = eng.Engine(configuration=cfg, model_runner=both)
    for r in requests:
        engine.submit(r)
    engine.run_until_complete()
    assert runner.device_error() == 0
    assert both.checked > 6
    assert both.max_err <= max(1.5 * both.budget, 2e-2) and both.max_err < 0.1, \
        (both.max_err, both.budget)


def test_chunked_prefill_slices_in_a_mixed_step_match_whole_prefill():
    """A 700-token prompt prefilled as two slices (300, then 400 tokens that attend to the
    first 300 through the pool), the second slice sharing its step with 12 decodes, gives
    the same last-token logits as one whole-prompt prefill; the decodes match the
    reference-style packed runner (fp32) in the same step."""
    dev = torch.device("cuda")
    base = small_1p5b_attention_model(seed=3)
    ours_model = copy.deepcopy(base).to(dev, torch.bfloat16)
    bs, blocks = 16, 512
    rng = np.random.default_rng(21)
    prompt = tuple(int(x) for x in rng.integers(0, 1000, size=700))
    whole_blocks = tuple(range(100, 100 + 44))  # 44 blocks of 16 cover 700 tokens

    # whole-prompt prefill on its own pool
    st_a = PagedKVStorage(2, blocks, bs, 2, 128, torch.bfloat16, dev)
    run_a = B200PagedModelRunner(copy.deepcopy(ours_model), dev, st_a)
    seq_full = eng.SequenceState(eng.Request("p", prompt, 8))
    whole = run_a.forward([eng.ModelExecution(seq_full, eng.ExecutionPhase.PREFILL,
                                              block_ids=whole_blocks, block_size=bs)])

    # the same prompt in two slices on a second pool; step 2 also carries 12 decodes
    st_b = PagedKVStorage(2, blocks, bs, 2, 128, torch.bfloat16, dev)
    run_b = B200PagedModelRunner(ours_model, dev, st_b)
    seq_part = eng.SequenceState(eng.Request("p", prompt[:300], 8))
    run_b.forward([eng.ModelExecution(seq_part, eng.ExecutionPhase.PREFILL,
                                      block_ids=whole_blocks[:19], block_size=bs)])
    # decodes: prefill their prompts first (one step), then one decode token each
    dec = []
    for i in range(12):
        n = int(rng.integers(20, 200))
        toks = tuple(int(x) for x in rng.integers(0, 1000, size=n))
        blk = tuple(range(200 + i * 16, 200 + i * 16 + (n + 1 + bs - 1) // bs))
        dec.append((eng.SequenceState(eng.Request(f"d{i}", toks, 8)), blk))
    run_b.forward([eng.ModelExecution(s, eng.ExecutionPhase.PREFILL, block_ids=b, block_size=bs)
                   for s, b in dec])
    for s, _ in dec:
        s.append_token(7)
    step = [eng.ModelExecution(s, eng.ExecutionPhase.DECODE, block_ids=b, block_size=bs)
            for s, b in dec]
    step.append(eng.ModelExecution(seq_full, eng.ExecutionPhase.PREFILL, block_ids=whole_blocks,
                                   block_size=bs, query_length=400))
    got = run_b.forward(step).float().cpu()
    assert run_b.device_error() == 0 and run_a.device_error() == 0
    # the chunked prefill's last token == whole prefill's last token (bf16 path both times)
    w0 = whole[0].float().cpu()
    assert (got[-1] - w0).abs().max().item() < 5e-2
    top2 = torch.topk(w0, 2).values
    if (top2[0] - top2[1]).item() > 5e-2:  # a confident top-1 must agree
        assert got[-1].argmax().item() == w0.argmax().item()

    # the decode rows against the reference-style path in fp32 on the same weights
    ref_model = copy.deepcopy(base).float()
    kr = torch.zeros(2, blocks * bs, 2, 128)
    vr = torch.zeros(2, blocks * bs, 2, 128)
    reference = ReferencePackedRunner(ref_model, kr, vr, bs)
    for s, _ in dec:  # rebuild their history in the reference pool: prompt, then decode
        s.discard_generated()
    reference.forward([eng.ModelExecution(s, eng.ExecutionPhase.PREFILL, block_ids=b,
                                          block_size=bs) for s, b in dec])
    for s, _ in dec:
        s.append_token(7)
    want = reference.forward([eng.ModelExecution(s, eng.ExecutionPhase.DECODE, block_ids=b,
                                                 block_size=bs) for s, b in dec])
    assert (got[:12] - want).abs().max().item() < 5e-2


def qwen2_1p5b_model(dev):
    """Random-init Qwen2.5-1.5B architecture (28 layers, hidden 1536, 12/2 heads,
    head_dim 128, FFN 8960, vocab 151936, tied embeddings), fp32, initialised on `dev`."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=151936, hidden_size=1536, intermediate_size=8960,
                      num_hidden_layers=28, num_attention_heads=12, num_key_value_heads=2,
                      rope_theta=1_000_000.0, tie_word_embeddings=True,
                      max_position_embeddings=32768, attn_implementation="sdpa")
    torch.manual_seed(0)
    with torch.device(dev):
        return Qwen2ForCausalLM(cfg).eval()


def test_bf16_engine_through_tensor_core_kernels_config1_requests():
    """The configuration-1 requests (8 prompts of 16..128 tokens, 32 greedy tokens each) on
    a bf16 random-init Qwen2.5-1.5B, so that every step runs the tensor-core kernels: the
    fused write + decode (paged_decode_tc) for decode rows and paged_prefill_tc for prompts.

    * Every attention call of every layer and step is checked against the oracle's fp32
      attention over the same bf16 queries and pool contents (after the step's K/V writes):
      max-abs 2e-2 and mean-abs 2e-3, the parity bounds of this path.
    * Logits, every step, against the reference-style packed runner (gather + dense mask
      + SDPA) in fp32 on the same weights: within 1.5x the distance of that same runner in
      bf16 (the bf16 budget of the reference path itself), and the same top-1 token on
      every row whose fp32 top-2 margin exceeds twice that budget. The engine follows the
      fp32 runner's tokens.
    * No bf16 call took a CUDA-core kernel (the fallback counters do not move)."""
    from transformers import AttentionInterface

    from llm_engineering_b200 import ops
    from llm_engineering_b200 import runner as runner_mod
    from oracle import paged as ref

    golden = json.loads((GOLDEN / "greedy_c1.json").read_text())
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    dev = torch.device("cuda")
    base = qwen2_1p5b_model(dev)
    ours_model = copy.deepcopy(base).to(torch.bfloat16)
    budget_model = copy.deepcopy(base).to(torch.bfloat16)
    bs, blocks, layers = 16, 2048, 28
    storage = PagedKVStorage(layers, blocks, bs, 2, 128, torch.bfloat16, dev)
    ours = B200PagedModelRunner(ours_model, dev, storage)
    shape = (layers, blocks * bs, 2, 128)
    reference = ReferencePackedRunner(base, torch.zeros(shape, device=dev),
                                      torch.zeros(shape, device=dev), bs)
    reference_bf16 = ReferencePackedRunner(
        budget_model, torch.zeros(shape, dtype=torch.bfloat16, device=dev),
        torch.zeros(shape, dtype=torch.bfloat16, device=dev), bs)

    attn_stats = {"calls": 0, "max": 0.0, "decode_rows": 0, "prefill_rows": 0}

    def checked_attention(module, query, key, value, attention_mask, **kwargs):
        out, _ = runner_mod.paged_attention(module, query, key, value, attention_mask, **kwargs)
        b = runner_mod._active_batch.get()
        layer = module.layer_idx
        q = query[0].transpose(0, 1)
        scale = kwargs.get("scaling") or q.shape[-1] ** -0.5
        tables = [row[row >= 0].tolist() for row in b.block_tables.cpu().numpy()]
        ctx = b.context_lens.cpu().tolist()
        cu = b.cu_seqlens_q.cpu().tolist()
        nd = b.num_decode
        parts = []
        if nd:
            parts.append(ref.decode_attention(q[:nd], b.key_cache, b.value_cache, layer,
                                              tables[:nd], ctx[:nd], b.block_size, scale))
        if nd < b.num_execs:
            parts.append(ref.prefill_attention(q, b.key_cache, b.value_cache, layer, tables[nd:],
                                               cu[nd:], ctx[nd:], b.block_size, scale))
        want = torch.cat(parts, 0)
        diff = (out[0].float() - want).abs()
        assert diff.max().item() < 2e-2 and diff.mean().item() < 2e-3, (layer, diff.max().item())
        attn_stats["calls"] += 1
        attn_stats["max"] = max(attn_stats["max"], diff.max().item())
        attn_stats["decode_rows"] += nd
        attn_stats["prefill_rows"] += cu[-1] - cu[nd]
        return out, None

    class Both:
        def __init__(self):
            self.max_err = self.budget = 0.0
            self.checked = self.confident = 0

        def forward(self, executions):
            want = reference.forward(executions).float()
            got = ours.forward(executions).float()
            in_bf16 = reference_bf16.forward(executions).float()
            budget = (in_bf16 - want).abs().max().item()
            self.max_err = max(self.max_err, (got - want).abs().max().item())
            self.budget = max(self.budget, budget)
            top2 = torch.topk(want, 2, dim=-1).values
            confident = (top2[:, 0] - top2[:, 1]) > 2 * budget
            agree = got.argmax(-1) == want.argmax(-1)
            assert bool((agree | ~confident).all())
            self.checked += len(executions)
            self.confident += int(confident.sum().item())
            return want

    AttentionInterface.register(runner_mod.ATTENTION_NAME, checked_attention)
    fallbacks = ops.cuda_core_fallbacks()
    try:
        both = Both()
        cfg = eng.EngineConfiguration(device="cuda", block_size=bs, num_blocks=blocks,
                                      max_sequences=8, max_batched_tokens=2048, seed=0)
        engine = eng.Engine(configuration=cfg, model_runner=both)
        for r in golden["requests"]:
            engine.submit(eng.Request(request_id=r["request_id"],
                                      prompt_token_ids=tuple(r["prompt"]), max_new_tokens=32,
                                      ignore_eos=True))
        engine.run_until_complete()
    finally:
        AttentionInterface.register(runner_mod.ATTENTION_NAME, runner_mod.paged_attention)
    assert ops.cuda_core_fallbacks() == fallbacks  # every bf16 call ran on tensor cores
    assert both.checked == 8 * 32
    assert attn_stats["calls"] >= 32 * layers and attn_stats["decode_rows"] > 0
    assert attn_stats["prefill_rows"] > 0
    assert both.max_err <= max(1.5 * both.budget, 2e-2), (both.max_err, both.budget)
    assert both.confident > 0


class _ReferenceStyleSequence:
    """The fields of the reference's SequenceState (serving/engine/sequence.py) that a
    ModelRunner reads: the request, the generated tokens as a list, the current length."""

    def __init__(self, seq):
        self.request = seq.request
        self.generated_token_ids = list(seq.generated_token_ids)
        self.current_length = seq.current_length


class _ReferenceStyleExecution:
    """The reference's ModelExecution (serving/engine/execution.py:16-47): the sequence, a
    phase and the slot of every position of the whole history, nothing else."""

    def __init__(self, ex):
        self.sequence = _ReferenceStyleSequence(ex.sequence)
        self.phase = ex.phase
        self.slot_ids = tuple(ex.slot_ids)


def test_reference_style_executions_reproduce_config1_tokens():
    """The CUDA half of the drop-in under the reference's engine (whose CPU half, with the
    reference's own Engine / PagedKVCache, is tests/test_dropin_reference_cpu.py): every
    step reaches B200PagedModelRunner as the reference engine hands it over, executions
    with whole-history slot_ids only (engine.py:106-133), and the configuration-1 golden
    tokens of the reference engine come out token for token."""
    golden = json.loads((GOLDEN / "greedy_c1.json").read_text())
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda")
    model = c1_model().to(dev)
    storage = PagedKVStorage(num_layers=24, num_blocks=2048, block_size=16, num_kv_heads=2,
                             head_dim=64, dtype=torch.float32, device=dev)
    runner = B200PagedModelRunner(model, dev, storage)

    class AsReference:
        steps = 0

        def forward(self, executions):
            self.steps += 1
            return runner.forward([_ReferenceStyleExecution(ex) for ex in executions])

    cfg = eng.EngineConfiguration(device="cuda", block_size=16, num_blocks=2048, max_sequences=8,
                                  max_batched_tokens=2048, seed=0)
    adapter = AsReference()
    engine = eng.Engine(configuration=cfg, model_runner=adapter)
    for r in golden["requests"]:
        engine.submit(eng.Request(request_id=r["request_id"], prompt_token_ids=tuple(r["prompt"]),
                                  max_new_tokens=32, ignore_eos=True))
    engine.run_until_complete()
    assert adapter.steps == 32
    got = {s.request.request_id: list(s.generated_token_ids) for s in engine.finished_sequences}
    for rid, want in golden["generated"].items():
        assert got[rid] == want, (rid, got[rid], want)
