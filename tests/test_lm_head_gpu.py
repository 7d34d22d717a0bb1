"""K6 — the LM head fused with the greedy argmax — against torch on the same inputs.

The reference's greedy token of a row is ``argmax`` over the LM head's logits in the model
dtype (serving/engine/paged_model_runner.py:83-91 then serving/engine/sampling.py:78-79);
torch's argmax takes the lowest index among equal values. K6 computes the same logits in
fp32 on the tensor cores, rounds each to the model dtype and keeps the first maximum, so:

* its id equals torch's ``argmax((hidden @ weight.T).to(dtype))`` on every row whose two
  largest rounded logits differ (both paths then agree on the rounded values; they can
  only differ where cuBLAS's and K6's fp32 sums fall on opposite sides of a rounding
  boundary), and on every row the logit of its id is within one rounding step of the
  largest;
* exactly equal logits (duplicated weight rows) give the lowest index;
* the returned maximum is the rounded largest logit.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _inputs(rows, vocab, hidden, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    h = (torch.randn(rows, hidden, generator=g) * 0.5).to(dtype).cuda()
    w = (torch.randn(vocab, hidden, generator=g) / hidden ** 0.5).to(dtype).cuda()
    return h, w


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,vocab,hidden", [
    (1, 1000, 128), (7, 4099, 896), (128, 151936, 1536), (129, 20000, 1536),
    (192, 151936, 1536), (256, 9000, 896), (300, 33000, 1536),
])
def test_lm_head_argmax_matches_torch(ops, rows, vocab, hidden, dtype):
    h, w = _inputs(rows, vocab, hidden, dtype, seed=rows * 7 + vocab)
    ws = torch.zeros(ops.lm_head_argmax_workspace_size(rows), dtype=torch.uint8, device="cuda")
    out_max = torch.empty(rows, dtype=torch.float32, device="cuda")
    ids = ops.lm_head_argmax(h, w, ws, out_max=out_max)
    torch.cuda.synchronize()
    logits = (h @ w.T).float()                 # cuBLAS, rounded to dtype, as the LM head
    exact = (h.float() @ w.float().T)          # fp32 products for the tolerance check
    want = logits.argmax(-1)
    top2 = torch.topk(logits, 2, dim=-1).values
    distinct = top2[:, 0] > top2[:, 1]
    assert bool(((ids == want) | ~distinct).all()), int(((ids != want) & distinct).sum())
    step = torch.finfo(dtype).eps * exact.abs().max(-1).values
    got = exact.gather(1, ids.view(-1, 1)).squeeze(1)
    assert bool((got >= exact.max(-1).values - 2 * step).all())
    assert torch.allclose(out_max, top2[:, 0], rtol=0, atol=float(step.max()) * 2)
    assert int(ws.count_nonzero()) == 0        # the launch left its workspace zeroed


def test_lm_head_argmax_ties_go_to_the_lowest_index(ops):
    rows, vocab, hidden = 5, 3000, 256
    h, w = _inputs(rows, vocab, hidden, torch.bfloat16, seed=3)
    logits = (h @ w.T).float()
    best = logits.argmax(-1)
    # copy each row's winning weight row to later and earlier vocabulary entries: equal
    # logits, and the earliest copy must win
    for r in range(rows):
        src = int(best[r])
        for dst in (2999 - r, 1500 + r, 10 + r):
            w[dst] = w[src]
    ws = torch.zeros(ops.lm_head_argmax_workspace_size(rows), dtype=torch.uint8, device="cuda")
    ids = ops.lm_head_argmax(h, w, ws)
    want = (h @ w.T).float().argmax(-1)        # torch: first maximal index
    assert torch.equal(ids, want)


def test_lm_head_argmax_nan_row_gets_a_valid_token(ops):
    """A NaN hidden row makes every logit of the row NaN: its id is 0, as torch's argmax
    gives, never an invalid token; the other rows are unaffected."""
    rows, vocab, hidden = 6, 5000, 256
    h, w = _inputs(rows, vocab, hidden, torch.bfloat16, seed=11)
    h[2] = float("nan")
    ws = torch.zeros(ops.lm_head_argmax_workspace_size(rows), dtype=torch.uint8, device="cuda")
    out_max = torch.empty(rows, dtype=torch.float32, device="cuda")
    ids = ops.lm_head_argmax(h, w, ws, out_max=out_max)
    want = (h @ w.T).float().argmax(-1)
    assert int(ids[2]) == int(want[2]) == 0
    assert bool(out_max[2].isnan())
    keep = [0, 1, 3, 4, 5]
    assert torch.equal(ids[keep], want[keep])


def test_lm_head_argmax_unsupported_shapes_return_none(ops):
    h = torch.randn(4, 100, device="cuda").to(torch.bfloat16)  # hidden not a multiple of 64
    w = torch.randn(50, 100, device="cuda").to(torch.bfloat16)
    ws = torch.zeros(ops.lm_head_argmax_workspace_size(4), dtype=torch.uint8, device="cuda")
    assert ops.lm_head_argmax(h, w, ws) is None
    assert ops.lm_head_argmax(h.float()[:, :64].contiguous(), w.float()[:, :64].contiguous(),
                              ws) is None  # fp32 keeps the logits path


def test_engine_greedy_tokens_through_k6_equal_logits_path():
    """The configuration-1 requests on a bf16 random-init Qwen2.5-1.5B: the engine's greedy
    tokens through ``greedy_tokens`` (K6) equal those through ``forward`` + argmax."""
    from llm_engineering_b200 import engine as eng
    from llm_engineering_b200.runner import B200PagedModelRunner
    from llm_engineering_b200.storage import PagedKVStorage
    from test_runner_gpu import qwen2_1p5b_model

    golden = json.loads((GOLDEN / "greedy_c1.json").read_text())
    dev = torch.device("cuda")
    model = qwen2_1p5b_model(dev).to(torch.bfloat16)

    def run(fused: bool):
        storage = PagedKVStorage(28, 2048, 16, 2, 128, torch.bfloat16, dev)
        runner = B200PagedModelRunner(model, dev, storage)
        calls = {"k6": 0}
        if fused:
            inner = runner.greedy_tokens

            def counted(executions):
                calls["k6"] += 1
                out = inner(executions)
                assert out is not None
                return out
            runner.greedy_tokens = counted
        else:
            runner.greedy_tokens = lambda executions: None
        cfg = eng.EngineConfiguration(device="cuda", block_size=16, num_blocks=2048,
                                      max_sequences=8, max_batched_tokens=2048, seed=0)
        engine = eng.Engine(configuration=cfg, model_runner=runner)
        for r in golden["requests"]:
            engine.submit(eng.Request(request_id=r["request_id"],
                                      prompt_token_ids=tuple(r["prompt"]), max_new_tokens=32,
                                      ignore_eos=True))
        done = engine.run_until_complete()
        return {s.request.request_id: list(s.generated_token_ids) for s in done}, calls["k6"]

    with_k6, n = run(True)
    with_logits, _ = run(False)
    assert n > 0
    assert with_k6 == with_logits
