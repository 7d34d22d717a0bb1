"""Host logic of B200PagedModelRunner on CPU, against the reference-style packed runner.

The runner's kernel module is monkeypatched, in this file only, with a CPU stand-in built
from the oracle (the product has no such seam: its runner always calls the CUDA ops): the
test checks the runner's own work — per-step metadata, the HF cache hook, the
registered attention function, the decode/prefill split and the logit rows — on a tiny
random Qwen2, driving both runners with this package's engine. The CUDA kernels
themselves are checked on the GPU (test_kernels_gpu.py, test_runner_gpu.py).
"""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from llm_engineering_b200 import engine as eng
from llm_engineering_b200 import runner as runner_mod
from llm_engineering_b200.runner import B200PagedModelRunner
from oracle import paged as ref
from oracle.runner import ReferencePackedRunner


class CpuKernels:
    """The ops API of llm_engineering_b200.ops, computed on the CPU with the oracle."""

    @staticmethod
    def kv_write(kc, vc, layer, slot_mapping, keys, values, err_flag=None):
        s = slot_mapping.long()
        keep = s >= 0
        kc[layer][s[keep]] = keys[keep]
        vc[layer][s[keep]] = values[keep]

    @staticmethod
    def decode_workspace_size(*args):
        return 16

    @staticmethod
    def _tables(bt, n):
        return [row[row >= 0].tolist() for row in bt[:n]]

    def paged_decode(self, q, kc, vc, layer, bt, ctx, bs, scale, out=None, workspace=None,
                     err_flag=None):
        n = q.shape[0]
        res = ref.decode_attention(q, kc, vc, layer, self._tables(bt, n), ctx[:n].tolist(), bs,
                                   scale)
        out.copy_(res.to(out.dtype))
        return out

    def paged_decode_append(self, q, new_k, new_v, kc, vc, layer, bt, ctx, bs, scale, out=None,
                            workspace=None, err_flag=None):
        n = q.shape[0]
        for i in range(n):  # the new row goes to the slot of position ctx - 1
            pos = int(ctx[i]) - 1
            slot = int(bt[i, pos // bs]) * bs + pos % bs
            kc[layer][slot] = new_k[i]
            vc[layer][slot] = new_v[i]
        return self.paged_decode(q, kc, vc, layer, bt, ctx, bs, scale, out=out,
                                 workspace=workspace, err_flag=err_flag)

    def paged_prefill(self, q, kc, vc, layer, bt, cu, ctx, max_q, bs, scale, out=None,
                      err_flag=None, num_rows=None):
        cu_l = cu.tolist()
        n = len(cu_l) - 1
        res = ref.prefill_attention(q, kc, vc, layer, self._tables(bt, n), cu_l,
                                    ctx[:n].tolist(), bs, scale)
        out[cu_l[0]:cu_l[-1]] = res[cu_l[0]:cu_l[-1]].to(out.dtype) if res.shape[0] == q.shape[0] \
            else res.to(out.dtype)
        return out

    @staticmethod
    def build_metadata(qlens, ctx, rows, mirror, bs, total_q, max_blocks, err_flag=None):
        q = qlens.tolist()
        k = ctx.tolist()
        cu_q = np.concatenate([[0], np.cumsum(q)]).astype(np.int32)
        cu_k = np.concatenate([[0], np.cumsum(k)]).astype(np.int32)
        pos, slots = [], []
        for i, (qi, ki) in enumerate(zip(q, k, strict=True)):
            table = mirror[int(rows[i])]
            p = np.arange(ki - qi, ki)
            pos.append(p)
            slots.append(table.numpy()[p // bs].astype(np.int64) * bs + p % bs)
        # padded per-execution tables gathered from the mirror rows (-1 past each need)
        width = max(max_blocks, 1)
        bt = torch.full((len(q), width), -1, dtype=torch.int32)
        for i, ki in enumerate(k):
            nblk = min(-(-ki // bs), width, mirror.shape[1])
            bt[i, :nblk] = mirror[int(rows[i]), :nblk]
        return {
            "cu_seqlens_q": torch.from_numpy(cu_q),
            "cu_seqlens_k": torch.from_numpy(cu_k),
            "positions": torch.from_numpy(np.concatenate(pos).astype(np.int64)),
            "slot_mapping": torch.from_numpy(np.concatenate(slots).astype(np.int32)),
            "logit_indices": torch.from_numpy((cu_q[1:] - 1).astype(np.int64)),
            "block_tables": bt,
        }


@pytest.fixture(autouse=True)
def cpu_kernels(monkeypatch):
    monkeypatch.setattr(runner_mod, "_ops", CpuKernels())


def tiny_model(seed=0):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=97, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, rope_theta=10000.0,
                      max_position_embeddings=512, attn_implementation="sdpa")
    torch.manual_seed(seed)
    return Qwen2ForCausalLM(cfg).eval()


def pool(layers, blocks, bs, hkv, d):
    return (torch.zeros(layers, blocks * bs, hkv, d), torch.zeros(layers, blocks * bs, hkv, d))


def run_engine(runner, requests, cfg):
    engine = eng.Engine(configuration=cfg, model_runner=runner)
    for r in requests:
        engine.submit(r)
    engine.run_until_complete()
    return {s.request.request_id: list(s.generated_token_ids) for s in engine.finished_sequences}


@pytest.mark.parametrize("block_size,num_blocks", [(4, 64), (4, 12)])
def test_runner_matches_reference_packed_path(block_size, num_blocks):
    model = tiny_model()
    rng = np.random.default_rng(3)
    requests = [eng.Request(request_id=f"r{i}",
                            prompt_token_ids=tuple(int(x) for x in rng.integers(0, 97, size=int(n))),
                            max_new_tokens=6, ignore_eos=True)
                for i, n in enumerate([5, 9, 3, 13])]
    cfg = eng.EngineConfiguration(block_size=block_size, num_blocks=num_blocks, max_sequences=3,
                                  max_batched_tokens=40)
    kc, vc = pool(2, num_blocks, block_size, 2, 16)
    ours = B200PagedModelRunner(copy.deepcopy(model), torch.device("cpu"),
                                _Storage(kc, vc, block_size))
    kr, vr = pool(2, num_blocks, block_size, 2, 16)
    theirs = ReferencePackedRunner(copy.deepcopy(model), kr, vr, block_size)
    got = run_engine(ours, requests, cfg)
    expect = run_engine(theirs, requests, cfg)
    assert got == expect
    assert all(len(v) == 6 for v in got.values())


def test_runner_logits_match_for_mixed_step_and_reference_style_slots():
    """Reference ModelExecution objects (slot_ids only), decode + prefill in one step."""
    model = tiny_model(1)
    bs = 4
    kc, vc = pool(2, 32, bs, 2, 16)
    kr, vr = pool(2, 32, bs, 2, 16)
    ours = B200PagedModelRunner(copy.deepcopy(model), torch.device("cpu"), _Storage(kc, vc, bs))
    theirs = ReferencePackedRunner(copy.deepcopy(model), kr, vr, bs)

    def execs(phase_a):
        ra = eng.Request("a", (1, 2, 3, 4, 5), 8)
        sa = eng.SequenceState(ra, generated_token_ids=[6] if phase_a == "decode" else [])
        rb = eng.Request("b", (7, 8, 9), 8)
        sb = eng.SequenceState(rb)
        a_slots = tuple(5 * bs + p for p in range(sa.current_length))
        b_slots = (2 * bs, 2 * bs + 1, 2 * bs + 2)
        return [eng.ModelExecution(sa, phase_a, a_slots),
                eng.ModelExecution(sb, eng.ExecutionPhase.PREFILL, b_slots)]

    for step in (execs("prefill"), execs("decode")):
        got = ours.forward(step)
        want = theirs.forward(step)
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)
    # non-block-structured slot ids (one slot per block) take the same path
    ra = eng.Request("c", (3, 1, 4, 1, 5, 9), 8)
    sc = eng.SequenceState(ra)
    odd = (1, 30, 7, 12, 99, 64)
    got = ours.forward([eng.ModelExecution(sc, eng.ExecutionPhase.PREFILL, odd)])
    want = theirs.forward([eng.ModelExecution(sc, eng.ExecutionPhase.PREFILL, odd)])
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def test_chunked_prefill_runs_give_the_tokens_of_whole_prefill():
    """Prompts longer than the step budget, prefilled in chunks by this package's engine
    through the B200 runner (chunked queries attend to the whole history in the pool), give
    the same greedy tokens as whole-prompt prefill with a budget that fits them."""
    model = tiny_model(2)
    bs, nb = 4, 96
    rng = np.random.default_rng(9)
    requests = [eng.Request(request_id=f"r{i}",
                            prompt_token_ids=tuple(int(x) for x in rng.integers(0, 97, size=n)),
                            max_new_tokens=5, ignore_eos=True)
                for i, n in enumerate([37, 6, 21, 50])]
    whole_cfg = eng.EngineConfiguration(block_size=bs, num_blocks=nb, max_sequences=4,
                                        max_batched_tokens=128)
    kc, vc = pool(2, nb, bs, 2, 16)
    whole = B200PagedModelRunner(copy.deepcopy(model), torch.device("cpu"), _Storage(kc, vc, bs))
    expect = run_engine(whole, requests, whole_cfg)
    chunk_cfg = eng.EngineConfiguration(block_size=bs, num_blocks=nb, max_sequences=4,
                                        max_batched_tokens=12, enable_chunked_prefill=True)
    kc2, vc2 = pool(2, nb, bs, 2, 16)
    chunked = B200PagedModelRunner(copy.deepcopy(model), torch.device("cpu"),
                                   _Storage(kc2, vc2, bs))
    assert run_engine(chunked, requests, chunk_cfg) == expect


def test_runner_rejects_empty_batch():
    kc, vc = pool(2, 8, 4, 2, 16)
    ours = B200PagedModelRunner(tiny_model(), torch.device("cpu"), _Storage(kc, vc, 4))
    with pytest.raises(ValueError, match="At least one execution is required."):
        ours.forward([])


class _Storage:
    def __init__(self, kc, vc, bs):
        self.key_cache, self.value_cache, self.block_size = kc, vc, bs


def test_block_table_mirror_tracks_appends_readmissions_and_growth():
    """The runner's device mirror of block tables, driven by a random step sequence: tables
    that grow by appended blocks, sequences that leave and come back under a new admission
    with new blocks, more rows and columns than the first allocation. After every step each
    live row must hold exactly its sequence's block list."""
    from llm_engineering_b200.runner import _TableMirror

    rng = np.random.default_rng(17)
    mirror = _TableMirror(torch.device("cpu"), rows=4, cols=2)
    tables: dict[tuple[str, int], list[int]] = {}
    admissions = {f"r{i}": 1 for i in range(40)}
    next_block = 0
    for _ in range(200):
        running = [f"r{i}" for i in rng.choice(40, size=int(rng.integers(1, 12)), replace=False)]
        keys, lists = [], []
        for rid in running:
            if rng.random() < 0.1:  # preempted and re-admitted: a new table
                admissions[rid] += 1
            key = (rid, admissions[rid])
            t = tables.setdefault(key, [])
            for _ in range(int(rng.integers(0, 3)) + (0 if t else 1)):
                t.append(next_block)
                next_block += 1
            keys.append(key)
            lists.append(tuple(t))
        rows = mirror.sync(keys, lists)
        assert len(set(rows)) == len(rows)
        for row, blocks in zip(rows, lists):
            assert mirror.table[row, :len(blocks)].tolist() == list(blocks)
    assert mirror.table.shape[0] >= 12 and mirror.table.shape[1] > 2


def test_wait_timeout_resets_every_scratch_buffer(monkeypatch):
    """After a bounded wait gave up (B2P_DEV_WAIT_TIMEOUT) a launch may have left split-K
    counters or greedy-pick keys set: device_error() zeroes the decode workspace and the K6
    workspace and resets the prefill claim counters, then reports the bits once."""
    from llm_engineering_b200._lib import DEV_BLOCK_RANGE, DEV_WAIT_TIMEOUT

    kc, vc = pool(2, 8, 4, 2, 16)
    ours = B200PagedModelRunner(tiny_model(), torch.device("cpu"), _Storage(kc, vc, 4))
    resets = []
    monkeypatch.setattr(runner_mod._ops, "reset_scratch", lambda dev: resets.append(dev),
                        raising=False)
    ours._workspace.fill_(7)
    ours._k6_workspace = torch.full((64,), 3, dtype=torch.uint8)
    ours._err.fill_(DEV_WAIT_TIMEOUT | DEV_BLOCK_RANGE)
    assert ours.device_error() == DEV_WAIT_TIMEOUT | DEV_BLOCK_RANGE
    assert int(ours._workspace.count_nonzero()) == 0
    assert int(ours._k6_workspace.count_nonzero()) == 0
    assert resets == [torch.device("cpu")]
    assert ours.device_error() == 0  # the bits were cleared
    # a block-range error alone leaves the scratch buffers as they are
    ours._workspace.fill_(7)
    ours._err.fill_(DEV_BLOCK_RANGE)
    assert ours.device_error() == DEV_BLOCK_RANGE
    assert int(ours._workspace.count_nonzero()) == ours._workspace.numel()
