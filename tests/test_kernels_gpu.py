"""GPU parity of the four kernels against the CPU oracle (called through the C ABI).

Tolerances (the parity contract of this path): bf16/f16 attention within max-abs 2e-2 and
mean-abs 2e-3 of the fp32 oracle; fp32 attention within 1e-4; KV writes and metadata
bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import paged as ref

pytestmark = pytest.mark.gpu

BF16_MAX, BF16_MEAN = 2e-2, 2e-3
F32_MAX = 1e-4


def make_pool(seed, layers, num_blocks, bs, hkv, d, dtype):
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(layers, num_blocks * bs, hkv, d, generator=g).to(dtype)
    vc = torch.randn(layers, num_blocks * bs, hkv, d, generator=g).to(dtype)
    return kc, vc


def make_tables(seed, ctx, bs, num_blocks):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(num_blocks)
    tables, used = [], 0
    for c in ctx:
        n = (c + bs - 1) // bs
        tables.append(perm[used:used + n].tolist())
        used += n
    assert used <= num_blocks
    width = max(1, max(len(t) for t in tables))
    bt = np.full((len(ctx), width), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    return tables, torch.from_numpy(bt)


def close(got, expect, dtype):
    err = (got.float().cpu() - expect).abs()
    if dtype == torch.float32:
        assert err.max().item() < F32_MAX, err.max().item()
    else:
        assert err.max().item() < BF16_MAX, err.max().item()
        assert err.mean().item() < BF16_MEAN, err.mean().item()


# ------------------------------------------------------------------ K1 KV write
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_kv_write_bit_exact_with_hf_layout(ops, dtype):
    dev = torch.device("cuda")
    layers, nb, bs, hkv, d = 3, 40, 16, 2, 64
    kc, vc = make_pool(1, layers, nb, bs, hkv, d, dtype)
    n = 57
    g = torch.Generator().manual_seed(2)
    # HF states are (1, kv_heads, tokens, head_dim); the cache adapter hands the kernel
    # the transposed (tokens, kv_heads, head_dim) view, as hf_batched_paged_cache.py:115.
    hf_k = torch.randn(1, hkv, n, d, generator=g).to(dtype)
    hf_v = torch.randn(1, hkv, n, d, generator=g).to(dtype)
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int32)
    kd, vd = kc.to(dev), vc.to(dev)
    ops.kv_write(kd, vd, 2, slots.to(dev), hf_k.to(dev)[0].transpose(0, 1),
                 hf_v.to(dev)[0].transpose(0, 1))
    ref.scatter(kc, vc, 2, slots.tolist(), hf_k[0].transpose(0, 1), hf_v[0].transpose(0, 1))
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)


def test_kv_write_skips_padding_and_flags_out_of_range(ops):
    dev = torch.device("cuda")
    kc, vc = make_pool(3, 1, 8, 16, 2, 128, torch.bfloat16)
    keys = torch.randn(4, 2, 128).to(torch.bfloat16)
    vals = torch.randn(4, 2, 128).to(torch.bfloat16)
    slots = torch.tensor([5, -1, 9, 8 * 16 + 3], dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    kd, vd = kc.to(dev), vc.to(dev)
    ops.kv_write(kd, vd, 0, slots.to(dev), keys.to(dev), vals.to(dev), err)
    ref.scatter(kc, vc, 0, [5, 9], keys[[0, 2]], vals[[0, 2]])
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)
    assert int(err.item()) & 1  # B2P_DEV_SLOT_RANGE


def test_kv_write_rejects_bad_layer(ops):
    dev = torch.device("cuda")
    kc, vc = make_pool(3, 2, 4, 16, 2, 64, torch.float16)
    k = torch.zeros(1, 2, 64, dtype=torch.float16, device=dev)
    with pytest.raises(ValueError):
        ops.kv_write(kc.to(dev), vc.to(dev), 2, torch.zeros(1, dtype=torch.int32, device=dev),
                     k, k)


# ------------------------------------------------------------------ K2 decode
DECODE_SHAPES = [
    # (hq, hkv, d, bs)
    (12, 2, 128, 16),   # Qwen2.5-1.5B
    (14, 2, 64, 16),    # Qwen2.5-0.5B
    (28, 4, 128, 16),   # Qwen2.5-7B
    (12, 2, 128, 32),   # two sub-blocks per block
    (8, 1, 128, 16),    # group of 8
    (32, 2, 128, 16),   # group of 16 (two query-head tiles)
    (4, 4, 64, 16),     # no GQA
]


@pytest.mark.parametrize("shape", DECODE_SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_matches_oracle(ops, shape, dtype):
    hq, hkv, d, bs = shape
    dev = torch.device("cuda")
    ctx = [1, 15, 16, 17, 33, 100, 511, 1024, 2049, 3000]
    nb = sum((c + bs - 1) // bs for c in ctx) + 7
    kc, vc = make_pool(10, 2, nb, bs, hkv, d, dtype)
    tables, bt = make_tables(11, ctx, bs, nb)
    q = torch.randn(len(ctx), hq, d, generator=torch.Generator().manual_seed(12)).to(dtype)
    out = ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), 1, bt.to(dev),
                           torch.tensor(ctx, dtype=torch.int32, device=dev), bs, d ** -0.5)
    expect = ref.decode_attention(q, kc, vc, 1, tables, ctx, bs, d ** -0.5)
    close(out, expect, dtype)


@pytest.mark.parametrize("bs,d", [(16, 128), (8, 64), (1, 32), (16, 96)])
def test_decode_fp32_and_generic_shapes(ops, bs, d):
    dev = torch.device("cuda")
    hq, hkv = 14, 2
    ctx = [1, 7, 64, 130]
    nb = sum((c + bs - 1) // bs for c in ctx) + 3
    for dtype in (torch.float32, torch.bfloat16):
        kc, vc = make_pool(20, 1, nb, bs, hkv, d, dtype)
        tables, bt = make_tables(21, ctx, bs, nb)
        q = torch.randn(len(ctx), hq, d, generator=torch.Generator().manual_seed(22)).to(dtype)
        out = ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                               torch.tensor(ctx, dtype=torch.int32, device=dev), bs, d ** -0.5)
        close(out, ref.decode_attention(q, kc, vc, 0, tables, ctx, bs, d ** -0.5), dtype)


def test_decode_many_short_sequences_cross_cta_merge(ops):
    """Hundreds of sequences of mixed lengths: ranges cut sequences in many places."""
    dev = torch.device("cuda")
    hq, hkv, d, bs = 12, 2, 128, 16
    rng = np.random.default_rng(5)
    ctx = rng.integers(1, 6000, size=300).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 1
    kc, vc = make_pool(30, 1, nb, bs, hkv, d, torch.bfloat16)
    tables, bt = make_tables(31, ctx, bs, nb)
    q = torch.randn(len(ctx), hq, d, generator=torch.Generator().manual_seed(32)).to(torch.bfloat16)
    ws = ops.make_decode_workspace(len(ctx), hq, hkv, d, dev)
    args = (q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
            torch.tensor(ctx, dtype=torch.int32, device=dev), bs, d ** -0.5)
    out1 = ops.paged_decode(*args, workspace=ws).clone()
    out2 = ops.paged_decode(*args, workspace=ws)  # the counters came back to zero
    assert torch.equal(out1, out2)  # deterministic
    close(out1, ref.decode_attention(q, kc, vc, 0, tables, ctx, bs, d ** -0.5), torch.bfloat16)


def test_decode_reused_workspace_with_growing_sequence_counts(ops):
    """One workspace serves launches whose sequence count grows from step to step (as the
    engine's decode batches do): every output row is written on every launch. The counters
    must never land on bytes where an earlier, smaller launch left partial records."""
    dev = torch.device("cuda")
    hq, hkv, d, bs = 12, 2, 128, 16
    rng = np.random.default_rng(17)
    ctx = rng.integers(1, 5000, size=400).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 1
    kc, vc = make_pool(18, 1, nb, bs, hkv, d, torch.bfloat16)
    tables, bt = make_tables(19, ctx, bs, nb)
    q = torch.randn(len(ctx), hq, d, generator=torch.Generator().manual_seed(20))
    q = q.to(torch.bfloat16)
    expect = ref.decode_attention(q, kc, vc, 0, tables, ctx, bs, d ** -0.5)
    qd, kd, vd, btd = q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev)
    lens = torch.tensor(ctx, dtype=torch.int32, device=dev)
    ws = ops.make_decode_workspace(len(ctx), hq, hkv, d, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for n in (4, 8, 60, 98, 150, 400, 30, 400):
        out = torch.full((n, hq, d), float("nan"), dtype=torch.bfloat16, device=dev)
        ops.paged_decode(qd[:n], kd, vd, 0, btd[:n], lens[:n], bs, d ** -0.5, out=out,
                         workspace=ws, err_flag=err)
        assert not bool(out.isnan().any()), n
        close(out, expect[:n], torch.bfloat16)
    assert int(err.item()) == 0


def _decode_case(ops, ctx, seed, hq=12, hkv=2, d=128, bs=16, workspace=None, err=None):
    dev = torch.device("cuda")
    nb = sum((c + bs - 1) // bs for c in ctx) + 1
    kc, vc = make_pool(seed, 1, nb, bs, hkv, d, torch.bfloat16)
    tables, bt = make_tables(seed + 1, ctx, bs, nb)
    q = torch.randn(len(ctx), hq, d, generator=torch.Generator().manual_seed(seed + 2))
    q = q.to(torch.bfloat16)
    out = ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                           torch.tensor(ctx, dtype=torch.int32, device=dev), bs, d ** -0.5,
                           workspace=workspace, err_flag=err)
    return out, ref.decode_attention(q, kc, vc, 0, tables, ctx, bs, d ** -0.5)


def test_decode_many_sequences(ops):
    """1,500 sequences: more sequences than stream units, most ranges hold several."""
    ctx = np.random.default_rng(61).integers(1, 2500, size=1500).tolist()
    out, expect = _decode_case(ops, ctx, 60)
    close(out, expect, torch.bfloat16)


def test_decode_one_long_sequence_and_a_long_tail(ops):
    """A 200k-token history split over every stream unit, and a mix of long and tiny ones."""
    for ctx in ([200_000], [150_000, 10, 5_000, 60_000, 1, 33_000]):
        out, expect = _decode_case(ops, ctx, 70)
        close(out, expect, torch.bfloat16)


def test_decode_empty_history_writes_zeros_and_flags(ops):
    dev = torch.device("cuda")
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ctx = [0, 50, 0, 3000, 17]
    out, expect = _decode_case(ops, ctx, 80, err=err)
    assert int(err.item()) & 8  # B2P_DEV_LENGTH
    assert torch.equal(out[0].float().cpu(), torch.zeros_like(out[0].float().cpu()))
    assert torch.equal(out[2].float().cpu(), torch.zeros_like(out[2].float().cpu()))
    keep = [1, 3, 4]
    close(out[keep], expect[keep], torch.bfloat16)


def test_decode_workspace_sizes(ops):
    """Any workspace the call accepts gives the same results; one too small for the
    device's stream units is refused with a workspace error before anything runs."""
    dev = torch.device("cuda")
    ctx = np.random.default_rng(91).integers(1, 4000, size=400).tolist()
    full = ops.decode_workspace_size(len(ctx), 12, 2, 128)
    accepted = 0
    for size in (2 * full, full, full - 64, full // 2, full // 16):
        ws = torch.zeros(max(size, 16), dtype=torch.uint8, device=dev)
        try:
            out, expect = _decode_case(ops, ctx, 90, workspace=ws)
        except ValueError as exc:
            assert "workspace" in str(exc).lower()
            assert size < full
            continue
        accepted += 1
        close(out, expect, torch.bfloat16)
    assert accepted >= 2


def test_decode_garbage_past_context_is_masked(ops):
    """Slots past a sequence's length may hold NaN/Inf (the pool is not cleared)."""
    dev = torch.device("cuda")
    hq, hkv, d, bs = 12, 2, 128, 16
    ctx = [5, 21]
    kc, vc = make_pool(40, 1, 4, bs, hkv, d, torch.bfloat16)
    tables = [[2], [0, 3]]
    bt = torch.tensor([[2, -1], [0, 3]], dtype=torch.int32)
    kc[0, 2 * bs + 5:3 * bs] = float("nan")
    vc[0, 2 * bs + 5:3 * bs] = float("inf")
    vc[0, 3 * bs + 5:4 * bs] = float("nan")
    q = torch.randn(2, hq, d, generator=torch.Generator().manual_seed(41)).to(torch.bfloat16)
    out = ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                           torch.tensor(ctx, dtype=torch.int32, device=dev), bs, d ** -0.5)
    assert torch.isfinite(out.float()).all()
    close(out, ref.decode_attention(q, kc, vc, 0, tables, ctx, bs, d ** -0.5), torch.bfloat16)


def test_decode_out_of_range_block_is_flagged(ops):
    dev = torch.device("cuda")
    hq, hkv, d, bs = 12, 2, 128, 16
    kc, vc = make_pool(50, 1, 4, bs, hkv, d, torch.bfloat16)
    bt = torch.tensor([[1, 99]], dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    q = torch.randn(1, hq, d).to(torch.bfloat16)
    ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                     torch.tensor([20], dtype=torch.int32, device=dev), bs, d ** -0.5,
                     err_flag=err)
    assert int(err.item()) & 2  # B2P_DEV_BLOCK_RANGE


def test_decode_full_benchmark_workload(ops):
    """The benchmark's 256-sequence, 65,536-block workload at full size."""
    import bench

    dev = torch.device("cuda")
    w = bench.make_workload(1234, None)
    kd, vd = w["kc"].to(dev), w["vc"].to(dev)
    ops.kv_write(kd, vd, 0, torch.from_numpy(w["slots"]).to(dev), w["new_k"].to(dev),
                 w["new_v"].to(dev))
    out = ops.paged_decode(w["q"].to(dev), kd, vd, 0, torch.from_numpy(w["tables"]).to(dev),
                           torch.from_numpy(w["ctx"]).to(dev), bench.BLOCK_SIZE,
                           bench.HEAD_DIM ** -0.5)
    kc, vc = w["kc"], w["vc"]
    ref.scatter(kc, vc, 0, w["slots"].tolist(), w["new_k"], w["new_v"])
    tables = [row[row >= 0].tolist() for row in w["tables"]]
    expect = ref.decode_attention(w["q"], kc, vc, 0, tables, w["ctx"].tolist(), bench.BLOCK_SIZE,
                                  bench.HEAD_DIM ** -0.5)
    close(out, expect, torch.bfloat16)


@pytest.mark.parametrize("shape,dtype", [((12, 2, 128, 16), torch.bfloat16),
                                         ((28, 4, 128, 16), torch.bfloat16),
                                         ((12, 2, 128, 32), torch.float16),
                                         ((14, 2, 64, 16), torch.bfloat16),
                                         ((14, 2, 64, 16), torch.float32)])
def test_decode_append_equals_write_then_decode(ops, shape, dtype):
    """The fused call stores the same pool rows as K1 with the block-table slot mapping and
    returns exactly what K2 returns after that write (the CUDA-core fallback for fp32)."""
    hq, hkv, d, bs = shape
    dev = torch.device("cuda")
    rng = np.random.default_rng(41)
    ctx = [1, 16, 17, 32, 100, 511, 512, 1024, 2049] + rng.integers(1, 3000, size=120).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 5
    kc, vc = make_pool(42, 2, nb, bs, hkv, d, dtype)
    tables, bt = make_tables(43, ctx, bs, nb)
    g = torch.Generator().manual_seed(44)
    q = torch.randn(len(ctx), hq, d, generator=g).to(dtype).to(dev)
    new_k = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(dev)
    new_v = torch.randn(len(ctx), hkv, d, generator=g).to(dtype).to(dev)
    slots = torch.tensor([t[(c - 1) // bs] * bs + (c - 1) % bs for t, c in zip(tables, ctx)],
                         dtype=torch.int32, device=dev)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
    ka, va = kc.to(dev), vc.to(dev)
    kb, vb = ka.clone(), va.clone()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.kv_write(ka, va, 1, slots, new_k, new_v, err)
    out_a = ops.paged_decode(q, ka, va, 1, bt.to(dev), ctx_d, bs, d ** -0.5, err_flag=err)
    out_b = ops.paged_decode_append(q, new_k, new_v, kb, vb, 1, bt.to(dev), ctx_d, bs, d ** -0.5,
                                    err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(ka, kb) and torch.equal(va, vb)
    assert torch.equal(out_a, out_b)
    ref.scatter(kc, vc, 1, slots.tolist(), new_k.cpu(), new_v.cpu())
    close(out_b, ref.decode_attention(q.cpu(), kc, vc, 1, tables, ctx, bs, d ** -0.5), dtype)


def churned_tables(rng, ctx, bs, num_blocks, churn=0.3):
    """Block tables after allocation churn: blocks are handed out from a FIFO free list,
    30% of them are freed in random order and handed out again, so every table mixes
    runs of old and recycled blocks (as after preemption and completion in the engine)."""
    need = [(c + bs - 1) // bs for c in ctx]
    free = list(range(num_blocks))
    tables = [[] for _ in ctx]
    # interleaved first allocation (sequences grow together under continuous batching)
    pending = list(range(len(ctx)))
    while pending:
        for i in list(pending):
            tables[i].append(free.pop(0))
            if len(tables[i]) == need[i]:
                pending.remove(i)
    # free 30% of all allocated blocks in random order, then reallocate them at the
    # positions they were taken from (FIFO order of the free list)
    taken = [(i, j) for i, t in enumerate(tables) for j in range(len(t))]
    victims = [taken[k] for k in rng.permutation(len(taken))[: int(churn * len(taken))]]
    for i, j in victims:
        free.append(tables[i][j])
        tables[i][j] = None
    for i, j in victims:
        tables[i][j] = free.pop(0)
    width = max(len(t) for t in tables)
    bt = np.full((len(ctx), width), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    return tables, torch.from_numpy(bt)


def test_decode_long_context_churned_tables_7b_shape(ops):
    """Qwen2.5-7B attention shape (28 Q / 4 KV heads, group 7), 16 sequences with contexts
    U[8192, 32768], block tables fragmented by allocation churn."""
    dev = torch.device("cuda")
    hq, hkv, d, bs = 28, 4, 128, 16
    rng = np.random.default_rng(97)
    ctx = rng.integers(8192, 32769, size=16).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 64
    tables, bt = churned_tables(rng, ctx, bs, nb)
    kc, vc = make_pool(98, 1, nb, bs, hkv, d, torch.bfloat16)
    q = torch.randn(len(ctx), hq, d, generator=torch.Generator().manual_seed(99)).to(torch.bfloat16)
    out = ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                           torch.tensor(ctx, dtype=torch.int32, device=dev), bs, d ** -0.5)
    close(out, ref.decode_attention(q, kc, vc, 0, tables, ctx, bs, d ** -0.5), torch.bfloat16)


# ------------------------------------------------------------------ K3 prefill
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(12, 2, 128, 16), (14, 2, 64, 16), (28, 4, 128, 32),
                                   (6, 2, 128, 16),   # odd GQA group: a lone head per group
                                   (4, 4, 128, 16)])  # no GQA: every query head alone
def test_prefill_matches_oracle(ops, dtype, shape):
    hq, hkv, d, bs = shape
    dev = torch.device("cuda")
    # whole-history prefills plus two chunked-prefill runs (q_len < ctx)
    ctx = [1, 17, 64, 130, 300, 77]
    qlen = [1, 17, 64, 130, 45, 1]
    cu = np.concatenate([[0], np.cumsum(qlen)]).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 2
    kc, vc = make_pool(60, 1, nb, bs, hkv, d, dtype)
    tables, bt = make_tables(61, ctx, bs, nb)
    q = torch.randn(cu[-1], hq, d, generator=torch.Generator().manual_seed(62)).to(dtype)
    out = ops.paged_prefill(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                            torch.tensor(cu, dtype=torch.int32, device=dev),
                            torch.tensor(ctx, dtype=torch.int32, device=dev), max(qlen), bs,
                            d ** -0.5)
    close(out, ref.prefill_attention(q, kc, vc, 0, tables, cu, ctx, bs, d ** -0.5), dtype)


# ------------------------------------------------------------------ K4 metadata
def test_metadata_bit_exact(ops):
    dev = torch.device("cuda")
    rng = np.random.default_rng(70)
    bs = 16
    n = 37
    lengths = rng.integers(1, 300, size=n)
    phases = [ref.PREFILL if rng.random() < 0.3 else ref.DECODE for _ in range(n)]
    # decode executions come first, as in Engine.step (engine.py:156-171)
    order = sorted(range(n), key=lambda i: phases[i] != ref.DECODE)
    phases = [phases[i] for i in order]
    lengths = [int(lengths[i]) for i in order]
    mirror_rows = n + 5
    width = 32
    perm = rng.permutation(4096)
    mirror = np.full((mirror_rows, width), -1, dtype=np.int32)
    rows = rng.permutation(mirror_rows)[:n]
    used = 0
    tables = []
    for i, L in enumerate(lengths):
        nb = (L + bs - 1) // bs
        mirror[rows[i], :nb] = perm[used:used + nb]
        tables.append(perm[used:used + nb].tolist())
        used += nb
    qlens = [ref.query_length(p, L) for p, L in zip(phases, lengths)]
    total_q = sum(qlens)
    md = ops.build_metadata(torch.tensor(qlens, dtype=torch.int32, device=dev),
                            torch.tensor(lengths, dtype=torch.int32, device=dev),
                            torch.tensor(rows, dtype=torch.int32, device=dev),
                            torch.from_numpy(mirror).to(dev), bs, total_q, width)
    lay = ref.batch_layout(phases, lengths)
    assert md["cu_seqlens_q"].cpu().tolist() == [*lay["query_offsets"], lay["total_query_tokens"]]
    assert md["cu_seqlens_k"].cpu().tolist() == [*lay["key_offsets"], lay["total_key_tokens"]]
    assert md["logit_indices"].cpu().tolist() == list(lay["logit_indices"])
    assert md["positions"].cpu().numpy().tolist() == ref.packed_positions(phases, lengths).tolist()
    hist = [ref.history_slots(t, L, bs) for t, L in zip(tables, lengths)]
    assert md["slot_mapping"].cpu().numpy().tolist() == ref.write_slots(phases, hist).tolist()
    bt = md["block_tables"].cpu().numpy()
    for i, t in enumerate(tables):
        assert bt[i, :len(t)].tolist() == t and (bt[i, len(t):] == -1).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(12, 2, 128), (14, 2, 64)])
def test_prefill_tensor_core_long_prompts_and_chunks(ops, dtype, shape):
    """Prompts up to 2,100 tokens (several 128-row tiles, many 128-key tiles), fragmented
    blocks, whole-history and chunked runs, NaN in the pool slots past every context; the
    Qwen2.5-1.5B/7B head size (128) and the Qwen2.5-0.5B one (64)."""
    hq, hkv, d = shape
    bs = 16
    dev = torch.device("cuda")
    rng = np.random.default_rng(80)
    ctx = [2100, 64, 129, 1000, 777, 300, 16]
    qlen = [2100, 64, 129, 1000, 200, 1, 16]
    cu = np.concatenate([[0], np.cumsum(qlen)]).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 5
    kc, vc = make_pool(81, 1, nb, bs, hkv, d, dtype)
    tables, bt = make_tables(82, ctx, bs, nb)
    for t, c in zip(tables, ctx):
        tail = c % bs
        if tail:
            kc[0, t[-1] * bs + tail:(t[-1] + 1) * bs] = float("nan")
            vc[0, t[-1] * bs + tail:(t[-1] + 1) * bs] = float("nan")
    q = torch.randn(cu[-1], hq, d, generator=torch.Generator().manual_seed(83)).to(dtype)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.paged_prefill(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                            torch.tensor(cu, dtype=torch.int32, device=dev),
                            torch.tensor(ctx, dtype=torch.int32, device=dev), max(qlen), bs,
                            d ** -0.5, err_flag=err)
    assert int(err.item()) == 0
    assert torch.isfinite(out.float()).all()
    close(out, ref.prefill_attention(q, kc, vc, 0, tables, cu, ctx, bs, d ** -0.5), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(12, 2, 128), (14, 2, 64)])
def test_prefill_running_max_jumps(ops, dtype, shape):
    """Scores that grow along the keys, so rows keep finding a larger max in later KV tiles
    (the kernel moves its reference max and rescales O, l and stored P). In the first
    prompt the larger half of every 128-key tile is keys 64..127, in the second keys
    0..63; the third grows smoothly; the fourth is a chunked prefill.

    Such peaked rows put most of the weight on a few V rows, so the bf16 rounding of P and
    V shows up in the max error: 2.4e-2 against the fp32 oracle for this input, the same
    for a kernel that takes each tile's exact max before the exponentials. The bf16 max
    bound here is 3e-2 (mean and f16 bounds as elsewhere). Head sizes 128 and 64 (where P
    has tensor-memory columns of its own, so the rescale of stored P takes another path)."""
    hq, hkv, d = shape
    bs = 16
    dev = torch.device("cuda")
    ctx = [900, 777, 1300, 1000]
    qlen = [900, 777, 1300, 300]
    cu = np.concatenate([[0], np.cumsum(qlen)]).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 3
    kc, vc = make_pool(91, 1, nb, bs, hkv, d, torch.float32)
    tables, bt = make_tables(92, ctx, bs, nb)
    for i, (t, c) in enumerate(zip(tables, ctx)):
        pos = np.arange(c)
        tile, half = pos // 128, (pos % 128) // 64
        if i == 0:
            mult = 1.0 + 2.5 * tile + 1.5 * half
        elif i == 1:
            mult = 1.0 + 2.5 * tile + 1.5 * (1 - half)
        else:
            mult = 1.0 + pos / 40.0
        slots = np.array(t)[pos // bs] * bs + pos % bs
        kc[0, torch.from_numpy(slots)] *= torch.from_numpy(mult).float()[:, None, None]
    kc, vc = kc.to(dtype), vc.to(dtype)
    q = torch.randn(cu[-1], hq, d, generator=torch.Generator().manual_seed(93)).to(dtype)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.paged_prefill(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                            torch.tensor(cu, dtype=torch.int32, device=dev),
                            torch.tensor(ctx, dtype=torch.int32, device=dev), max(qlen), bs,
                            d ** -0.5, err_flag=err)
    assert int(err.item()) == 0
    assert torch.isfinite(out.float()).all()
    expect = ref.prefill_attention(q, kc, vc, 0, tables, cu, ctx, bs, d ** -0.5)
    diff = (out.float().cpu() - expect).abs()
    assert diff.max().item() < (3e-2 if dtype == torch.bfloat16 else BF16_MAX), diff.max().item()
    assert diff.mean().item() < BF16_MEAN, diff.mean().item()


def test_prefill_scheduler_limits_many_prompts_and_long_history(ops):
    """Past the scheduler's shared-memory tables (more than 1,024 sequences; a query tile
    needing more than 1,024 KV tiles, i.e. a history past 131,072 tokens) the work items
    are ordered from cu_seqlens and the context lengths read in global memory. Both cases
    must still cover every query tile once: 1,100 short prompts, and a 300-token chunk
    appended to a 140,000-token history next to two ordinary prompts."""
    hq, hkv, d, bs = 12, 2, 128, 16
    dev = torch.device("cuda")
    rng = np.random.default_rng(95)
    cases = [
        [int(x) for x in rng.integers(1, 40, size=1100)],
        None,
    ]
    for case in cases:
        if case is not None:
            ctx = case
            qlen = list(case)
        else:
            ctx = [140_000, 200, 77]
            qlen = [300, 200, 77]
        cu = np.concatenate([[0], np.cumsum(qlen)]).tolist()
        nb = sum((c + bs - 1) // bs for c in ctx) + 2
        kc, vc = make_pool(96, 1, nb, bs, hkv, d, torch.bfloat16)
        tables, bt = make_tables(97, ctx, bs, nb)
        q = torch.randn(cu[-1], hq, d, generator=torch.Generator().manual_seed(98)).to(torch.bfloat16)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        out = torch.full((cu[-1], hq, d), float("nan"), dtype=torch.bfloat16, device=dev)
        ops.paged_prefill(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                          torch.tensor(cu, dtype=torch.int32, device=dev),
                          torch.tensor(ctx, dtype=torch.int32, device=dev), max(qlen), bs,
                          d ** -0.5, out=out, err_flag=err)
        assert int(err.item()) == 0
        assert torch.isfinite(out.float()).all()  # every row written
        close(out, ref.prefill_attention(q, kc, vc, 0, tables, cu, ctx, bs, d ** -0.5),
              torch.bfloat16)


def test_prefill_trailing_slice_of_packed_batch(ops):
    """The runner's call: decode rows first, prefill rows run with views of the metadata."""
    hq, hkv, d, bs = 12, 2, 128, 16
    dev = torch.device("cuda")
    ctx = [50, 33, 300, 140]
    qlen = [1, 1, 300, 12]
    cu = np.concatenate([[0], np.cumsum(qlen)]).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 2
    kc, vc = make_pool(90, 1, nb, bs, hkv, d, torch.bfloat16)
    tables, bt = make_tables(91, ctx, bs, nb)
    q = torch.randn(cu[-1], hq, d, generator=torch.Generator().manual_seed(92)).to(torch.bfloat16)
    cu_d = torch.tensor(cu, dtype=torch.int32, device=dev)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
    bt_d = bt.to(dev)
    out = torch.zeros(cu[-1], hq, d, dtype=torch.bfloat16, device=dev)
    ops.paged_prefill(q.to(dev), kc.to(dev), vc.to(dev), 0, bt_d[2:], cu_d[2:], ctx_d[2:], 300, bs,
                      d ** -0.5, out=out)
    expect = ref.prefill_attention(q, kc, vc, 0, tables[2:], cu[2:], ctx[2:], bs, d ** -0.5)
    close(out[2:], expect, torch.bfloat16)
    assert torch.count_nonzero(out[:2].float()) == 0  # decode rows untouched


# ------------------------------------------------------------------ parity at benchmark sizes
def test_decode_large_values_in_split_sequences(ops):
    """V rows around 4e5 (N(0,1) x 1e5 + 4e5: representable in bf16, far past fp16's
    65,504) in sequences cut across many stream units, so that every partial record the
    merge reads holds values beyond fp16's range. Outputs must be finite and within a
    bf16-sized relative error of the fp32 oracle: at most 1e-2 for any element and 3e-3
    on average (one bf16 rounding of the output is up to 2.6e-3 relative here)."""
    dev = torch.device("cuda")
    hq, hkv, d, bs = 12, 2, 128, 16
    rng = np.random.default_rng(130)
    ctx = [120_000, 9_000] + rng.integers(2_000, 6_000, size=40).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 3
    kc, vc = make_pool(131, 1, nb, bs, hkv, d, torch.float32)
    vc = (vc * 1.0e5 + 4.0e5).to(torch.bfloat16)
    kc = kc.to(torch.bfloat16)
    tables, bt = make_tables(132, ctx, bs, nb)
    q = torch.randn(len(ctx), hq, d, generator=torch.Generator().manual_seed(133)).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), 0, bt.to(dev),
                           torch.tensor(ctx, dtype=torch.int32, device=dev), bs, d ** -0.5,
                           err_flag=err)
    assert int(err.item()) == 0
    assert torch.isfinite(out.float()).all()
    expect = ref.decode_attention(q, kc, vc, 0, tables, ctx, bs, d ** -0.5)
    assert expect.abs().min().item() > 65504.0  # beyond what fp16 records could hold
    rel = (out.float().cpu() - expect).abs() / expect.abs()
    assert rel.max().item() < 1e-2, rel.max().item()
    assert rel.mean().item() < 3e-3, rel.mean().item()


def test_decode_7b_long_context_churn_full_size(ops):
    """The long-context configuration at its full per-GPU size: Qwen2.5-7B attention shape
    (28 Q / 4 KV heads, head_dim 128), 64 sequences with contexts U[8192, 32768], block
    size 16, tables fragmented by 30% alloc/free churn; the fused write + decode call the
    benchmark runs, against the oracle's scatter + decode."""
    import bench

    dev = torch.device("cuda")
    w = bench.make_longctx_workload(2024, dev, layers=1)
    hq, hkv, d, bs = bench.LC_HQ, bench.LC_HKV, bench.HEAD_DIM, bench.BLOCK_SIZE
    kd, vd = w["kc"], w["vc"]
    tables = w["table_lists"]
    ctx = w["ctx"].tolist()
    kc, vc = kd.cpu(), vd.cpu()  # the pool before the fused call stores the new rows
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = ops.paged_decode_append(w["q"][0], w["new_k"][0], w["new_v"][0], kd, vd, 0,
                                  torch.from_numpy(w["tables"]).to(dev),
                                  torch.from_numpy(w["ctx"]).to(dev), bs, d ** -0.5,
                                  err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    slots = [t[(c - 1) // bs] * bs + (c - 1) % bs for t, c in zip(tables, ctx)]
    ref.scatter(kc, vc, 0, slots, w["new_k"][0].cpu(), w["new_v"][0].cpu())
    rows = torch.tensor(slots, dtype=torch.long)
    assert torch.equal(kd[0, rows.to(dev)].cpu(), kc[0, rows])
    assert torch.equal(vd[0, rows.to(dev)].cpu(), vc[0, rows])
    expect = ref.decode_attention(w["q"][0].cpu(), kc, vc, 0, tables, ctx, bs, d ** -0.5)
    close(out, expect, torch.bfloat16)
    assert (hq, hkv) == (28, 4) and len(ctx) == 64 and min(ctx) >= 8192 and max(ctx) <= 32768


def test_prefill_full_benchmark_workload_and_chunks(ops):
    """The prefill benchmark's workload at full size (32 prompts log-uniform in [64, 8192],
    49,659 packed tokens, fragmented pool, bf16, 12/2 heads, head_dim 128): K1 writes every
    prompt token, K3 runs the packed causal attention, and the result is compared with the
    oracle's scatter + per-prompt causal attention. Then the prompts longer than 2,048
    tokens are run again as chunked-prefill slices (a middle slice and the last 512 rows of
    each, packed into one launch, attending to the history already in the pool), whose rows
    must match the same rows of the whole-prompt oracle."""
    import bench

    dev = torch.device("cuda")
    w = bench.make_prefill_workload(4321, dev)
    bs, d = bench.BLOCK_SIZE, bench.HEAD_DIM
    lens = w["lens"].astype(np.int64)
    cu = w["cu"].tolist()
    ctx = lens.astype(np.int32)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    slots = torch.from_numpy(w["slots"]).to(dev)
    ops.kv_write(w["kc"], w["vc"], 0, slots, w["k"], w["v"], err)
    bt = torch.from_numpy(w["tables"]).to(dev)
    out = ops.paged_prefill(w["q"], w["kc"], w["vc"], 0, bt,
                            torch.from_numpy(w["cu"]).to(dev), torch.from_numpy(ctx).to(dev),
                            int(lens.max()), bs, d ** -0.5, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(lens.sum()) == 49_659 and int(lens.max()) == 6_818

    tables = [row[row >= 0].tolist() for row in w["tables"]]
    kc = torch.zeros(w["kc"].shape, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q_cpu = w["q"].cpu()
    ref.scatter(kc, vc, 0, w["slots"].tolist(), w["k"].cpu(), w["v"].cpu())
    assert torch.equal(w["kc"].cpu(), kc) and torch.equal(w["vc"].cpu(), vc)
    expect = ref.prefill_attention(q_cpu, kc, vc, 0, tables, cu, lens.tolist(), bs, d ** -0.5)
    close(out, expect, torch.bfloat16)

    # chunked-prefill slices of the long prompts, packed into one launch
    rows, c_tables, c_ctx, c_cu = [], [], [], [0]
    for i, n in enumerate(lens.tolist()):
        if n <= 2048:
            continue
        for a, b in ((n // 2 - 300, n // 2 + 100), (n - 512, n)):
            rows.append(np.arange(cu[i] + a, cu[i] + b))
            c_tables.append(w["tables"][i])
            c_ctx.append(b)
            c_cu.append(c_cu[-1] + (b - a))
    rows = np.concatenate(rows)
    assert len(c_ctx) >= 8
    q_chunks = w["q"][torch.from_numpy(rows).to(dev)]
    out_c = ops.paged_prefill(q_chunks, w["kc"], w["vc"], 0,
                              torch.from_numpy(np.stack(c_tables)).to(dev),
                              torch.tensor(c_cu, dtype=torch.int32, device=dev),
                              torch.tensor(c_ctx, dtype=torch.int32, device=dev), 512, bs,
                              d ** -0.5, err_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    close(out_c, expect[torch.from_numpy(rows)], torch.bfloat16)
