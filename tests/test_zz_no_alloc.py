"""The scratch-free decode entry point against the ordinary one.

b2p_paged_decode_noalloc exists for callers that cannot give the library device scratch
(a runtime whose device memory is entirely held by its own arena, a binding from a
language with no device allocator). It keeps the split-K scratch in an array compiled
into the library instead. These tests call it through the C ABI and check that two calls
in a row give the results of b2p_paged_decode with a caller-allocated workspace, within
the bf16 tolerance used by the other decode tests, and those of the fp32 oracle, and that
a problem too large for the array is refused before anything is queued. The file is named
to be collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from llm_engineering_b200 import _lib
from oracle import paged as ref


def _call_noalloc(q, kc, vc, bt, ctx, out, bs, scale, err):
    lib = _lib.load()
    layers, slots, hkv, d = kc.shape
    n, hq, _ = q.shape
    return lib.b2p_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), 0, layers, slots,
        bt.data_ptr(), bt.stride(0), ctx.data_ptr(), n, hq, hkv, d, bs, float(scale),
        out.data_ptr(), out.stride(0), out.stride(1), _lib.B2P_BF16, err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.gpu
def test_noalloc_decode_matches_workspace_decode_twice(ops):
    dev = torch.device("cuda")
    hq, hkv, d, bs = 12, 2, 128, 16
    rng = np.random.default_rng(123)
    # mixed lengths so that many sequences are split across stream units (partials + merge)
    ctx = rng.integers(1, 5000, size=200).tolist()
    nb = sum((c + bs - 1) // bs for c in ctx) + 3
    g = torch.Generator().manual_seed(124)
    kc = torch.randn(1, nb * bs, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    vc = torch.randn(1, nb * bs, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    perm = rng.permutation(nb)
    width = max((c + bs - 1) // bs for c in ctx)
    bt = np.full((len(ctx), width), -1, dtype=np.int32)
    used = 0
    for i, c in enumerate(ctx):
        k = (c + bs - 1) // bs
        bt[i, :k] = perm[used:used + k]
        used += k
    bt = torch.from_numpy(bt).to(dev)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
    q = torch.randn(len(ctx), hq, d, generator=g).to(torch.bfloat16).to(dev)
    scale = d ** -0.5

    expect = ops.paged_decode(q, kc, vc, 0, bt, ctx_d, bs, scale)
    tables = [row[row >= 0].tolist() for row in bt.cpu().numpy()]
    oracle = ref.decode_attention(q.cpu(), kc.cpu(), vc.cpu(), 0, tables, ctx, bs, scale)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        out = torch.full_like(q, float("nan"))
        rc = _call_noalloc(q, kc, vc, bt, ctx_d, out, bs, scale, err)
        assert rc == _lib.B2P_OK, _lib.status_text(rc)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        for want in (expect.float(), oracle.to(dev)):
            diff = (out.float() - want).abs()
            assert diff.max().item() < 2e-2 and diff.mean().item() < 2e-3


@pytest.mark.gpu
def test_noalloc_decode_refuses_when_only_the_counters_fit(ops):
    """Counters that fit the array but split-K records that do not: the call is refused
    with a workspace error and leaves the output untouched (nothing was queued)."""
    dev = torch.device("cuda")
    hq, hkv, d, bs = 12, 2, 128, 16
    # 15.2 MB of counters fit the 16 MiB array; with the split-K records of 148 SMs
    # (~4.4 MB for this shape) the call needs more
    n = 1_900_000
    need = ops.decode_workspace_size(n, hq, hkv, d)
    assert need > (16 << 20) and hkv * n * 4 < (16 << 20)
    kc = torch.zeros(1, 4 * bs, hkv, d, dtype=torch.bfloat16, device=dev)
    bt = torch.zeros(n, 1, dtype=torch.int32, device=dev)
    ctx_d = torch.ones(n, dtype=torch.int32, device=dev)
    q = torch.zeros(n, hq, d, dtype=torch.bfloat16, device=dev)
    out = torch.full_like(q, 7.0)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = _call_noalloc(q, kc, kc, bt, ctx_d, out, bs, d ** -0.5, err)
    torch.cuda.synchronize()
    assert rc == _lib.B2P_EWORKSPACE
    assert bool((out == 7.0).all()) and int(err.item()) == 0


def test_noalloc_decode_refuses_oversized_problem_without_a_gpu_call():
    """More sequences than the built-in array has counter room for: refused up front."""
    lib = _lib.load()
    too_many = (16 << 20) // (4 * 2) + 1024  # counters for 2 KV heads exceed 16 MiB
    rc = lib.b2p_paged_decode_noalloc(
        ctypes.c_void_p(16), 0, 0, ctypes.c_void_p(16), ctypes.c_void_p(16), 0, 1, 16,
        ctypes.c_void_p(16), 1, ctypes.c_void_p(16), too_many, 12, 2, 128, 16, 1.0,
        ctypes.c_void_p(16), 0, 0, _lib.B2P_BF16, None, None)
    assert rc == _lib.B2P_EWORKSPACE
