"""Torch-facing wrappers of the C-ABI kernels.

Each function takes CUDA tensors, checks shapes/dtypes on the host, passes raw device
pointers, element strides and ``torch.cuda.current_stream()`` to the library, and
returns without synchronising. Nothing here computes attention itself: a tensor on the
wrong device or a missing library raises instead of falling back.
"""

from __future__ import annotations

import torch

from . import _lib

_DTYPE_CODES = {
    torch.bfloat16: _lib.B2P_BF16,
    torch.float16: _lib.B2P_F16,
    torch.float32: _lib.B2P_F32,
}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported KV dtype {dtype}") from exc


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); the paged kernels have "
                         "no CPU path.")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _tok_head_strides(name: str, t: torch.Tensor) -> tuple[int, int]:
    if t.dim() != 3:
        raise ValueError(f"{name} must have shape (tokens, heads, head_dim)")
    if t.stride(2) != 1:
        raise ValueError(f"{name} must have a contiguous head_dim")
    return t.stride(0), t.stride(1)


def _check_pool(key_cache: torch.Tensor, value_cache: torch.Tensor) -> None:
    _require_cuda("key_cache", key_cache)
    _require_cuda("value_cache", value_cache)
    if key_cache.shape != value_cache.shape or key_cache.dim() != 4:
        raise ValueError("key_cache/value_cache must both be [layers, slots, kv_heads, head_dim]")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("key_cache/value_cache must be contiguous")
    if key_cache.dtype != value_cache.dtype:
        raise ValueError("key_cache/value_cache dtypes differ")


def _int32(name: str, t: torch.Tensor) -> None:
    _require_cuda(name, t)
    if t.dtype != torch.int32 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous int32 CUDA tensor")


def kv_write(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer_index: int,
    slot_mapping: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    err_flag: torch.Tensor | None = None,
) -> None:
    """K1: write row t of keys/values into slot slot_mapping[t] of layer ``layer_index``.

    keys/values: (tokens, kv_heads, head_dim) views (any token/head strides).
    slot_mapping: int32 (tokens,); negative entries are skipped.
    """
    _check_pool(key_cache, value_cache)
    _require_cuda("keys", keys)
    _require_cuda("values", values)
    _int32("slot_mapping", slot_mapping)
    layers, slots, hkv, d = key_cache.shape
    if keys.shape != values.shape or keys.dim() != 3 or tuple(keys.shape[1:]) != (hkv, d):
        raise ValueError(f"keys/values must have shape (tokens, {hkv}, {d})")
    if keys.dtype != key_cache.dtype or values.dtype != key_cache.dtype:
        raise ValueError("keys/values dtype must match the KV-cache dtype")
    if slot_mapping.numel() != keys.shape[0]:
        raise ValueError("slot_mapping must have one entry per token")
    kt, kh = _tok_head_strides("keys", keys)
    vt, vh = _tok_head_strides("values", values)
    rc = _lib.load().b2p_kv_write(
        keys.data_ptr(), kt, kh, values.data_ptr(), vt, vh, key_cache.data_ptr(),
        value_cache.data_ptr(), slot_mapping.data_ptr(), keys.shape[0], layer_index, layers,
        slots, hkv, d, dtype_code(key_cache.dtype), _ptr(err_flag), _stream(key_cache.device),
    )
    _lib.check(rc, "b2p_kv_write")


def cuda_core_fallbacks() -> tuple[int, int]:
    """bf16/f16 launches of (decode, prefill) so far that ran on the CUDA-core kernels
    because the tensor-core kernels' preconditions were not met."""
    lib = _lib.load()
    return int(lib.b2p_cuda_core_fallbacks(2)), int(lib.b2p_cuda_core_fallbacks(3))


def reset_scratch(device: torch.device) -> None:
    """Zero the library's device-resident prefill claim counters on ``device`` (on its
    current stream), after a launch whose bounded waits gave up."""
    with torch.cuda.device(device):
        _lib.check(_lib.load().b2p_reset_scratch(_stream(torch.device(device))),
                   "b2p_reset_scratch")


def decode_workspace_size(num_seqs: int, num_q_heads: int, num_kv_heads: int, head_dim: int) -> int:
    return int(_lib.load().b2p_paged_decode_workspace_size(num_seqs, num_q_heads, num_kv_heads,
                                                            head_dim))


def make_decode_workspace(max_seqs: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                          device: torch.device) -> torch.Tensor:
    """Zero-filled scratch for the split-K decode kernel (reusable across launches)."""
    n = decode_workspace_size(max_seqs, num_q_heads, num_kv_heads, head_dim)
    return torch.zeros(max(n, 16), dtype=torch.uint8, device=device)


def paged_decode(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer_index: int,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    block_size: int,
    scale: float,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    err_flag: torch.Tensor | None = None,
) -> torch.Tensor:
    """K2: one query token per sequence attends its paged history.

    q: (num_seqs, num_q_heads, head_dim); returns out of the same shape.
    """
    _check_pool(key_cache, value_cache)
    _require_cuda("q", q)
    _int32("block_tables", block_tables)
    _int32("context_lens", context_lens)
    layers, slots, hkv, d = key_cache.shape
    n, hq, dq = q.shape
    if dq != d or q.dtype != key_cache.dtype:
        raise ValueError("q must match the pool's head_dim and dtype")
    if block_tables.dim() != 2 or block_tables.shape[0] < n or context_lens.numel() < n:
        raise ValueError("block_tables/context_lens must cover every sequence")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    qt, qhs = _tok_head_strides("q", q)
    ot, ohs = _tok_head_strides("out", out)
    if workspace is None:
        workspace = make_decode_workspace(n, hq, hkv, d, q.device)
    rc = _lib.load().b2p_paged_decode(
        q.data_ptr(), qt, qhs, key_cache.data_ptr(), value_cache.data_ptr(), layer_index, layers,
        slots, block_tables.data_ptr(), block_tables.stride(0), context_lens.data_ptr(), n, hq,
        hkv, d, block_size, float(scale), out.data_ptr(), ot, ohs, workspace.data_ptr(),
        workspace.numel(), dtype_code(q.dtype), _ptr(err_flag), _stream(q.device),
    )
    _lib.check(rc, "b2p_paged_decode")
    return out


def paged_decode_append(
    q: torch.Tensor,
    new_keys: torch.Tensor,
    new_values: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer_index: int,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    block_size: int,
    scale: float,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    err_flag: torch.Tensor | None = None,
) -> torch.Tensor:
    """K1 + K2 for decode rows in one launch: stores each sequence's new K/V row (position
    ``context_lens[i] - 1``, slot from its block table) into the pool and attends over the
    whole history. q: (num_seqs, HQ, D); new_keys / new_values: (num_seqs, Hkv, D)."""
    _check_pool(key_cache, value_cache)
    _require_cuda("q", q)
    _int32("block_tables", block_tables)
    _int32("context_lens", context_lens)
    layers, slots, hkv, d = key_cache.shape
    n, hq, dq = q.shape
    if dq != d or q.dtype != key_cache.dtype:
        raise ValueError("q must match the pool's head_dim and dtype")
    for name, t in (("new_keys", new_keys), ("new_values", new_values)):
        _require_cuda(name, t)
        if t.dtype != key_cache.dtype or t.dim() != 3 or t.shape[0] < n or t.shape[1:] != (hkv, d):
            raise ValueError(f"{name} must be (num_seqs, num_kv_heads, head_dim) in the pool dtype")
        if t.stride(-1) != 1:
            raise ValueError(f"{name} must have a contiguous head_dim")
    if block_tables.dim() != 2 or block_tables.shape[0] < n or context_lens.numel() < n:
        raise ValueError("block_tables/context_lens must cover every sequence")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    qt, qhs = _tok_head_strides("q", q)
    ot, ohs = _tok_head_strides("out", out)
    if workspace is None:
        workspace = make_decode_workspace(n, hq, hkv, d, q.device)
    rc = _lib.load().b2p_paged_decode_append(
        q.data_ptr(), qt, qhs, new_keys.data_ptr(), new_keys.stride(0), new_keys.stride(1),
        new_values.data_ptr(), new_values.stride(0), new_values.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(), layer_index, layers, slots,
        block_tables.data_ptr(), block_tables.stride(0), context_lens.data_ptr(), n, hq, hkv, d,
        block_size, float(scale), out.data_ptr(), ot, ohs, workspace.data_ptr(),
        workspace.numel(), dtype_code(q.dtype), _ptr(err_flag), _stream(q.device),
    )
    _lib.check(rc, "b2p_paged_decode_append")
    return out


def paged_prefill(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer_index: int,
    block_tables: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    context_lens: torch.Tensor,
    max_q_len: int,
    block_size: int,
    scale: float,
    out: torch.Tensor | None = None,
    err_flag: torch.Tensor | None = None,
) -> torch.Tensor:
    """K3: packed variable-length causal attention over the paged history.

    q: (rows, num_q_heads, head_dim); sequence i owns rows [cu_seqlens_q[i],
    cu_seqlens_q[i+1]) of q (int32, num_seqs + 1 entries, need not start at 0, so a
    trailing slice of a packed batch can be run with views of its metadata).
    """
    _check_pool(key_cache, value_cache)
    _require_cuda("q", q)
    _int32("block_tables", block_tables)
    _int32("cu_seqlens_q", cu_seqlens_q)
    _int32("context_lens", context_lens)
    layers, slots, hkv, d = key_cache.shape
    total_q, hq, dq = q.shape
    if dq != d or q.dtype != key_cache.dtype:
        raise ValueError("q must match the pool's head_dim and dtype")
    num_seqs = cu_seqlens_q.numel() - 1
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    qt, qhs = _tok_head_strides("q", q)
    ot, ohs = _tok_head_strides("out", out)
    rc = _lib.load().b2p_paged_prefill(
        q.data_ptr(), qt, qhs, key_cache.data_ptr(), value_cache.data_ptr(), layer_index, layers,
        slots, block_tables.data_ptr(), block_tables.stride(0), cu_seqlens_q.data_ptr(),
        context_lens.data_ptr(), num_seqs, total_q, max_q_len, hq, hkv, d, block_size,
        float(scale), out.data_ptr(), ot, ohs, dtype_code(q.dtype), _ptr(err_flag),
        _stream(q.device),
    )
    _lib.check(rc, "b2p_paged_prefill")
    return out


def build_metadata(
    query_lens: torch.Tensor,
    context_lens: torch.Tensor,
    table_rows: torch.Tensor,
    block_mirror: torch.Tensor,
    block_size: int,
    total_q: int,
    max_blocks_per_seq: int,
    err_flag: torch.Tensor | None = None,
) -> dict[str, torch.Tensor]:
    """K4: packed batch metadata from a per-step execution descriptor (all int32 CUDA)."""
    for name, t in (("query_lens", query_lens), ("context_lens", context_lens),
                    ("table_rows", table_rows), ("block_mirror", block_mirror)):
        _int32(name, t)
    n = query_lens.numel()
    dev = query_lens.device
    out = {
        "cu_seqlens_q": torch.empty(n + 1, dtype=torch.int32, device=dev),
        "cu_seqlens_k": torch.empty(n + 1, dtype=torch.int32, device=dev),
        "positions": torch.empty(total_q, dtype=torch.int64, device=dev),
        "slot_mapping": torch.empty(total_q, dtype=torch.int32, device=dev),
        "logit_indices": torch.empty(n, dtype=torch.int64, device=dev),
        "block_tables": torch.empty((n, max(max_blocks_per_seq, 1)), dtype=torch.int32,
                                    device=dev),
    }
    rc = _lib.load().b2p_build_metadata(
        query_lens.data_ptr(), context_lens.data_ptr(), table_rows.data_ptr(), n,
        block_mirror.data_ptr(), block_mirror.stride(0), block_mirror.shape[0], block_size,
        out["cu_seqlens_q"].data_ptr(), out["cu_seqlens_k"].data_ptr(),
        out["positions"].data_ptr(), out["slot_mapping"].data_ptr(),
        out["logit_indices"].data_ptr(), out["block_tables"].data_ptr(), max_blocks_per_seq,
        total_q, _ptr(err_flag), _stream(dev),
    )
    _lib.check(rc, "b2p_build_metadata")
    return out


def lm_head_argmax_workspace_size(rows: int) -> int:
    """Bytes of the K6 workspace for up to ``rows`` rows (keys and a counter; rows are
    counted rounded up to the kernel's 128-row tiles)."""
    return int(_lib.load().b2p_lm_head_argmax_workspace_size(rows + (-rows) % 128))


def lm_head_argmax(
    hidden: torch.Tensor,
    weight: torch.Tensor,
    workspace: torch.Tensor,
    out_ids: torch.Tensor | None = None,
    out_max: torch.Tensor | None = None,
    err_flag: torch.Tensor | None = None,
    rows: int | None = None,
) -> torch.Tensor | None:
    """K6: greedy token ids ``argmax_v round(hidden[r] . weight[v])`` for the first ``rows``
    rows of hidden (default: all).

    hidden (n, hidden_size) and weight (vocab, hidden_size) are bf16 or f16 CUDA tensors
    with contiguous rows; the logits are rounded to their dtype before the argmax (the LM
    head's own output type) and never written. The kernel takes rows in tiles of 128: a
    hidden whose n is a multiple of 128 is used as it is (rows past ``rows`` are computed
    and dropped), any other is copied into a zero-padded one first. ``workspace`` is a uint8
    CUDA tensor of at least ``lm_head_argmax_workspace_size(n rounded up to 128)`` bytes,
    zero before its first use (each launch leaves it zero). Returns the int64 ids of the
    first ``rows`` rows, or None when the dtype or shape is outside what the kernel takes
    (the caller then computes logits).
    """
    _require_cuda("hidden", hidden)
    _require_cuda("weight", weight)
    _require_cuda("workspace", workspace)
    if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
        raise ValueError("hidden must be (rows, hidden_size) and weight (vocab, hidden_size)")
    if hidden.dtype != weight.dtype:
        raise ValueError("hidden and weight dtypes differ")
    if hidden.stride(1) != 1 or weight.stride(1) != 1:
        raise ValueError("hidden and weight rows must be contiguous")
    if hidden.dtype not in (torch.bfloat16, torch.float16) or hidden.shape[1] % 64:
        return None
    n = hidden.shape[0]
    rows = n if rows is None else rows
    if not 0 <= rows <= n:
        raise ValueError("rows must lie within hidden's rows")
    if n % 128:
        padded = hidden.new_zeros((n + (-n) % 128, hidden.shape[1]))
        padded[:n] = hidden
        hidden = padded
    n = hidden.shape[0]
    dev = hidden.device
    for name, t, dt in (("out_ids", out_ids, torch.int64), ("out_max", out_max, torch.float32)):
        if t is not None and (t.dtype != dt or not t.is_contiguous() or t.numel() < rows):
            raise ValueError(f"{name} must be a contiguous {dt} tensor of at least rows entries")
    # the kernel writes one entry per padded row: the caller's tensors when they are large
    # enough, else scratch whose first rows are copied back
    ids = out_ids if out_ids is not None and out_ids.numel() >= n else \
        torch.empty(n, dtype=torch.int64, device=dev)
    mx = out_max if out_max is None or out_max.numel() >= n else \
        torch.empty(n, dtype=torch.float32, device=dev)
    rc = _lib.load().b2p_lm_head_argmax(
        hidden.data_ptr(), hidden.stride(0), weight.data_ptr(), weight.stride(0), n,
        weight.shape[0], hidden.shape[1], dtype_code(hidden.dtype), ids.data_ptr(),
        _ptr(mx), workspace.data_ptr(), workspace.numel(), _ptr(err_flag), _stream(dev),
    )
    if rc == _lib.B2P_EUNSUPPORTED:
        return None
    _lib.check(rc, "b2p_lm_head_argmax")
    if out_ids is not None and ids is not out_ids:
        out_ids[:rows].copy_(ids[:rows])
        ids = out_ids
    if out_max is not None and mx is not out_max:
        out_max[:rows].copy_(mx[:rows])
    return ids[:rows]
