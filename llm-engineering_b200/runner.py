"""B200 paged model runner — the drop-in for the reference's ``PagedModelRunner``.

Reference path replaced (serving/engine/paged_model_runner.py:44-91): one packed HF
forward per engine step, with ``HFBatchedPagedCache`` (serving/engine/
hf_batched_paged_cache.py:52-148) scattering new K/V, gathering every history and
concatenating it, a dense additive block-diagonal mask (serving/engine/attention_mask.py),
and HF SDPA over all packed keys.

Here the same ``ModelRunner.forward(executions) -> (B, vocab)`` interface
(serving/engine/model_runner.py:11-26) drives:
  * K4 (``ops.build_metadata``): cu_seqlens, positions, write slots and logit rows built on
    the GPU from a per-step descriptor (query length, key length, table row per execution)
    and the step's block tables;
  * ``B200PagedCache.update`` (the HF ``Cache`` hook, transformers/models/qwen2/
    modeling_qwen2.py:225): K1 writes the step's prefill K/V rows into the pool and
    returns without gathering anything;
  * ``paged_attention`` (registered with HF's ``AttentionInterface`` under
    ``ATTENTION_NAME``; the model calls it at modeling_qwen2.py:227-240): the fused K1 + K2
    call for the leading decode executions (it stores their new K/V rows and attends in one
    launch) and K3 for the prefill / chunked-prefill ones, reading the pool in place
    through block tables. A registered name outside HF's mask registry also makes HF skip
    building any mask.
  * ``logits_to_keep`` restricts the LM head to each execution's last query row, which is
    exactly the rows the reference keeps with ``index_select`` (paged_model_runner.py:85-91).
  * ``greedy_tokens`` (an addition to the interface, used by this package's engine when
    every row of a step is greedy): K6 (``ops.lm_head_argmax``) computes the LM head over
    those rows and keeps only each row's arg-max, in place of ``forward`` + ``argmax``
    (serving/engine/sampling.py:78-79).

Executions may come from the reference engine (``slot_ids`` over the whole history) or
from this package's engine (``block_ids``). Slot ids that follow the block structure
(``slot = block * block_size + pos % block_size``, which is what the reference's
``BlockTable`` produces) become block tables; any other slot list is run as a table of
one-slot blocks, which the CUDA-core attention kernel accepts.
"""

from __future__ import annotations

import contextlib
import contextvars
import warnings
from collections.abc import Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch
from transformers.cache_utils import Cache

from . import ops as _ops
from ._lib import DEV_WAIT_TIMEOUT

ATTENTION_NAME = "b200_paged"
PREFILL, DECODE = "prefill", "decode"

_active_batch: contextvars.ContextVar[StepBatch | None] = contextvars.ContextVar(
    "b200_paged_step", default=None)


@dataclass
class StepBatch:
    """Device metadata of one packed forward."""

    kernels: Any
    key_cache: torch.Tensor
    value_cache: torch.Tensor
    block_size: int
    total_q: int
    num_execs: int
    num_decode: int       # leading executions that are single-token decodes
    max_q_len: int
    slot_mapping: torch.Tensor   # int32 [total_q]
    positions: torch.Tensor      # int64 [total_q]
    cu_seqlens_q: torch.Tensor   # int32 [B + 1]
    context_lens: torch.Tensor   # int32 [B]
    block_tables: torch.Tensor   # int32 [B, W]
    logit_indices: torch.Tensor  # int64 [B]
    workspace: torch.Tensor
    err: torch.Tensor
    # Decode rows take the fused K1 + K2 call: the cache hook then writes only the
    # prefill rows, and the attention function stores the decode rows' new K/V itself.
    fused_decode: bool = False


def _phase_of(execution) -> str:
    phase = getattr(execution.phase, "value", execution.phase)
    if phase not in (PREFILL, DECODE):
        raise ValueError(f"Unsupported execution phase: {execution.phase}")
    return phase


def paged_attention(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                    value: torch.Tensor, attention_mask: torch.Tensor | None,
                    dropout: float = 0.0, scaling: float | None = None, **kwargs: Any):
    """HF attention-interface function: paged attention of the packed query rows.

    query: (1, HQ, Tq, D) after RoPE. ``key``/``value`` are this step's new rows; the
    prefill rows are already in the pool (``B200PagedCache.update``), and the decode rows
    are stored by the fused decode call when the step uses it. The kernels read every
    history from the pool. Returns (attn_output (1, Tq, HQ, D), None) like HF's SDPA path.
    """
    del attention_mask, kwargs
    batch = _active_batch.get()
    if batch is None:
        raise RuntimeError(f"{ATTENTION_NAME} attention used outside B200PagedModelRunner.forward")
    if dropout:
        raise ValueError("paged attention does not implement dropout")
    layer = module.layer_idx
    q = query[0].transpose(0, 1)  # (Tq, HQ, D) view, head_dim contiguous
    if scaling is None:
        scaling = q.shape[-1] ** -0.5
    k = batch.kernels
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    nd = batch.num_decode
    if nd and batch.fused_decode:
        k.paged_decode_append(q[:nd], key[0].transpose(0, 1)[:nd], value[0].transpose(0, 1)[:nd],
                              batch.key_cache, batch.value_cache, layer, batch.block_tables[:nd],
                              batch.context_lens[:nd], batch.block_size, scaling, out=out[:nd],
                              workspace=batch.workspace, err_flag=batch.err)
    elif nd:
        k.paged_decode(q[:nd], batch.key_cache, batch.value_cache, layer, batch.block_tables[:nd],
                       batch.context_lens[:nd], batch.block_size, scaling, out=out[:nd],
                       workspace=batch.workspace, err_flag=batch.err)
    if nd < batch.num_execs:
        k.paged_prefill(q, batch.key_cache, batch.value_cache, layer, batch.block_tables[nd:],
                        batch.cu_seqlens_q[nd:], batch.context_lens[nd:], batch.max_q_len,
                        batch.block_size, scaling, out=out, err_flag=batch.err)
    return out.unsqueeze(0), None


def _register_attention() -> None:
    from transformers import AttentionInterface

    AttentionInterface.register(ATTENTION_NAME, paged_attention)


class B200PagedCache(Cache):
    """HF cache hook: writes each layer's new prefill K/V rows into the pool (K1; decode
    rows are stored by the fused decode call) and returns the states unchanged — there is
    no gathered history to hand back."""

    def __init__(self, batch: StepBatch) -> None:
        super().__init__(layers=[])
        self._batch = batch

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               *args: Any, **kwargs: Any) -> tuple[torch.Tensor, torch.Tensor]:
        del args, kwargs
        if key_states.ndim != 4:
            raise ValueError("key_states must have shape (batch, kv_heads, tokens, head_dim).")
        if value_states.ndim != 4:
            raise ValueError("value_states must have shape (batch, kv_heads, tokens, head_dim).")
        if key_states.shape != value_states.shape:
            raise ValueError("key_states and value_states must have matching shapes.")
        if key_states.shape[0] != 1:
            raise ValueError("Packed execution must use one Hugging Face batch row.")
        if key_states.shape[2] != self._batch.total_q:
            raise ValueError(
                "Packed KV query length does not match BatchLayout: "
                f"expected {self._batch.total_q}, got {key_states.shape[2]}.")
        b = self._batch
        first = b.num_decode if b.fused_decode else 0  # decode rows: stored by the fused call
        if first < b.total_q:
            b.kernels.kv_write(b.key_cache, b.value_cache, layer_idx, b.slot_mapping[first:],
                               key_states[0].transpose(0, 1)[first:],
                               value_states[0].transpose(0, 1)[first:], b.err)
        return key_states, value_states

    def get_seq_length(self, layer_idx: int = 0) -> int:
        raise RuntimeError(
            "B200PagedCache does not expose one scalar sequence length for packed execution "
            f"(layer {layer_idx}).")

    def get_query_offset(self, layer_idx: int = 0) -> int:
        raise RuntimeError(
            "B200PagedCache does not expose one scalar query offset for packed execution "
            f"(layer {layer_idx}).")

    def get_mask_sizes(self, query_length: int, layer_idx: int) -> tuple[int, int]:
        raise RuntimeError(
            "B200PagedCache builds no attention mask; cache-derived mask sizing is unsupported "
            f"(query_length={query_length}, layer={layer_idx}).")


def _storage_of(paged_cache) -> Any:
    return getattr(paged_cache, "storage", paged_cache)


class _TableMirror:
    """Device-resident copy of the block tables of the sequences a step runs, one row per
    (request, admission), updated with only the blocks each table gained since its last
    step (the engine appends to a table between admissions and never rewrites it). Rows of
    sequences a step does not run are released; a sequence that comes back gets a fresh
    row and a whole upload. Per step this moves a few bytes per new block instead of the
    whole [B, W] table, and the host walks only the new blocks."""

    def __init__(self, device: torch.device, rows: int = 256, cols: int = 64) -> None:
        self.device = device
        self.table = torch.full((rows, cols), -1, dtype=torch.int32, device=device)
        self._rows: dict[object, list[int]] = {}  # key -> [row, blocks uploaded]
        self._free = list(range(rows - 1, -1, -1))

    def _grow(self, rows: int, cols: int) -> None:
        old = self.table
        self.table = torch.full((rows, cols), -1, dtype=torch.int32, device=self.device)
        self.table[:old.shape[0], :old.shape[1]] = old
        self._free = list(range(rows - 1, old.shape[0] - 1, -1)) + self._free

    def sync(self, keys: Sequence, block_lists: Sequence) -> list[int]:
        """Rows of `keys` (one per execution), after uploading their new blocks."""
        live = set(keys)
        for key in [k for k in self._rows if k not in live]:
            self._free.append(self._rows.pop(key)[0])
        need_cols = max(len(b) for b in block_lists)
        need_rows = len(self._rows) + sum(1 for k in live if k not in self._rows)
        rows_cap, cols_cap = self.table.shape
        while rows_cap < need_rows:
            rows_cap *= 2
        while cols_cap < need_cols:
            cols_cap *= 2
        if (rows_cap, cols_cap) != tuple(self.table.shape):
            self._grow(rows_cap, cols_cap)
        stride = self.table.shape[1]
        rows, idx, vals = [], [], []
        for key, blocks in zip(keys, block_lists, strict=True):
            entry = self._rows.get(key)
            if entry is None:
                entry = [self._free.pop(), 0]
                self._rows[key] = entry
            row, done = entry
            if len(blocks) > done:
                base = row * stride
                idx.extend(range(base + done, base + len(blocks)))
                vals.extend(blocks[done:])
                entry[1] = len(blocks)
            rows.append(row)
        if idx:
            packed = torch.from_numpy(np.asarray([idx, vals], dtype=np.int64))
            if self.device.type == "cuda":
                packed = packed.pin_memory()
            packed = packed.to(self.device, non_blocking=True)
            self.table.view(-1).index_copy_(0, packed[0], packed[1].to(torch.int32))
        return rows


class B200PagedModelRunner:
    """``ModelRunner`` implementation running the packed forward on the paged kernels.

    Args:
        model: a Hugging Face causal LM whose attention goes through ``AttentionInterface``
            (Qwen2 and the other functional-attention models).
        device: CUDA device of the model and the pool.
        paged_cache: the reference's ``PagedKVCache`` (or anything with ``.storage``) or a
            storage object exposing ``key_cache``, ``value_cache`` and ``block_size``
            (the reference's ``PagedKVStorage`` or ``llm_engineering_b200.storage``).

    Every ``forward`` reads the kernels' device error word once the step's logits are
    computed (one synchronisation, which the caller's sampling would make anyway) and
    raises ``RuntimeError`` if a kernel reported bad data (a slot or block id outside the
    pool, a context length that does not fit, a bounded wait that gave up): the logits of
    such a step are not returned.
    """

    def __init__(self, model, device: torch.device, paged_cache) -> None:
        self._model = model
        self._device = torch.device(device)
        self._storage = _storage_of(paged_cache)
        self._warned_fallback = False
        _register_attention()
        model.set_attn_implementation(ATTENTION_NAME)
        model.eval()
        cfg = model.config
        self._hq = cfg.num_attention_heads
        self._hkv = cfg.num_key_value_heads
        self._head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self._workspace = torch.zeros(16, dtype=torch.uint8, device=self._device)
        self._err = torch.zeros(1, dtype=torch.int32, device=self._device)
        self._mirror: _TableMirror | None = None
        self._k6_hidden: torch.Tensor | None = None
        self._k6_workspace: torch.Tensor | None = None

    # ------------------------------------------------------------------ host metadata
    @staticmethod
    def _token_ids(seq, start: int, stop: int) -> np.ndarray:
        """Token ids of positions [start, stop) without building the whole history."""
        take = getattr(seq, "token_slice", None)
        if take is not None:  # this package's sequences keep the history as one array
            return take(start, stop)
        prompt = seq.request.prompt_token_ids
        n = len(prompt)
        if stop <= n:
            return np.asarray(prompt[start:stop], dtype=np.int64)
        gen = seq.generated_token_ids
        if start >= n:
            return np.asarray(gen[start - n:stop - n], dtype=np.int64)
        return np.concatenate([np.asarray(prompt[start:], dtype=np.int64),
                               np.asarray(gen[:stop - n], dtype=np.int64)])

    def _describe(self, executions: Sequence) -> dict:
        bs = self._storage.block_size
        # Executions of this package's engine (block lists, sequences that count their
        # admissions) keep their tables in the device mirror, updated with new blocks only.
        mirrored = all(getattr(ex, "block_ids", None) is not None
                       and hasattr(ex.sequence, "admissions") for ex in executions)
        phases, qlens, lengths, tables, is_slots, token_parts = [], [], [], [], [], []
        for ex in executions:
            phase = _phase_of(ex)
            length = getattr(ex, "length", None) or ex.sequence.current_length
            qlen = getattr(ex, "query_length", None)
            if qlen is None:  # reference ModelExecution: BatchLayout semantics
                qlen = length if phase == PREFILL else 1
            blocks = getattr(ex, "block_ids", None)
            slot_list = False
            if blocks is None:
                slots = np.asarray(ex.slot_ids, dtype=np.int64)
                if len(slots) != length:
                    raise ValueError("slot_ids length must equal the sequence current length.")
                cand = slots[::bs] // bs
                pos = np.arange(length, dtype=np.int64)
                if np.array_equal(cand[pos // bs] * bs + pos % bs, slots):
                    blocks = cand
                else:  # not block-structured: keep the per-position slots
                    blocks, slot_list = slots, True
            tables.append(blocks if mirrored else np.asarray(blocks, dtype=np.int64))
            is_slots.append(slot_list)
            token_parts.append(self._token_ids(ex.sequence, length - qlen, length))
            phases.append(phase)
            qlens.append(qlen)
            lengths.append(length)
        if any(is_slots):  # express every table as one-slot blocks (block size 1)
            expanded = []
            for t, n, sl in zip(tables, lengths, is_slots, strict=True):
                if sl:
                    expanded.append(t)
                else:
                    pos = np.arange(n, dtype=np.int64)
                    expanded.append(t[pos // bs] * bs + pos % bs)
            tables, bs = expanded, 1
        return {"phases": phases, "qlens": qlens, "lengths": lengths, "tables": tables,
                "tokens": np.concatenate(token_parts), "block_size": bs, "mirrored": mirrored}

    def _build_batch(self, executions: Sequence) -> tuple[StepBatch, torch.Tensor]:
        d = self._describe(executions)
        n = len(executions)
        dev = self._device
        num_decode = 0
        while num_decode < n and d["phases"][num_decode] == DECODE:
            num_decode += 1
        kernels = _ops
        bs = d["block_size"]
        if d["mirrored"]:
            # rows of the device mirror (new blocks uploaded by sync); K4 gathers this step's
            # padded [n, width] tables from them
            keys = [(ex.sequence.request.request_id, ex.sequence.admissions) for ex in executions]
            if self._mirror is None:
                self._mirror = _TableMirror(dev)
            mirror_rows = self._mirror.sync(keys, d["tables"])
            width = max(1, max(-(-length // bs) for length in d["lengths"]))
            host = np.empty((3 * n,), dtype=np.int32)
            host[2 * n:3 * n] = mirror_rows
        else:
            width = max(1, max(len(t) for t in d["tables"]))
            host = np.full((3 * n + n * width,), -1, dtype=np.int32)
            host[2 * n:3 * n] = np.arange(n, dtype=np.int32)
            tab = host[3 * n:].reshape(n, width)
            for i, t in enumerate(d["tables"]):
                tab[i, :len(t)] = t
        host[0:n] = d["qlens"]
        host[n:2 * n] = d["lengths"]
        staged = torch.from_numpy(host)
        tokens = torch.from_numpy(d["tokens"])
        if dev.type == "cuda":
            staged = staged.pin_memory()
            tokens = tokens.pin_memory()
        dev_i32 = staged.to(dev, non_blocking=True)
        input_ids = tokens.to(dev, non_blocking=True)
        qlens = dev_i32[0:n]
        ctx = dev_i32[n:2 * n]
        rows = dev_i32[2 * n:3 * n]
        total_q = int(sum(d["qlens"]))
        if d["mirrored"]:
            md = kernels.build_metadata(qlens, ctx, rows, self._mirror.table, bs, total_q, width,
                                        self._err)
            tables = md["block_tables"]
        else:
            tables = dev_i32[3 * n:].view(n, width)
            md = kernels.build_metadata(qlens, ctx, rows, tables, bs, total_q, 0, self._err)
        need = kernels.decode_workspace_size(max(num_decode, 1), self._hq, self._hkv,
                                             self._head_dim)
        if self._workspace.numel() < need:
            self._workspace = torch.zeros(need, dtype=torch.uint8, device=dev)
        batch = StepBatch(
            kernels=kernels, key_cache=self._storage.key_cache,
            value_cache=self._storage.value_cache, block_size=d["block_size"], total_q=total_q,
            num_execs=n, num_decode=num_decode, max_q_len=max(d["qlens"]),
            slot_mapping=md["slot_mapping"], positions=md["positions"],
            cu_seqlens_q=md["cu_seqlens_q"], context_lens=ctx, block_tables=tables,
            logit_indices=md["logit_indices"], workspace=self._workspace, err=self._err,
            fused_decode=num_decode > 0 and hasattr(kernels, "paged_decode_append"))
        return batch, input_ids

    # ------------------------------------------------------------------ ModelRunner
    def forward(self, executions: Sequence) -> torch.Tensor:
        """Next-token logits (B, vocab) for the executions, in their order."""
        out = self._run(executions, lambda batch, input_ids, cache: self._model(
            input_ids=input_ids.unsqueeze(0), position_ids=batch.positions.unsqueeze(0),
            attention_mask=None, past_key_values=cache, use_cache=True,
            logits_to_keep=batch.logit_indices))
        return out.logits[0]

    def greedy_tokens(self, executions: Sequence) -> torch.Tensor | None:
        """Greedy next-token ids (B,) int64 on the device, in the executions' order.

        The same forward as ``forward`` up to the final norm, then K6 (the LM head fused with
        the argmax, ``ops.lm_head_argmax``) on each execution's last row: the ids equal the
        argmax of the logits ``forward`` returns (the rounding to the model dtype included),
        and the (B, vocab) logits are never written. Returns None, without running
        anything, when the model has no plain bias-free LM head over a ``model`` body or its
        dtype / hidden size is outside what K6 takes (the caller then uses ``forward``).
        """
        head = self._lm_head()
        if head is None:
            return None
        n = len(executions)
        padded = n + (-n) % 128  # K6 takes rows in tiles of 128
        if self._k6_hidden is None or self._k6_hidden.shape[0] < padded:
            self._k6_hidden = torch.zeros((max(padded, 256), head.shape[1]), dtype=head.dtype,
                                          device=self._device)
            self._k6_workspace = torch.zeros(
                _ops.lm_head_argmax_workspace_size(self._k6_hidden.shape[0]), dtype=torch.uint8,
                device=self._device)

        def run(batch, input_ids, cache):
            out = self._model.model(input_ids=input_ids.unsqueeze(0),
                                    position_ids=batch.positions.unsqueeze(0), attention_mask=None,
                                    past_key_values=cache, use_cache=True)
            # last rows into the padded buffer (rows past n hold earlier steps' states, whose
            # ids are computed and dropped)
            hidden = self._k6_hidden[:padded]
            torch.index_select(out.last_hidden_state[0], 0, batch.logit_indices, out=hidden[:n])
            return _ops.lm_head_argmax(hidden, head, self._k6_workspace, err_flag=self._err,
                                       rows=n)
        return self._run(executions, run)

    def _lm_head(self) -> torch.Tensor | None:
        """The LM head weight when K6 can stand in for it (else None)."""
        lm = getattr(self._model, "lm_head", None)
        body = getattr(self._model, "model", None)
        if not isinstance(lm, torch.nn.Linear) or lm.bias is not None or body is None:
            return None
        w = lm.weight
        if (w.dtype not in (torch.bfloat16, torch.float16) or not w.is_cuda
                or w.shape[1] % 64 != 0 or w.stride(1) != 1
                or getattr(self._model.config, "final_logit_softcapping", None)):
            return None
        return w

    def _run(self, executions: Sequence, fn):
        """One packed step: batch metadata, the model call ``fn``, the device-error check."""
        if not executions:
            raise ValueError("At least one execution is required.")
        fallbacks = self._fallbacks()
        batch, input_ids = self._build_batch(executions)
        cache = B200PagedCache(batch)
        token = _active_batch.set(batch)
        try:
            with torch.inference_mode():
                out = fn(batch, input_ids, cache)
        finally:
            _active_batch.reset(token)
        bits = self.device_error()
        if bits:
            raise RuntimeError(
                f"paged-attention kernels reported device error bits {bits:#x} "
                f"({', '.join(_error_names(bits))}) in this step; its logits are discarded")
        if fallbacks is not None and not self._warned_fallback and self._fallbacks() != fallbacks:
            self._warned_fallback = True
            warnings.warn(
                f"{self._storage.key_cache.dtype} paged attention ran on the CUDA-core kernels "
                "(block size, head_dim, GQA group or row alignment outside what the tensor-core "
                "kernels take); expect a large slowdown", RuntimeWarning, stacklevel=3)
        return out

    @staticmethod
    def _fallbacks() -> tuple[int, int] | None:
        """bf16/f16 launches that took the CUDA-core kernels so far (decode, prefill)."""
        count = getattr(_ops, "cuda_core_fallbacks", None)
        return None if count is None else count()

    def device_error(self) -> int:
        """Bits the kernels reported since the last call (0 = none); clears them.

        After a bounded wait gave up (``B2P_DEV_WAIT_TIMEOUT``) a launch may have left
        split-K counters or greedy-pick keys set: the decode workspace, the K6 workspace and
        the prefill claim counters are then zeroed before the next step."""
        v = int(self._err.item())
        if v:
            self._err.zero_()
            if v & DEV_WAIT_TIMEOUT:
                self._workspace.zero_()
                if self._k6_workspace is not None:
                    self._k6_workspace.zero_()
                reset = getattr(_ops, "reset_scratch", None)
                if reset is not None:
                    reset(self._device)
        return v


_ERROR_BITS = ((1, "slot id outside the pool"), (2, "block id outside the pool"),
               (4, "a bounded wait gave up"), (8, "a length that does not fit"))


def _error_names(bits: int) -> list[str]:
    return [name for bit, name in _ERROR_BITS if bits & bit] or ["unknown"]



@contextlib.contextmanager
def active(batch: StepBatch):
    """Make ``batch`` the current step for ``paged_attention`` (used by tests)."""
    token = _active_batch.set(batch)
    try:
        yield
    finally:
        _active_batch.reset(token)
