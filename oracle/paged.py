"""CPU restatement of the reference's paged KV and packed-attention computations.

Test infrastructure only (see ``oracle/__init__.py``). Every function cites the
reference file:line it restates (paths relative to the reference project root).
Integer work is done in numpy / plain Python; attention in fp32 torch on the CPU.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

PREFILL = "prefill"
DECODE = "decode"


# --------------------------------------------------------------------- KV storage
def scatter(key_cache: torch.Tensor, value_cache: torch.Tensor, layer: int,
            slot_ids: Sequence[int], keys: torch.Tensor, values: torch.Tensor) -> None:
    """``PagedKVStorage.scatter`` (serving/engine/paged_kv_storage.py:76-136): row t of
    keys/values goes to physical slot slot_ids[t] of one layer (index_copy_, :135-136)."""
    num_slots = key_cache.shape[1]
    if not 0 <= layer < key_cache.shape[0]:
        raise ValueError("layer_index must be within the configured layers.")
    if any(s < 0 or s >= num_slots for s in slot_ids):
        raise ValueError("slot_ids must be within the configured physical slots.")
    idx = torch.as_tensor(list(slot_ids), dtype=torch.long, device=key_cache.device)
    key_cache[layer].index_copy_(0, idx, keys.to(key_cache.device))
    value_cache[layer].index_copy_(0, idx, values.to(value_cache.device))


def gather(key_cache: torch.Tensor, value_cache: torch.Tensor, layer: int,
           slot_ids: Sequence[int]) -> tuple[torch.Tensor, torch.Tensor]:
    """``PagedKVStorage.gather`` (serving/engine/paged_kv_storage.py:138-174): rows of the
    given slots in logical order (index_select, :171-172)."""
    num_slots = key_cache.shape[1]
    if not 0 <= layer < key_cache.shape[0]:
        raise ValueError("layer_index must be within the configured layers.")
    if any(s < 0 or s >= num_slots for s in slot_ids):
        raise ValueError("slot_ids must be within the configured physical slots.")
    idx = torch.as_tensor(list(slot_ids), dtype=torch.long, device=key_cache.device)
    return key_cache[layer].index_select(0, idx), value_cache[layer].index_select(0, idx)


# --------------------------------------------------------------------- slots and layout
def slot_for_position(blocks: Sequence[int], position: int, block_size: int) -> int:
    """``BlockTable.slot_for_position`` (serving/engine/block.py:370-405)."""
    if position < 0:
        raise ValueError("token_position must not be negative.")
    logical = position // block_size
    if logical >= len(blocks):
        raise ValueError(f"No physical block exists for token position: {position!r}")
    return blocks[logical] * block_size + position % block_size


def history_slots(blocks: Sequence[int], length: int, block_size: int) -> np.ndarray:
    """``Engine._build_model_execution`` slot ids (serving/engine/engine.py:121-127): the
    slot of every position 0..length-1, vectorised."""
    pos = np.arange(length, dtype=np.int64)
    b = np.asarray(blocks, dtype=np.int64)
    if length and (length - 1) // block_size >= len(b):
        raise ValueError(f"No physical block exists for token position: {length - 1!r}")
    return b[pos // block_size] * block_size + pos % block_size


def query_length(phase: str, current_length: int) -> int:
    """``BatchLayout._query_length`` (serving/engine/batch_layout.py:84-109)."""
    if phase == PREFILL:
        return current_length
    if phase == DECODE:
        return 1
    raise ValueError(f"Unsupported execution phase: {phase}")


def exclusive_offsets(lengths: Sequence[int]) -> tuple[int, ...]:
    """``BatchLayout._offsets`` (serving/engine/batch_layout.py:112-137)."""
    out, cur = [], 0
    for n in lengths:
        out.append(cur)
        cur += n
    return tuple(out)


def batch_layout(phases: Sequence[str], current_lengths: Sequence[int]) -> dict:
    """``BatchLayout`` properties (serving/engine/batch_layout.py:40-81)."""
    if not phases:
        raise ValueError("BatchLayout requires at least one execution.")
    q = tuple(query_length(p, n) for p, n in zip(phases, current_lengths, strict=True))
    k = tuple(current_lengths)
    qo = exclusive_offsets(q)
    ko = exclusive_offsets(k)
    return {
        "query_lengths": q,
        "key_lengths": k,
        "query_offsets": qo,
        "key_offsets": ko,
        "logit_indices": tuple(o + n - 1 for o, n in zip(qo, q, strict=True)),
        "total_query_tokens": sum(q),
        "total_key_tokens": sum(k),
    }


def packed_positions(phases: Sequence[str], current_lengths: Sequence[int]) -> np.ndarray:
    """position_ids of ``build_packed_inputs`` (serving/engine/packed_inputs.py:106-131)."""
    parts = []
    for p, n in zip(phases, current_lengths, strict=True):
        if p == PREFILL:
            parts.append(np.arange(n, dtype=np.int64))
        elif p == DECODE:
            parts.append(np.array([n - 1], dtype=np.int64))
        else:
            raise ValueError(f"Unsupported execution phase: {p}")
    return np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)


def packed_input_ids(phases: Sequence[str], token_histories: Sequence[Sequence[int]]) -> np.ndarray:
    """input_ids of ``build_packed_inputs`` (serving/engine/packed_inputs.py:81-103)."""
    parts = []
    for p, toks in zip(phases, token_histories, strict=True):
        parts.append(np.asarray(toks if p == PREFILL else toks[-1:], dtype=np.int64))
    return np.concatenate(parts)


def write_slots(phases: Sequence[str], slot_histories: Sequence[Sequence[int]]) -> np.ndarray:
    """Slots written per step: ``PagedKVCache.update_and_gather``
    (serving/engine/paged_kv_cache.py:51-58) — prefill writes every slot of the history,
    decode the last one; concatenated in execution order."""
    parts = []
    for p, s in zip(phases, slot_histories, strict=True):
        s = np.asarray(s, dtype=np.int64)
        if p == PREFILL:
            parts.append(s)
        elif p == DECODE:
            parts.append(s[-1:])
        else:
            raise ValueError(f"Unsupported execution phase: {p}")
    return np.concatenate(parts)


def attention_mask(phases: Sequence[str], current_lengths: Sequence[int]) -> torch.Tensor:
    """``build_attention_mask`` (serving/engine/attention_mask.py:9-77): dense bool
    (total_q, total_k), block diagonal, tril for prefill, ones for decode."""
    lay = batch_layout(phases, current_lengths)
    mask = torch.zeros((lay["total_query_tokens"], lay["total_key_tokens"]), dtype=torch.bool)
    for i, p in enumerate(phases):
        qo, ko = lay["query_offsets"][i], lay["key_offsets"][i]
        ql, kl = lay["query_lengths"][i], lay["key_lengths"][i]
        block = torch.ones((ql, kl), dtype=torch.bool)
        if p == PREFILL:
            block = torch.tril(block)
        mask[qo:qo + ql, ko:ko + kl] = block
    return mask


def additive_mask(mask: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """``semantic_to_additive_attention_mask`` (serving/engine/attention_mask.py:80-120)."""
    add = torch.zeros(mask.shape, dtype=dtype)
    add.masked_fill_(~mask, torch.finfo(dtype).min)
    return add.unsqueeze(0).unsqueeze(0)


# --------------------------------------------------------------------- attention
def dense_packed_attention(q: torch.Tensor, k_hist: torch.Tensor, v_hist: torch.Tensor,
                           mask_add: torch.Tensor, scale: float) -> torch.Tensor:
    """The reference's packed attention: HF attention over the concatenated histories with
    the additive block-diagonal mask (transformers/models/qwen2/modeling_qwen2.py:161-184,
    softmax in fp32; SDPA at transformers/integrations/sdpa_attention.py:40-104 computes the
    same function). GQA heads via repeat_kv (modeling_qwen2.py:149-158).

    q: (Tq, HQ, D); k_hist/v_hist: (Tk, HKV, D); mask_add: (1, 1, Tq, Tk).
    Returns (Tq, HQ, D) in fp32.
    """
    hq, hkv = q.shape[1], k_hist.shape[1]
    group = hq // hkv
    qf = q.float().transpose(0, 1)                       # (HQ, Tq, D)
    kf = k_hist.float().transpose(0, 1).repeat_interleave(group, dim=0)  # (HQ, Tk, D)
    vf = v_hist.float().transpose(0, 1).repeat_interleave(group, dim=0)
    scores = torch.matmul(qf, kf.transpose(1, 2)) * scale + mask_add[0].float()
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32)
    return torch.matmul(probs, vf).transpose(0, 1).contiguous()


def _attend(qf: torch.Tensor, kf: torch.Tensor, vf: torch.Tensor, scale: float,
            causal_offset: int | None) -> torch.Tensor:
    """fp32 attention of q (Tq, HQ, D) over one sequence's keys (Tk, HKV, D)."""
    hq, hkv = qf.shape[1], kf.shape[1]
    group = hq // hkv
    qh = qf.transpose(0, 1)
    kh = kf.transpose(0, 1).repeat_interleave(group, dim=0)
    vh = vf.transpose(0, 1).repeat_interleave(group, dim=0)
    s = torch.matmul(qh, kh.transpose(1, 2)) * scale
    if causal_offset is not None:
        tq, tk = s.shape[1], s.shape[2]
        qpos = torch.arange(tq, device=s.device).unsqueeze(1) + causal_offset
        kpos = torch.arange(tk, device=s.device).unsqueeze(0)
        s = s.masked_fill(kpos > qpos, float("-inf"))
    p = torch.softmax(s, dim=-1, dtype=torch.float32)
    return torch.matmul(p, vh).transpose(0, 1)


def decode_attention(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                     layer: int, tables: Sequence[Sequence[int]], context_lens: Sequence[int],
                     block_size: int, scale: float) -> torch.Tensor:
    """Decode rows of the reference's packed attention, one sequence at a time: gather the
    history (paged_kv_storage.py:138-174, slots from engine.py:121-127) and attend with
    the all-ones decode block of the mask (attention_mask.py:47-52). Equal to
    ``dense_packed_attention`` restricted to decode rows; per-sequence so that it stays
    O(sum ctx) at benchmark sizes. Returns (num_seqs, HQ, D) fp32."""
    out = []
    for i, ctx in enumerate(context_lens):
        slots = history_slots(tables[i], ctx, block_size)
        k, v = gather(key_cache, value_cache, layer, slots.tolist())
        out.append(_attend(q[i:i + 1].float(), k.float(), v.float(), scale, None))
    return torch.cat(out, dim=0)


def prefill_attention(q: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                      layer: int, tables: Sequence[Sequence[int]], cu_seqlens_q: Sequence[int],
                      context_lens: Sequence[int], block_size: int, scale: float) -> torch.Tensor:
    """Prefill rows of the reference's packed attention, one sequence at a time, with the
    tril block of the mask (attention_mask.py:41-45). For a query run shorter than the
    history (chunked prefill) query j sits at position ctx - q_len + j — the
    generalisation the reference's mask comment asks for (attention_mask.py:20-22).
    Returns (total_q, HQ, D) fp32."""
    out = []
    for i, ctx in enumerate(context_lens):
        a, b = cu_seqlens_q[i], cu_seqlens_q[i + 1]
        slots = history_slots(tables[i], ctx, block_size)
        k, v = gather(key_cache, value_cache, layer, slots.tolist())
        out.append(_attend(q[a:b].float(), k.float(), v.float(), scale, ctx - (b - a)))
    return torch.cat(out, dim=0)


# --------------------------------------------------------------------- greedy sampling
def greedy_tokens(hidden: torch.Tensor, weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's greedy pick for each row: the LM head over the row's last hidden
    state (``lm_head`` + ``index_select`` of the logit rows,
    serving/engine/paged_model_runner.py:83-91), whose logits come out in the model dtype,
    then ``argmax`` (serving/engine/sampling.py:78-79; torch returns the first of equal
    maxima). Computed on the CPU in fp32, rounded to the weight dtype. Returns (ids, max)."""
    logits = (hidden.float().cpu() @ weight.float().cpu().T).to(weight.dtype).float()
    best = logits.max(-1).values
    ids = torch.argmax(logits, -1)
    return ids, best
