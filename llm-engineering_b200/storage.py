"""Paged KV storage with the reference layout, written through the K1 kernel.

Interface of ``PagedKVStorage`` (serving/engine/paged_kv_storage.py:6-174): the same
constructor, attributes (``key_cache``/``value_cache`` of shape
``[num_layers, num_blocks * block_size, num_kv_heads, head_dim]``, ``num_slots`` ...) and
``ValueError`` messages. ``scatter`` runs the CUDA KV-write kernel; ``gather`` exists for
callers that still want materialised histories (the paged attention kernels never call
it).
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from . import ops


class PagedKVStorage:
    def __init__(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                 head_dim: int, dtype: torch.dtype, device: torch.device) -> None:
        for name, value in (("num_layers", num_layers), ("num_blocks", num_blocks),
                            ("block_size", block_size), ("num_kv_heads", num_kv_heads),
                            ("head_dim", head_dim)):
            if value <= 0:
                raise ValueError(f"{name} must be greater than zero.")
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device)
        self.num_slots = num_blocks * block_size
        shape = (num_layers, self.num_slots, num_kv_heads, head_dim)
        self.key_cache = torch.empty(shape, dtype=dtype, device=self.device)
        self.value_cache = torch.empty(shape, dtype=dtype, device=self.device)

    def _check_layer(self, layer_index: int) -> None:
        if not 0 <= layer_index < self.num_layers:
            raise ValueError("layer_index must be within the configured layers.")

    def _slot_tensor(self, slot_ids: Sequence[int] | torch.Tensor) -> torch.Tensor:
        if isinstance(slot_ids, torch.Tensor):
            arr = slot_ids.detach().to("cpu", torch.int64).numpy()
        else:
            arr = np.asarray(slot_ids, dtype=np.int64).reshape(-1)
        if arr.size and (arr.min() < 0 or arr.max() >= self.num_slots):
            raise ValueError("slot_ids must be within the configured physical slots.")
        return torch.from_numpy(arr.astype(np.int32)).to(self.key_cache.device, non_blocking=True)

    def scatter(self, layer_index: int, slot_ids: Sequence[int] | torch.Tensor,
                keys: torch.Tensor, values: torch.Tensor) -> None:
        """Write row t of keys/values into slot slot_ids[t] of one layer (K1)."""
        self._check_layer(layer_index)
        slots = self._slot_tensor(slot_ids)
        expected = (slots.numel(), self.num_kv_heads, self.head_dim)
        if tuple(keys.shape) != expected:
            raise ValueError(f"keys must have shape {expected}.")
        if tuple(values.shape) != expected:
            raise ValueError(f"values must have shape {expected}.")
        if keys.dtype != self.dtype:
            raise ValueError("keys dtype must match the KV-cache dtype.")
        if values.dtype != self.dtype:
            raise ValueError("values dtype must match the KV-cache dtype.")
        if keys.device != self.key_cache.device:
            raise ValueError("keys device must match the KV-cache device.")
        if values.device != self.key_cache.device:
            raise ValueError("values device must match the KV-cache device.")
        ops.kv_write(self.key_cache, self.value_cache, layer_index, slots, keys, values)

    def gather(self, layer_index: int,
               slot_ids: Sequence[int] | torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Rows of the given slots in logical order (materialised copy)."""
        self._check_layer(layer_index)
        idx = self._slot_tensor(slot_ids).long()
        return (self.key_cache[layer_index].index_select(0, idx),
                self.value_cache[layer_index].index_select(0, idx))
