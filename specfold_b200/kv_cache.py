"""Preallocated prefix KV cache for the folded verify forward and the block commit.

The reference keeps the prefix in a transformers ``DynamicCache``.  Every committed
block appends through ``DynamicCache.update`` (transformers 4.57.3, called from the
attention layers, ``modeling_ministral.py:154-158``; the commit forward is
``nld_generation.py:279-289`` / ``fastdllm_v2_generation.py:560-575``), which is a
``torch.cat`` per layer: the whole prefix is reallocated and copied for every block
(O(P) per block), and the tensors move, so nothing keyed on their addresses survives
a commit.

This cache allocates ``capacity`` rows per layer and kv head once and appends in place
on the GPU (``sf_kv_append``).  The prefix views it hands out keep their addresses
until the capacity is exceeded (then it grows by doubling, one copy), so the folded
forward's per-configuration state and CUDA graph are reused across the verify steps of
a block, and only the prefix length changes from block to block.

It implements what the folded forward and a decoder layer call on ``past_key_values``:
``get_seq_length``, ``len``, ``[li] -> (k, v)`` with k, v shaped [1, Hkv, P, hd] (rows
contiguous per head, heads ``capacity * hd`` apart), iteration, and
``update(key_states, value_states, layer_idx, cache_kwargs=None) -> (k, v)`` with the
``DynamicCache.update`` meaning (append, return the whole prefix of that layer), plus
``crop``.  Batch 1 only, like the reference's running prefix.
"""

from __future__ import annotations

from typing import Iterator, List, Optional, Tuple

import torch

from . import kernels as K


class PreallocatedKVCache:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, capacity: int,
                 dtype: torch.dtype = torch.bfloat16, device="cuda"):
        if num_layers <= 0 or num_kv_heads <= 0 or head_dim <= 0 or capacity <= 0:
            raise ValueError("layers, kv heads, head dim and capacity must be positive")
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("the preallocated KV cache lives on a CUDA device")
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.dtype, self.device = dtype, device
        self.capacity = 0
        self._store: Optional[torch.Tensor] = None       # [L, 2, Hkv, capacity, hd]
        self._len: List[int] = [0] * num_layers
        self._grow(capacity)

    # ---------------------------------------------------------------- construction
    @classmethod
    def from_cache(cls, cache, capacity: Optional[int] = None) -> "PreallocatedKVCache":
        """Copy a cache with the ``len`` / ``[li] -> (k, v)`` interface (a DynamicCache
        shim, or another prefix cache) into a new preallocated cache with room for
        ``capacity`` rows (default: twice the current length, at least 256)."""
        L = len(cache)
        k0, _ = cache[0]
        _, Hkv, P, hd = k0.shape
        out = cls(L, Hkv, hd, capacity or max(256, 2 * P), dtype=k0.dtype, device=k0.device)
        for li in range(L):
            k, v = cache[li]
            out.update(k, v, li)
        return out

    def _grow(self, capacity: int) -> None:
        store = torch.zeros(self.num_layers, 2, self.num_kv_heads, capacity, self.head_dim,
                            dtype=self.dtype, device=self.device)
        if self._store is not None:
            n = max(self._len)
            store[:, :, :, :n].copy_(self._store[:, :, :, :n])
        self._store = store
        self.capacity = capacity

    # ---------------------------------------------------------------- read side
    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._len[layer_idx]

    def __len__(self) -> int:
        return self.num_layers

    def __getitem__(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        n = self._len[layer_idx]
        return (self._store[layer_idx, 0, :, :n].unsqueeze(0),
                self._store[layer_idx, 1, :, :n].unsqueeze(0))

    def __iter__(self) -> Iterator[Tuple[torch.Tensor, torch.Tensor]]:
        return (self[li] for li in range(self.num_layers))

    def buffers(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Layer ``layer_idx``'s whole key and value buffers [Hkv, capacity, hd]: the
        addresses the forward keys its state on (they change only when the cache grows)."""
        return self._store[layer_idx, 0], self._store[layer_idx, 1]

    # ---------------------------------------------------------------- write side
    def reserve(self, n: int) -> None:
        """Make room for ``n`` more rows in every layer (grows by doubling)."""
        need = max(self._len) + n
        if need > self.capacity:
            cap = self.capacity
            while cap < need:
                cap *= 2
            self._grow(cap)

    def advance(self, n: int) -> None:
        """Count ``n`` rows that a commit forward wrote in place (at the current length of
        every layer, within the reserved capacity) as part of the prefix."""
        if any(x + n > self.capacity for x in self._len):
            raise ValueError("advance past the cache capacity")
        self._len = [x + n for x in self._len]

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append ``key_states`` / ``value_states`` [1, Hkv, n, hd] to layer
        ``layer_idx`` and return that layer's whole prefix (``DynamicCache.update``)."""
        if key_states.shape != value_states.shape or key_states.dim() != 4 or key_states.shape[0] != 1:
            raise ValueError(f"expected [1, Hkv, n, hd] key/value states, got {tuple(key_states.shape)}")
        _, Hkv, n, hd = key_states.shape
        if Hkv != self.num_kv_heads or hd != self.head_dim:
            raise ValueError(f"cache holds {self.num_kv_heads} kv heads of {self.head_dim}, "
                             f"got {Hkv} x {hd}")
        if key_states.dtype != self.dtype or value_states.dtype != self.dtype:
            raise ValueError(f"cache dtype {self.dtype}, got {key_states.dtype}")
        P = self._len[layer_idx]
        if P + n > self.capacity:
            cap = self.capacity
            while cap < P + n:
                cap *= 2
            self._grow(cap)
        if n > 0:
            nk, nv = key_states[0], value_states[0]

            def rows_ok(t):
                return t.stride(2) == 1 and (n == 1 or t.stride(1) == hd)

            if not (rows_ok(nk) and rows_ok(nv) and nk.stride(0) == nv.stride(0)):
                # one [Hkv, n, hd] layout for both (torch keeps odd strides on size-1 dims)
                nk = torch.empty((Hkv, n, hd), dtype=self.dtype, device=self.device).copy_(nk)
                nv = torch.empty((Hkv, n, hd), dtype=self.dtype, device=self.device).copy_(nv)
            K.kv_append(self._store[layer_idx, 0], self._store[layer_idx, 1], nk, nv, P)
        self._len[layer_idx] = P + n
        return self[layer_idx]

    def crop(self, max_length: int) -> None:
        """Keep the first ``max_length`` rows of every layer (``DynamicCache.crop``; a
        negative value drops that many rows from the end)."""
        for li in range(self.num_layers):
            n = self._len[li]
            self._len[li] = max(0, n + max_length) if max_length < 0 else min(n, max_length)
