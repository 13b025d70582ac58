"""Decode-side KV cache that stores each KV head once.

After ``CircuitKVCluster.update_kv`` the reference's attention forward hands the
compressed K / V to ``past_key_value.update(key, value, layer_idx, cache_kwargs)``
(KVCache-Factory/pyramidkv/llama_model.py:2918-2928) and, at every decode step, the new
token's K / V the same way (llama_model.py:2931).  Its forward calls ``repeat_kv`` before
the cache, so an HF ``DynamicCache`` there stores every KV head ``num_key_value_groups``
times (4 times for Llama-3-8B).

``DistinctKVCache`` has the same ``update`` / ``get_seq_length`` / ``get_usable_length``
surface but keeps ``[B, Hkv, T, D]``: inputs that carry all query heads (the repeat_kv
layout, whose heads ``g * groups .. g * groups + groups - 1`` are equal) are reduced to
their distinct heads as they come in, and prefill outputs made with
``CircuitKVCluster(distinct_kv_heads=True)`` arrive that way already.  ``update`` returns
the layer's whole cache in the distinct layout for a GQA-aware attention (e.g.
``flash_attn_func`` with ``num_heads_k = Hkv``), or repeated to all query heads with
``repeat=True`` for one that is not.  Memory and decode reads: 1 / groups of the
repeated cache.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch


class DistinctKVCache:
    def __init__(self, num_key_value_heads: int, num_key_value_groups: int, repeat: bool = False):
        if num_key_value_groups < 1 or num_key_value_heads < 1:
            raise ValueError("num_key_value_heads and num_key_value_groups must be >= 1")
        self.kv_heads = int(num_key_value_heads)
        self.groups = int(num_key_value_groups)
        self.repeat = bool(repeat)
        self.key_cache: List[torch.Tensor] = []
        self.value_cache: List[torch.Tensor] = []
        self._seen_tokens = 0

    def _distinct(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 4:
            raise ValueError("expected [batch, heads, tokens, head_dim]")
        if x.shape[1] == self.kv_heads:
            return x
        if x.shape[1] == self.kv_heads * self.groups:
            return x[:, :: self.groups]   # the repeat_kv layout: equal heads in groups
        raise ValueError(f"expected {self.kv_heads} or {self.kv_heads * self.groups} heads, got {x.shape[1]}")

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Appends this call's tokens to layer ``layer_idx`` and returns its whole cache."""
        k = self._distinct(key_states)
        v = self._distinct(value_states)
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[-2]
        if layer_idx < len(self.key_cache):
            self.key_cache[layer_idx] = torch.cat([self.key_cache[layer_idx], k], dim=-2)
            self.value_cache[layer_idx] = torch.cat([self.value_cache[layer_idx], v], dim=-2)
        else:
            while len(self.key_cache) < layer_idx:   # layers this rank does not hold stay empty
                self.key_cache.append(torch.empty(0))
                self.value_cache.append(torch.empty(0))
            self.key_cache.append(k.contiguous())
            self.value_cache.append(v.contiguous())
        return self.layer(layer_idx)

    def layer(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        k, v = self.key_cache[layer_idx], self.value_cache[layer_idx]
        if self.repeat and self.groups > 1:
            return (k.repeat_interleave(self.groups, dim=1), v.repeat_interleave(self.groups, dim=1))
        return k, v

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if layer_idx >= len(self.key_cache) or self.key_cache[layer_idx].dim() != 4:
            return 0
        return self.key_cache[layer_idx].shape[-2]

    def get_usable_length(self, new_seq_length: int, layer_idx: int = 0) -> int:
        return self.get_seq_length(layer_idx)

    def __len__(self) -> int:
        return len(self.key_cache)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.key_cache + self.value_cache)
