"""Attention and cache contracts shared by model adapters and operators.

Same contract surface as the reference (``models/attention_contracts.py:11-60``
and ``cache/contracts.py:11-31``): an indexer returns a logical block or
token selection relative to the request; main attention consumes that
selection through a cache access object that does not expose physical
placement (so an offloading backend can overlap fetches with compute).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Protocol

import torch


@dataclass(frozen=True)
class BlockSelection:
    """Logical block ids [query, head_or_group, selected_block] (+ optional valid mask)."""

    block_ids: torch.Tensor
    block_size: int
    valid_mask: torch.Tensor | None = None


@dataclass(frozen=True)
class TokenSelection:
    """Logical token ids [query, selected_token]; -1 marks padding."""

    token_ids: torch.Tensor


@dataclass(frozen=True)
class AttentionContext:
    layer_idx: int
    query_start: int
    query_length: int
    auxiliary_state: Any = None


class CacheAccess(Protocol):
    """Committed token count and capacity of one request, plus per-layer state."""

    @property
    def length(self) -> int: ...

    @property
    def max_seq_len(self) -> int: ...

    def get_layer_state(self, layer_idx: int) -> object | None: ...

    def set_layer_state(self, layer_idx: int, state: object) -> None: ...


class CacheSession(Protocol):
    @property
    def released(self) -> bool: ...

    def release(self) -> None: ...


class Indexer(Protocol):
    def __call__(self, q: torch.Tensor, cache_access: CacheAccess,
                 context: AttentionContext) -> BlockSelection | TokenSelection: ...


class MainAttention(Protocol):
    def __call__(self, q: torch.Tensor, selection: BlockSelection | TokenSelection | None,
                 cache_access: CacheAccess, context: AttentionContext) -> torch.Tensor: ...


@dataclass
class SimpleCacheAccess:
    """Minimal :class:`CacheAccess` for a single request."""

    length: int
    max_seq_len: int
    states: dict | None = None

    def get_layer_state(self, layer_idx):
        return (self.states or {}).get(layer_idx)

    def set_layer_state(self, layer_idx, state):
        if self.states is None:
            self.states = {}
        self.states[layer_idx] = state
