"""Generic per-request resident caches with step transactions.

Reference: ``cache/manager.py:23-257`` (``CacheSpec``, ``ResidentCache`` with
begin/write/commit/abort, ``CacheManager``).  A step reserves rows after the
committed length; writes land in place; ``commit`` publishes them, ``abort``
forgets them (the next step overwrites the rows).  Used for per-layer
auxiliary records (e.g. the indexer's FP8 keys) next to the main KV cache.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class CacheSpec:
    name: str
    shape: tuple[int, ...]      # per-token record shape
    dtype: torch.dtype
    capacity: int

    def bytes(self) -> int:
        n = self.capacity
        for d in self.shape:
            n *= d
        return n * torch.empty((), dtype=self.dtype).element_size()


class ResidentCache:
    def __init__(self, spec: CacheSpec, device="cuda"):
        self.spec = spec
        self.data = torch.zeros((spec.capacity, *spec.shape), dtype=spec.dtype, device=device)
        self.length = 0
        self._pending = None

    def begin(self, count: int) -> slice:
        if self._pending is not None:
            raise RuntimeError(f"{self.spec.name}: a step is already open")
        if count < 1 or self.length + count > self.spec.capacity:
            raise ValueError(f"{self.spec.name}: step exceeds capacity")
        self._pending = slice(self.length, self.length + count)
        return self._pending

    def write(self, rows: slice, values: torch.Tensor):
        if self._pending is None or rows.start < self._pending.start or rows.stop > self._pending.stop:
            raise ValueError(f"{self.spec.name}: write outside the open step")
        self.data[rows] = values

    def commit(self):
        if self._pending is None:
            raise RuntimeError(f"{self.spec.name}: no open step")
        self.length = self._pending.stop
        self._pending = None

    def abort(self):
        self._pending = None

    def truncate(self, length: int):
        if self._pending is not None or not 0 <= length <= self.length:
            raise ValueError(f"{self.spec.name}: invalid truncation")
        self.length = length

    def view(self, end: int | None = None) -> torch.Tensor:
        return self.data[: self.length if end is None else end]


class CacheManager:
    """A named set of resident caches that begin/commit/abort together."""

    def __init__(self, specs, device="cuda"):
        self.caches = {s.name: ResidentCache(s, device) for s in specs}

    def __getitem__(self, name) -> ResidentCache:
        return self.caches[name]

    def begin(self, count):
        return {n: c.begin(count) for n, c in self.caches.items()}

    def commit(self):
        for c in self.caches.values():
            c.commit()

    def abort(self):
        for c in self.caches.values():
            c.abort()

    def nbytes(self) -> int:
        return sum(c.spec.bytes() for c in self.caches.values())
