"""Resident FP8 indexer key cache of one session x layer.

The lightning indexer scans every visible key each step, so its 132-byte
records (128 E4M3 values + one FP32 scale) stay resident in HBM even when the
main MLA records are offloaded (reference: ``cache/indexer_cache.py:60-286``
and the resident arrays of ``models/deepseek_v32/attention.py:56-61``).
Candidate (transient) tokens use rows after the committed history and are
discarded with the step.
"""

from __future__ import annotations

import torch


class IndexerCache:
    def __init__(self, capacity: int, dim: int = 128, *, device="cuda"):
        self.capacity = capacity
        self.keys = torch.zeros((capacity, dim), dtype=torch.float8_e4m3fn, device=device)
        self.scales = torch.zeros(capacity, dtype=torch.float32, device=device)
        # offset[0]: prefill mean hint; offset[1]: decode EMA of the k-th score.
        self.offset = torch.zeros(16, dtype=torch.float32, device=device)
        self.length = 0

    @property
    def record_bytes(self) -> int:
        return self.keys.shape[1] + 4

    def rows(self, start: int, count: int):
        if start < 0 or start + count > self.capacity:
            raise ValueError("indexer rows exceed the session capacity")
        return self.keys[start:start + count], self.scales[start:start + count]

    def pred_ids(self, end: int) -> torch.Tensor:
        """Scratch list [end] of predicted history rows, reset to -1 (no host sync)."""
        if getattr(self, "_pred", None) is None or self._pred.numel() < end:
            self._pred = torch.empty(self.capacity, dtype=torch.int32, device=self.keys.device)
        view = self._pred[:end]
        view.fill_(-1)
        return view

    def visible(self, end: int):
        return self.keys[:end], self.scales[:end]

    def commit(self, length: int):
        self.length = length

    def truncate(self, length: int):
        self.length = min(self.length, length)

    def snapshot(self) -> dict:
        return {"length": self.length, "offset": self.offset.clone()}

    def restore(self, state: dict):
        self.length = state["length"]
        self.offset.copy_(state["offset"])

    def nbytes(self) -> int:
        return self.keys.numel() + self.scales.numel() * 4 + self.offset.numel() * 4
