"""Batched indexer over independent resident sequences (one query each).

Reference: ``operators/deepseek_v32/indexer/resident_batch.py:73-216``
(``prepare_keys`` / ``paged_logits`` / ``single_sequence_logits`` /
``mask_causal_``), an observation API over Hopper's paged DeepGEMM indexer.
Here sequences keep contiguous FP8 keys (no page packing); each sequence's
logits come from the same indexer kernel as the model, its keys split over
all SMs, and ``mask_causal_`` writes -inf past each sequence's length.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import indexer_logits


@dataclass(frozen=True)
class PreparedKeys:
    keys: torch.Tensor      # FP8 [B, N, 128]
    scales: torch.Tensor    # FP32 [B, N]
    lengths: torch.Tensor   # int64 [B] (host), valid keys per sequence

    @property
    def batch_size(self) -> int:
        return self.keys.shape[0]


def prepare_keys(keys: torch.Tensor, scales: torch.Tensor, *, lengths=None) -> PreparedKeys:
    """Validate ``[B, N, 128]`` FP8 keys and ``[B, N]`` scales; ``lengths`` defaults to N each."""
    if keys.dim() != 3 or keys.shape[2] != 128 or keys.dtype != torch.float8_e4m3fn:
        raise ValueError("keys must be FP8 [B, N, 128]")
    if scales.shape != keys.shape[:2] or scales.dtype != torch.float32:
        raise ValueError("scales must be FP32 [B, N]")
    B, N = keys.shape[:2]
    lengths = torch.full((B,), N, dtype=torch.int64) if lengths is None else torch.as_tensor(lengths).long().cpu()
    if lengths.shape != (B,) or bool((lengths < 1).any()) or bool((lengths > N).any()):
        raise ValueError("lengths must be in [1, N] per sequence")
    return PreparedKeys(keys.contiguous(), scales.contiguous(), lengths)


def single_sequence_logits(q, keys, weights, scales, length: int) -> torch.Tensor:
    """Logits [Q, length] of Q queries at the end of one sequence (causal)."""
    Q = q.shape[0]
    return indexer_logits(q, keys[:length], weights, scales[:length], length - Q)


def paged_logits(prepared: PreparedKeys, q: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """One query per sequence: q FP8 [B, 64, 128], weights FP32 [B, 64] -> logits [B, N]
    (columns at or past a sequence's length are -inf)."""
    B, N = prepared.keys.shape[:2]
    if q.shape[0] != B or weights.shape[0] != B:
        raise ValueError("one query (and head-weight row) per sequence")
    out = torch.full((B, N), -torch.inf, dtype=torch.float32, device=q.device)
    for b in range(B):
        n = int(prepared.lengths[b])
        out[b, :n] = single_sequence_logits(q[b:b + 1], prepared.keys[b], weights[b:b + 1], prepared.scales[b], n)[0]
    return out


def mask_causal_(logits: torch.Tensor, lengths) -> torch.Tensor:
    """In place: -inf at columns >= each row's length."""
    lengths = torch.as_tensor(lengths, device=logits.device).long()
    cols = torch.arange(logits.shape[1], device=logits.device)[None, :]
    return logits.masked_fill_(cols >= lengths[:, None], -torch.inf)
