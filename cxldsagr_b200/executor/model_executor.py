"""Single-request chunked inference over any model with a request cache.

Behavioural parity with ``executor/model_executor.py:18-125`` of the
reference: ``run_chunks`` feeds a token tensor through ``model(chunk, cache,
...)`` in chunks of ``chunk_size`` and returns only the last chunk's output
(hidden states of every token of that chunk, or logits through the model's
``logits_to_keep`` option); :class:`ModelExecutor` adds the empty/nonempty
cache rules of prefill and extend and the cache allocation hooks.
"""

from __future__ import annotations

from typing import Any, Literal

import torch

Output = Literal["hidden", "logits"]


def _check_chunk(chunk_size):
    if isinstance(chunk_size, bool) or not isinstance(chunk_size, int) or chunk_size < 1:
        raise ValueError("chunk_size must be a positive integer")


def run_chunks(model: Any, ids: torch.Tensor, cache: Any, chunk_size: int, *, output: Output = "hidden",
               logits_to_keep: int = 0) -> torch.Tensor:
    _check_chunk(chunk_size)
    if not isinstance(ids, torch.Tensor) or ids.ndim != 1 or ids.numel() == 0 or ids.dtype != torch.long:
        raise ValueError("ids must be a nonempty 1-D torch.long tensor")
    if output not in ("hidden", "logits"):
        raise ValueError("output must be 'hidden' or 'logits'")
    if isinstance(logits_to_keep, bool) or not isinstance(logits_to_keep, int) or logits_to_keep < 0:
        raise ValueError("logits_to_keep must be a nonnegative integer")
    if output == "hidden" and logits_to_keep:
        raise ValueError("hidden output returns all final-chunk features; do not set logits_to_keep")
    end = cache.length + ids.numel()
    if end > cache.max_seq_len:
        raise ValueError("KV cache capacity exceeded by the complete input")
    if end > model.config.max_position_embeddings:
        raise ValueError("Input exceeds model.config.max_position_embeddings")
    result = None
    with torch.inference_mode():
        for start in range(0, ids.numel(), chunk_size):
            chunk = ids[start:start + chunk_size]
            if output == "hidden":
                result = model(chunk, cache, return_hidden=True)
            else:
                result = model(chunk, cache, logits_to_keep=logits_to_keep)
    return result


class ModelExecutor:
    """Prefill/extend token tensors against a model and a request-level cache."""

    def __init__(self, model: Any, *, cache_manager: Any = None, chunk_size: int = 1024):
        _check_chunk(chunk_size)
        self.model = model
        self.cache_manager = cache_manager if cache_manager is not None else getattr(model, "cache_manager", None)
        self.chunk_size = chunk_size

    @property
    def max_seq_len(self) -> int:
        return self.model.config.max_position_embeddings

    def allocate(self, max_seq_len: int) -> Any:
        if self.cache_manager is not None:
            return self.cache_manager.allocate(max_seq_len)
        return self.model.new_cache(max_seq_len)

    def release(self, cache: Any) -> None:
        if self.cache_manager is not None:
            self.cache_manager.release(cache)

    def prefill(self, ids, cache, *, output: Output = "hidden", logits_to_keep: int = 0):
        if cache.length != 0:
            raise ValueError("prefill requires an empty cache")
        return run_chunks(self.model, ids, cache, self.chunk_size, output=output, logits_to_keep=logits_to_keep)

    def extend(self, ids, cache, *, output: Output = "hidden", logits_to_keep: int = 0):
        """Append one or more tokens (single-token decode included)."""
        if cache.length <= 0:
            raise ValueError("extend requires a nonempty cache")
        return run_chunks(self.model, ids, cache, self.chunk_size, output=output, logits_to_keep=logits_to_keep)
