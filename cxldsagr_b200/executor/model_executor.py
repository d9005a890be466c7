"""Single-request chunked inference over any model with a request cache.

Same job as the reference's ``executor/model_executor.py``: split a token
tensor into chunks, feed each chunk through ``model(chunk, cache, ...)`` so
the cache grows chunk by chunk, and hand back what the last chunk produced
(the hidden states of all its tokens, or the logits of its last
``logits_to_keep`` tokens).  :class:`ModelExecutor` adds the prefill
(empty cache) / extend (nonempty cache) rules and the cache allocation hooks.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Literal

import torch

Output = Literal["hidden", "logits"]


def _is_count(value: Any, *, minimum: int) -> bool:
    return isinstance(value, int) and not isinstance(value, bool) and value >= minimum


@dataclass(frozen=True)
class ChunkSchedule:
    """Chunk boundaries of one request: tokens [start, start + size) per step."""

    total: int
    chunk_size: int

    def __post_init__(self):
        if not _is_count(self.chunk_size, minimum=1):
            raise ValueError(f"chunk_size must be an int >= 1, got {self.chunk_size!r}")

    def spans(self):
        for start in range(0, self.total, self.chunk_size):
            yield start, min(self.chunk_size, self.total - start)

    @property
    def steps(self) -> int:
        return -(-self.total // self.chunk_size)


def _check_request(ids: Any, output: str, logits_to_keep: Any) -> None:
    if not (isinstance(ids, torch.Tensor) and ids.ndim == 1 and ids.numel() > 0 and ids.dtype == torch.long):
        raise ValueError("ids: expected a nonempty 1-D tensor of dtype torch.long")
    if output not in ("hidden", "logits"):
        raise ValueError(f"output must be 'hidden' or 'logits', got {output!r}")
    if not _is_count(logits_to_keep, minimum=0):
        raise ValueError(f"logits_to_keep must be an int >= 0, got {logits_to_keep!r}")
    if output == "hidden" and logits_to_keep:
        raise ValueError("logits_to_keep applies to logits output only (hidden output returns the whole last chunk)")


def _check_capacity(model: Any, cache: Any, new_tokens: int) -> None:
    end = cache.length + new_tokens
    if end > cache.max_seq_len:
        raise ValueError(f"the request needs {end} cache rows, the cache holds {cache.max_seq_len}")
    limit = model.config.max_position_embeddings
    if end > limit:
        raise ValueError(f"the request reaches position {end}, beyond max_position_embeddings = {limit}")


def run_chunks(model: Any, ids: torch.Tensor, cache: Any, chunk_size: int, *, output: Output = "hidden",
               logits_to_keep: int = 0) -> torch.Tensor:
    schedule = ChunkSchedule(ids.numel() if isinstance(ids, torch.Tensor) else 0, chunk_size)
    _check_request(ids, output, logits_to_keep)
    _check_capacity(model, cache, ids.numel())
    kwargs = {"return_hidden": True} if output == "hidden" else {"logits_to_keep": logits_to_keep}
    last = None
    with torch.inference_mode():
        for start, size in schedule.spans():
            last = model(ids.narrow(0, start, size), cache, **kwargs)
    return last


class ModelExecutor:
    """Prefill/extend token tensors against a model and a request-level cache."""

    def __init__(self, model: Any, *, cache_manager: Any = None, chunk_size: int = 1024):
        ChunkSchedule(0, chunk_size)  # validates chunk_size
        self.model = model
        self.cache_manager = cache_manager if cache_manager is not None else getattr(model, "cache_manager", None)
        self.chunk_size = chunk_size

    @property
    def max_seq_len(self) -> int:
        return self.model.config.max_position_embeddings

    def allocate(self, max_seq_len: int) -> Any:
        manager = self.cache_manager
        return manager.allocate(max_seq_len) if manager is not None else self.model.new_cache(max_seq_len)

    def release(self, cache: Any) -> None:
        if self.cache_manager is not None:
            self.cache_manager.release(cache)

    def _run(self, ids, cache, output, logits_to_keep):
        return run_chunks(self.model, ids, cache, self.chunk_size, output=output, logits_to_keep=logits_to_keep)

    def prefill(self, ids, cache, *, output: Output = "hidden", logits_to_keep: int = 0):
        if cache.length:
            raise ValueError(f"prefill starts from an empty cache; this one holds {cache.length} tokens")
        return self._run(ids, cache, output, logits_to_keep)

    def extend(self, ids, cache, *, output: Output = "hidden", logits_to_keep: int = 0):
        """Append one or more tokens (single-token decode included)."""
        if cache.length <= 0:
            raise ValueError("extend continues a cache that already holds tokens; prefill first")
        return self._run(ids, cache, output, logits_to_keep)
