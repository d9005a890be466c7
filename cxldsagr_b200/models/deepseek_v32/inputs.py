"""Validation of one token sequence before it reaches the model.

Reference: ``models/deepseek_v32/inputs.py:6-26``.  Values are checked on the
tensor's own device with a single (min, max) transfer; only an accepted
sequence is copied to the execution device (asynchronously: the forward's
stream consumes the copy in order).
"""

from __future__ import annotations

import torch


def prepare_token_ids(token_ids, *, device, vocab_size: int, max_tokens: int) -> torch.Tensor:
    if isinstance(token_ids, torch.Tensor):
        ids = token_ids.to(dtype=torch.long)
    else:
        ids = torch.as_tensor(token_ids, dtype=torch.long, device="cpu")
    if ids.ndim != 1 or not 0 < ids.numel() <= max_tokens:
        raise ValueError("expected a nonempty single sequence fitting cache capacity")
    bounds = torch.stack(torch.aminmax(ids))
    if bounds.device.type != "cpu":
        bounds = bounds.cpu()
    low, high = (int(v) for v in bounds)
    if low < 0 or high >= vocab_size:
        raise ValueError("token ID is outside the checkpoint vocabulary")
    return ids.to(device=device, non_blocking=True)
