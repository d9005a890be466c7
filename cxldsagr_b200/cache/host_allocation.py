"""Pinned host allocation and its accounting.

The CUDA caching host allocator rounds pinned blocks up to powers of two, so a
ledger that wants the real DRAM footprint must count the rounded size
(reference: ``cache/host_allocation.py:14-56``).
"""

from __future__ import annotations

import torch


def pinned_allocation_bytes(nbytes: int) -> int:
    """Bytes the pinned caching allocator reserves for a request of ``nbytes``."""
    if nbytes <= 0:
        return 0
    return 1 << (int(nbytes) - 1).bit_length()


def allocate_host_tensor(shape, *, dtype, pin_memory: bool) -> torch.Tensor:
    """Zeroed host tensor; pinned (page-locked, device-mapped under UVA) when asked."""
    t = torch.empty(shape, dtype=dtype, pin_memory=pin_memory)
    t.zero_()
    return t


def tensor_bytes(tensors) -> dict:
    """{"hbm": bytes, "dram": bytes} of the distinct storages among ``tensors``."""
    seen, out = set(), {"hbm": 0, "dram": 0}
    for t in tensors:
        if t is None:
            continue
        storage = t.untyped_storage()
        key = (t.device, storage.data_ptr())
        if key in seen:
            continue
        seen.add(key)
        n = storage.nbytes()
        if t.device.type == "cpu" and t.is_pinned():
            n = pinned_allocation_bytes(n)
        out["hbm" if t.device.type == "cuda" else "dram"] += n
    return out
