"""Layer placement over the GPUs of one process.

The reference's own multi-GPU mode (``models/deepseek_v32/model.py:34-60``
plan, ``:142`` placement, ``:874-894`` loop): the checkpoint's layers are
split into contiguous runs, one run per device in the given order (every
device gets at least one layer), minimising the largest run's resident
weight bytes subject to each device's memory budget; the forward pass runs
the layers in order and moves the hidden / residual rows between devices.
:class:`~cxldsagr_b200.models.deepseek_v32.model.DeepSeekV32Model` takes it
with ``devices=[...]``.  It is the simple scale-out path (one request, layers
in sequence); the throughput paths are data parallel and the sequence /
expert parallel layout of :mod:`.groups`.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from ..checkpoint import layer_tensor_specs
from ..config import ModelConfig


def plan_layer_devices(sizes: Sequence[int], devices: Sequence, budgets: Sequence[int]) -> list:
    """Device of each layer: contiguous runs over ``devices`` in order, each
    non-empty, minimising the largest run's bytes with every run within its
    device's budget.  Among equally good plans the last run starts as early
    as possible (the reference's choice).

    Raises ``ValueError`` for inconsistent arguments and ``RuntimeError`` when
    no plan fits the budgets.
    """
    n, g = len(sizes), len(devices)
    if not 1 <= g <= n or len(budgets) != g:
        raise ValueError("one memory budget per nonempty device partition is required")
    prefix = [0]
    for s in sizes:
        prefix.append(prefix[-1] + int(s))
    # plans[e] for the first j devices: (largest run, run ends) covering layers [0, e).
    plans: dict[int, tuple[int, tuple[int, ...]]] = {0: (0, ())}
    for j in range(1, g + 1):
        nxt: dict[int, tuple[int, tuple[int, ...]]] = {}
        for e in range(j, n - (g - j) + 1):  # leave one layer for each later device
            best = None
            for s in range(j - 1, e):
                prev = plans.get(s)
                if prev is None:
                    continue
                w = prefix[e] - prefix[s]
                if w > budgets[j - 1]:
                    continue
                cand = (max(prev[0], w), prev[1] + (e,))
                if best is None or cand[0] < best[0]:
                    best = cand
            if best is not None:
                nxt[e] = best
        plans = nxt
    if n not in plans:
        raise RuntimeError("available GPU memory cannot hold the complete FP8 checkpoint plus reserve")
    ends = plans[n][1]
    mapping, start = [], 0
    for device, end in zip(devices, ends):
        mapping.extend([device] * (end - start))
        start = end
    return mapping


_BYTES = {"linear": 1, "fp32": 4, "bias": 4, "norm": 4, "bf16": 2}


def layer_weight_bytes(cfg: ModelConfig, layer: int, *, fp8: bool = True) -> int:
    """Resident bytes of one layer's weights: FP8 linears (1 byte per element
    plus one FP32 scale per 128 x 128 block) or BF16, FP32 norms / gates."""
    total = 0
    for _, (shape, kind) in layer_tensor_specs(cfg, layer).items():
        numel = 1
        for d in shape:
            numel *= d
        if kind == "linear":
            if fp8 and len(shape) == 2:
                total += numel + ((shape[0] + 127) // 128) * ((shape[1] + 127) // 128) * 4
            else:
                total += numel * 2
        else:
            total += numel * _BYTES.get(kind, 4)
    return total


def device_budgets(devices: Sequence[torch.device], reserve_bytes: int, endpoints: tuple[int, int] = (0, 0)) -> list[int]:
    """Free memory per device minus ``reserve_bytes``; the first device also
    holds ``endpoints[0]`` bytes (embedding), the last ``endpoints[1]`` (LM
    head).  CPU devices have no limit."""
    out = []
    for d in devices:
        d = torch.device(d)
        if d.type == "cuda":
            free, _ = torch.cuda.mem_get_info(d)
            out.append(int(free) - int(reserve_bytes))
        else:
            out.append(1 << 62)
    out[0] -= endpoints[0]
    out[-1] -= endpoints[1]
    return out
