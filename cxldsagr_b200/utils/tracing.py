"""Scope hooks threaded through every forward (reference: the ``scope(name)``
callback of ``models/deepseek_v32/model.py:657`` bound to NVTX ranges).

* :func:`null_scope` - zero-cost default;
* :class:`NvtxScope` - NVTX ranges for an external timeline profiler;
* :class:`EventScope` - CUDA-event timing per scope name on the launching
  stream, summed after one synchronisation (device time, not wall clock).
"""

from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager, nullcontext

import torch


def null_scope(_name: str):
    return nullcontext()


class NvtxScope:
    def __call__(self, name: str):
        return torch.cuda.nvtx.range(name)


class EventScope:
    """Collect (start, end) CUDA events per scope; ``summary()`` syncs and sums ms."""

    def __init__(self, device=None):
        self.device = device
        self.events = defaultdict(list)
        self.stack = []

    @contextmanager
    def __call__(self, name: str):
        full = "/".join(self.stack + [name])
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        self.stack.append(name)
        try:
            yield
        finally:
            self.stack.pop()
            e.record()
            self.events[full].append((s, e))

    def summary(self) -> dict:
        torch.cuda.synchronize(self.device)
        out = {}
        for name, pairs in self.events.items():
            out[name] = {"ms": sum(s.elapsed_time(e) for s, e in pairs), "calls": len(pairs)}
        return dict(sorted(out.items(), key=lambda kv: -kv[1]["ms"]))

    def reset(self):
        self.events.clear()
