"""Double-buffered staging of whole-layer history (dense prefetch method).

Reference: ``cache/staging.py:49-376``.  Two device buffers alternate between
layers: while layer l computes from buffer l % 2, the copy engine fills
buffer (l + 1) % 2 with layer l+1's history from pinned host memory.  A
lease hands out a buffer; ``prefetch`` enqueues the host->device copy on
the staging stream and records a ready event; ``wait_ready`` makes the
compute stream wait for it (no host synchronisation).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class StagingLease:
    staging: "DoubleBufferStaging"
    index: int
    rows: int = 0
    event: object = None

    @property
    def buffer(self) -> torch.Tensor:
        return self.staging.buffers[self.index][: self.rows]

    def prefetch(self, host: torch.Tensor, rows: int):
        st = self.staging
        if rows > st.buffers[self.index].shape[0]:
            raise ValueError("history exceeds the staging buffer")
        self.rows = rows
        if st.stream is None:
            st.buffers[self.index][:rows].copy_(host[:rows])
            return self
        # The buffer may still be read by the layer that used it two steps ago.
        if st.consumed[self.index] is not None:
            st.stream.wait_event(st.consumed[self.index])
        with torch.cuda.stream(st.stream):
            st.buffers[self.index][:rows].copy_(host[:rows], non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(st.stream)
        return self

    def prefetch_runs(self, host: torch.Tensor, runs, rows: int, *, before=None):
        """Copy host rows into this buffer: ``runs`` yields (buffer row, count, host row).

        ``before`` runs on the staging stream first (e.g. waits for pending
        host writes).  One cudaMemcpyAsync per contiguous run.
        """
        st = self.staging
        if rows > st.buffers[self.index].shape[0]:
            raise ValueError("history exceeds the staging buffer")
        self.rows = rows
        buf = st.buffers[self.index]
        if st.stream is None:
            for lo, n, h in runs:
                buf[lo:lo + n].copy_(host[h:h + n])
            return self
        if st.consumed[self.index] is not None:
            st.stream.wait_event(st.consumed[self.index])
        with torch.cuda.stream(st.stream):
            if before is not None:
                before()
            for lo, n, h in runs:
                buf[lo:lo + n].copy_(host[h:h + n], non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(st.stream)
        return self

    def wait_ready(self) -> torch.Tensor:
        if self.event is not None:
            torch.cuda.current_stream(self.staging.device).wait_event(self.event)
        return self.buffer

    def release(self):
        st = self.staging
        if st.stream is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(st.device))
            st.consumed[self.index] = ev


class DoubleBufferStaging:
    def __init__(self, rows: int, width: int, *, device="cuda", dtype=torch.bfloat16):
        self.device = torch.device(device)
        self.buffers = [torch.zeros((rows, width), dtype=dtype, device=self.device) for _ in range(2)]
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self.consumed = [None, None]
        self._next = 0

    def lease(self) -> StagingLease:
        lease = StagingLease(self, self._next)
        self._next ^= 1
        return lease

    def nbytes(self) -> int:
        return sum(b.numel() * b.element_size() for b in self.buffers)
