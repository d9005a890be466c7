"""Double-buffered staging of whole-layer history (dense prefetch method).

Reference: ``cache/staging.py:49-376``.  Two device buffers alternate between
layers: while layer l computes from buffer l % 2, the copy engine fills
buffer (l + 1) % 2 with layer l+1's history from pinned host memory.  A
lease hands out a buffer; ``prefetch`` enqueues the host->device copy on
the staging stream and records a ready event; ``wait_ready`` makes the
compute stream wait for it (no host synchronisation).

FP8 records (``fp8_records=True``): the host arena holds 656-byte records;
the copy engine fills a packed staging buffer and ``wait_ready`` dequantizes
the staged rows into the BF16 buffer on the compute stream.
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

    def _target(self) -> torch.Tensor:
        st = self.staging
        return st.packed[self.index] if st.packed is not None else st.buffers[self.index]

    def prefetch(self, host: torch.Tensor, rows: int):
        st = self.staging
        if rows > st.buffers[self.index].shape[0]:
            raise ValueError("history exceeds the staging buffer")
        self.rows = rows
        target = self._target()
        if st.stream is None:
            target[:rows].copy_(host[:rows])
            return self
        st.order_after_use(self.index)
        with torch.cuda.stream(st.stream):
            target[:rows].copy_(host[:rows], non_blocking=True)
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
        buf = self._target()
        if st.stream is None:
            for lo, n, h in runs:
                buf[lo:lo + n].copy_(host[h:h + n])
            return self
        st.order_after_use(self.index)
        with torch.cuda.stream(st.stream):
            if before is not None:
                before()
            for lo, n, h in runs:
                buf[lo:lo + n].copy_(host[h:h + n], non_blocking=True)
            self.event = torch.cuda.Event()
            self.event.record(st.stream)
        return self

    def wait_ready(self) -> torch.Tensor:
        st = self.staging
        if self.event is not None:
            torch.cuda.current_stream(st.device).wait_event(self.event)
        if st.packed is not None and self.rows:
            from .. import ops

            ops.dequant_kv_rows(st.packed[self.index], st.buffers[self.index], count=self.rows,
                                latent_dim=st.latent_dim)
        return self.buffer

    def release(self):
        st = self.staging
        if st.stream is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(st.device))
            st.consumed[self.index] = ev


class DoubleBufferStaging:
    def __init__(self, rows: int, width: int, *, device="cuda", dtype=torch.bfloat16, fp8_records: bool = False,
                 latent_dim: int = 512):
        from ..ops.reference import fp8_record_bytes

        self.device = torch.device(device)
        self.latent_dim = latent_dim
        self.buffers = [torch.zeros((rows, width), dtype=dtype, device=self.device) for _ in range(2)]
        rb = fp8_record_bytes(latent_dim, width - latent_dim)
        self.packed = ([torch.zeros((rows, rb), dtype=torch.uint8, device=self.device) for _ in range(2)]
                       if fp8_records else None)
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self.consumed = [None, None]
        self._next = 0

    def order_after_use(self, index: int):
        """Order the staging stream after the last reader of buffer ``index``.

        Eagerly: its consumed event (the layer that used it two steps ago),
        or, with none recorded (first use, or after a capture, whose graph may
        still be reading it), everything enqueued on the compute stream.
        Inside a CUDA-graph capture: the compute stream's work so far, which
        also brings the staging stream into the capture (events recorded
        before the capture cannot be waited on inside it)."""
        cur = torch.cuda.current_stream(self.device)
        if torch.cuda.is_current_stream_capturing() or self.consumed[index] is None:
            self.stream.wait_stream(cur)
        else:
            self.stream.wait_event(self.consumed[index])

    def end_capture(self):
        """Forget the consumed events recorded inside a capture (they never ran eagerly)."""
        self.consumed = [None, None]

    def lease(self) -> StagingLease:
        lease = StagingLease(self, self._next)
        self._next ^= 1
        return lease

    def nbytes(self) -> int:
        return sum(b.numel() * b.element_size() for b in self.buffers + (self.packed or []))
