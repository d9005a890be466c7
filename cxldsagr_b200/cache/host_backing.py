"""Host-backed record cache: device working rows + a pinned DRAM backing copy.

Reference: ``cache/host_backing.py:13-233``.  Appended records are written to
the device rows and copied to pinned host memory on a side copy stream; the
host copy is the durable one.  ``commit`` records the new length only after
the writeback of the step was enqueued (the device copy may be evicted
later); ``ensure_resident`` copies a range back (copy engine) when the device
rows were reused.  Write-back completion is tracked by CUDA events, and a
reader must call :meth:`wait_writeback` before touching host rows.
"""

from __future__ import annotations

import torch

from .host_allocation import allocate_host_tensor


class HostBackingCache:
    def __init__(self, capacity: int, width: int, *, device="cuda", dtype=torch.bfloat16, device_rows=None):
        self.device = torch.device(device)
        self.capacity = capacity
        pin = self.device.type == "cuda"
        self.host = allocate_host_tensor((capacity, width), dtype=dtype, pin_memory=pin)
        self.rows = device_rows or capacity
        self.device_records = torch.zeros((self.rows, width), dtype=dtype, device=self.device)
        self.resident_start = 0  # logical row held at device row 0
        self.length = 0
        self._pending = None
        self._stream = torch.cuda.Stream(device=self.device) if pin else None
        self._events = []

    def begin(self, count):
        if self._pending is not None or self.length + count > self.capacity:
            raise ValueError("invalid host-backed step")
        self._pending = (self.length, self.length + count)

    def append(self, records: torch.Tensor):
        s, e = self._pending
        if records.shape[0] != e - s:
            raise ValueError("records must fill the open step")
        # device rows hold a sliding window of the most recent `rows` records
        if e - self.resident_start > self.rows:
            self.resident_start = max(0, e - self.rows)
        lo = s - self.resident_start
        if lo >= 0:
            self.device_records[lo:lo + records.shape[0]] = records
        if self._stream is None:
            self.host[s:e] = records.to(self.host.dtype)
            return
        self._stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self._stream):
            self.host[s:e].copy_(records, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self._stream)
        records.record_stream(self._stream)
        self._events.append(ev)

    def wait_writeback(self):
        if self._stream is not None:
            cur = torch.cuda.current_stream(self.device)
            for ev in self._events:
                cur.wait_event(ev)
            self._events.clear()

    def commit(self):
        self.length = self._pending[1]
        self._pending = None

    def rollback(self):
        self._pending = None

    def ensure_resident(self, start: int, end: int) -> torch.Tensor:
        """Device view of logical rows [start, end), recalling from host if needed."""
        if end - start > self.rows:
            raise ValueError("range exceeds the device working rows")
        if not (self.resident_start <= start and end <= self.resident_start + self.rows):
            self.wait_writeback()
            self.resident_start = start
            self.device_records[: end - start].copy_(self.host[start:end], non_blocking=True)
        return self.device_records[start - self.resident_start:end - self.resident_start]

    def drain(self):
        if self._stream is not None:
            self._stream.synchronize()
        self._events.clear()
