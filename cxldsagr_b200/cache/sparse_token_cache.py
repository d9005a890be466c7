"""Per-(session, layer) KV view: resident storage or a shared pool + host backing.

Transactions (reference: ``cache/sparse_token_cache.py:33-981``):

* ``begin_step(n)`` opens a step of n new tokens; ``append`` writes their
  records; ``commit`` makes them history; ``rollback`` truncates back;
* ``begin_transient(n)`` opens a candidate step whose records live only in the
  pool's GPU tail rows ``[P+1, P+1+C)`` (no host pages, never committed);
  ``discard_transient`` drops them and leaves history unchanged;
* ``ensure(ids)`` maps logical selections [Q, K] to physical rows of
  ``records`` recalling exact misses from host DRAM (free slots first, then
  FIFO victims that are not part of this selection); ``WorkingSetTooLarge``
  asks the caller to split the query batch.

The resident mode keeps logical row i at physical row i.
"""

from __future__ import annotations

from dataclasses import dataclass, asdict

import torch

from ..ops.reference import fp8_record_bytes
from .sparse_token_pool import MISSING, PAGE_SIZE, SharedSparseTokenPool, SparseTokenSession, _device


class WorkingSetTooLarge(ValueError):
    """The exact selection union exceeds the pool; split the query batch."""


@dataclass
class CacheStats:
    written_records: int = 0
    transient_written_records: int = 0
    recalled_records: int = 0
    prefetched_records: int = 0
    evicted_records: int = 0
    max_working_set: int = 0
    capacity_splits: int = 0
    selection_records: int = 0
    resident_selection_records: int = 0
    host_to_device_bytes: int = 0
    device_to_host_bytes: int = 0


# Device counters of a cache (accumulated by the pool kernels / tensor ops, no host sync):
_SELECTED, _RESIDENT, _EVICTED, _RECALLED, _PREFETCHED = 0, 1, 2, 3, 5


class SparseTokenCache:
    def __init__(self, capacity: int, width: int, *, device="cuda", dtype=torch.bfloat16,
                 slots: int | None = None, candidate_slots: int = 0, kv_format: str = "bf16",
                 latent_dim: int | None = None):
        """Standalone cache: resident (``slots`` None) or a private pool of ``slots`` rows.

        ``kv_format="fp8"``: rows are FP8-quantized once on write (the resident
        rows hold the dequantized values, a pool's host arena the 656-byte records)."""
        if capacity < 1 or width < 1:
            raise ValueError("capacity and width must be positive")
        self._init_stats(device)
        if slots is not None:
            host = ((capacity + PAGE_SIZE - 1) // PAGE_SIZE) * PAGE_SIZE
            pool = SharedSparseTokenPool(host, width, 1, slots, device=device, dtype=dtype,
                                         candidate_slots=candidate_slots, kv_format=kv_format, latent_dim=latent_dim)
            session = pool.allocate_session(capacity)
            self._bind(session, 0)
            session._layers[0] = self
            return
        if kv_format not in ("bf16", "fp8"):
            raise ValueError("kv_format must be 'bf16' or 'fp8'")
        self.kv_format = kv_format
        self.latent_dim = SharedSparseTokenPool._split(width, latent_dim)[0] if kv_format == "fp8" else None
        self._pool = None
        self.session = None
        self.layer_id = 0
        self.capacity, self.width = capacity, width
        self.device = _device(device)
        self.offload = False
        self.slots = capacity
        self.candidate_slots = candidate_slots
        self.records = torch.zeros((capacity + candidate_slots, width), dtype=dtype, device=self.device)
        self.length = self.written = 0
        self._step_end = None
        self.transient_start = None

    @classmethod
    def shared(cls, session: SparseTokenSession, layer: int) -> "SparseTokenCache":
        self = object.__new__(cls)
        self._init_stats(session.pool.device)
        self._bind(session, layer)
        return self

    def _init_stats(self, device):
        self._stats = CacheStats()
        self._dev = torch.zeros(8, dtype=torch.int64, device=_device(device))
        self._scratch = torch.zeros(8, dtype=torch.int64, device=_device(device))

    @property
    def stats(self) -> CacheStats:
        """Counters (device-counted fields are read back here, which synchronises)."""
        d = self._dev.tolist()
        st = self._stats
        st.selection_records, st.resident_selection_records = d[_SELECTED], d[_RESIDENT]
        st.evicted_records, st.recalled_records, st.prefetched_records = d[_EVICTED], d[_RECALLED], d[_PREFETCHED]
        st.host_to_device_bytes = (d[_RECALLED] + d[_PREFETCHED]) * self.record_bytes
        return st

    @property
    def native(self) -> bool:
        """Pool metadata handled by the device kernels (CUDA pools)."""
        return self._pool is not None and self.device.type == "cuda"

    def _bind(self, session, layer):
        pool = session.pool
        self._pool, self.session, self.layer_id = pool, session, layer
        self.kv_format, self.latent_dim = pool.kv_format, pool.latent_dim
        self.capacity, self.width, self.slots = session.capacity, pool.width, pool.slots
        self.candidate_slots = pool.candidate_slots
        self.device, self.offload = pool.device, True
        self.records = pool.layers[layer].records
        self.length = self.written = 0
        self._step_end = None
        self.transient_start = None

    # ---------------------------------------------------------------- helpers
    @property
    def record_bytes(self) -> int:
        """Bytes of one record as it crosses PCIe (656 for FP8 records)."""
        if self.kv_format == "fp8":
            return fp8_record_bytes(self.latent_dim, self.width - self.latent_dim)
        return self.width * self.records.element_size()

    def packed_rows(self, count: int):
        """A fresh [count, record bytes] uint8 buffer for kv_finish's FP8 records (None for BF16 caches)."""
        if self.kv_format != "fp8":
            return None
        return torch.empty((count, self.record_bytes), dtype=torch.uint8, device=self.device)

    # Set by a serving backend for borrowed session caches: raises unless the
    # owning session's own operation is active (see ResourceLifecycle.check_active).
    access_check = None

    def _check(self):
        if self.access_check is not None:
            self.access_check()
        if self._pool is not None:
            self.session._check()

    def operation(self):
        if self._pool is None:
            from contextlib import nullcontext

            return nullcontext()
        return self._pool.operation(self.session, self.layer_id)

    def logical_to_global(self, logical):
        return self.session.logical_to_global(logical)

    @property
    def all_history_resident(self) -> bool:
        if self._pool is None:
            return True
        if self.length == 0:
            return True
        g = self.logical_to_global(torch.arange(self.length, device=self.device))
        return bool((self._pool.layers[self.layer_id].h2d[g] != MISSING).all())

    # ----------------------------------------------------------- transactions
    def begin_step(self, count: int):
        self._check()
        if self._step_end is not None:
            raise RuntimeError("a cache step is already open")
        if count < 1 or self.length + count > self.capacity:
            raise ValueError("step exceeds the session capacity")
        self._step_end = self.length + count

    def begin_transient(self, count: int):
        """Candidate records after the committed history, kept only in GPU tail rows."""
        self._check()
        if self._step_end is not None:
            raise RuntimeError("a cache step is already open")
        if count < 1 or count > self.candidate_slots:
            raise ValueError("candidate step exceeds the transient tail rows")
        if self._pool is not None:
            owner = self._pool._transient_owner.get(self.layer_id)
            if owner is not None and owner != self.session.owner:
                raise RuntimeError("another session owns this layer's candidate rows")
            self._pool._transient_owner[self.layer_id] = self.session.owner
        self.transient_start = self.length
        self._step_end = self.length + count

    def discard_transient(self):
        if self.access_check is not None:
            self.access_check()
        if self.transient_start is None:
            raise RuntimeError("no transient step is open")
        self.written = self.length = self.transient_start
        self.transient_start = None
        self._step_end = None
        if self._pool is not None and self._pool._transient_owner.get(self.layer_id) == self.session.owner:
            del self._pool._transient_owner[self.layer_id]

    def commit(self):
        self._check()
        if self.transient_start is not None:
            raise RuntimeError("transient candidate KV is discarded, not committed")
        if self._step_end is None or self.written != self._step_end:
            raise RuntimeError("cannot commit an incomplete cache step")
        self.length = self.written
        self._step_end = None

    def rollback(self):
        self._check()
        if self.transient_start is not None:
            self.discard_transient()
            return
        if self._step_end is None:
            raise RuntimeError("no open cache step")
        self._step_end = None
        self.truncate(self.length)

    def truncate(self, length: int):
        self._check()
        if self._step_end is not None:
            raise RuntimeError("roll back the open step before truncating")
        if not 0 <= length <= max(self.length, self.written):
            raise ValueError("truncate length must not extend history")
        if self._pool is not None:
            self._pool.drain()
            top = max(self.written, self.length)
            if top > length:
                ids = self.logical_to_global(torch.arange(length, top, device=self.device))
                self._pool.release_ids(self.layer_id, ids)
        self.length = self.written = length

    def reset(self):
        if self._step_end is not None:
            self.rollback()
        self.truncate(0)
        self._stats = CacheStats()
        self._dev.zero_()

    # ----------------------------------------------------------------- append
    def destination_rows(self, count: int) -> torch.Tensor:
        """Physical rows the next ``count`` appended records will occupy (allocating them).

        Lets the projection epilogue write records straight into the pool;
        call :meth:`finish_append` afterwards.
        """
        self._check()
        if self._step_end is None or self.written + count > self._step_end:
            raise ValueError("append exceeds the open step")
        start = self.written
        from .. import ops

        if self._pool is None:
            return ops.arange_cached(start, start + count, device=self.device)
        if self.transient_start is not None:
            first = self.slots + 1 + start - self.transient_start
            return ops.arange_cached(first, first + count, device=self.device)
        if count > self.slots:
            raise WorkingSetTooLarge("new KV batch exceeds the shared pool")
        with self.operation():
            glob = self.logical_to_global(torch.arange(start, start + count, device=self.device))
            pool = self._pool.layers[self.layer_id]
            if self.native:
                from .. import ops

                ops.lib().pool_select(pool.h2d, pool.d2h, pool.priority, pool.meta, pool.mark, pool.miss_list,
                                      pool.victims, self._dev, count, -1, glob, -1)
                return pool.victims[:count].clone()
            chosen = self._pool.available_slots(self.layer_id, glob, count)
            self._dev[_EVICTED] += self._pool.evict(self.layer_id, chosen)
            pool.h2d[glob] = chosen.int()
            pool.d2h[chosen] = glob
            self._pool.stamp(self.layer_id, chosen)
        return chosen

    def finish_append(self, rows: torch.Tensor, packed: torch.Tensor | None = None):
        """Complete an append whose records were written into ``records[rows]``
        (``packed``: their 656-byte FP8 records, required for FP8 caches)."""
        start, count = self.written, rows.numel()
        if self.kv_format == "fp8" and packed is None:
            raise ValueError("an FP8 cache append needs the packed records")
        if self._pool is not None and self.transient_start is None:
            source = packed[:count] if self.kv_format == "fp8" else self.records[rows]
            self._pool.write_host(self.session, self.layer_id, start, source)
            self._stats.device_to_host_bytes += count * self.record_bytes
        if self.transient_start is not None:
            self._stats.transient_written_records += count
        self.written = start + count
        self._stats.written_records += count
        return start

    def append(self, records: torch.Tensor) -> int:
        if records.ndim != 2 or records.shape[1] != self.width or not len(records):
            raise ValueError("invalid appended records")
        rows = self.destination_rows(len(records))
        packed = None
        with self.operation():
            if self.kv_format == "fp8":
                from .. import ops

                records, packed = ops.fp8_kv_records(records.to(self.records.dtype), self.latent_dim)
            self.records[rows] = records.to(self.records.dtype)
        return self.finish_append(rows, packed)

    # ----------------------------------------------------------------- recall
    def ensure(self, indices: torch.Tensor) -> torch.Tensor:
        """Logical ids [Q, K] (-1 = padding) -> physical rows of ``records``.

        Recalls the exact missing union from host memory.  History rows are
        protected from eviction while this selection is being made resident.
        """
        self._check()
        if self._pool is None:
            return torch.where((indices >= 0) & (indices < self.written), indices, -1).int()
        if self.native:
            return self._ensure_native(indices)
        flat = indices.reshape(-1).long()
        uniq = torch.unique(flat[flat >= 0])
        if uniq.numel() and int(uniq[-1]) >= self.written:
            raise ValueError("selection references unwritten records")
        history = uniq if self.transient_start is None else uniq[uniq < self.transient_start]
        if history.numel() > self.slots:
            raise WorkingSetTooLarge(f"{history.numel()} selected records exceed {self.slots} slots")
        self._stats.max_working_set = max(self._stats.max_working_set, int(uniq.numel()))
        pool = self._pool.layers[self.layer_id]
        with self.operation():
            glob = self.logical_to_global(history)
            mapped = pool.h2d[glob]
            missing = glob[mapped == MISSING]
            self._dev[_SELECTED] += int(uniq.numel())
            self._dev[_RESIDENT] += int(uniq.numel() - missing.numel())
            if missing.numel():
                self._pool.wait_host(self.session, self.layer_id)
                chosen = self._pool.available_slots(self.layer_id, glob, missing.numel())
                self._dev[_EVICTED] += self._pool.evict(self.layer_id, chosen)
                from .. import ops

                ops.gather_host_records(pool.host, pool.records, missing, chosen, fp8_scratch=self._pool.fp8_scratch,
                                        latent_dim=self._pool.latent_dim)
                pool.h2d[missing] = chosen.int()
                pool.d2h[chosen] = missing
                self._dev[_RECALLED] += int(missing.numel())
            # One protection event for the whole selection (hits and recalls).
            self._pool.stamp(self.layer_id, pool.h2d[glob].long())
            if self.transient_start is None:
                phys = pool.h2d[self.logical_to_global(indices.clamp_min(0))].long()
            else:
                is_hist = (indices >= 0) & (indices < self.transient_start)
                phys_h = pool.h2d[self.logical_to_global(torch.where(is_hist, indices, 0))].long()
                tail = self.slots + 1 + indices.long() - self.transient_start
                phys = torch.where(is_hist, phys_h, tail)
            return torch.where(indices >= 0, phys, -1).int()

    def prefetch(self, logical: torch.Tensor, limit: int | None = None) -> int:
        """Make a predicted subset of history resident ahead of exact recall.

        Used by the indexer-fused prefetch method: ``logical`` are ids the
        predictor proved to be in the coming top-k.  Returns records copied.
        """
        if self.access_check is not None:
            self.access_check()
        if self._pool is None or not logical.numel():
            return 0
        if self.native:
            return self._prefetch_native(logical, limit)
        logical = torch.unique(logical.long())
        logical = logical[(logical >= 0) & (logical < self.length)]
        if limit is not None:
            logical = logical[:limit]
        pool = self._pool.layers[self.layer_id]
        with self.operation():
            glob = self.logical_to_global(logical)
            missing = glob[pool.h2d[glob] == MISSING]
            if not missing.numel():
                return 0
            if missing.numel() > self.slots:
                missing = missing[: self.slots]
            self._pool.wait_host(self.session, self.layer_id)
            chosen = self._pool.available_slots(self.layer_id, glob, missing.numel())
            self._dev[_EVICTED] += self._pool.evict(self.layer_id, chosen)
            from .. import ops

            ops.gather_host_records(pool.host, pool.records, missing, chosen, fp8_scratch=self._pool.fp8_scratch,
                                        latent_dim=self._pool.latent_dim)
            pool.h2d[missing] = chosen.int()
            pool.d2h[chosen] = missing
            self._pool.stamp(self.layer_id, chosen)
            n = int(missing.numel())
            self._dev[_PREFETCHED] += n
            return n

    # ---------------------------------------------------------- native paths
    def _recall_native(self, ids32: torch.Tensor, hist_end: int, *, k_limit: int, count_slot: int, stats):
        """One device-side event: classify ``ids32`` (stamp hits, list misses), choose
        slots for the misses, copy their host rows in.  No host synchronisation."""
        from .. import ops

        pool = self._pool.layers[self.layer_id]
        # Host rows written by earlier appends must be complete before a slot they
        # still back can be evicted (select) or a row is read back (gather).
        self._pool.wait_host(self.session, self.layer_id)
        # classify -> select -> gather in one native call (csrc/host/recall_dispatch.h).
        ops.lib().pool_recall_dispatch(ids32, hist_end, self.session.page_table, pool.h2d, pool.d2h, pool.priority,
                                       pool.meta, pool.mark, pool.miss_list, pool.victims, stats,
                                       self._dev if stats is self._scratch else stats, k_limit, count_slot,
                                       pool.host, pool.records, self._pool.fp8_scratch)
        return pool

    def _ensure_native(self, indices: torch.Tensor) -> torch.Tensor:
        from .. import ops

        ids = indices.reshape(-1)
        ids32 = ids if ids.dtype == torch.int32 and ids.is_contiguous() else ids.to(torch.int32).contiguous()
        hist_end = self.transient_start if self.transient_start is not None else self.written
        with self.operation():
            pool = self._recall_native(ids32, hist_end, k_limit=-1, count_slot=_RECALLED, stats=self._dev)
            out = torch.empty_like(ids32)
            ops.lib().pool_map(ids32, hist_end, self.slots + 1, self.written, self.session.page_table, pool.h2d, out)
            # The union can only exceed the pool when the selection is larger than it.
            if min(ids32.numel(), hist_end) > self.slots and int(pool.meta[3]):
                raise WorkingSetTooLarge("selected records exceed the device working set")
        return out.view(indices.shape)

    def _prefetch_native(self, logical: torch.Tensor, limit: int | None) -> int:
        ids32 = logical.to(torch.int32).contiguous()
        with self.operation():
            self._recall_native(ids32, self.length, k_limit=-1 if limit is None else int(limit),
                                count_slot=_PREFETCHED, stats=self._scratch)
        return -1   # placed on the device; the count is in the prefetched counter

    # ---------------------------------------------------------- diagnostics
    def metrics(self) -> dict:
        return asdict(self.stats)

    def _state(self) -> dict:
        return {"length": self.length, "written": self.written}

    def _restore(self, st: dict):
        self.length, self.written = st["length"], st["written"]
        self._step_end = None
        self.transient_start = None
