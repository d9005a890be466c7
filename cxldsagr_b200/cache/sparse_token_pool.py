"""Shared per-layer HBM token pools backed by a pinned host-DRAM arena.

Layout per layer (reference semantics: ``cache/sparse_token_pool.py:98-906``):

* ``host``     [NH, W]    pinned DRAM arena, owned by sessions in 64-token pages
  (``kv_format="fp8"``: [NH, 656] uint8, the packed FP8 records);
* ``records``  [P+1+C, W] HBM pool: slot 0 is a never-allocated padding
  sentinel, slots 1..P hold history records, the C tail slots hold a
  session's transient candidate records (no host pages, no maps);
* ``h2d``      [NH] int32  global host id -> physical slot (MISSING = INT32_MAX);
* ``d2h``      [P+1] int64 physical slot -> global host id (MISSING);
* ``priority`` [P+1] int64 FIFO clock stamp of each slot (-1 = free);
  eviction takes the smallest stamp first (oldest insertion / protection).

A layer lease (:meth:`operation`) is exclusive: indexer, append, recall and
attention of one layer of one session run under it.  Host writeback of
appended records runs on a dedicated copy stream with at most
``max_inflight_writes`` outstanding events; readers wait for the writes of
their (session, layer) before touching host rows.  Failed CUDA bookkeeping
poisons the pool (no silent reuse of possibly inconsistent maps).
"""

from __future__ import annotations

from bisect import bisect_right
from collections import deque
from contextlib import contextmanager
from dataclasses import dataclass, field

import torch

from ..ops.reference import fp8_record_bytes
from .host_allocation import allocate_host_tensor, pinned_allocation_bytes, tensor_bytes

PAGE_SIZE = 64
MISSING = torch.iinfo(torch.int32).max


def _device(device) -> torch.device:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


# int64 words of a layer's device metadata: 8 state words + the victim
# selection's scratch (2 snapshot words, 6 spare, 2 x 64 per-block counts).
POOL_META_WORDS = 8 + 8 + 2 * 64


@dataclass
class LayerPool:
    host: torch.Tensor
    records: torch.Tensor
    h2d: torch.Tensor
    d2h: torch.Tensor
    priority: torch.Tensor
    # Device-resident metadata of the native (no host sync) path:
    # meta = [clock, epoch, miss count, overflow, ...; words 8+ are the victim
    # selection's scratch (event snapshot and per-block slot counts)]; mark [NH] epoch marks;
    # miss_list / victims [P+1] scratch of one event.
    meta: torch.Tensor = None
    mark: torch.Tensor = None
    miss_list: torch.Tensor = None
    victims: torch.Tensor = None
    lease_owner: int | None = None

    @property
    def clock(self):
        """The clock as a 0-d tensor (device-resident; reading it as an int synchronises)."""
        return self.meta[0]


@dataclass
class _HostWrite:
    owner: int
    layer: int
    event: object
    source: torch.Tensor


@dataclass(eq=False)
class PoolSnapshot:
    """HBM maps + records of every layer; host / indexer prefixes are not copied."""

    pool_id: int
    topology: int
    layers: list
    sessions: dict
    valid: bool = True
    reason: str = ""


class SharedSparseTokenPool:
    @staticmethod
    def _validate(host_capacity, width, layers, slots, candidate_slots):
        if any(type(x) is not int or x < 1 for x in (host_capacity, width, layers, slots)):
            raise ValueError("host_capacity, width, layers and slots must be positive integers")
        if host_capacity % PAGE_SIZE:
            raise ValueError("host_capacity must be a multiple of 64 tokens")
        if type(candidate_slots) is not int or candidate_slots < 0:
            raise ValueError("candidate_slots must be a nonnegative integer")
        if host_capacity >= MISSING or slots + candidate_slots >= MISSING:
            raise ValueError("pool ids must fit the int32 map domain")

    @classmethod
    def estimate_shared_bytes(cls, host_capacity, width, layers, slots, *, dtype=torch.bfloat16,
                              device="cuda", candidate_slots=0, kv_format="bf16", latent_dim=None) -> dict:
        """Exact persistent bytes of the pool ({"hbm", "dram"}) before allocating it."""
        cls._validate(host_capacity, width, layers, slots, candidate_slots)
        size = torch.empty((), dtype=dtype).element_size()
        fp8_row = fp8_record_bytes(*cls._split(width, latent_dim)) if kv_format == "fp8" else 0
        host_row = fp8_row if kv_format == "fp8" else width * size
        host = host_capacity * host_row
        if torch.device(device).type == "cuda":
            host = pinned_allocation_bytes(host)
        per_layer = ((slots + 1 + candidate_slots) * width * size + host_capacity * 8 + (slots + 1) * 32
                     + POOL_META_WORDS * 8)
        hbm = layers * per_layer + ((slots + 1) * fp8_row if kv_format == "fp8" else 0)  # + one recall scratch
        if torch.device(device).type == "cpu":
            return {"hbm": 0, "dram": hbm + layers * host}
        return {"hbm": hbm, "dram": layers * host}

    @staticmethod
    def _split(width: int, latent_dim: int | None) -> tuple[int, int]:
        """(latent, rope) widths of a KV row (V3.2: 512 + 64)."""
        L = latent_dim if latent_dim is not None else (512 if width == 576 else None)
        if L is None or not 0 < L < width:
            raise ValueError("FP8 records need the latent width of the KV row")
        return L, width - L

    def __init__(self, host_capacity, width, layers, slots, *, device="cuda", dtype=torch.bfloat16,
                 candidate_slots=0, max_inflight_writes=2, kv_format="bf16", latent_dim=None):
        self._validate(host_capacity, width, layers, slots, candidate_slots)
        if kv_format not in ("bf16", "fp8"):
            raise ValueError("kv_format must be 'bf16' or 'fp8'")
        if kv_format == "fp8" and dtype != torch.bfloat16:
            raise ValueError("FP8 records cover BF16 MLA KV rows")
        self.kv_format = kv_format
        self.latent_dim = self._split(width, latent_dim)[0] if kv_format == "fp8" else None
        host_row = fp8_record_bytes(self.latent_dim, width - self.latent_dim) if kv_format == "fp8" else 0
        self.device = _device(device)
        self.host_capacity, self.width, self.num_layers, self.slots = host_capacity, width, layers, slots
        self.candidate_slots = candidate_slots
        self.dtype = dtype
        self.max_inflight_writes = max_inflight_writes
        pin = self.device.type == "cuda"
        self.layers: list[LayerPool] = []
        for _ in range(layers):
            priority = torch.full((slots + 1,), -1, dtype=torch.int64, device=self.device)
            priority[0] = MISSING
            host_shape, host_dtype = ((host_capacity, host_row), torch.uint8) if kv_format == "fp8" else \
                ((host_capacity, width), dtype)
            self.layers.append(LayerPool(
                host=allocate_host_tensor(host_shape, dtype=host_dtype, pin_memory=pin),
                records=torch.zeros((slots + 1 + candidate_slots, width), dtype=dtype, device=self.device),
                h2d=torch.full((host_capacity,), MISSING, dtype=torch.int32, device=self.device),
                d2h=torch.full((slots + 1,), MISSING, dtype=torch.int64, device=self.device),
                priority=priority,
                meta=torch.zeros(POOL_META_WORDS, dtype=torch.int64, device=self.device),
                mark=torch.zeros(host_capacity, dtype=torch.int32, device=self.device),
                miss_list=torch.zeros(slots + 1, dtype=torch.int64, device=self.device),
                victims=torch.zeros(slots + 1, dtype=torch.int64, device=self.device),
            ))
        # FP8 host records cross PCIe into this dense scratch and are dequantized
        # into their slots (one recall event at a time per pool).
        self.fp8_scratch = (torch.zeros((slots + 1, host_row), dtype=torch.uint8, device=self.device)
                            if kv_format == "fp8" else None)
        self._free_pages = list(range(host_capacity // PAGE_SIZE - 1, -1, -1))
        self._sessions: dict[int, SparseTokenSession] = {}
        self._next_owner = 0
        self._topology = 0
        self._active: tuple[int, int] | None = None
        self._transient_owner: dict[int, int] = {}
        self._writes: deque[_HostWrite] = deque()
        self._captured: list[_HostWrite] = []
        self._copy_stream = torch.cuda.Stream(device=self.device) if pin else None
        self._last_stream = None
        self.closed = False
        self.poisoned = False

    # ------------------------------------------------------------ accounting
    @property
    def free_host_pages(self) -> int:
        return len(self._free_pages)

    def shared_bytes(self) -> dict:
        ts = []
        for layer in self.layers:
            ts += [layer.host, layer.records, layer.h2d, layer.d2h, layer.priority, layer.meta, layer.mark,
                   layer.miss_list, layer.victims]
        if self.fp8_scratch is not None:
            ts.append(self.fp8_scratch)
        return tensor_bytes(ts)

    def _check(self):
        if self.closed:
            raise RuntimeError("shared token pool is closed")
        if self.poisoned:
            raise RuntimeError("shared token pool is poisoned after a failure")

    # --------------------------------------------------------------- sessions
    def allocate_session(self, capacity: int) -> "SparseTokenSession":
        self._check()
        if self._active is not None:
            raise RuntimeError("session allocation requires a quiescent pool")
        if type(capacity) is not int or capacity < 1:
            raise ValueError("session capacity must be positive")
        pages = (capacity + PAGE_SIZE - 1) // PAGE_SIZE
        if pages > len(self._free_pages):
            raise ValueError("insufficient host pages for the session capacity")
        chosen = [self._free_pages.pop() for _ in range(pages)]
        owner = self._next_owner
        self._next_owner += 1
        session = SparseTokenSession(self, owner, capacity, chosen)
        self._sessions[owner] = session
        self._topology += 1
        return session

    acquire_session = allocate_session

    def release_session(self, session: "SparseTokenSession"):
        session._check()
        if self._active is not None:
            raise RuntimeError("session release requires a quiescent pool")
        self.drain()
        ids = session.global_ids()
        for layer in range(self.num_layers):
            self.release_ids(layer, ids)
            if self._transient_owner.get(layer) == session.owner:
                del self._transient_owner[layer]
        self._free_pages.extend(reversed(session.pages))
        del self._sessions[session.owner]
        session.released = True
        self._topology += 1

    # ----------------------------------------------------------------- leases
    @contextmanager
    def operation(self, session: "SparseTokenSession", layer: int):
        """Exclusive lease of one layer's shared pool state for one session."""
        session._check()
        ident = (session.owner, layer)
        owner = self._transient_owner.get(layer)
        if owner is not None and owner != session.owner:
            raise RuntimeError("another session owns this layer's transient candidate rows")
        if self._active is not None and self._active != ident:
            raise RuntimeError("the shared pool workspace is leased by another layer call")
        outer = self._active is None
        if outer:
            self._wait_previous()
            self.layers[layer].lease_owner = session.owner
            self._active = ident
        try:
            yield
        finally:
            if outer:
                if self.device.type == "cuda":
                    self._last_stream = torch.cuda.current_stream(self.device)
                self._active = None

    def _wait_previous(self):
        if self.device.type != "cuda" or self._last_stream is None:
            return
        current = torch.cuda.current_stream(self.device)
        if current != self._last_stream:
            current.wait_stream(self._last_stream)

    # ------------------------------------------------------------- host writes
    def _reap(self, make_room=False):
        while self._writes:
            ticket = self._writes[0]
            if make_room and len(self._writes) >= self.max_inflight_writes:
                ticket.event.synchronize()
            elif not ticket.event.query():
                break
            self._writes.popleft()

    def write_host(self, session, layer: int, start: int, source: torch.Tensor):
        """Copy appended records (logical rows start..) into the session's host pages."""
        host = self.layers[layer].host
        if self.device.type == "cpu":
            for lo, n, hstart in session.host_runs(start, len(source)):
                host[hstart:hstart + n].copy_(source[lo:lo + n])
            return
        capturing = torch.cuda.is_current_stream_capturing()
        if not capturing:
            self._reap(make_room=True)
        stream = torch.cuda.current_stream(self.device)
        self._copy_stream.wait_stream(stream)
        with torch.cuda.stream(self._copy_stream):
            for lo, n, hstart in session.host_runs(start, len(source)):
                host[hstart:hstart + n].copy_(source[lo:lo + n], non_blocking=True)
            event = torch.cuda.Event()
            event.record(self._copy_stream)
        if capturing:
            # Inside a CUDA graph the copy is a graph node; the graph joins it back
            # (join_writes) and the source lives in the graph's private pool.
            self._captured.append(_HostWrite(session.owner, layer, event, source))
            return
        source.record_stream(self._copy_stream)
        self._writes.append(_HostWrite(session.owner, layer, event, source))

    def join_writes(self):
        """Make the current stream wait for every host write issued so far (no host sync)."""
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).wait_stream(self._copy_stream)

    def end_capture(self):
        """Forget the host-write tickets recorded inside a graph capture."""
        self._captured.clear()

    def wait_host(self, session, layer: int):
        """Make the current stream wait for this (session, layer)'s pending host writes."""
        if self.device.type != "cuda":
            return
        stream = torch.cuda.current_stream(self.device)
        if torch.cuda.is_current_stream_capturing():
            for t in self._captured:
                if t.owner == session.owner and t.layer == layer:
                    stream.wait_event(t.event)
            return
        self._reap()
        for t in self._writes:
            if t.owner == session.owner and t.layer == layer:
                stream.wait_event(t.event)

    def drain(self):
        try:
            if self.device.type == "cuda":
                if self._last_stream is not None:
                    self._last_stream.synchronize()
                for t in self._writes:
                    t.event.synchronize()
                self._copy_stream.synchronize()
            self._writes.clear()
        except BaseException:
            self.poisoned = True
            raise

    # ------------------------------------------------------------- FIFO clock
    def stamp(self, layer: int, physical: torch.Tensor):
        """One FIFO event: stamp ``physical`` slots with the current clock value."""
        pool = self.layers[layer]
        if physical.numel():
            pool.priority[physical.long()] = pool.meta[0]
        pool.meta[0] += 1
        pool.priority[0] = MISSING

    def release_ids(self, layer: int, global_ids: torch.Tensor):
        pool = self.layers[layer]
        phys = pool.h2d[global_ids.long()].long()
        phys = phys[phys != MISSING]
        pool.h2d[global_ids.long()] = MISSING
        if phys.numel():
            pool.d2h[phys] = MISSING
            pool.priority[phys] = -1

    def available_slots(self, layer: int, protected_global: torch.Tensor, count: int) -> torch.Tensor:
        """``count`` slots to (re)use: free first, then the oldest stamps, never a
        slot that holds one of ``protected_global`` or the sentinel."""
        if count == 0:
            return torch.empty(0, dtype=torch.int64, device=self.device)
        pool = self.layers[layer]
        keep = torch.zeros(self.slots + 1, dtype=torch.bool, device=self.device)
        keep[0] = True
        if protected_global.numel():
            mapped = pool.h2d[protected_global.long()].long()
            keep[mapped[mapped != MISSING]] = True
        rank = torch.where(pool.d2h == MISSING, torch.full_like(pool.priority, -2), pool.priority)
        rank = rank.masked_fill(keep, torch.iinfo(torch.int64).max)
        order = torch.argsort(rank, stable=True)[:count]
        if bool((rank[order] == torch.iinfo(torch.int64).max).any()):
            from .sparse_token_cache import WorkingSetTooLarge

            raise WorkingSetTooLarge("protected records exceed the device working set")
        return order

    def evict(self, layer: int, slots: torch.Tensor) -> int:
        pool = self.layers[layer]
        old = pool.d2h[slots]
        valid = old != MISSING
        if bool(valid.any()):
            pool.h2d[old[valid]] = MISSING
        pool.d2h[slots] = MISSING
        pool.priority[slots] = -1
        return int(valid.sum())

    # -------------------------------------------------------- snapshot/restore
    def snapshot(self) -> PoolSnapshot:
        self._check()
        if self._active is not None:
            raise RuntimeError("snapshot requires a quiescent pool")
        self.drain()
        layers = [
            {"records": l.records.clone(), "h2d": l.h2d.clone(), "d2h": l.d2h.clone(),
             "priority": l.priority.clone(), "meta": l.meta.clone()}
            for l in self.layers
        ]
        sessions = {o: [s.layer(i)._state() for i in range(self.num_layers)] for o, s in self._sessions.items()}
        return PoolSnapshot(id(self), self._topology, layers, sessions)

    def restore(self, snap: PoolSnapshot):
        self._check()
        if snap.pool_id != id(self) or snap.topology != self._topology:
            raise ValueError("snapshot belongs to another pool or session set")
        if not snap.valid:
            raise ValueError(snap.reason)
        self.drain()
        for layer, state in zip(self.layers, snap.layers):
            for name in ("records", "h2d", "d2h", "priority", "meta"):
                getattr(layer, name).copy_(state[name])
        for owner, states in snap.sessions.items():
            for i, st in enumerate(states):
                self._sessions[owner].layer(i)._restore(st)

    snapshot_prefix, restore_prefix = snapshot, restore

    def close(self):
        if self.closed:
            return
        self.drain()
        for s in list(self._sessions.values()):
            self.release_session(s)
        self.layers.clear()
        self.closed = True


class SparseTokenSession:
    """One user's host pages (64 tokens each) and its per-layer cache views."""

    def __init__(self, pool: SharedSparseTokenPool, owner: int, capacity: int, pages: list[int]):
        self.pool, self.owner, self.capacity = pool, owner, capacity
        self.pages = pages
        self.page_table = torch.tensor(pages, dtype=torch.int32, device=pool.device)
        runs = []
        for lp, hp in enumerate(pages):
            start = lp * PAGE_SIZE
            if runs and runs[-1][2] + (start - runs[-1][0]) == hp * PAGE_SIZE:
                runs[-1] = (runs[-1][0], start + PAGE_SIZE, runs[-1][2])
            else:
                runs.append((start, start + PAGE_SIZE, hp * PAGE_SIZE))
        self._runs = runs
        self._run_ends = [r[1] for r in runs]
        self._layers: dict = {}
        self.released = False

    def _check(self):
        self.pool._check()
        if self.released or self.pool._sessions.get(self.owner) is not self:
            raise RuntimeError("session was released or is stale")

    def host_runs(self, start: int, count: int):
        """Yield (offset in source, rows, host row start) covering logical [start, start+count)."""
        pos, done = start, 0
        run = bisect_right(self._run_ends, pos)
        while done < count:
            lo, hi, hstart = self._runs[run]
            n = min(hi - pos, count - done)
            yield done, n, hstart + pos - lo
            pos += n
            done += n
            run += 1

    def logical_to_global(self, logical: torch.Tensor) -> torch.Tensor:
        logical = logical.long()
        return self.page_table[logical // PAGE_SIZE].long() * PAGE_SIZE + logical % PAGE_SIZE

    def global_ids(self) -> torch.Tensor:
        local = torch.arange(len(self.pages) * PAGE_SIZE, device=self.pool.device)
        return self.logical_to_global(local)

    def layer(self, index: int):
        self._check()
        if index not in self._layers:
            from .sparse_token_cache import SparseTokenCache

            self._layers[index] = SparseTokenCache.shared(self, index)
        return self._layers[index]

    def release(self):
        self.pool.release_session(self)

    def session_bytes(self) -> dict:
        return tensor_bytes([self.page_table])
