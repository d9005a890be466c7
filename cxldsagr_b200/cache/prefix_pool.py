"""Per-user LRU retention of prefilled histories under one admission ledger.

Reference semantics (``cache/prefix_pool.py:36-301``): each user key maps to
one cached session; a request for a key whose history signature matches hits
(the prefix is reused); otherwise whole users are evicted least-recently-used
first until the new session's reservation fits.  Admission is checked against
either a byte budget (HBM + DRAM) or fixed pools (host pages and/or HBM
tokens).  A lease stays unpublished until ``mark_ready`` after the prefix is
built; on any failure the caller discards it.  An impossible request never
evicts existing users.
"""

from __future__ import annotations

from collections import OrderedDict
from collections.abc import Callable, Hashable
from dataclasses import dataclass
from typing import Any

from .capacity import CacheBudgetExceeded, CacheFootprint, ResourceUsage, SessionPlan


@dataclass
class PrefixEntry:
    key: Hashable
    signature: Hashable
    session: Any
    capacity: int
    reservation: CacheFootprint
    host_pages: int = 0
    hbm_tokens: int = 0
    ready: bool = False


@dataclass
class PrefixLease:
    entry: PrefixEntry
    hit: bool
    evicted: tuple  # user keys evicted to admit this lease

    @property
    def session(self):
        return self.entry.session


class PrefixSessionPool:
    def __init__(self, budget: CacheFootprint | None, *, allocate: Callable, release: Callable,
                 measure: Callable, shared: CacheFootprint | None = None,
                 measure_shared: Callable | None = None,
                 host_page_capacity: int = 0, hbm_token_capacity: int = 0):
        shared = shared or CacheFootprint()
        if budget is None and host_page_capacity == 0 and hbm_token_capacity == 0:
            raise ValueError("fixed-pool admission needs a host-page or HBM-token capacity")
        if budget is not None and not shared.fits(budget):
            raise CacheBudgetExceeded(f"shared cache {shared} exceeds the cache budget {budget}")
        self.budget, self.shared = budget, shared
        self.host_page_capacity, self.hbm_token_capacity = host_page_capacity, hbm_token_capacity
        self._allocate, self._release, self._measure = allocate, release, measure
        self._measure_shared = measure_shared
        self._entries: "OrderedDict[Hashable, PrefixEntry]" = OrderedDict()
        self.evictions = 0
        self.hits = 0
        self.misses = 0

    # ---------------------------------------------------------- accounting
    def __len__(self):
        return len(self._entries)

    def __contains__(self, key):
        return key in self._entries

    @property
    def session_reserved(self) -> CacheFootprint:
        out = CacheFootprint()
        for e in self._entries.values():
            out = out + e.reservation
        return out

    @property
    def reserved(self) -> CacheFootprint:
        return self.shared + self.session_reserved

    @property
    def reserved_host_pages(self) -> int:
        return sum(e.host_pages for e in self._entries.values())

    @property
    def reserved_hbm_tokens(self) -> int:
        return sum(e.hbm_tokens for e in self._entries.values())

    def _fits(self, reservation, host_pages, hbm_tokens) -> bool:
        if self.budget is not None and not (self.reserved + reservation).fits(self.budget):
            return False
        if self.host_page_capacity and self.reserved_host_pages + host_pages > self.host_page_capacity:
            return False
        if self.hbm_token_capacity and self.reserved_hbm_tokens + hbm_tokens > self.hbm_token_capacity:
            return False
        return True

    # -------------------------------------------------------------- admit
    def discard(self, key: Hashable) -> None:
        entry = self._entries.pop(key, None)
        if entry is not None:
            self._release(entry.session)

    def acquire(self, key: Hashable, signature: Hashable, capacity: int, reservation: CacheFootprint, *,
                host_pages: int = 0, hbm_tokens: int = 0, plan: SessionPlan | None = None) -> PrefixLease:
        if type(capacity) is not int or capacity <= 0:
            raise ValueError("capacity must be a positive integer")
        if plan is not None and (plan.retained_capacity != capacity or plan.history_identity != signature
                                 or plan.reservation != reservation):
            raise ValueError("admission arguments must match the session plan")
        # An impossible request must not destroy reusable state.
        if self.budget is not None and not (self.shared + reservation).fits(self.budget):
            raise CacheBudgetExceeded(f"one session needs {reservation}, the budget is {self.budget}")
        if self.host_page_capacity and host_pages > self.host_page_capacity:
            raise CacheBudgetExceeded("one session exceeds the host page pool")
        if self.hbm_token_capacity and hbm_tokens > self.hbm_token_capacity:
            raise CacheBudgetExceeded("one session exceeds the HBM token pool")
        entry = self._entries.get(key)
        if entry is not None and entry.ready and entry.signature == signature and entry.capacity >= capacity:
            self._entries.move_to_end(key)
            self.hits += 1
            return PrefixLease(entry, True, ())
        if entry is not None:  # stale history for this user
            self.discard(key)
        self.misses += 1
        evicted = []
        while not self._fits(reservation, host_pages, hbm_tokens):
            victim_key = next(iter(self._entries))
            self.discard(victim_key)
            evicted.append(victim_key)
            self.evictions += 1
        session = self._allocate(plan if plan is not None else capacity)
        entry = PrefixEntry(key, signature, session, capacity, reservation, host_pages, hbm_tokens)
        self._entries[key] = entry
        return PrefixLease(entry, False, tuple(evicted))

    def mark_ready(self, lease_or_key):
        """Publish a built prefix (by its lease or its user key)."""
        if isinstance(lease_or_key, PrefixLease):
            entry = lease_or_key.entry
            if self._entries.get(entry.key) is not entry:
                raise RuntimeError("lease was evicted or replaced before it became ready")
        else:
            entry = self._entries.get(lease_or_key)
            if entry is None:
                raise RuntimeError("no pending lease for this user")
        entry.ready = True

    def shared_bytes(self) -> CacheFootprint:
        """Measured bytes of the shared (all-user) cache structures."""
        if self._measure_shared is None:
            return self.shared
        return ResourceUsage.coerce(self._measure_shared()).bytes

    def audit(self) -> dict:
        """Measured per-session usage must stay within each reservation."""
        report = {"sessions": len(self._entries), "reserved": self.reserved, "violations": []}
        for key, e in self._entries.items():
            used = ResourceUsage.coerce(self._measure(e.session))
            if not used.bytes.fits(e.reservation):
                report["violations"].append((key, used.bytes, e.reservation))
        if report["violations"]:
            raise RuntimeError(f"session usage exceeds its reservation: {report['violations']}")
        return report

    def close(self):
        for key in list(self._entries):
            self.discard(key)
