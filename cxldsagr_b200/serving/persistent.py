"""Serial GR service with bounded cross-request prefix reuse.

The service the reference runs in ``serving/persistent.py`` (one request at
a time; only each user's stable history survives between requests), built
here as a small request pipeline:

* ``_parse``     checks the request (user id, token ids, stable prefix) and
                 packs the ids once; the prefix digest is the history identity;
* ``_admit``     plans the session and leases it from the LRU
                 :class:`PrefixSessionPool` (a hit reuses the retained
                 session; a miss evicts least-recently-used users until the
                 reservation fits);
* ``_prefix``    builds the history on a miss;
* ``_candidates`` runs the candidate suffix and cuts the session back to its
                 history, auditing the cache ledger at both ends;
* ``_report``    turns the request's clock marks and ledger into metrics.

A :class:`_Clock` synchronises the device before each mark, so the phases
(admission / prefix / extend / cleanup) are device-complete wall times; the
whole latency covers validation and the host-to-device copy too.  A failure
anywhere in the leased part discards the user's session.  Omitting both byte
budgets selects fixed-pool admission (host pages / HBM tokens).
"""

from __future__ import annotations

import hashlib
import sys
import time
from array import array
from collections import Counter
from collections.abc import Iterable, Iterator, Mapping
from dataclasses import dataclass
from typing import Any

import torch

from ..cache.capacity import CacheBudgetExceeded, CacheFootprint, CapacityPolicy
from ..cache.prefix_pool import PrefixSessionPool
from ..executor.contracts import RequestShape, ServingBackend
from ..executor.runtime import TokenRuntime
from . import token_validation


def token_digest(ids: list) -> str:
    """SHA-256 of the ids as little-endian int64."""
    packed = array("q", ids)
    if sys.byteorder != "little":
        packed.byteswap()
    return hashlib.sha256(packed.tobytes()).hexdigest()


def _pack(ids: list, prefix: int):
    """One private int64 buffer for both the prefix digest and the CPU tensor."""
    packed = array("q", ids)
    if packed.itemsize != 8:
        raise RuntimeError("token encoding requires an eight-byte signed long long")
    if sys.byteorder == "little":
        digest = hashlib.sha256(memoryview(packed)[:prefix]).hexdigest()
    else:
        head = packed[:prefix]
        head.byteswap()
        digest = hashlib.sha256(head).hexdigest()
    return (prefix, digest), torch.frombuffer(packed, dtype=torch.long)


@dataclass
class ServingResult:
    metrics: dict
    hidden: torch.Tensor


@dataclass(frozen=True)
class _Request:
    uid: Any
    ids: list
    prefix: int

    @property
    def shape(self) -> RequestShape:
        return RequestShape(self.prefix, len(self.ids) - self.prefix)


class _Clock:
    """Named perf_counter marks; each mark first waits for the device."""

    def __init__(self, synchronize):
        self._sync = synchronize
        self.marks: dict[str, float] = {}

    def mark(self, name: str, *, sync: bool = True) -> None:
        if sync:
            self._sync()
        self.marks[name] = time.perf_counter()

    def ms(self, begin: str, end: str) -> float:
        return (self.marks[end] - self.marks[begin]) * 1e3


@dataclass
class _Candidates:
    hidden: torch.Tensor
    ledger_during: CacheFootprint | None = None  # measured bytes with the candidate tail present
    ledger_after: CacheFootprint | None = None   # measured bytes after the cut


class PersistentGRRunner:
    def __init__(self, backend: ServingBackend, *, hbm_budget_bytes: int | None = None,
                 dram_budget_bytes: int | None = None, resource_limits: Mapping[str, int] | None = None,
                 native_token_validation: bool = False):
        if (hbm_budget_bytes is None) is not (dram_budget_bytes is None):
            raise ValueError("give both cache byte budgets (HBM and DRAM) or neither (fixed pools)")
        self.backend = backend
        self.pool: PrefixSessionPool | None = None
        self.closed = True
        self._owner_bound = False
        self._closed_fully = False
        self._rollback_on_close = False
        budget = None if hbm_budget_bytes is None else CacheFootprint(hbm_budget_bytes, dram_budget_bytes)
        self.resource_mode = "budget" if budget is not None else "fixed_pools"
        self.resource_limits = self._limits(backend, resource_limits)
        policy = CapacityPolicy.byte_budget(budget) if budget is not None else CapacityPolicy.fixed_pools()
        self.runtime = TokenRuntime(backend.runtime_driver(policy))
        self.driver = self.runtime.driver
        self.resource_plan = self.runtime.plan_resources(policy, self.resource_limits)
        self._check_plan(self.resource_plan, budget)
        self._valid_ids = token_validation.prepare() if native_token_validation else token_validation.reference
        self.token_validation_identity = {"backend": "python_reference", "fallback_reason": None,
                                          "requested_native": native_token_validation}
        if native_token_validation:
            self.token_validation_identity.update(token_validation.runtime_info())
        self._open(budget)
        self.visits: Counter = Counter()
        self.closed = False

    # ------------------------------------------------------------ set-up
    @staticmethod
    def _limits(backend, extra: Mapping[str, int] | None) -> dict:
        limits = {"max_seq_len": backend.max_seq_len, "max_session_capacity": backend.max_seq_len}
        limits.update(extra or {})
        bad = {k: v for k, v in limits.items() if type(v) is not int or v <= 0}
        if bad:
            raise ValueError(f"resource limits must be positive integers: {bad}")
        return limits

    def _check_plan(self, plan, budget) -> None:
        if budget is not None:
            if not plan.shared.fits(budget):
                raise CacheBudgetExceeded(f"the shared cache alone needs {plan.shared}; budget is {budget}")
            return
        if plan.host_pages == 0 and plan.hbm_tokens == 0:
            raise ValueError("fixed-pools admission needs a shared backend with host pages or HBM tokens")
        pages, tokens = self.driver.maximum_session_quota(plan)
        if pages == 0 and tokens == 0:
            raise ValueError("fixed-pools admission needs sessions that take host pages or HBM tokens")
        for need, have, what in ((pages, plan.host_pages, "host arena"), (tokens, plan.hbm_tokens, "HBM pool")):
            if need > have:
                raise CacheBudgetExceeded(f"the fixed {what} ({have}) is smaller than one maximum-size session "
                                          f"({need})")

    def _open(self, budget) -> None:
        """Bind ownership, allocate and build the session pool; undo on failure."""
        plan = self.resource_plan
        try:
            self.driver.bind_owner(self)
            self._owner_bound = True
            self.runtime.allocate_resources(plan)
            self.pool = PrefixSessionPool(
                budget, allocate=self.runtime.create_session, release=self.runtime.release_session,
                measure=self.runtime.session_usage, shared=plan.shared,
                measure_shared=lambda: self.runtime.shared_usage().as_mapping(),
                host_page_capacity=plan.host_pages, hbm_token_capacity=plan.hbm_tokens)
            self.pool.audit()
        except BaseException as failure:
            self._undo(failure, "runner set-up failed and so did its cleanup (ownership kept)",
                       lambda: self._close(rollback=True))
            raise

    @staticmethod
    def _undo(failure: BaseException, message: str, cleanup) -> None:
        """Run ``cleanup`` after ``failure``; if it fails too, raise both together."""
        try:
            cleanup()
        except BaseException as second:  # noqa: BLE001 - report both failures
            raise BaseExceptionGroup(message, [failure, second]) from None

    # --------------------------------------------------------- one request
    def _parse(self, request: Mapping) -> _Request:
        uid = request["user_id"]
        if isinstance(uid, bool) or not isinstance(uid, (str, int)):
            raise TypeError(f"user_id must be an int or a str, got {type(uid).__name__}")
        ids = request["input_ids"]
        if not isinstance(ids, (list, tuple)) or len(ids) == 0:
            raise ValueError("input_ids must be a nonempty list of token ids")
        ids = list(ids)
        if not self._valid_ids(ids):
            raise ValueError("input_ids may only hold nonnegative integers")
        prefix = request["stable_prefix_tokens"]
        if type(prefix) is not int or prefix <= 0 or prefix >= len(ids):
            raise ValueError(f"stable_prefix_tokens={prefix!r} must be in [1, {len(ids) - 1}] (nonempty suffix)")
        parsed = _Request(uid, ids, prefix)
        self.resource_plan.limits.validate(parsed.shape)
        return parsed

    def _admit(self, req: _Request, signature):
        plan = self.runtime.plan_session(req.shape, signature)
        return self.pool.acquire(req.uid, signature, plan.retained_capacity, plan.reservation,
                                 host_pages=plan.host_pages, hbm_tokens=plan.hbm_tokens, plan=plan)

    def _prefix(self, lease, req: _Request, ids: torch.Tensor) -> None:
        if lease.hit:
            return
        self.runtime.prefill(lease.session, ids[:req.prefix])
        self.backend.synchronize()
        self.pool.mark_ready(req.uid)

    def _candidates(self, lease, req: _Request, ids: torch.Tensor, clock: _Clock) -> _Candidates:
        out = _Candidates(hidden=None)

        def on_stage(stage):
            # The audit checks every session against its reservation; the
            # ledger is what the caches hold at that point.
            if stage == "executed":
                clock.mark("extended", sync=False)   # the runtime synchronised already
                self.pool.audit()
                out.ledger_during = self._ledger()
            else:
                self.pool.audit()
                out.ledger_after = self._ledger()
                clock.mark("finished", sync=False)

        out.hidden = self.runtime.candidate(lease.session, ids[req.prefix:], observer=on_stage).hidden
        return out

    def execute(self, request: Mapping) -> ServingResult:
        if self.closed:
            raise RuntimeError("this runner is closed")
        clock = _Clock(self.backend.synchronize)
        clock.mark("start")
        req = self._parse(request)
        signature, cpu_ids = _pack(req.ids, req.prefix)
        ids = cpu_ids.to(device=self.backend.device)
        del cpu_ids
        lease = self._admit(req, signature)
        try:
            clock.mark("admitted")
            self._prefix(lease, req, ids)
            clock.mark("prefixed", sync=False)
            done = self._candidates(lease, req, ids, clock)
        except BaseException as failure:
            self._undo(failure, "the request failed and discarding its session failed too",
                       lambda: self.pool.discard(req.uid))
            raise
        return ServingResult(self._report(request, req, lease, clock, done), done.hidden)

    # -------------------------------------------------------------- report
    def _ledger(self) -> CacheFootprint:
        """Measured bytes of the shared structures plus every retained session."""
        total = self.pool.shared_bytes()
        for entry in self.pool._entries.values():
            total = total + self.runtime.session_usage(entry.session).bytes
        return total

    def _report(self, request: Mapping, req: _Request, lease, clock: _Clock, done: _Candidates) -> dict:
        diagnostics = self.driver.diagnostics(lease.session)   # read after the timed part
        visit = self.visits[req.uid]
        self.visits[req.uid] += 1
        pool, plan, budget = self.pool, self.resource_plan, self.pool.budget
        after, during = done.ledger_after, done.ledger_during
        shared = pool.shared_bytes()
        hit_tier = ("hbm" if self.backend.scheme == "hbm" else "dram") if lease.hit else "miss"
        timing = {
            "latency_ms": clock.ms("start", "finished"), "admission_ms": clock.ms("start", "admitted"),
            "prefix_ms": clock.ms("admitted", "prefixed"), "extend_ms": clock.ms("prefixed", "extended"),
            "cleanup_ms": clock.ms("extended", "finished"),
        }
        visit_info = {
            "scheme": self.backend.scheme, "user_id": req.uid, "visit_index": visit, "visit_number": visit + 1,
            "is_revisit": visit > 0, "prefix_hit_tier": hit_tier, "prefix_cache_hit": lease.hit,
            "evicted_users": list(lease.evicted), "stable_prefix_tokens": req.prefix,
            "candidate_suffix_tokens": len(req.ids) - req.prefix,
        }
        ledger = {
            "resource_mode": self.resource_mode,
            "hbm_budget_bytes": budget.hbm if budget is not None else None,
            "dram_budget_bytes": budget.dram if budget is not None else None,
            "cache_hbm_bytes": after.hbm, "cache_dram_bytes": after.dram,
            "request_cache_hbm_bytes": during.hbm, "request_cache_dram_bytes": during.dram,
            "reserved_hbm_bytes": pool.reserved.hbm, "reserved_dram_bytes": pool.reserved.dram,
            "shared_cache_hbm_bytes": shared.hbm, "shared_cache_dram_bytes": shared.dram,
            "shared_reserved_hbm_bytes": pool.shared.hbm, "shared_reserved_dram_bytes": pool.shared.dram,
            "session_reserved_hbm_bytes": pool.session_reserved.hbm,
            "session_reserved_dram_bytes": pool.session_reserved.dram,
            "cache_host_pages": pool.reserved_host_pages, "host_page_capacity": pool.host_page_capacity,
            "session_host_pages": lease.entry.host_pages, "cache_hbm_tokens": pool.reserved_hbm_tokens,
            "hbm_token_capacity": pool.hbm_token_capacity, "session_hbm_tokens": lease.entry.hbm_tokens,
            "host_page_tokens": plan.page_size, "cache_pool_scope": plan.metadata.get("pool_scope", "session"),
            "cache_diagnostics": diagnostics, "cached_users": len(pool),
        }
        passthrough = {k: v for k, v in request.items() if k not in ("input_ids", "attention_mask", "prompt")}
        return {**passthrough, **visit_info, **timing, **ledger}

    def run(self, requests: Iterable[Mapping]) -> Iterator[ServingResult]:
        for request in requests:
            yield self.execute(request)

    # ---------------------------------------------------------------- close
    def _close(self, *, rollback=False):
        if self._closed_fully:
            return
        self.closed = True
        self._rollback_on_close |= rollback
        if self.pool is not None:
            self.pool.close()
        if self._owner_bound:
            self.driver.unbind_owner(self, rollback=self._rollback_on_close)
            self._owner_bound = False
        self.runtime.retire()
        self._closed_fully = True

    def close(self):
        self._close()

    def __enter__(self):
        return self

    def __exit__(self, exc_type, error, tb):
        try:
            self.close()
        except BaseException as cleanup_error:
            if error is not None:
                raise BaseExceptionGroup("the runner body and its close both failed", [error, cleanup_error]) \
                    from None
            raise
