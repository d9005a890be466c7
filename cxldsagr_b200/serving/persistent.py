"""Serial GR service with bounded cross-request prefix reuse.

Reference semantics (``serving/persistent.py:56-319``).  One request runs at
a time; only each user's stable history survives between requests:

1. validate the request (user id, token ids, stable prefix length) and pack
   the ids once (the prefix digest is the history identity);
2. admit the user through the LRU :class:`PrefixSessionPool` (hit: reuse the
   retained session; miss: evict least-recently-used users until the new
   reservation fits, then prefill the prefix);
3. run the candidate suffix (GPU-transient tails) and restore the session to
   its history;
4. report latency split into admission / prefix / extend / cleanup plus the
   cache ledger.

Latency covers input validation and transfer, admission and eviction, prefix
construction on a miss, all candidate hidden states and the rollback.  Any
failure discards the user's session (never reused after a failure).  Omitting
both byte budgets selects fixed-pool admission (host pages / HBM tokens).
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


class PersistentGRRunner:
    def __init__(self, backend: ServingBackend, *, hbm_budget_bytes: int | None = None,
                 dram_budget_bytes: int | None = None, resource_limits: Mapping[str, int] | None = None,
                 native_token_validation: bool = False):
        self.backend = backend
        self.pool: PrefixSessionPool | None = None
        self.closed = True
        self._owner_bound = False
        self._closed_fully = False
        self._rollback_on_close = False
        if (hbm_budget_bytes is None) != (dram_budget_bytes is None):
            raise ValueError("provide both cache byte budgets or omit both for fixed pools")
        budget = None if hbm_budget_bytes is None else CacheFootprint(hbm_budget_bytes, dram_budget_bytes)
        self.resource_mode = "fixed_pools" if budget is None else "budget"
        limits = {"max_seq_len": backend.max_seq_len, "max_session_capacity": backend.max_seq_len,
                  **(resource_limits or {})}
        if any(type(v) is not int or v <= 0 for v in limits.values()):
            raise ValueError("resource limits must be positive integers")
        self.resource_limits = limits
        policy = CapacityPolicy.fixed_pools() if budget is None else CapacityPolicy.byte_budget(budget)
        self.runtime = TokenRuntime(backend.runtime_driver(policy))
        self.driver = self.runtime.driver
        self.resource_plan = self.runtime.plan_resources(policy, limits)
        plan = self.resource_plan
        if budget is not None and not plan.shared.fits(budget):
            raise CacheBudgetExceeded(f"shared cache requires {plan.shared}, exceeds cache budget {budget}")
        if budget is None:
            if plan.host_pages == plan.hbm_tokens == 0:
                raise ValueError("fixed-pools admission requires a shared backend with host pages or HBM tokens")
            pages, tokens = self.driver.maximum_session_quota(plan)
            if pages == tokens == 0:
                raise ValueError("fixed-pools admission requires positive session host pages or HBM tokens")
            if pages > plan.host_pages:
                raise CacheBudgetExceeded("fixed host arena cannot hold one maximum-size session")
            if tokens > plan.hbm_tokens:
                raise CacheBudgetExceeded("fixed HBM pool cannot hold one maximum-size session")
        self.token_validation_identity = {"backend": "python_reference", "fallback_reason": None,
                                          "requested_native": native_token_validation}
        self._valid_ids = token_validation.reference
        if native_token_validation:
            self._valid_ids = token_validation.prepare()
            self.token_validation_identity.update(token_validation.runtime_info())
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
        except BaseException as init_error:
            try:
                self._close(rollback=True)
            except BaseException as cleanup_error:  # noqa: BLE001 - keep both failures
                raise BaseExceptionGroup("runner initialization cleanup failed; ownership retained",
                                         [init_error, cleanup_error]) from None
            raise
        self.visits: Counter = Counter()
        self.closed = False

    # --------------------------------------------------------------- request
    def _validate(self, request: Mapping):
        uid = request["user_id"]
        if isinstance(uid, bool) or not isinstance(uid, (str, int)):
            raise TypeError("user_id must be an integer or string")
        ids = request["input_ids"]
        if not isinstance(ids, (list, tuple)) or not ids:
            raise ValueError("input_ids must be a nonempty integer list")
        ids = list(ids)
        if not self._valid_ids(ids):
            raise ValueError("input_ids must contain nonnegative integers")
        prefix = request["stable_prefix_tokens"]
        if type(prefix) is not int or not 0 < prefix < len(ids):
            raise ValueError("stable_prefix_tokens must leave a nonempty suffix")
        self.resource_plan.limits.validate(RequestShape(prefix, len(ids) - prefix))
        return uid, ids, prefix

    def execute(self, request: Mapping) -> ServingResult:
        if self.closed:
            raise RuntimeError("runner has been closed")
        self.backend.synchronize()
        t0 = time.perf_counter()
        uid, raw, prefix = self._validate(request)
        signature, cpu_ids = _pack(raw, prefix)
        ids = cpu_ids.to(device=self.backend.device)
        del cpu_ids
        plan = self.runtime.plan_session(RequestShape(prefix, len(raw) - prefix), signature)
        lease = self.pool.acquire(uid, signature, plan.retained_capacity, plan.reservation,
                                  host_pages=plan.host_pages, hbm_tokens=plan.hbm_tokens, plan=plan)
        session = lease.session
        stamps = {}
        try:
            self.backend.synchronize()
            t_admit = time.perf_counter()
            if not lease.hit:
                self.runtime.prefill(session, ids[:prefix])
                self.backend.synchronize()
                self.pool.mark_ready(uid)
            t_prefix = time.perf_counter()

            def observe(stage):
                if stage == "executed":
                    stamps["extended"] = time.perf_counter()
                    stamps["request_usage"] = self.pool.audit()
                else:
                    stamps["usage"] = self.pool.audit()
                    stamps["finished"] = time.perf_counter()

            result = self.runtime.candidate(session, ids[prefix:], observer=observe)
        except BaseException as exec_error:
            try:
                self.pool.discard(uid)
            except BaseException as cleanup_error:  # noqa: BLE001 - keep both failures
                raise BaseExceptionGroup("request execution and session cleanup failed",
                                         [exec_error, cleanup_error]) from None
            raise
        diagnostics = self.driver.diagnostics(session)   # outside the timed interval
        visit = self.visits[uid]
        self.visits[uid] += 1
        usage = self._usage(stamps["usage"])
        req_usage = self._usage(stamps["request_usage"])
        shared_now = self.pool.shared_bytes()
        budget = self.pool.budget
        metrics = {k: v for k, v in request.items() if k not in ("input_ids", "attention_mask", "prompt")}
        metrics.update(
            scheme=self.backend.scheme, user_id=uid, visit_index=visit, visit_number=visit + 1,
            is_revisit=visit > 0,
            prefix_hit_tier=(("hbm" if self.backend.scheme == "hbm" else "dram") if lease.hit else "miss"),
            prefix_cache_hit=lease.hit, evicted_users=list(lease.evicted),
            latency_ms=(stamps["finished"] - t0) * 1e3, admission_ms=(t_admit - t0) * 1e3,
            prefix_ms=(t_prefix - t_admit) * 1e3, extend_ms=(stamps["extended"] - t_prefix) * 1e3,
            cleanup_ms=(stamps["finished"] - stamps["extended"]) * 1e3,
            stable_prefix_tokens=prefix, candidate_suffix_tokens=len(raw) - prefix,
            resource_mode=self.resource_mode,
            hbm_budget_bytes=None if budget is None else budget.hbm,
            dram_budget_bytes=None if budget is None else budget.dram,
            cache_hbm_bytes=usage.hbm, cache_dram_bytes=usage.dram,
            request_cache_hbm_bytes=req_usage.hbm, request_cache_dram_bytes=req_usage.dram,
            reserved_hbm_bytes=self.pool.reserved.hbm, reserved_dram_bytes=self.pool.reserved.dram,
            shared_cache_hbm_bytes=shared_now.hbm, shared_cache_dram_bytes=shared_now.dram,
            shared_reserved_hbm_bytes=self.pool.shared.hbm, shared_reserved_dram_bytes=self.pool.shared.dram,
            session_reserved_hbm_bytes=self.pool.session_reserved.hbm,
            session_reserved_dram_bytes=self.pool.session_reserved.dram,
            cache_host_pages=self.pool.reserved_host_pages, host_page_capacity=self.pool.host_page_capacity,
            session_host_pages=lease.entry.host_pages, cache_hbm_tokens=self.pool.reserved_hbm_tokens,
            hbm_token_capacity=self.pool.hbm_token_capacity, session_hbm_tokens=lease.entry.hbm_tokens,
            host_page_tokens=self.resource_plan.page_size,
            cache_pool_scope=self.resource_plan.metadata.get("pool_scope", "session"),
            cache_diagnostics=diagnostics, cached_users=len(self.pool),
        )
        return ServingResult(metrics, result.hidden)

    def _usage(self, audit_report) -> CacheFootprint:
        """Measured bytes summed over sessions + shared structures at an audit point."""
        total = self.pool.shared_bytes()
        for entry in self.pool._entries.values():
            used = self.runtime.session_usage(entry.session).bytes
            total = total + used
        return total

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
                raise BaseExceptionGroup("runner body and close both failed", [error, cleanup_error]) from None
            raise
