"""Model-neutral token runtime over a :class:`ModelDriver`.

Serves the same role as the reference's ``executor/runtime.py`` (request
runtime between a serving loop and one model driver): it owns the lifecycle
of the runtime (planned -> allocated -> closed) and of every session it
created (live -> failed), checks tokens and output contracts around each
driver call, and turns any exception raised inside a driver call into a
failed session that can only be released afterwards.

Candidate execution notifies an optional observer twice: ``"executed"`` once
the candidate's outputs exist (before the session is cut back to its
history) and ``"cleaned"`` after the cut, so callers can time the two parts.
"""

from __future__ import annotations

import enum
from collections.abc import Callable, Hashable, Mapping
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any

import torch

from ..cache.capacity import CapacityPolicy, ResourcePlan, SessionPlan
from .contracts import ExecutionResult, ModelDriver, OutputSpec, RequestShape, StageObserver


class _Stage(enum.Enum):
    NEW = "new"            # no plan yet
    PLANNED = "planned"    # plan_resources done, nothing allocated
    ALLOCATED = "allocated"
    CLOSED = "closed"


@dataclass
class _Entry:
    session: Any
    plan: SessionPlan
    failed: bool = False


def _check_token_tensor(ids: Any, device: torch.device) -> int:
    """Number of tokens in a valid 1-D integral tensor on ``device``."""
    ok_shape = isinstance(ids, torch.Tensor) and ids.ndim == 1 and ids.numel() > 0
    if not ok_shape:
        raise ValueError("token ids: expected a one-dimensional tensor with at least one token")
    if ids.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"token ids: integral dtype required, got {ids.dtype}")
    if ids.device != device:
        raise ValueError(f"token ids live on {ids.device}, the model runs on {device}")
    return ids.numel()


def _check_outputs(result: ExecutionResult, spec: OutputSpec, count: int) -> None:
    """The driver returned what ``spec`` promised for ``count`` tokens."""
    if spec.hidden != "none":
        want = count if spec.hidden == "all" else 1
        h = result.hidden
        if h is None or h.ndim != 2 or h.shape[0] != want:
            raise RuntimeError(f"driver returned hidden states {None if h is None else tuple(h.shape)}, "
                               f"expected {want} rows")
    if spec.logits == "last":
        lg = result.logits
        if lg is None or lg.ndim != 2 or lg.shape[0] != 1:
            raise RuntimeError("driver did not return the last token's logits")
    if result.ownership != spec.ownership:
        raise RuntimeError(f"driver returned {result.ownership} outputs, the spec asked for {spec.ownership}")


class TokenRuntime:
    def __init__(self, driver: ModelDriver):
        self.driver = driver
        self.plan: ResourcePlan | None = None
        self._stage = _Stage.NEW
        self._entries: dict[int, _Entry] = {}

    # ------------------------------------------------------------ lifecycle
    def _expect(self, *stages: _Stage, error: type[Exception], what: str) -> None:
        if self._stage not in stages:
            raise error(f"{what} is not possible while the runtime is {self._stage.value}")

    def plan_resources(self, policy: CapacityPolicy, limits: Mapping[str, int]) -> ResourcePlan:
        self._expect(_Stage.NEW, _Stage.PLANNED, error=RuntimeError, what="planning resources")
        self.plan = self.driver.plan_resources(policy, limits)
        self._stage = _Stage.PLANNED
        return self.plan

    def allocate_resources(self, plan: ResourcePlan) -> None:
        self._expect(_Stage.PLANNED, error=ValueError, what="allocating resources")
        if plan is not self.plan:
            raise ValueError("allocate_resources needs the plan object this runtime produced")
        self.driver.allocate_resources(plan)
        self._stage = _Stage.ALLOCATED

    def plan_session(self, shape: RequestShape, identity: Hashable) -> SessionPlan:
        self._expect(_Stage.ALLOCATED, error=RuntimeError, what="planning a session")
        self.plan.limits.validate(shape)
        return self.driver.plan_session(shape, identity)

    def create_session(self, plan: SessionPlan):
        self._expect(_Stage.ALLOCATED, error=ValueError, what="creating a session")
        if plan.resource_identity is not self.plan:
            raise ValueError("the session plan was made for other resources")
        session = self.driver.create_session(plan)
        self._entries[id(session)] = _Entry(session, plan)
        return session

    def release_session(self, session):
        self._lookup(session, failed_ok=True)
        self.driver.release_session(session)
        del self._entries[id(session)]

    def _finish(self, *, close_driver: bool) -> None:
        if self._entries:
            raise RuntimeError(f"{len(self._entries)} session(s) still open; release them first")
        if close_driver:
            self.driver.close()
        self._stage = _Stage.CLOSED

    def close(self):
        self._finish(close_driver=True)

    def retire(self):
        """End this runtime while the backend keeps its shared allocations."""
        self._finish(close_driver=False)

    # ------------------------------------------------------------- sessions
    def _lookup(self, session, *, failed_ok: bool = False) -> _Entry:
        entry = self._entries.get(id(session))
        if entry is None or entry.session is not session:
            raise ValueError("session unknown to this runtime (foreign or already released)")
        if self._stage is _Stage.CLOSED:
            raise RuntimeError("the runtime is closed")
        if entry.failed and not failed_ok:
            raise RuntimeError("the session failed earlier and can only be released")
        return entry

    def session_failed(self, session) -> bool:
        return self._lookup(session, failed_ok=True).failed

    def session_usage(self, session):
        self._lookup(session, failed_ok=True)
        return self.driver.session_usage(session)

    def shared_usage(self):
        return self.driver.shared_usage()

    @contextmanager
    def _transaction(self, entry: _Entry):
        """Any exception escaping a driver call poisons the session."""
        try:
            yield
        except BaseException:
            entry.failed = True
            raise

    def _spec(self, given: OutputSpec | None, default: OutputSpec, *, prefill: bool = False) -> OutputSpec:
        spec = given or default
        self.driver.validate_output(spec, prefill=prefill)
        return spec

    def _run_checked(self, entry: _Entry, call: Callable[[], ExecutionResult], spec: OutputSpec, count: int,
                     *, committed: int | None, sync: bool) -> ExecutionResult:
        """Run ``call``, then (when ``sync``) synchronise, check its outputs and
        (when ``committed`` is set) the session length it left."""
        with self._transaction(entry):
            with torch.inference_mode():
                result = call()
            if sync:
                self.driver.synchronize()
                _check_outputs(result, spec, count)
            if committed is not None and self.driver.session_length(entry.session) != committed:
                raise RuntimeError(f"driver left {self.driver.session_length(entry.session)} committed tokens, "
                                   f"expected {committed}")
            return result

    # ------------------------------------------------------------ execution
    def prefill(self, session, ids, output_spec: OutputSpec | None = None):
        entry = self._lookup(session)
        n = _check_token_tensor(ids, self.driver.device)
        if self.driver.session_length(session) != 0:
            raise ValueError("prefill needs an empty session")
        if n != entry.plan.history_tokens:
            raise ValueError(f"prefill got {n} tokens, the session was planned for {entry.plan.history_tokens}")
        spec = self._spec(output_spec, self.driver.prefill_output_spec, prefill=True)
        return self._run_checked(entry, lambda: self.driver.prefill(session, ids, spec), spec, n,
                                 committed=n, sync=False)

    def candidate(self, session, ids, output_spec: OutputSpec | None = None, *,
                  observer: StageObserver | None = None):
        entry = self._lookup(session)
        n = _check_token_tensor(ids, self.driver.device)
        history = self.driver.session_length(session)
        if history != entry.plan.history_tokens:
            raise ValueError(f"candidates run on the full planned history ({entry.plan.history_tokens} tokens), "
                             f"the session holds {history}")
        self.plan.limits.validate(RequestShape(history, n))
        if self.driver.candidate_mode == "append_truncate" and history + n > entry.plan.retained_capacity:
            raise ValueError("history + candidates exceed the session's allocated capacity")
        spec = self._spec(output_spec, self.driver.output_spec)
        notify = observer or (lambda stage: None)
        with self._transaction(entry):
            # The observer runs inside the transaction: if it raises, the
            # session (still holding the candidate tail) is poisoned too.
            result = self._run_checked(entry, lambda: self.driver.candidate(session, ids, spec), spec, n,
                                       committed=None, sync=True)
            notify("executed")
            self.driver.finish_candidate(session, history)
            self.driver.synchronize()
            if self.driver.session_length(session) != history:
                raise RuntimeError("the candidate cut did not restore the committed history length")
            notify("cleaned")
        return result

    def append(self, session, ids, output_spec: OutputSpec | None = None):
        entry = self._lookup(session)
        n = _check_token_tensor(ids, self.driver.device)
        before = self.driver.session_length(session)
        if before == 0:
            raise ValueError("append needs a committed prefix (run prefill first)")
        room = min(entry.plan.retained_capacity, self.plan.limits.context_tokens)
        if before + n > room:
            raise ValueError(f"append of {n} tokens to {before} exceeds the session capacity {room}")
        if n > self.plan.limits.candidate_tokens:
            raise ValueError(f"append of {n} tokens exceeds the planned per-call limit "
                             f"{self.plan.limits.candidate_tokens}")
        spec = self._spec(output_spec, self.driver.output_spec)
        return self._run_checked(entry, lambda: self.driver.append(session, ids, spec), spec, n,
                                 committed=before + n, sync=True)
