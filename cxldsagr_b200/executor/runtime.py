"""Model-neutral token runtime over a :class:`ModelDriver`.

Behavioural parity with ``executor/runtime.py:23-195`` of the reference: the
runtime validates tokens, plan identity and session state, checks that the
driver returned the outputs it promised, and marks a session failed on any
exception so that it can never execute again (only be released).  Candidate
execution reports two stages to an optional observer: ``executed`` after the
candidate hidden states are complete and ``cleaned`` after the session was
restored to its history.
"""

from __future__ import annotations

from collections.abc import Hashable, Mapping
from dataclasses import dataclass
from typing import Any

import torch

from ..cache.capacity import CapacityPolicy, ResourcePlan, SessionPlan
from .contracts import ModelDriver, OutputSpec, RequestShape, StageObserver


@dataclass
class _Tracked:
    session: Any
    plan: SessionPlan
    failed: bool = False


class TokenRuntime:
    def __init__(self, driver: ModelDriver):
        self.driver = driver
        self.plan: ResourcePlan | None = None
        self._tracked: dict[int, _Tracked] = {}
        self._allocated = False
        self._closed = False

    # ------------------------------------------------------------ resources
    def plan_resources(self, policy: CapacityPolicy, limits: Mapping[str, int]) -> ResourcePlan:
        if self._closed or self._allocated:
            raise RuntimeError("cannot replan a closed or allocated runtime")
        self.plan = self.driver.plan_resources(policy, limits)
        return self.plan

    def allocate_resources(self, plan: ResourcePlan) -> None:
        if self._closed or plan is not self.plan:
            raise ValueError("resource plan identity does not match this runtime")
        self.driver.allocate_resources(plan)
        self._allocated = True

    # ------------------------------------------------------------- sessions
    def plan_session(self, shape: RequestShape, identity: Hashable) -> SessionPlan:
        if self._closed or not self._allocated:
            raise RuntimeError("allocate resources before planning sessions")
        self.plan.limits.validate(shape)
        return self.driver.plan_session(shape, identity)

    def create_session(self, plan: SessionPlan):
        if self._closed or not self._allocated or plan.resource_identity is not self.plan:
            raise ValueError("session plan belongs to inactive or foreign resources")
        session = self.driver.create_session(plan)
        self._tracked[id(session)] = _Tracked(session, plan)
        return session

    def _state(self, session, *, allow_failed=False) -> _Tracked:
        st = self._tracked.get(id(session))
        if st is None or st.session is not session:
            raise ValueError("foreign or released runtime session")
        if self._closed or (st.failed and not allow_failed):
            raise RuntimeError("runtime session cannot execute after failure or close")
        return st

    def session_failed(self, session) -> bool:
        return self._state(session, allow_failed=True).failed

    def session_usage(self, session):
        self._state(session, allow_failed=True)
        return self.driver.session_usage(session)

    def shared_usage(self):
        return self.driver.shared_usage()

    def _check_tokens(self, ids):
        if not isinstance(ids, torch.Tensor) or ids.ndim != 1 or ids.numel() == 0:
            raise ValueError("tokens must be a nonempty one-dimensional tensor")
        if ids.dtype not in (torch.int32, torch.int64) or ids.device != self.driver.device:
            raise ValueError("tokens must be integral and on the backend device")

    @staticmethod
    def _check_result(result, spec: OutputSpec, count: int):
        if spec.hidden != "none":
            rows = count if spec.hidden == "all" else 1
            h = result.hidden
            if h is None or h.ndim != 2 or h.shape[0] != rows:
                raise RuntimeError("backend must return every selected token's hidden state")
        if spec.logits == "last":
            lg = result.logits
            if lg is None or lg.ndim != 2 or lg.shape[0] != 1:
                raise RuntimeError("backend must return the requested last-token logits")
        if result.ownership != spec.ownership:
            raise RuntimeError("backend output ownership differs from output spec")

    def _guard(self, st: _Tracked, fn):
        try:
            return fn()
        except BaseException:
            st.failed = True
            raise

    # ------------------------------------------------------------ execution
    def prefill(self, session, ids, output_spec: OutputSpec | None = None):
        st = self._state(session)
        self._check_tokens(ids)
        if self.driver.session_length(session) != 0:
            raise ValueError("prefill requires an empty session")
        if ids.numel() != st.plan.history_tokens:
            raise ValueError("prefill must build the planned history")
        spec = output_spec or self.driver.prefill_output_spec
        self.driver.validate_output(spec, prefill=True)

        def run():
            result = self.driver.prefill(session, ids, spec)
            if self.driver.session_length(session) != ids.numel():
                raise RuntimeError("prefill did not commit the complete history")
            return result

        return self._guard(st, run)

    def candidate(self, session, ids, output_spec: OutputSpec | None = None, *,
                  observer: StageObserver | None = None):
        st = self._state(session)
        self._check_tokens(ids)
        history = self.driver.session_length(session)
        if history != st.plan.history_tokens:
            raise ValueError("candidate requires the complete planned history")
        self.plan.limits.validate(RequestShape(history, ids.numel()))
        if self.driver.candidate_mode == "append_truncate" and history + ids.numel() > st.plan.retained_capacity:
            raise ValueError("candidate exceeds session allocation capacity")
        spec = output_spec or self.driver.output_spec
        self.driver.validate_output(spec)

        def run():
            with torch.inference_mode():
                result = self.driver.candidate(session, ids, spec)
            self.driver.synchronize()
            self._check_result(result, spec, ids.numel())
            if observer is not None:
                observer("executed")
            self.driver.finish_candidate(session, history)
            self.driver.synchronize()
            if self.driver.session_length(session) != history:
                raise RuntimeError("candidate changed committed history length")
            if observer is not None:
                observer("cleaned")
            return result

        return self._guard(st, run)

    def append(self, session, ids, output_spec: OutputSpec | None = None):
        st = self._state(session)
        self._check_tokens(ids)
        before = self.driver.session_length(session)
        if before == 0:
            raise ValueError("append requires a committed prefix")
        if before + ids.numel() > min(st.plan.retained_capacity, self.plan.limits.context_tokens):
            raise ValueError("append exceeds session allocation capacity")
        if ids.numel() > self.plan.limits.candidate_tokens:
            raise ValueError("append exceeds planned execution capacity")
        spec = output_spec or self.driver.output_spec
        self.driver.validate_output(spec)

        def run():
            with torch.inference_mode():
                result = self.driver.append(session, ids, spec)
            self.driver.synchronize()
            self._check_result(result, spec, ids.numel())
            if self.driver.session_length(session) != before + ids.numel():
                raise RuntimeError("append did not commit all tokens")
            return result

        return self._guard(st, run)

    # -------------------------------------------------------------- teardown
    def release_session(self, session):
        self._state(session, allow_failed=True)
        self.driver.release_session(session)
        del self._tracked[id(session)]

    def close(self):
        if self._tracked:
            raise RuntimeError("release runtime sessions before closing resources")
        self.driver.close()
        self._closed = True

    def retire(self):
        """End this runtime while the backend keeps its shared allocations."""
        if self._tracked:
            raise RuntimeError("release runtime sessions before retiring admission")
        self._closed = True
