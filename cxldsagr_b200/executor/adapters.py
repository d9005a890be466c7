"""Bridge from a model's serving backend to the :class:`ModelDriver` contract.

Plays the role of the reference's ``executor/adapters.py`` (the adapter a
DeepSeek serving backend is wrapped in before a :class:`TokenRuntime` drives
it).  The adapter adds no computation of its own: it checks at construction
which capabilities the backend offers (a capability table below), turns the
backend's resource plan into the runtime's limits, and forwards the
session and execution calls, passing the current owner along when the
backend asks for it.

Three choices are fixed by whoever builds the adapter: whether the backend
owns shared (all-user) storage, how candidates execute (``gpu_transient``:
candidate KV exists only in GPU tail rows; ``append_truncate``: candidates
are appended, then truncated away) and how a session's committed length is
read.
"""

from __future__ import annotations

from collections.abc import Callable, Hashable, Mapping
from dataclasses import dataclass, replace
from types import MappingProxyType
from typing import Any, Literal

from ..cache.capacity import CacheFootprint, CapacityPolicy, ResourcePlan, ResourceUsage, SessionPlan
from .contracts import ExecutionLimits, ExecutionResult, OutputSpec, RequestShape

CandidateMode = Literal["gpu_transient", "append_truncate"]

# Capability groups: (condition under which the group is needed, method names).
_CAPABILITIES: tuple[tuple[str, tuple[str, ...]], ...] = (
    ("always", ("estimate_session_bytes", "create_session", "prefill", "extend", "truncate",
                "session_bytes", "release_session", "synchronize")),
    ("shared", ("plan_resources", "allocate_shared", "bind_owner", "unbind_owner", "close",
                "shared_bytes", "estimate_session_host_pages", "session_host_pages")),
    ("gpu_transient", ("extend_candidate",)),
    ("hbm_tokens", ("estimate_session_hbm_tokens", "session_hbm_tokens")),
)

# Runtime limit -> (plan metadata keys that may cap it, in priority order).
_LIMIT_CAPS: tuple[tuple[str, str, tuple[str, ...]], ...] = (
    ("max_session_capacity", "request_tokens", ("max_session_capacity",)),
    ("max_history_tokens", "history_tokens", ("max_history_tokens",)),
    ("max_candidate_tokens", "candidate_tokens", ("max_candidate_tokens",)),
    ("max_query_tokens", "query_tokens", ("max_query_tokens", "workspace_query_tokens")),
)


def _missing(backend: Any, group: str) -> list[str]:
    names = dict(_CAPABILITIES)[group]
    return [n for n in names if not callable(getattr(backend, n, None))]


def _check_capabilities(backend: Any, *groups: str) -> None:
    absent = [n for g in groups for n in _missing(backend, g)]
    if absent:
        raise TypeError(f"backend {type(backend).__name__} lacks required method(s): {', '.join(absent)}")


def _count(value: Any, what: str) -> int:
    if type(value) is not int or value < 0:
        raise ValueError(f"{what}: expected an integer >= 0, got {value!r}")
    return value


@dataclass(frozen=True)
class _Options:
    """The builder's fixed choices, validated once."""

    shared: bool
    candidate_mode: CandidateMode
    run_lm_head: bool
    has_logits: bool
    custom_sessions: bool

    def __post_init__(self):
        if self.candidate_mode not in ("gpu_transient", "append_truncate"):
            raise ValueError(f"candidate_mode must be 'gpu_transient' or 'append_truncate', "
                             f"got {self.candidate_mode!r}")
        if not isinstance(self.shared, bool) or not isinstance(self.run_lm_head, bool):
            raise TypeError("shared and run_lm_head take booleans")
        if self.run_lm_head and not self.has_logits:
            raise ValueError("run_lm_head=True needs a last_logits callable to read the logits")


class BackendAdapter:
    def __init__(self, backend: Any, *, shared: bool, candidate_mode: CandidateMode,
                 session_length: Callable[[Any], int], chunk_size: int, run_lm_head: bool = False,
                 last_logits: Callable[[], Any] | None = None,
                 diagnostics: Callable[[Any], dict] | None = None, owner_aware: bool = False,
                 session_planner: Callable[[ResourcePlan, RequestShape, Hashable], SessionPlan] | None = None,
                 session_factory: Callable[..., Any] | None = None):
        if (session_planner is None) is not (session_factory is None):
            raise ValueError("session_planner and session_factory come as a pair (both or neither)")
        opts = _Options(shared, candidate_mode, run_lm_head, last_logits is not None, session_planner is not None)
        groups = ["always"] + (["shared"] if opts.shared else []) + \
                 (["gpu_transient"] if opts.candidate_mode == "gpu_transient" else [])
        _check_capabilities(backend, *groups)
        self._opts = opts
        self.backend = backend
        self.shared = opts.shared
        self.candidate_mode = opts.candidate_mode
        self.session_length = session_length
        self.device = backend.device
        self.max_seq_len = backend.max_seq_len
        self.chunk_size = chunk_size
        self.output_spec = OutputSpec(run_lm_head=run_lm_head)
        self.prefill_output_spec = OutputSpec(hidden="none", run_lm_head=run_lm_head)
        self._read_logits = last_logits
        self._diagnose = diagnostics
        self._owner_aware = owner_aware
        self._owner: Any = None
        self._custom = (session_planner, session_factory) if opts.custom_sessions else None
        self._plan: ResourcePlan | None = None        # what the runtime sees
        self._backend_plan: ResourcePlan | None = None  # what the backend allocates

    # ---------------------------------------------------------------- owner
    @property
    def _by_owner(self) -> dict:
        """Keyword arguments naming the current owner, for owner-aware backends."""
        return {"owner": self._owner} if self._owner_aware else {}

    def bind_owner(self, owner):
        if self.shared:
            self.backend.bind_owner(owner)
        self._owner = owner

    def unbind_owner(self, owner, *, rollback=False):
        if self.shared:
            self.backend.unbind_owner(owner, rollback=rollback)
        self._owner = None

    # ------------------------------------------------------------- planning
    def plan_resources(self, policy: CapacityPolicy, limits: Mapping[str, int]) -> ResourcePlan:
        if policy.mode == "fixed_pools" and not self.shared:
            raise ValueError("fixed-pools admission works only with a shared backend (host pages or HBM tokens)")
        asked = ExecutionLimits.from_mapping(limits, context=self.max_seq_len, chunk_size=self.chunk_size)
        backend_plan = self.backend.plan_resources(policy.budget, limits) if self.shared else ResourcePlan()
        if not isinstance(backend_plan, ResourcePlan):
            raise TypeError(f"backend plan_resources returned {type(backend_plan).__name__}, not a ResourcePlan")
        if backend_plan.hbm_tokens:
            _check_capabilities(self.backend, "hbm_tokens")
        meta = dict(backend_plan.metadata)
        granted = {"max_seq_len": asked.context_tokens}
        for key, field, cap_keys in _LIMIT_CAPS:
            value = getattr(asked, field)
            cap = next((meta[k] for k in cap_keys if meta.get(k) is not None), None)
            granted[key] = value if cap is None else min(value, cap)
        effective = ExecutionLimits.from_mapping(granted, context=asked.context_tokens, chunk_size=self.chunk_size)
        meta["candidate_persistence"] = "gpu_transient" if self.candidate_mode == "gpu_transient" else "committed"
        self._backend_plan = backend_plan
        self._plan = replace(backend_plan, policy=policy, limits=effective, metadata=MappingProxyType(meta))
        return self._plan

    def allocate_resources(self, plan: ResourcePlan) -> None:
        if plan is not self._plan:
            raise ValueError("allocate_resources takes the plan object plan_resources returned")
        if self.shared:
            self.backend.allocate_shared(self._backend_plan, **self._by_owner)

    def _retained(self, history: int, total: int) -> int:
        """Tokens a session keeps: the history alone for GPU-transient candidates."""
        return history if self.candidate_mode == "gpu_transient" else total

    def _quota(self, capacity: int) -> tuple[int, int]:
        plan = self._plan
        pages = self.backend.estimate_session_host_pages(capacity) if plan.host_pages else 0
        tokens = self.backend.estimate_session_hbm_tokens(capacity) if plan.hbm_tokens else 0
        return _count(pages, "session host pages"), _count(tokens, "session HBM tokens")

    def maximum_session_quota(self, plan: ResourcePlan) -> tuple[int, int]:
        return self._quota(self._retained(plan.limits.history_tokens, plan.limits.request_tokens))

    def plan_session(self, shape: RequestShape, identity: Hashable) -> SessionPlan:
        self._plan.limits.validate(shape)
        if self._custom is not None:
            plan = self._custom[0](self._plan, shape, identity)
            if not isinstance(plan, SessionPlan) or plan.resource_identity is not self._plan:
                raise ValueError("the custom session planner must return a SessionPlan tied to these resources")
            if plan.history_tokens != shape.history_tokens or plan.history_identity != identity:
                raise ValueError("the custom session planner must keep the request's history and identity")
            return plan
        capacity = self._retained(shape.history_tokens, shape.total_tokens)
        reservation = CacheFootprint.from_mapping(self.backend.estimate_session_bytes(capacity, shape.history_tokens))
        pages, tokens = self._quota(capacity)
        return SessionPlan(self._plan, identity, shape.history_tokens, capacity, reservation, pages, tokens,
                           model_plan=capacity)

    def create_session(self, plan: SessionPlan):
        if plan.resource_identity is not self._plan:
            raise ValueError("this session plan belongs to another resource plan")
        if self._custom is not None:
            return self._custom[1](plan, **self._by_owner)
        return self.backend.create_session(plan.model_plan, **self._by_owner)

    # ---------------------------------------------------------------- usage
    def session_usage(self, session) -> ResourceUsage:
        plan = self._plan
        return ResourceUsage(
            CacheFootprint.from_mapping(self.backend.session_bytes(session)),
            host_pages=self.backend.session_host_pages(session) if plan.host_pages else 0,
            hbm_tokens=self.backend.session_hbm_tokens(session) if plan.hbm_tokens else 0,
        )

    def shared_usage(self) -> ResourceUsage:
        if not self.shared:
            return ResourceUsage(CacheFootprint(), owner="shared")
        return ResourceUsage(CacheFootprint.from_mapping(self.backend.shared_bytes()), owner="shared")

    # ------------------------------------------------------------ execution
    def validate_output(self, output: OutputSpec, *, prefill=False):
        problems = [
            (output.run_lm_head != self.output_spec.run_lm_head, "the output spec may not switch the LM head"),
            (output.logits == "all", "only last-token logits are computed"),
            (output.ownership != "owned", "outputs are always owned by the caller"),
            (prefill and output.hidden != "none", "prefill returns no hidden states"),
        ]
        for bad, why in problems:
            if bad:
                raise ValueError(why)

    def _select(self, hidden, output: OutputSpec) -> ExecutionResult:
        kept = {"none": None, "last": None if hidden is None else hidden[-1:], "all": hidden}[output.hidden]
        logits = self._read_logits() if output.logits == "last" else None
        return ExecutionResult(kept, logits)

    def prefill(self, session, ids, output):
        self.validate_output(output, prefill=True)
        return self._select(self.backend.prefill(session, ids, **self._by_owner), output)

    def candidate(self, session, ids, output):
        self.validate_output(output)
        if self.candidate_mode == "gpu_transient":
            hidden = self.backend.extend_candidate(session, ids, **self._by_owner)
        else:
            hidden = self.backend.extend(session, ids, **self._by_owner)
        return self._select(hidden, output)

    def finish_candidate(self, session, history_tokens):
        self.backend.truncate(session, history_tokens, **self._by_owner)

    def append(self, session, ids, output):
        self.validate_output(output)
        return self._select(self.backend.extend(session, ids, **self._by_owner), output)

    def diagnostics(self, session):
        return self._diagnose(session) if self._diagnose is not None else {}

    def release_session(self, session):
        self.backend.release_session(session, **self._by_owner)

    def synchronize(self):
        self.backend.synchronize()

    def close(self):
        if self.shared:
            self.backend.close()
