"""Model-neutral token execution contracts.

Behavioural parity with the reference's ``executor/contracts.py:16-148``:
request shapes, planned execution limits, output selection, results, and the
two protocols a serving stack binds to — :class:`ModelDriver` (the operations
a runtime may invoke on one model) and :class:`ServingBackend` (a model entry
point that declares its driver before admission).  The field names and the
validation rules are kept identical so that configuration written for the
reference carries over unchanged.
"""

from __future__ import annotations

from collections.abc import Callable, Hashable, Mapping
from dataclasses import dataclass, fields
from typing import TYPE_CHECKING, Any, Literal, Protocol

from ..cache.capacity import CapacityPolicy, ResourcePlan, ResourceUsage, SessionPlan

if TYPE_CHECKING:  # pragma: no cover
    import torch


def _positive(value, name):
    if type(value) is not int or value <= 0:
        raise ValueError(f"{name} must be a positive integer")


@dataclass(frozen=True)
class RequestShape:
    """A GR request: a stable history followed by a candidate suffix."""

    history_tokens: int
    candidate_tokens: int

    def __post_init__(self):
        _positive(self.history_tokens, "history_tokens")
        _positive(self.candidate_tokens, "candidate_tokens")

    @property
    def total_tokens(self) -> int:
        return self.history_tokens + self.candidate_tokens


@dataclass(frozen=True)
class ExecutionLimits:
    """Planned per-request limits of one allocated runtime."""

    context_tokens: int
    request_tokens: int
    history_tokens: int
    candidate_tokens: int
    history_chunk_tokens: int
    query_tokens: int

    def __post_init__(self):
        for f in fields(self):
            _positive(getattr(self, f.name), f.name)
        if self.request_tokens > self.context_tokens:
            raise ValueError("planned request exceeds backend context limit")
        if max(self.history_tokens, self.candidate_tokens) > self.request_tokens:
            raise ValueError("history/candidate limit exceeds planned request capacity")

    @classmethod
    def from_mapping(cls, values: Mapping[str, int], *, context: int, chunk_size: int) -> "ExecutionLimits":
        """Limits from the user-facing keys (``max_seq_len``, ``max_session_capacity`` ...)."""
        for v in values.values():
            if type(v) is not int or v <= 0:
                raise ValueError("resource limits must be positive integers")
        total = values.get("max_session_capacity", context)
        query = values.get("max_query_tokens", values.get("workspace_query_tokens", total))
        return cls(
            context_tokens=min(context, values.get("max_seq_len", context)),
            request_tokens=total,
            history_tokens=values.get("max_history_tokens", total),
            candidate_tokens=values.get("max_candidate_tokens", total),
            history_chunk_tokens=chunk_size,
            query_tokens=query,
        )

    def validate(self, shape: RequestShape) -> None:
        checks = (
            (shape.total_tokens > self.context_tokens, "request exceeds backend context limit"),
            (shape.total_tokens > self.request_tokens, "request exceeds planned session capacity"),
            (shape.history_tokens > self.history_tokens, "history exceeds planned retained capacity"),
            (shape.candidate_tokens > self.candidate_tokens, "candidate suffix exceeds planned execution capacity"),
        )
        for failed, message in checks:
            if failed:
                raise ValueError(message)


_SELECT = ("none", "last", "all")


@dataclass(frozen=True)
class OutputSpec:
    """Which per-token outputs a call returns."""

    hidden: Literal["none", "last", "all"] = "all"
    logits: Literal["none", "last", "all"] = "none"
    run_lm_head: bool = False
    ownership: Literal["owned", "borrowed"] = "owned"

    def __post_init__(self):
        if self.hidden not in _SELECT or self.logits not in _SELECT:
            raise ValueError("output selection must be none, last or all")
        if type(self.run_lm_head) is not bool:
            raise TypeError("run_lm_head must be boolean")
        if self.logits != "none" and not self.run_lm_head:
            raise ValueError("logits require LM head execution")
        if self.ownership not in ("owned", "borrowed"):
            raise ValueError("output ownership must be owned or borrowed")


@dataclass(frozen=True)
class ExecutionResult:
    hidden: "torch.Tensor | None" = None
    logits: "torch.Tensor | None" = None
    ownership: Literal["owned", "borrowed"] = "owned"


StageObserver = Callable[[Literal["executed", "cleaned"]], None]


class ModelDriver(Protocol):
    """Operations a :class:`~cxldsagr_b200.executor.runtime.TokenRuntime` drives.

    A driver keeps its own compute loop, device leases, synchronisation and
    commit scope; the runtime never commits model state a second time.
    """

    device: "torch.device"
    max_seq_len: int
    chunk_size: int
    output_spec: OutputSpec
    prefill_output_spec: OutputSpec
    candidate_mode: Literal["gpu_transient", "append_truncate"]

    def plan_resources(self, policy: CapacityPolicy, limits: Mapping[str, int]) -> ResourcePlan: ...
    def allocate_resources(self, plan: ResourcePlan) -> None: ...
    def bind_owner(self, owner: Any) -> None: ...
    def unbind_owner(self, owner: Any, *, rollback: bool = False) -> None: ...
    def maximum_session_quota(self, plan: ResourcePlan) -> tuple[int, int]: ...
    def plan_session(self, shape: RequestShape, identity: Hashable) -> SessionPlan: ...
    def create_session(self, plan: SessionPlan) -> Any: ...
    def session_usage(self, session: Any) -> ResourceUsage: ...
    def shared_usage(self) -> ResourceUsage: ...
    def session_length(self, session: Any) -> int: ...
    def prefill(self, session: Any, ids: "torch.Tensor", output: OutputSpec) -> ExecutionResult: ...
    def candidate(self, session: Any, ids: "torch.Tensor", output: OutputSpec) -> ExecutionResult: ...
    def finish_candidate(self, session: Any, history_tokens: int) -> None: ...
    def append(self, session: Any, ids: "torch.Tensor", output: OutputSpec) -> ExecutionResult: ...
    def validate_output(self, output: OutputSpec, *, prefill: bool = False) -> None: ...
    def diagnostics(self, session: Any) -> dict: ...
    def release_session(self, session: Any) -> None: ...
    def synchronize(self) -> None: ...
    def close(self) -> None: ...


class ServingBackend(Protocol):
    """A model entry point that declares its complete runtime driver before admission."""

    scheme: str
    device: "torch.device"
    max_seq_len: int

    def runtime_driver(self, policy: CapacityPolicy) -> ModelDriver: ...
    def describe(self) -> dict: ...
