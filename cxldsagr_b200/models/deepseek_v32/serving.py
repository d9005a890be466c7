"""DeepSeek-V3.2 serving backend: retained user sessions on one model replica.

Reference: ``models/deepseek_v32/execution/adapter.py:70-1116``
(``DeepSeekServingBackend``).  One physical model (optionally a replay of
checkpoint layers 0-2, see :mod:`.replay`) serves many users; every user
history is a :class:`~.model.ModelSession` whose allocations are fixed when it
is created, so the admission ledger can reserve their upper bound first.

B200 design choices:

* Candidates always execute as GPU-transient tails for every scheme (the
  resident ``hbm`` cache has candidate tail rows too), so a request never
  appends-and-truncates committed history.
* Offload schemes share one per-layer sparse-token pool sized by the plan
  (host arena pages from the DRAM budget or the fixed-pool configuration).
* Every model operation runs inside the backend's exclusive, non-blocking
  lifecycle operation; a failure whose device drain cannot be confirmed
  poisons the backend.
"""

from __future__ import annotations

from pathlib import Path

import torch

from ...cache.capacity import CacheFootprint, ResourcePlan, SessionPlan
from ...cache.host_allocation import tensor_bytes
from ...cache.lifecycle import ResourceLifecycle
from ...checkpoint import CheckpointReader
from ...config import CacheConfig, ModelConfig
from ...executor.adapters import BackendAdapter
from . import planning
from .model import DeepSeekV32Model, ModelSession
from .replay import ReplayLayout, replay_parameter_count

SCHEMES = ("hbm", "echo", "serial_sparse", "dense_prefetch")


class DeepSeekServingBackend:
    def __init__(self, model_path=None, *, source=None, cfg: ModelConfig | None = None, scheme: str = "hbm",
                 device="cuda:0", num_layers: int = 3, chunk_size: int = 2048, extend_chunk_size: int | None = None,
                 sparse_pool_tokens: int = 32768, host_arena_tokens: int | None = None,
                 workspace_query_tokens: int | None = None, candidate_tokens: int | None = None, scope=None,
                 kv_format: str = "bf16"):
        if scheme not in SCHEMES:
            raise ValueError(f"scheme must be one of {SCHEMES}")
        if chunk_size < 1 or (scheme != "hbm" and sparse_pool_tokens < chunk_size):
            raise ValueError("chunk_size must be positive and fit in sparse_pool_tokens")
        if host_arena_tokens is not None and (host_arena_tokens < 64 or host_arena_tokens % 64):
            raise ValueError("host_arena_tokens must be a positive multiple of 64")
        if workspace_query_tokens is not None and workspace_query_tokens < chunk_size:
            raise ValueError("workspace query bound cannot be smaller than prefill chunk")
        if extend_chunk_size is not None and extend_chunk_size < 1:
            raise ValueError("extend_chunk_size must be positive or None for a whole batch")
        if (model_path is None) == (source is None):
            raise ValueError("give exactly one of model_path or source")
        self.device = torch.device(device)
        if self.device.type == "cuda":
            if self.device.index is None:
                self.device = torch.device("cuda", torch.cuda.current_device())
            if torch.cuda.get_device_capability(self.device)[0] != 10:
                raise ValueError("the CUDA serving path is built for sm_100 (B200)")
        if model_path is not None:
            self.path = Path(model_path)
            source = CheckpointReader(self.path)
            cfg = cfg or source.config
        else:
            self.path = None
        if cfg is None:
            raise ValueError("a model config is required")
        if cfg.first_k_dense_replace < 3 and num_layers >= 3:
            raise ValueError("checkpoint layers 0, 1, 2 must all have dense MLPs")
        self.cfg = cfg
        self.scheme = scheme
        self.max_seq_len = cfg.max_seq_len
        self.num_layers = num_layers
        self.chunk_size = chunk_size
        self.extend_chunk_size = extend_chunk_size
        self.slots = sparse_pool_tokens
        self.host_arena_tokens = host_arena_tokens
        self.kv_format = kv_format
        self.workspace_query_tokens = workspace_query_tokens or max(chunk_size, extend_chunk_size or 0)
        self.candidate_tokens = candidate_tokens or self.workspace_query_tokens
        self.lifecycle = ResourceLifecycle("DeepSeek", drain=self.synchronize)
        self.plan: ResourcePlan | None = None
        layers = list(ReplayLayout.repeated_sources(num_layers).source_layers) if num_layers >= 3 else list(range(num_layers))
        self.parameter_counts = replay_parameter_count(source, num_layers) if num_layers >= 3 else None
        cache = CacheConfig(method=scheme, capacity=self.max_seq_len, pool_tokens=sparse_pool_tokens,
                            host_tokens=host_arena_tokens, candidate_tokens=self.candidate_tokens,
                            chunk_size=chunk_size, kv_format=kv_format)
        self.model = DeepSeekV32Model(cfg, source, device=self.device, cache=cache, layers=layers,
                                      replay=num_layers >= 3, allocate_default_session=False,
                                      allocate_pool=False, scope=scope)
        self.last_logits = None
        self._sessions: set[int] = set()

    # -------------------------------------------------------------- driver
    def runtime_driver(self, policy) -> BackendAdapter:
        return BackendAdapter(
            self, shared=True, owner_aware=True, candidate_mode="gpu_transient",
            session_length=lambda s: s.length, chunk_size=self.chunk_size, run_lm_head=True,
            last_logits=lambda: self.last_logits, diagnostics=self.session_metrics,
            session_planner=self.plan_runtime_session, session_factory=self.create_planned_session,
        )

    def _planning_config(self) -> planning.ServingResourceConfig:
        return planning.ServingResourceConfig(
            scheme=self.scheme, cfg=self.cfg, num_layers=self.num_layers, max_seq_len=self.max_seq_len,
            slots=self.slots, chunk_size=self.chunk_size, workspace_query_tokens=self.workspace_query_tokens,
            host_arena_tokens=self.host_arena_tokens, extend_chunk_size=self.extend_chunk_size,
            device=str(self.device), kv_format=self.kv_format)

    def plan_resources(self, budget: CacheFootprint | None, limits) -> ResourcePlan:
        return planning.plan_serving_resources(self._planning_config(), budget, limits)

    def allocate_shared(self, plan: ResourcePlan, *, owner=None):
        self.lifecycle.check_access(owner, allow_closed=True)
        if not isinstance(plan, ResourcePlan):
            raise TypeError("allocate_shared needs a ResourcePlan")
        if self.model.pool is not None:
            raise RuntimeError("shared resources are already allocated")
        if self.scheme != "hbm":
            self.model.attach_pool(self.model.make_pool(plan.metadata["host_arena_tokens"], self.slots))
        self.plan = plan
        self.lifecycle.closed = False

    def shared_bytes(self) -> dict:
        out = {"hbm": 0, "dram": 0}
        if self.model.pool is not None:
            out = dict(self.model.pool.shared_bytes())
        for buf in self.model._logits_buf.values():
            out["hbm" if buf.is_cuda else "dram"] += buf.numel() * 4
        return out

    # ------------------------------------------------------------ sessions
    def estimate_session_host_pages(self, capacity: int) -> int:
        return planning.padded_tokens(capacity) // planning.PAGE if self.scheme != "hbm" else 0

    def estimate_session_hbm_tokens(self, capacity: int) -> int:
        return capacity if self.scheme == "hbm" else 0

    def session_hbm_tokens(self, session: ModelSession) -> int:
        self._check_session(session)
        return session.capacity if self.scheme == "hbm" else 0

    def session_host_pages(self, session: ModelSession) -> int:
        self._check_session(session)
        return len(session.pool_session.pages) if session.pool_session is not None else 0

    def estimate_session_bytes(self, capacity: int, prefix_tokens: int = 0) -> dict:
        fp = planning.session_bytes(self._planning_config(), capacity, self.candidate_tokens)
        return {"hbm": fp.hbm, "dram": fp.dram}

    def plan_runtime_session(self, resources: ResourcePlan, shape, identity) -> SessionPlan:
        resources.limits.validate(shape)
        capacity = shape.history_tokens
        reservation = CacheFootprint.from_mapping(self.estimate_session_bytes(capacity, capacity))
        return SessionPlan(resources, identity, shape.history_tokens, capacity, reservation,
                           self.estimate_session_host_pages(capacity) if resources.host_pages else 0,
                           self.estimate_session_hbm_tokens(capacity) if resources.hbm_tokens else 0,
                           model_plan=capacity)

    def create_planned_session(self, plan: SessionPlan, *, owner=None) -> ModelSession:
        if not isinstance(plan, SessionPlan) or plan.model_plan != plan.retained_capacity:
            raise TypeError("DeepSeek session allocation requires its own SessionPlan")
        return self.create_session(plan.retained_capacity, owner=owner)

    def create_session(self, capacity: int, *, owner=None) -> ModelSession:
        self.lifecycle.check_access(owner, allow_closed=self.scheme == "hbm")
        if self.scheme != "hbm" and self.model.pool is None:
            raise RuntimeError("allocate shared resources before creating offload sessions")
        session = self.model.new_session(capacity)
        session.generation = self.lifecycle.generation
        self._sessions.add(id(session))
        self.lifecycle.register(session)
        session.bind_serving(self.lifecycle)
        return session

    def _check_session(self, session):
        if id(session) not in self._sessions or session.released:
            raise ValueError("foreign or released session")

    def session_bytes(self, session: ModelSession) -> dict:
        self._check_session(session)
        tensors = []
        for layer in session.layers:
            tensors += [layer.index.keys, layer.index.scales, layer.index.offset]
            if session.pool_session is None:
                tensors.append(layer.kv.records)
        if session.pool_session is not None:
            tensors.append(session.pool_session.page_table)
        return tensor_bytes(tensors)

    def release_session(self, session: ModelSession, *, owner=None):
        self._check_session(session)
        with self.lifecycle.operation(session, "release", owner=owner):
            session.release()
        self._sessions.discard(id(session))
        self.lifecycle.release(session)

    # ----------------------------------------------------------- execution
    def _run(self, session, ids, owner, kind, **kw):
        self._check_session(session)
        with self.lifecycle.operation(session, kind, owner=owner):
            result = self.model.forward(ids, session=session, **kw)
        self.last_logits = result.logits
        return result.hidden

    def prefill(self, session, token_ids, *, owner=None):
        return self._run(session, token_ids, owner, "prefill", chunk_size=self.chunk_size)

    def extend(self, session, token_ids, *, owner=None):
        return self._run(session, token_ids, owner, "extend", return_hidden=True,
                         chunk_size=self.extend_chunk_size or token_ids.numel())

    def extend_candidate(self, session, token_ids, *, owner=None):
        if token_ids.numel() > self.candidate_tokens:
            raise ValueError("candidate suffix exceeds the planned candidate tail rows")
        return self._run(session, token_ids, owner, "candidate", transient=True, return_hidden=True)

    def truncate(self, session, prefix_tokens: int, *, owner=None):
        self._check_session(session)
        if session.length != prefix_tokens:
            with self.lifecycle.operation(session, "truncate", owner=owner):
                session.truncate(prefix_tokens)

    def session_metrics(self, session) -> dict:
        stats = [layer.kv.stats for layer in session.layers]
        keys = ("written_records", "recalled_records", "prefetched_records", "evicted_records",
                "capacity_splits", "selection_records", "resident_selection_records")
        return {k: sum(getattr(s, k, 0) for s in stats) for k in keys} | {"length": session.length}

    # ------------------------------------------------------------ ownership
    def bind_owner(self, owner):
        self.lifecycle.bind_owner(owner)

    def unbind_owner(self, owner, *, rollback: bool = False):
        if rollback:
            self._release_shared()
        self.lifecycle.unbind_owner(owner)

    def _release_shared(self):
        pool = self.model.pool
        if pool is not None:
            pool.close()
            self.model.attach_pool(None)
        self.plan = None

    def close(self):
        self.synchronize()
        self._release_shared()
        self.lifecycle.close()

    def synchronize(self):
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def describe(self) -> dict:
        return {
            "scheme": self.scheme,
            "model": str(self.path) if self.path else "in-memory",
            "num_layers": self.num_layers,
            "chunk_size": self.chunk_size,
            "sparse_pool_tokens": self.slots,
            "host_arena_tokens": None if self.plan is None else self.plan.metadata.get("host_arena_tokens"),
            "parameter_counts": self.parameter_counts,
            "device": str(self.device),
        }
