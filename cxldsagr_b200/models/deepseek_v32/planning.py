"""Serving resource planning for the DeepSeek-V3.2 backend.

Reference: ``models/deepseek_v32/execution/planning.py:37-544`` and
``execution/cache_resources.py:43-180``.  Given the scheme, the model shape and
either byte budgets (HBM + DRAM) or fixed pools, decide

* the shared (all-user) footprint: the per-layer sparse-token pool (HBM rows,
  global maps, pinned host arena) for offload schemes, the execution workspace
  (indexer logits, activations of one query chunk), and
* the per-session footprint: resident KV rows (``hbm``) or page tables, plus
  the resident FP8 indexer keys that every scheme keeps in HBM.

With a byte budget and no explicit host arena, the largest arena (in 64-token
pages) that leaves room for one maximum-size session is found by bisection.
Byte formulas mirror the allocations the model actually makes, so the audit
(measured <= reserved) holds by construction.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ...cache.capacity import CacheBudgetExceeded, CacheFootprint, ResourcePlan
from ...cache.host_allocation import pinned_allocation_bytes
from ...cache.sparse_token_pool import POOL_META_WORDS
from ...config import ModelConfig
from ...ops.reference import fp8_record_bytes

PAGE = 64
CACHE_POLICY_REVISION = "b200-v1"


def padded_tokens(tokens: int) -> int:
    return (tokens + PAGE - 1) // PAGE * PAGE


@dataclass(frozen=True)
class ServingResourceConfig:
    scheme: str
    cfg: ModelConfig
    num_layers: int
    max_seq_len: int
    slots: int                       # sparse pool rows P per layer (offload schemes)
    chunk_size: int
    workspace_query_tokens: int
    host_arena_tokens: int | None = None
    extend_chunk_size: int | None = None
    device: str = "cuda"
    kv_format: str = "bf16"

    @property
    def width(self) -> int:
        return self.cfg.kv_lora_rank + self.cfg.qk_rope_head_dim

    @property
    def host_row_bytes(self) -> int:
        """Bytes of one KV record in the pinned-DRAM arena (656 for V3.2 FP8 records)."""
        if self.kv_format == "fp8":
            return fp8_record_bytes(self.cfg.kv_lora_rank, self.cfg.qk_rope_head_dim)
        return self.width * 2

    @property
    def offload(self) -> bool:
        return self.scheme != "hbm"

    @property
    def on_gpu(self) -> bool:
        return str(self.device).startswith("cuda")


def indexer_record_bytes(cfg: ModelConfig) -> int:
    return cfg.index_head_dim + 4


def execution_workspace(config: ServingResourceConfig, capacity: int, candidate: int) -> CacheFootprint:
    """Activation + indexer-logit workspace of one query chunk (an upper bound)."""
    cfg, q = config.cfg, config.workspace_query_tokens
    logits = q * ((capacity + candidate + 3) // 4 * 4) * 4
    per_token = (
        cfg.dim * 2 * 6                         # hidden, residual, normed, summed, quantised copies
        + cfg.q_lora_rank * 4 + cfg.n_heads * cfg.qk_head_dim * 2 * 3  # q_a, q_b, absorbed q, MLA out
        + cfg.index_n_heads * (cfg.index_head_dim + 8) * 2
        + max(cfg.intermediate_size, cfg.moe_intermediate_size * cfg.num_experts_per_tok) * 2 * 3
        + cfg.index_topk * 8                    # top-k ids + values
    )
    return CacheFootprint(logits + q * per_token if config.on_gpu else 0, 0 if config.on_gpu else logits)


def shared_pool_bytes(config: ServingResourceConfig, host_tokens: int, candidate: int) -> CacheFootprint:
    """Bytes of the per-layer shared pool (exactly the tensors SharedSparseTokenPool allocates)."""
    L, P, w = config.num_layers, config.slots, config.width
    rows = (P + 1 + candidate) * w * 2
    maps = host_tokens * 8 + (P + 1) * 8 * 4 + POOL_META_WORDS * 8   # h2d + marks, d2h + priority + miss list + victims, meta
    hb = config.host_row_bytes
    host = pinned_allocation_bytes(host_tokens * hb) if config.on_gpu else host_tokens * hb
    scratch = (P + 1) * hb if config.kv_format == "fp8" else 0   # one FP8 recall scratch per pool
    if config.on_gpu:
        return CacheFootprint(L * (rows + maps) + scratch, L * host)
    return CacheFootprint(0, L * (rows + maps + host) + scratch)


def session_bytes(config: ServingResourceConfig, capacity: int, candidate: int) -> CacheFootprint:
    """Private bytes of one session (resident KV for ``hbm``; indexer keys always)."""
    cfg, L = config.cfg, config.num_layers
    index = (capacity + candidate) * indexer_record_bytes(cfg) + 16 * 4
    kv = (capacity + candidate) * config.width * 2 if not config.offload else 0
    table = (padded_tokens(capacity) // PAGE) * 4 if config.offload else 0
    total = L * (index + kv) + table
    return CacheFootprint(total, 0) if config.on_gpu else CacheFootprint(0, total)


def plan_serving_resources(config: ServingResourceConfig, budget: CacheFootprint | None, limits) -> ResourcePlan:
    capacity = limits["max_session_capacity"]
    if capacity > config.max_seq_len:
        raise ValueError("planned session exceeds model context limit")
    queries = config.workspace_query_tokens
    candidate = limits.get("max_candidate_tokens", min(capacity, queries))
    history = limits.get("max_history_tokens", capacity)
    if type(candidate) is not int or not 0 < candidate <= capacity:
        raise ValueError("candidate limit must satisfy 0 < A <= C")
    if type(history) is not int or not 0 < history <= capacity:
        raise ValueError("history limit must satisfy 0 < H <= context capacity")
    if candidate > queries:
        raise CacheBudgetExceeded("candidate limit exceeds whole-batch query workspace")
    if config.extend_chunk_size is not None and config.extend_chunk_size > queries:
        raise CacheBudgetExceeded("extend chunk exceeds query workspace")
    if config.offload:
        if config.slots < min(config.cfg.index_topk, capacity):
            raise CacheBudgetExceeded("sparse pool must fit one query's full exact selection")
        if queries > config.slots:
            raise CacheBudgetExceeded("query workspace exceeds the per-layer device pool")
        if budget is None and config.host_arena_tokens is None:
            raise ValueError("fixed-pools admission requires explicit host_arena_tokens")
    elif budget is None and history > config.slots:
        raise CacheBudgetExceeded("the fixed HBM token pool must fit one complete history")
    workspace = execution_workspace(config, history, candidate)
    meta = {
        "cache_policy_revision": CACHE_POLICY_REVISION,
        "resource_mode": "fixed_pools" if budget is None else "budget",
        "max_session_capacity": capacity,
        "max_history_tokens": history,
        "max_candidate_tokens": candidate,
        "candidate_persistence": "gpu_transient",
        "candidate_slots": candidate,
        "workspace_query_tokens": queries,
        "sparse_pool_tokens": config.slots,
        "workspace_bytes": workspace.hbm + workspace.dram,
        "max_inflight_writes": 2,
    }
    if not config.offload:
        return ResourcePlan(shared=workspace, hbm_tokens=config.slots if budget is None else 0,
                            metadata={**meta, "pool_scope": "session"})

    one_session = session_bytes(config, history, candidate)
    minimum = padded_tokens(history)

    def estimate(tokens):
        return shared_pool_bytes(config, tokens, candidate) + workspace

    def fits(tokens):
        return (estimate(tokens) + one_session).fits(budget)

    if budget is None:
        tokens = config.host_arena_tokens
        if tokens < minimum:
            raise CacheBudgetExceeded("fixed host arena cannot hold one maximum-size session")
    elif config.host_arena_tokens is not None:
        tokens = config.host_arena_tokens
        if tokens < minimum or not fits(tokens):
            raise CacheBudgetExceeded("configured host arena plus one session exceeds budgets")
    else:
        per_token = config.num_layers * config.host_row_bytes
        upper = max(minimum, (budget.dram // max(per_token, 1)) // PAGE * PAGE)
        if not fits(minimum):
            raise CacheBudgetExceeded("shared pool, workspace and one session do not fit budgets")
        lo, hi = minimum // PAGE, upper // PAGE
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if fits(mid * PAGE):
                lo = mid
            else:
                hi = mid - 1
        tokens = lo * PAGE
    return ResourcePlan(
        shared=estimate(tokens),
        host_pages=tokens // PAGE,
        metadata={**meta, "pool_scope": "backend_per_layer", "shared_token_pool": True,
                  "host_arena_tokens": tokens,
                  "dense_contiguous": config.scheme == "dense_prefetch"},
    )


def bytes_of(tensors) -> int:
    return sum(t.numel() * t.element_size() for t in tensors if isinstance(t, torch.Tensor))
