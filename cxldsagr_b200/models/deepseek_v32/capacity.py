"""Static capacity planning for a fixed-pool GR session population.

Reference: ``models/deepseek_v32/execution/capacity.py:39-386``
(``EchoCapacityPlanner``): hold one of the two pool capacities fixed -- the
per-layer HBM sparse pool ``P`` (rows) or the pinned host arena ``NH``
(tokens, whole sessions of ``ceil(H / 64)`` pages) -- and find the largest
value of the other whose reservation fits the HBM and DRAM budgets.

The ledger is this build's own byte model: the shared pool, the execution
workspace and a session's private bytes come from :mod:`.planning`, whose
formulas are the tensors :class:`~cxldsagr_b200.cache.sparse_token_pool.SharedSparseTokenPool`,
:class:`~cxldsagr_b200.cache.indexer_cache.IndexerCache` and the model
allocate.  Every retained session (``NH // padded(H)`` of them) keeps its FP8
indexer keys in HBM, so raising ``NH`` also costs HBM.  On top of the
reservation comes an allocator allowance: the PyTorch caching allocator
rounds each persistent allocation up (512 B below 1 MiB, 2 MiB segments
above), charged per allocation, plus a fixed scratch headroom (64 MiB by
default, a planning policy rather than a proven bound).

Nothing is allocated: the result is a reservation for the current serving
implementation, not a measured process peak.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass

from ...cache.host_allocation import pinned_allocation_bytes
from ...config import ModelConfig
from . import planning

INT32_MAX = (1 << 31) - 1
# Host ids and slot ids are int32 in the pool metadata kernels; INT32_MAX is the
# MISSING sentinel and slot 0 the padding row.
MAX_HOST_TOKENS = (INT32_MAX - 1) // planning.PAGE * planning.PAGE
MAX_DEVICE_SLOTS = INT32_MAX - 2
DEFAULT_ALLOCATOR_HEADROOM = 64 << 20
# Persistent allocations: per pool layer (records, h2d, d2h, priority, meta,
# mark, miss list, victims), per session layer (indexer keys, scales, hint
# slab, prediction scratch), per session (page table).
POOL_TENSORS_PER_LAYER = 8
SESSION_TENSORS_PER_LAYER = 4
SESSION_TENSORS = 1


def allocator_tail(nbytes: int) -> int:
    """Upper bound on the caching allocator's rounding of one allocation."""
    if nbytes <= 0:
        return 0
    unit = 512 if nbytes < (1 << 20) else 2 << 20
    return -nbytes % unit if nbytes % unit else 0


def _int(name, value, minimum=0):
    if type(value) is not int or value < minimum:
        raise ValueError(f"{name} must be an integer >= {minimum}")
    return value


@dataclass
class CapacityPlanner:
    """Largest ``P`` for a fixed ``NH`` or largest ``NH`` for a fixed ``P``.

    The HBM envelope is ``floor(total_hbm * hbm_fraction) - model_hbm``;
    ``noncache_headroom`` is deducted from it once.  ``scheme`` is one of the
    offload schemes (the ``hbm`` scheme has no shared pool to size).
    """

    cfg: ModelConfig
    num_layers: int
    history_tokens: int
    candidate_tokens: int
    chunk_size: int
    total_hbm_bytes: int
    model_hbm_bytes: int
    dram_budget_bytes: int
    hbm_fraction: float = 0.9
    noncache_headroom_bytes: int = 0
    allocator_headroom_bytes: int = DEFAULT_ALLOCATOR_HEADROOM
    scheme: str = "echo"

    def __post_init__(self):
        for name in ("num_layers", "history_tokens", "candidate_tokens", "chunk_size"):
            _int(name, getattr(self, name), 1)
        for name in ("total_hbm_bytes", "model_hbm_bytes", "dram_budget_bytes", "noncache_headroom_bytes",
                     "allocator_headroom_bytes"):
            _int(name, getattr(self, name))
        f = float(self.hbm_fraction)
        if not (0 < f <= 1):
            raise ValueError("hbm_fraction must satisfy 0 < f <= 1")
        if self.scheme == "hbm":
            raise ValueError("the hbm scheme keeps KV per session; there is no shared pool to size")
        self.context_tokens = self.history_tokens + self.candidate_tokens
        if self.context_tokens > self.cfg.max_seq_len:
            raise ValueError("H + A exceeds the model context")
        self.page_tokens = planning.padded_tokens(self.history_tokens)
        self.query_tokens = max(self.chunk_size, self.candidate_tokens)
        self.min_slots = max(self.query_tokens, min(self.cfg.index_topk, self.context_tokens))
        self.max_slots = MAX_DEVICE_SLOTS - self.candidate_tokens
        self.fraction_limit = int(self.total_hbm_bytes * f)
        self.envelope = max(0, self.fraction_limit - self.model_hbm_bytes)
        self.width = self.cfg.kv_lora_rank + self.cfg.qk_rope_head_dim

    @property
    def budgets(self) -> dict:
        return {"total_hbm_bytes": self.total_hbm_bytes, "model_hbm_bytes": self.model_hbm_bytes,
                "hbm_fraction": self.hbm_fraction, "fraction_hbm_limit_bytes": self.fraction_limit,
                "hbm_envelope_bytes": self.envelope,
                "cache_hbm_budget_bytes": self.envelope - self.noncache_headroom_bytes,
                "noncache_headroom_bytes": self.noncache_headroom_bytes,
                "dram_budget_bytes": self.dram_budget_bytes,
                "allocator_scratch_headroom_bytes": self.allocator_headroom_bytes}

    def _config(self, p: int, nh: int) -> planning.ServingResourceConfig:
        return planning.ServingResourceConfig(
            scheme=self.scheme, cfg=self.cfg, num_layers=self.num_layers, max_seq_len=self.cfg.max_seq_len,
            slots=p, chunk_size=self.chunk_size, workspace_query_tokens=self.query_tokens, host_arena_tokens=nh)

    def estimate(self, *, sparse_pool_tokens: int, host_arena_tokens: int) -> dict:
        """JSON ledger for one (P, NH), including the checks it fails (``feasible``)."""
        p = _int("sparse_pool_tokens", sparse_pool_tokens, 1)
        nh = _int("host_arena_tokens", host_arena_tokens, planning.PAGE)
        if nh % planning.PAGE:
            raise ValueError("host_arena_tokens must be a multiple of 64")
        conf = self._config(p, nh)
        L, A, H, w = self.num_layers, self.candidate_tokens, self.history_tokens, self.width
        users, unused = divmod(nh, self.page_tokens)
        pool = planning.shared_pool_bytes(conf, nh, A)
        work = planning.execution_workspace(conf, H, A)
        session = planning.session_bytes(conf, H, A)
        index_rows = H + A
        hbm = {
            "pool_records": L * (p + 1 + A) * w * 2,
            "pool_maps": pool.hbm - L * (p + 1 + A) * w * 2,
            "execution_workspace": work.hbm,
            "session_private": users * session.hbm,
        }
        # Allocator rounding of every persistent allocation.
        pool_sizes = [(p + 1 + A) * w * 2, nh * 4, (p + 1) * 8, (p + 1) * 8, 8 * 64, nh * 4, (p + 1) * 8,
                      (p + 1) * 8]
        sess_sizes = [index_rows * self.cfg.index_head_dim, index_rows * 4, 64, index_rows * 4]
        tails = (L * sum(allocator_tail(s) for s in pool_sizes)
                 + users * L * sum(allocator_tail(s) for s in sess_sizes)
                 + users * allocator_tail(self.page_tokens // planning.PAGE * 4))
        reservation = sum(hbm.values())
        cache_total = reservation + tails + self.allocator_headroom_bytes
        total = cache_total + self.noncache_headroom_bytes
        host_bin = pinned_allocation_bytes(nh * w * 2)
        dram = {"host_records_pinned_bins": L * host_bin, "session_cpu_page_tables": users * 8}
        dram_total = sum(dram.values())
        violated = []
        if total > self.envelope:
            violated.append("hbm_budget")
        if dram_total > self.dram_budget_bytes:
            violated.append("dram_budget")
        if p > self.max_slots:
            violated.append("native_device_index_limit")
        if nh > MAX_HOST_TOKENS:
            violated.append("native_host_index_limit")
        if p < self.min_slots:
            violated.append("minimum_device_pool")
        if users < 1:
            violated.append("full_session_fit")
        return {
            "status": "static_reservation_not_measured_peak", "feasible": not violated,
            "violated_constraints": violated, "sparse_pool_tokens": p, "host_arena_tokens": nh,
            "full_sessions": users, "unused_host_tokens": unused, "useful_device_slots": min(p, nh),
            "num_layers": L, "history_tokens": H, "candidate_tokens": A, "chunk_size": self.chunk_size,
            "workspace_query_tokens": self.query_tokens, "session_page_tokens": self.page_tokens,
            "minimum_device_slots": self.min_slots, "maximum_device_slots": self.max_slots,
            "record_width": w, "budgets": self.budgets,
            "hbm": {"components": hbm, "reservation_bytes": reservation, "allocator_tail_bytes": tails,
                    "allocator_headroom_bytes": self.allocator_headroom_bytes, "cache_total_bytes": cache_total,
                    "total_bytes": total, "budget_bytes": self.envelope, "remaining_bytes": self.envelope - total},
            "dram": {"components": dram, "host_record_logical_bytes": L * nh * w * 2, "total_bytes": dram_total,
                     "budget_bytes": self.dram_budget_bytes,
                     "remaining_bytes": self.dram_budget_bytes - dram_total},
        }

    def _search(self, variable: str, fixed: int, lo: int, hi: int) -> dict:
        """Largest feasible value in [lo, hi] by bisection (feasibility is monotone in both)."""
        def ev(v):
            if variable == "NH":
                return self.estimate(sparse_pool_tokens=fixed, host_arena_tokens=v * self.page_tokens)
            return self.estimate(sparse_pool_tokens=v, host_arena_tokens=fixed)

        first = ev(lo)
        if not first["feasible"]:
            selected, following = None, first
        else:
            hi = max(lo, hi)
            while lo < hi:
                mid = (lo + hi + 1) // 2
                if ev(mid)["feasible"]:
                    lo = mid
                else:
                    hi = mid - 1
            selected, following = ev(lo), ev(lo + 1)
        return {"status": "static_reservation_not_measured_peak", "search_variable": variable,
                "feasible": selected is not None, "budgets": self.budgets, "selected": selected,
                "next_candidate": following, "limiting_constraints": following["violated_constraints"]}

    def max_host_capacity(self, *, sparse_pool_tokens: int) -> dict:
        """Largest NH (whole sessions) for a fixed P."""
        p = _int("sparse_pool_tokens", sparse_pool_tokens, 1)
        if not self.min_slots <= p <= self.max_slots:
            raise ValueError("fixed P violates the query/top-k or native indexing bound")
        upper = min(MAX_HOST_TOKENS // self.page_tokens,
                    self.dram_budget_bytes // (self.num_layers * self.width * 2 * self.page_tokens))
        r = self._search("NH", p, 1, upper)
        sel = r["selected"]
        r.update(fixed_P=p, max_host_arena_tokens=sel["host_arena_tokens"] if sel else 0,
                 max_full_sessions=sel["full_sessions"] if sel else 0, step_tokens=self.page_tokens)
        return r

    def max_device_capacity(self, *, host_arena_tokens: int) -> dict:
        """Largest allocated P for a fixed NH; ``useful_max_P`` caps it at NH (rows past NH hold nothing new)."""
        nh = _int("host_arena_tokens", host_arena_tokens, planning.PAGE)
        if nh % planning.PAGE or nh > MAX_HOST_TOKENS:
            raise ValueError("fixed NH must be page aligned and within the native indexing bound")
        if nh < self.page_tokens:
            raise ValueError("fixed NH cannot hold one complete session")
        room = max(0, self.envelope - self.noncache_headroom_bytes)
        upper = min(self.max_slots, room // (self.num_layers * self.width * 2))
        r = self._search("P", nh, self.min_slots, upper)
        sel = r["selected"]
        raw = sel["sparse_pool_tokens"] if sel else 0
        useful = min(raw, nh)
        r.update(fixed_NH=nh, raw_alloc_max_P=raw, useful_max_P=useful,
                 useful_selected=(self.estimate(sparse_pool_tokens=useful, host_arena_tokens=nh)
                                  if useful >= self.min_slots else None),
                 useful_limiting_constraints=["host_token_capacity"] if raw > nh else r["limiting_constraints"],
                 step_tokens=1)
        return r


def main(argv=None):
    """``python -m cxldsagr_b200.models.deepseek_v32.capacity --history 65536 --candidate 1280 --fixed-p 65536``"""
    from ...config import v32_config

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--num-layers", type=int, default=61)
    ap.add_argument("--history", type=int, required=True)
    ap.add_argument("--candidate", type=int, required=True)
    ap.add_argument("--chunk-size", type=int, default=2048)
    ap.add_argument("--total-hbm-gib", type=float, default=178.4)
    ap.add_argument("--model-hbm-gib", type=float, default=0.0)
    ap.add_argument("--dram-gib", type=float, default=1024.0)
    ap.add_argument("--hbm-fraction", type=float, default=0.9)
    ap.add_argument("--scheme", default="echo", choices=("echo", "serial_sparse", "dense_prefetch"))
    g = ap.add_mutually_exclusive_group(required=True)
    g.add_argument("--fixed-p", type=int, help="maximise NH for this P")
    g.add_argument("--fixed-nh", type=int, help="maximise P for this NH")
    a = ap.parse_args(argv)
    planner = CapacityPlanner(v32_config(a.num_layers), a.num_layers, a.history, a.candidate, a.chunk_size,
                              int(a.total_hbm_gib * 2**30), int(a.model_hbm_gib * 2**30), int(a.dram_gib * 2**30),
                              hbm_fraction=a.hbm_fraction, scheme=a.scheme)
    out = (planner.max_host_capacity(sparse_pool_tokens=a.fixed_p) if a.fixed_p is not None
           else planner.max_device_capacity(host_arena_tokens=a.fixed_nh))
    print(json.dumps(out))


if __name__ == "__main__":
    main()
