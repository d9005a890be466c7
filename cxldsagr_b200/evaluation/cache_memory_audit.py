"""Cache memory audit: measured storage against the admission plan.

Reference: ``evaluation/cache_memory_audit.py:47-887``.  The ledger that admits
users (``cache.prefix_pool``) reserves bytes from a plan; this audit walks the
tensors that actually hold cache state (shared pool, sessions, staging,
workspace), groups them by category and device tier, counts each storage
once, and reports any category whose measured bytes exceed its reservation.
The pinned-host allocator rounds up to powers of two, so DRAM is measured as
charged bytes (``cache.host_allocation.pinned_allocation_bytes``).
"""

from __future__ import annotations

import argparse
import json
from dataclasses import dataclass, field

import torch

from ..cache.capacity import CacheFootprint
from ..cache.host_allocation import pinned_allocation_bytes

CATEGORIES = ("shared_pool", "session", "staging", "workspace", "other")


def scope_category(name: str) -> str:
    for c in CATEGORIES:
        if name.startswith(c):
            return c
    return "other"


def storage_inventory(tensors: dict) -> dict:
    """{category: {"hbm": bytes, "dram": bytes}} over distinct storages (aliases counted once)."""
    seen = set()
    out = {c: {"hbm": 0, "dram": 0} for c in CATEGORIES}
    for name, t in tensors.items():
        if t is None:
            continue
        st = t.untyped_storage()
        key = (str(t.device), st.data_ptr())
        if key in seen:
            continue
        seen.add(key)
        n = st.nbytes()
        if t.device.type == "cuda":
            out[scope_category(name)]["hbm"] += n
        else:
            out[scope_category(name)]["dram"] += pinned_allocation_bytes(n) if t.is_pinned() else n
    return out


def model_cache_tensors(model, sessions=()) -> dict:
    """Name -> tensor for every cache-holding tensor of a DeepSeekV32Model and its sessions."""
    out = {}
    pool = getattr(model, "pool", None)
    if pool is not None:
        for i, layer in enumerate(pool.layers):
            for attr in ("host", "records", "h2d", "d2h", "priority"):
                out[f"shared_pool.{i}.{attr}"] = getattr(layer, attr)
    for s_idx, sess in enumerate(sessions):
        for i, layer in enumerate(sess.layers):
            out[f"session.{s_idx}.{i}.index_keys"] = layer.index.keys
            out[f"session.{s_idx}.{i}.index_scales"] = layer.index.scales
            if sess.pool_session is None:
                out[f"session.{s_idx}.{i}.records"] = layer.kv.records
        if sess.pool_session is not None:
            out[f"session.{s_idx}.page_table"] = sess.pool_session.page_table
    st = getattr(model, "dense_staging", None)
    if st is not None:
        for i, b in enumerate(st.buffers):
            out[f"staging.{i}"] = b
    for d, buf in (getattr(model, "_logits_buf", None) or {}).items():
        out["workspace.logits" if d == model.device else f"workspace.logits.{d}"] = buf
    return out


@dataclass
class CacheMemoryAudit:
    """Compare an inventory against reservations per category."""

    reservations: dict = field(default_factory=dict)   # category -> CacheFootprint

    def check(self, inventory: dict) -> dict:
        violations = []
        for cat, used in inventory.items():
            res = self.reservations.get(cat)
            if res is None:
                continue
            if not CacheFootprint(used["hbm"], used["dram"]).fits(res):
                violations.append({"category": cat, "used": used, "reserved": {"hbm": res.hbm, "dram": res.dram}})
        total = {"hbm": sum(v["hbm"] for v in inventory.values()), "dram": sum(v["dram"] for v in inventory.values())}
        return {"inventory": inventory, "total": total, "violations": violations, "ok": not violations}


def cuda_allocator_snapshot(device=None) -> dict:
    """Allocator totals (reserved / allocated / peak) for the audit report."""
    if not torch.cuda.is_available():
        return {}
    s = torch.cuda.memory_stats(device)
    return {k: s.get(k, 0) for k in ("allocated_bytes.all.current", "allocated_bytes.all.peak",
                                     "reserved_bytes.all.current", "reserved_bytes.all.peak")}


def main(argv=None):
    p = argparse.ArgumentParser(description="Audit a serving run's JSONL output: per-request cache bytes vs budget.")
    p.add_argument("jsonl", help="output of python -m cxldsagr_b200.serving.run_multi_user")
    a = p.parse_args(argv)
    worst, n = {"hbm": 0, "dram": 0}, 0
    violations = []
    with open(a.jsonl) as f:
        for line in f:
            row = json.loads(line)
            if row.get("status") != "completed":
                continue
            m = row["metrics"]
            n += 1
            for tier in ("hbm", "dram"):
                used = m[f"request_cache_{tier}_bytes"]
                worst[tier] = max(worst[tier], used)
                budget = m.get(f"{tier}_budget_bytes")
                if budget is not None and used > budget:
                    violations.append((m["request_id"] if "request_id" in m else n, tier, used, budget))
    print(json.dumps({"requests": n, "peak_request_cache_bytes": worst, "violations": violations,
                      "ok": not violations}))
    return 0 if not violations else 1


if __name__ == "__main__":
    raise SystemExit(main())
