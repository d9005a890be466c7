"""Cache memory audit: fixed cache storage and per-scope transient device memory
against the admission plan.

Reference behaviour: ``evaluation/cache_memory_audit.py:47-887`` (an
allocator-event audit of the cache paths with a workspace allowance per
transaction).  Three measurements, none of them part of a latency sample:

* **Fixed storage** (:func:`storage_inventory`): the tensors that hold cache
  state (shared pool, sessions, staging, workspace buffers), grouped by
  category and tier, each storage counted once.  With a CUDA allocator
  snapshot the allocator block behind every storage is charged as well, so
  rounding padding shows; pinned host storage is charged at the caching host
  allocator's power-of-two size.
* **Transient memory per scope** (:class:`ScopeMemoryTracker`): installed as a
  model's ``scope`` hook, it reads the CUDA caching allocator's counters at
  every scope boundary (host side, no device synchronisation) and records per
  scope name the peak bytes above the bytes live at entry (nested scopes
  included), the bytes still live at exit (retained) and the bytes allocated.
  Peak counters are reset at each boundary and folded into the enclosing
  scope, so nested scopes do not hide each other's peaks.
* **Allowance** (:class:`WorkspaceAllowance`): the transient bytes one chunk
  of one layer may take per component, computed from the buffers this
  framework's kernels use (fused selection: sampled logits, thresholds,
  candidate lists, counts, outputs; full-logits selection; MLA output and
  split-K partials; FP8 recall scratch; pool metadata lists).
  :func:`audit_scopes` compares the tracker's peaks with it.

What this does not see: memory outside the PyTorch caching allocator (the
symmetric heap's ``cudaMalloc``, CUDA graph private pools' reuse), CPU malloc
overhead, and allocator fragmentation beyond block rounding.

CLI::

    python -m cxldsagr_b200.evaluation.cache_memory_audit run.jsonl     # serving log: per-request bytes vs budget
    python -m cxldsagr_b200.evaluation.cache_memory_audit model --history 16384 --extend 128 --method serial_sparse
"""

from __future__ import annotations

import argparse
import json
from contextlib import contextmanager
from dataclasses import asdict, dataclass, field

import torch

from ..cache.capacity import CacheFootprint
from ..cache.host_allocation import pinned_allocation_bytes

CATEGORIES = ("shared_pool", "session", "staging", "workspace", "other")

# Scope names of the attention path and the allowance component they draw on.
SCOPE_COMPONENTS = {
    "indexer_select": "selection",
    "indexer": "selection",
    "exact_topk": "selection",
    "indexer_cp": "selection",
    "indexer_prefetch": "selection",
    "prefetch_hint": "selection",
    "sparse_mla": "attention",
}


def scope_category(name: str) -> str:
    for c in CATEGORIES:
        if name.startswith(c):
            return c
    return "other"


# ------------------------------------------------------------ fixed storage
def allocator_blocks(snapshot) -> dict:
    """(device, address) -> allocator block bytes of every active allocation in a
    ``torch.cuda.memory_snapshot()``."""
    blocks = {}
    for seg in snapshot or ():
        addr = seg["address"]
        for blk in seg["blocks"]:
            start = blk.get("address", addr)
            if blk["state"] == "active_allocated":
                blocks[(f"cuda:{seg['device']}", start)] = blk["size"]
            addr = start + blk["size"]
    return blocks


def storage_inventory(tensors: dict, *, snapshot=None) -> dict:
    """{category: {"hbm", "hbm_allocator", "dram"}} over distinct storages (aliases counted once).

    ``hbm_allocator`` charges the caching allocator's block for each CUDA
    storage when a snapshot is given (else the storage size)."""
    blocks = allocator_blocks(snapshot) if snapshot is not None else {}
    seen = set()
    out = {c: {"hbm": 0, "hbm_allocator": 0, "dram": 0} for c in CATEGORIES}
    for name, t in tensors.items():
        if t is None:
            continue
        st = t.untyped_storage()
        key = (str(t.device), st.data_ptr())
        if key in seen or st.nbytes() == 0:
            continue
        seen.add(key)
        n = st.nbytes()
        row = out[scope_category(name)]
        if t.device.type == "cuda":
            row["hbm"] += n
            row["hbm_allocator"] += max(n, blocks.get(key, n))
        else:
            row["dram"] += pinned_allocation_bytes(n) if t.is_pinned() else n
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
            hbm = max(used["hbm"], used.get("hbm_allocator", 0))
            if not CacheFootprint(hbm, used["dram"]).fits(res):
                violations.append({"category": cat, "used": used, "reserved": {"hbm": res.hbm, "dram": res.dram}})
        total = {t: sum(v.get(t, 0) for v in inventory.values()) for t in ("hbm", "hbm_allocator", "dram")}
        return {"inventory": inventory, "total": total, "violations": violations, "ok": not violations}


def cuda_allocator_snapshot(device=None) -> dict:
    """Allocator totals (reserved / allocated / peak) for the audit report."""
    if not torch.cuda.is_available():
        return {}
    s = torch.cuda.memory_stats(device)
    return {k: s.get(k, 0) for k in ("allocated_bytes.all.current", "allocated_bytes.all.peak",
                                     "reserved_bytes.all.current", "reserved_bytes.all.peak")}


# ------------------------------------------------------------ allowances
def _c4(n: int) -> int:
    return max(4, (n + 3) // 4 * 4)


def _blk(n: int) -> int:
    """An n-byte request rounded to the caching allocator's 512-byte granule (at least the bytes requested)."""
    return (n + 511) // 512 * 512


@dataclass(frozen=True)
class WorkspaceAllowance:
    """Transient device bytes one chunk of one layer may hold, per component.

    The components are additive admission terms; scopes are attribution only
    (a scope's peak is compared with the component it draws on)."""

    selection: int      # indexer + exact top-k working set
    attention: int      # MLA query projection, output, split-K partials, recall scratch
    metadata: int       # pool classify / map lists of one step

    @property
    def total(self) -> int:
        return self.selection + self.attention + self.metadata

    @classmethod
    def for_chunk(cls, cfg, *, queries: int, context: int, method: str = "hbm", kv_format: str = "bf16",
                  fused_select: bool = True, logits_preallocated: bool = True, cand_cap: int = 8192,
                  sample_stride: int = 32, splits: int = 1, offload: bool = False) -> "WorkspaceAllowance":
        if min(queries, context) < 1:
            raise ValueError("queries and context must be positive")
        k = cfg.index_topk
        width = min(k, context)
        out_ids = _blk(queries * width * 4) * 2            # values FP32 + ids int32
        if fused_select and method != "echo":
            sel = (_blk(queries * _c4(-(-context // sample_stride)) * 4)   # sampled logits
                   + _blk(queries * 4)                                     # thresholds
                   + _blk(queries * max(cand_cap, 2 * k) * 8)              # candidate composites
                   + _blk((queries + 1) * 4) + _blk(2 * queries * 4)       # counts + any-flag, flags + overflow
                   + out_ids)
        else:
            sel = out_ids + _blk(queries * 4)                        # outputs + two-pass overflow words
            if method == "echo":
                sel += _blk(context * 4)                             # predicted-row list
        if not logits_preallocated:
            sel += _blk(queries * _c4(context) * 4)                  # [Q, N] FP32 logits (or fallback rows)
        H, D = cfg.n_heads, cfg.kv_lora_rank
        qk = D + cfg.qk_rope_head_dim
        att = _blk(queries * H * qk * 2) + _blk(queries * H * D * 2)  # absorbed query, latent output (BF16)
        if splits > 1:
            att += _blk(splits * queries * H * D * 4) + _blk(splits * queries * H * 4)  # FP32 partials + LSE
        meta = 0
        if offload:
            rows = queries * width
            att += _blk(rows * 4)                                    # physical slot ids
            if kv_format == "fp8":
                att += _blk(min(rows, context) * 656)                # 656-byte records gathered before dequant
            meta = 3 * _blk(rows * 4)                                # classify / select / map lists
        return cls(int(sel), int(att), int(meta))


# ------------------------------------------------------------ transient tracker
@dataclass
class ScopeMemory:
    calls: int = 0
    peak_transient: int = 0     # max over calls: peak live bytes above the bytes live at entry
    retained: int = 0           # sum over calls: bytes still live at exit beyond entry
    allocated: int = 0          # sum over calls: bytes handed out inside the scope
    block_peak_transient: int = 0   # peak_transient in allocator blocks (requests plus the cache's slack)


class ScopeMemoryTracker:
    """Per-scope allocator accounting from the caching allocator's counters.

    ``stats_fn`` returns a dict with ``<counter>.all.current``, ``.peak`` and
    ``.allocated``; ``reset_fn`` sets the peak to the current value (defaults:
    the CUDA allocator of ``device``).  Use :meth:`scope` as the model's scope
    hook.  The default counter, ``requested_bytes``, counts the bytes the code
    asked for; ``allocated_bytes`` counts the caching allocator's blocks, which
    add its slack: sizes round up to 512 bytes, and a request served from a
    cached block of the large pool takes the whole block when the remainder
    would be under 1 MiB, so the same step can charge different bytes
    depending on what the cache held."""

    def __init__(self, device=None, *, stats_fn=None, reset_fn=None, counter: str = "requested_bytes"):
        self.CUR, self.PEAK, self.CUM = (f"{counter}.all.current", f"{counter}.all.peak", f"{counter}.all.allocated")
        self.BCUR, self.BPEAK = "allocated_bytes.all.current", "allocated_bytes.all.peak"
        self.stats_fn = stats_fn or (lambda: torch.cuda.memory_stats(device))
        self.reset_fn = reset_fn or (lambda: torch.cuda.reset_peak_memory_stats(device))
        # [name, entry_current, running_peak, entry_cumulative, block_entry, block_running_peak]
        self._stack: list[list] = []
        self.rows: dict[str, ScopeMemory] = {}

    def _block(self, s: dict, key: str) -> int:
        return s.get(key, 0)

    def _enter(self, name: str):
        s = self.stats_fn()
        if self._stack:
            top = self._stack[-1]
            top[2] = max(top[2], s[self.PEAK])
            top[5] = max(top[5], self._block(s, self.BPEAK))
        self.reset_fn()
        b = self._block(s, self.BCUR)
        self._stack.append([name, s[self.CUR], s[self.CUR], s[self.CUM], b, b])

    def _exit(self):
        s = self.stats_fn()
        name, entry, peak, cum, bentry, bpeak = self._stack.pop()
        peak = max(peak, s[self.PEAK])
        bpeak = max(bpeak, self._block(s, self.BPEAK))
        row = self.rows.setdefault(name, ScopeMemory())
        row.calls += 1
        row.peak_transient = max(row.peak_transient, peak - entry)
        row.block_peak_transient = max(row.block_peak_transient, bpeak - bentry)
        row.retained += s[self.CUR] - entry
        row.allocated += s[self.CUM] - cum
        if self._stack:
            self._stack[-1][2] = max(self._stack[-1][2], peak)
            self._stack[-1][5] = max(self._stack[-1][5], bpeak)
        self.reset_fn()

    @contextmanager
    def scope(self, name: str):
        self._enter(name)
        try:
            yield
        finally:
            self._exit()

    def __call__(self, name: str):
        return self.scope(name)

    def summary(self) -> dict:
        return {n: asdict(r) for n, r in sorted(self.rows.items())}


def audit_scopes(rows: dict, allowance: WorkspaceAllowance, *, mapping=None) -> dict:
    """Compare each mapped scope's peak transient with its allowance component."""
    mapping = SCOPE_COMPONENTS if mapping is None else mapping
    limits = asdict(allowance)
    checked, violations = {}, []
    for name, row in rows.items():
        comp = mapping.get(name)
        if comp is None:
            continue
        r = row if isinstance(row, dict) else asdict(row)
        peak = r["peak_transient"]
        checked[name] = {"component": comp, "peak_transient": peak, "allowance": limits[comp],
                         "block_peak_transient": r.get("block_peak_transient", peak)}
        if peak > limits[comp]:
            violations.append(name)
    return {"checked": checked, "violations": violations, "ok": not violations, "allowance": limits}


# ------------------------------------------------------------ CLI
def audit_serving_log(path: str) -> int:
    worst, n = {"hbm": 0, "dram": 0}, 0
    violations = []
    with open(path) as f:
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


def audit_model(a) -> int:
    """Prefill + extend of a random-init V3.2 model under the tracker (CUDA)."""
    from ..checkpoint import RandomSource
    from ..config import CacheConfig, v32_config
    from ..models.deepseek_v32.model import DeepSeekV32Model

    dev = torch.device(a.device)
    cfg = v32_config(layers=a.layers)
    H, A = a.history, a.extend
    offload = a.method in ("serial_sparse", "echo")
    cache = CacheConfig(method=a.method, capacity=H + A, chunk_size=a.chunk, candidate_tokens=A,
                        pool_tokens=(H + A) if offload else None, host_tokens=H + A, kv_format=a.kv_format)
    model = DeepSeekV32Model(cfg, RandomSource(cfg, layers=range(a.layers), seed=0, device=dev), device=dev,
                             cache=cache)
    g = torch.Generator().manual_seed(11)
    hist = torch.randint(0, cfg.vocab_size, (H,), generator=g).to(dev)
    ext = torch.randint(0, cfg.vocab_size, (A,), generator=g).to(dev)
    model.prefill(hist)            # warm-up: kernels, cached buffers
    model.reset()
    torch.cuda.synchronize(dev)
    report = {}
    for phase, fn, queries, context in (("prefill", lambda: model.prefill(hist), min(a.chunk, H), H),
                                        ("extend", lambda: model.extend(ext), A, H + A)):
        tracker = ScopeMemoryTracker(dev)
        model.scope = tracker
        fn()
        model.scope = None
        torch.cuda.synchronize(dev)
        from ..ops import mla_splits

        allowance = WorkspaceAllowance.for_chunk(cfg, queries=queries, context=context, method=a.method,
                                                 kv_format=a.kv_format, offload=offload,
                                                 splits=mla_splits(queries, min(cfg.index_topk, context)))
        rows = tracker.summary()
        report[phase] = {"scopes": rows, "audit": audit_scopes(rows, allowance)}
    inv = storage_inventory(model_cache_tensors(model, [model.session]), snapshot=torch.cuda.memory_snapshot())
    report["fixed"] = CacheMemoryAudit().check(inv)
    report["allocator"] = cuda_allocator_snapshot(dev)
    report["config"] = {"history": H, "extend": A, "method": a.method, "layers": a.layers, "chunk": a.chunk,
                        "kv_format": a.kv_format}
    ok = report["prefill"]["audit"]["ok"] and report["extend"]["audit"]["ok"]
    report["ok"] = ok
    print(json.dumps(report))
    return 0 if ok else 1


def main(argv=None):
    import sys

    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "model":
        p = argparse.ArgumentParser(prog="cache_memory_audit model",
                                    description="per-scope transient memory of a model step vs the allowance")
        p.add_argument("--history", type=int, default=16384)
        p.add_argument("--extend", type=int, default=128)
        p.add_argument("--chunk", type=int, default=2048)
        p.add_argument("--layers", type=int, default=3)
        p.add_argument("--method", default="hbm", choices=("hbm", "serial_sparse", "echo", "dense_prefetch"))
        p.add_argument("--kv-format", choices=("bf16", "fp8"), default="bf16")
        p.add_argument("--device", default="cuda:0")
        return audit_model(p.parse_args(argv[1:]))
    p = argparse.ArgumentParser(description="Audit a serving run's JSONL output: per-request cache bytes vs budget.")
    p.add_argument("jsonl", help="output of python -m cxldsagr_b200.serving.run_multi_user")
    return audit_serving_log(p.parse_args(argv).jsonl)


if __name__ == "__main__":
    raise SystemExit(main())
