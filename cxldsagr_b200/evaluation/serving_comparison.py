"""Compare serving runs (cache schemes, versions) on the same GR workload.

Reference: ``evaluation/serving_comparison.py:27-350``.  Input: the JSONL
outputs of ``serving.run_multi_user`` for two or more runs.  Output: per run,
latency summaries (mean / p50 / p90 / p99, first visits vs revisits), hit and
eviction counts, peak cache bytes; and whether the runs served the same
workload (identical ``workload_sha256`` in their ``started`` records).

    python -m cxldsagr_b200.evaluation.serving_comparison hbm.jsonl echo.jsonl --markdown
"""

from __future__ import annotations

import argparse
import json
import math


def percentile(values, q: float) -> float | None:
    if not values:
        return None
    xs = sorted(values)
    k = (len(xs) - 1) * q
    lo, hi = math.floor(k), math.ceil(k)
    return xs[lo] if lo == hi else xs[lo] + (xs[hi] - xs[lo]) * (k - lo)


def summarize(values) -> dict:
    if not values:
        return {"n": 0}
    return {"n": len(values), "mean": sum(values) / len(values), "p50": percentile(values, 0.5),
            "p90": percentile(values, 0.9), "p99": percentile(values, 0.99), "max": max(values)}


def collect_run(path: str) -> dict:
    started, rows = None, []
    with open(path) as f:
        for line in f:
            r = json.loads(line)
            if r.get("status") == "started":
                started = r
            elif r.get("status") == "completed":
                rows.append(r["metrics"])
    lat = [m["latency_ms"] for m in rows]
    rev = [m["latency_ms"] for m in rows if m["is_revisit"]]
    first = [m["latency_ms"] for m in rows if not m["is_revisit"]]
    return {
        "path": path,
        "scheme": started.get("scheme") if started else None,
        "workload_sha256": started.get("workload_sha256") if started else None,
        "latency_ms": summarize(lat),
        "first_visit_ms": summarize(first),
        "revisit_ms": summarize(rev),
        "prefix_hits": sum(m["prefix_cache_hit"] for m in rows),
        "evictions": sum(len(m["evicted_users"]) for m in rows),
        "peak_cache_hbm_bytes": max((m["request_cache_hbm_bytes"] for m in rows), default=0),
        "peak_cache_dram_bytes": max((m["request_cache_dram_bytes"] for m in rows), default=0),
    }


def compare(runs: list[dict]) -> dict:
    ids = {r["workload_sha256"] for r in runs}
    base = runs[0]
    out = {"same_workload": len(ids) == 1 and None not in ids, "runs": runs, "speedup_vs_first": {}}
    for r in runs[1:]:
        a, b = base["revisit_ms"].get("mean"), r["revisit_ms"].get("mean")
        out["speedup_vs_first"][r["scheme"] or r["path"]] = (a / b) if a and b else None
    return out


def markdown(result: dict) -> str:
    lines = ["| scheme | mean ms | p50 | p90 | revisit mean | hits | evictions |", "|---|---|---|---|---|---|---|"]
    for r in result["runs"]:
        lat, rev = r["latency_ms"], r["revisit_ms"]
        fmt = lambda v: "-" if v is None else f"{v:.2f}"  # noqa: E731
        lines.append(f"| {r['scheme']} | {fmt(lat.get('mean'))} | {fmt(lat.get('p50'))} | {fmt(lat.get('p90'))} | "
                     f"{fmt(rev.get('mean'))} | {r['prefix_hits']} | {r['evictions']} |")
    lines.append("")
    lines.append(f"same workload: {result['same_workload']}")
    return "\n".join(lines)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("runs", nargs="+")
    p.add_argument("--markdown", action="store_true")
    a = p.parse_args(argv)
    result = compare([collect_run(r) for r in a.runs])
    print(markdown(result) if a.markdown else json.dumps(result, indent=2))


if __name__ == "__main__":
    main()
