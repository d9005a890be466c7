"""GR workload analysis: user-heat statistics, sampled access traces and
histograms reconstructed from saved heat curves (CPU only, no model).

Reference: ``GR/analyze_heat.py:25-335`` (population statistics and the
``heat_curves.csv`` export), ``GR/sample_distribution.py:45-270`` (a request
trace sampled from a heat curve with the serving scheduler),
``GR/reconstruct_histogram.py:34-257`` (an integer visits histogram that
preserves every saved cumulative point) and ``GR/dataset.py:18`` (catalog
titles).  Outputs are CSV / JSON; the reference's figures need matplotlib,
which this image does not ship, so no plots are drawn.

    python -m cxldsagr_b200.gr.analysis summarize --industrial users.csv --output out/
    python -m cxldsagr_b200.gr.analysis sample --users 64 256 --requests 4096 --output out/
    python -m cxldsagr_b200.gr.analysis reconstruct --curve-path heat_curves.csv --dataset industrial_10M \\
        --field pv_int --users 10000000 --visits 123456789 --output out/
"""

from __future__ import annotations

import argparse
import csv
import hashlib
import json
import math
import pickle
from collections import Counter
from dataclasses import asdict
from fractions import Fraction
from pathlib import Path

import numpy as np

from .heat import INDUSTRIAL_FIELDS, HeatPopulation
from .scheduling import ScheduleConfig, schedule

TOP_PERCENTS = (1, 5, 10, 20, 50)
# Visit-count bins of a sampled trace: (label, lo, hi) inclusive.
VISIT_BINS = (("0", 0, 0), ("1", 1, 1), ("2-4", 2, 4)) + tuple(
    (f"{2 ** p + 1}-{2 ** (p + 1)}", 2 ** p + 1, 2 ** (p + 1)) for p in range(2, 8)) + (("257+", 257, math.inf),)


# ------------------------------------------------------------ statistics
def summarize_weights(weights, dataset: str, field: str, *, curve_points: int = 800) -> tuple[dict, dict]:
    """Concentration statistics of positive user weights and a downsampled cumulative curve.

    Gini uses the ascending-rank formula ``(n + 1 - 2 * sum_i r_i w_(i) / W) / n``
    with weights sorted in DEcreasing order and ranks from 1 (equivalent form);
    effective users = ``W^2 / sum w^2``; top-x% shares round the user count up.
    """
    w = np.sort(np.asarray(weights, dtype=np.float64))[::-1]
    if w.size == 0 or not np.all(np.isfinite(w)) or np.any(w <= 0):
        raise ValueError(f"{dataset}/{field}: expected finite, positive user weights")
    n = w.size
    cum = np.cumsum(w)
    total = float(cum[-1])
    share = cum / total
    ranks = np.arange(1, n + 1, dtype=np.float64)
    q = np.quantile(w, [0.0, 0.5, 0.9, 0.99, 1.0])
    row = {
        "dataset": dataset, "field": field, "users": n, "total_weight": total, "mean_weight": total / n,
        "min_weight": float(q[0]), "median_weight": float(q[1]), "p90_weight": float(q[2]),
        "p99_weight": float(q[3]), "max_weight": float(q[4]),
        "gini": (n + 1 - 2 * float(ranks @ w) / total) / n,
        "effective_users": total * total / float(w @ w),
        "users_for_50pct_traffic_pct": 100.0 * (int(np.searchsorted(share, 0.5)) + 1) / n,
    }
    for pct in TOP_PERCENTS:
        row[f"top_{pct}pct_traffic_pct"] = 100.0 * float(share[math.ceil(n * pct / 100) - 1])
    pts = np.unique(np.concatenate(([1, n], np.geomspace(1, n, min(n, curve_points)).astype(np.int64))))
    curve = {"user_fraction": pts / n, "traffic_fraction": share[pts - 1], "relative_weight": w[pts - 1] / (total / n)}
    return row, curve


def interaction_weights(path: Path) -> np.ndarray:
    """Per-user interaction counts summed over a ``{item: [[user, count], ...]}`` JSON map."""
    users: Counter = Counter()
    for pairs in json.loads(Path(path).read_text()).values():
        for uid, count in pairs:
            if type(count) is not int or count <= 0:
                raise ValueError(f"{path}: invalid frequency {count!r}")
            users[int(uid)] += count
    return np.fromiter(users.values(), dtype=np.float64, count=len(users))


def industrial_weights(path: Path) -> dict[str, np.ndarray]:
    """The three weight columns of an industrial users CSV (``user_id`` + fields)."""
    cols = {f: [] for f in INDUSTRIAL_FIELDS}
    with Path(path).open(newline="", encoding="utf-8") as f:
        for row in csv.DictReader(f):
            for k in INDUSTRIAL_FIELDS:
                cols[k].append(float(row[k]))
    return {k: np.asarray(v, dtype=np.float64) for k, v in cols.items()}


def fingerprint(path: Path) -> dict:
    data = Path(path).read_bytes()
    return {"path": str(Path(path).resolve()), "bytes": len(data), "sha256": hashlib.sha256(data).hexdigest()}


def write_heat_artifacts(rows: list[dict], curves: dict, output: Path, sources: list[dict]):
    """``heat_summary.{csv,json}``, ``heat_curves.csv`` (the curve format :class:`HeatPopulation` reads)
    and ``heat_provenance.json``."""
    output.mkdir(parents=True, exist_ok=True)
    with (output / "heat_summary.csv").open("w", newline="") as f:
        wr = csv.DictWriter(f, fieldnames=list(rows[0]), lineterminator="\n")
        wr.writeheader()
        wr.writerows(rows)
    (output / "heat_summary.json").write_text(json.dumps(rows, indent=2) + "\n")
    with (output / "heat_curves.csv").open("w", newline="") as f:
        wr = csv.writer(f, lineterminator="\n")
        wr.writerow(["dataset", "field", "user_fraction", "traffic_fraction", "relative_weight"])
        for (dataset, field), c in curves.items():
            for x, y, z in zip(c["user_fraction"], c["traffic_fraction"], c["relative_weight"], strict=True):
                wr.writerow([dataset, field, float(x), float(y), float(z)])
    (output / "heat_provenance.json").write_text(json.dumps({
        "sources": sources, "numpy": np.__version__, "quantile_method": "numpy linear",
        "top_fraction_rounding": "ceil", "population": "all users in each input file"}, indent=2) + "\n")


# ------------------------------------------------------- sampled traces
def _quantile(sorted_vals, frac):
    pos = frac * (len(sorted_vals) - 1)
    lo, hi = math.floor(pos), math.ceil(pos)
    return sorted_vals[lo] + (sorted_vals[hi] - sorted_vals[lo]) * (pos - lo)


def sample_population(population: HeatPopulation, requests: int, cfg: ScheduleConfig):
    """Sample ``requests`` with the serving scheduler; return (trace, per-user rows, histogram, summary)."""
    if type(requests) is not int or requests < 1:
        raise ValueError("requests must be an integer >= 1")
    users = sorted(population.weights)
    ranked = sorted(users, key=lambda u: (-population.weights[u], u))
    rank = {u: i + 1 for i, u in enumerate(ranked)}
    wsum = math.fsum(population.weights.values())
    counts: Counter = Counter()
    first, last, trace = {}, {}, []
    for i, (uid, ts) in enumerate(schedule(users, population.weights, requests, cfg)):
        prev = last.get(uid)
        trace.append({"request_id": i, "user_id": uid, "heat_rank": rank[uid], "visit_index": counts[uid],
                      "is_revisit": int(counts[uid] > 0), "previous_request_id": prev,
                      # distinct users seen since this user's previous request
                      "reuse_distance_users": None if prev is None else sum(p > prev for p in last.values()),
                      "synthetic_timestamp": ts})
        counts[uid] += 1
        first.setdefault(uid, i)
        last[uid] = i
    per_user = [{"pool_users": len(users), "user_id": u, "heat_rank": rank[u],
                 "probability": population.weights[u] / wsum,
                 "expected_visits": requests * population.weights[u] / wsum, "visits": counts[u],
                 "revisits": max(0, counts[u] - 1), "first_request_id": first.get(u),
                 "last_request_id": last.get(u)} for u in ranked]
    hist = []
    for label, lo, hi in VISIT_BINS:
        members = [u for u in users if lo <= counts[u] <= hi]
        hist.append({"pool_users": len(users), "visit_count_bin": label, "users": len(members),
                     "user_fraction": len(members) / len(users), "requests": sum(counts[u] for u in members)})
    vals = sorted(counts[u] for u in users)
    visited = sum(v > 0 for v in vals)
    top = math.ceil(0.1 * len(users))
    summary = {
        "pool_users": len(users), "requests": len(trace), "visited_users": visited,
        "unvisited_users": len(users) - visited, "one_visit_users": sum(v == 1 for v in vals),
        "returning_users": sum(v > 1 for v in vals), "revisits": len(trace) - visited,
        "revisit_request_fraction": (len(trace) - visited) / max(len(trace), 1),
        "visits_mean_all_pool_users": len(trace) / len(users), "visits_min_all_pool_users": vals[0],
        "visits_median_all_pool_users": _quantile(vals, 0.5), "visits_p95_all_pool_users": _quantile(vals, 0.95),
        "visits_max": vals[-1], "top10pct_users_ceiling": top,
        "top10pct_expected_request_fraction": sum(r["probability"] for r in per_user[:top]),
        "top10pct_observed_request_fraction": sum(r["visits"] for r in per_user[:top]) / max(len(trace), 1),
        "schedule": asdict(cfg), "population": population.metadata,
    }
    return trace, per_user, hist, summary


# ------------------------------------------------- curve reconstruction
def _exact_count(fraction, scale: int) -> int:
    v = Fraction(str(fraction)) * scale
    n = round(v)
    if abs(v - n) > Fraction(1, 10**6):
        raise ValueError("the saved curve does not resolve integer user / visit counts")
    return int(n)


def reconstruct_histogram(points, users: int, visits: int):
    """Integer ``{visits per user: users}`` histogram through every saved cumulative point.

    Between consecutive points the segment's visits are split as evenly as
    integers allow (``floor`` for most users, ``floor + 1`` for the
    remainder), so every point, the user total and the visit total are
    exact.  It approximates the unavailable raw data; it is not that data.
    """
    hist: Counter = Counter()
    segments = []
    pr = pv = 0
    for p in points:
        r = _exact_count(p["user_fraction"], users)
        c = _exact_count(p["traffic_fraction"], visits)
        su, sv = r - pr, c - pv
        if su <= 0 or sv < su:
            raise ValueError("expected increasing ranks and at least one visit per user")
        low, extra = divmod(sv, su)
        hist[low] += su - extra
        if extra:
            hist[low + 1] += extra
        segments.append({"first_rank": pr + 1, "last_rank": r, "users": su, "visits": sv,
                         "floor_visits_per_user": low, "floor_users": su - extra, "ceil_users": extra})
        pr, pv = r, c
    if (pr, pv) != (users, visits):
        raise ValueError("curve endpoints disagree with the population totals")
    return hist, segments


def read_curve_points(path: Path, dataset: str, field: str) -> list[dict]:
    with Path(path).open(newline="", encoding="utf-8") as f:
        pts = [{"user_fraction": r["user_fraction"], "traffic_fraction": r["traffic_fraction"]}
               for r in csv.DictReader(f) if r["dataset"] == dataset and r["field"] == field]
    if not pts:
        raise ValueError(f"{path}: no curve for {dataset}/{field}")
    return pts


# ------------------------------------------------------------- titles
class _PlainUnpickler(pickle.Unpickler):
    def find_class(self, module, name):  # plain dict / list / str / int data only
        raise ValueError(f"unsupported pickle object: {module}.{name}")


def load_titles(path: Path) -> dict[int, str]:
    """Catalog titles (``{"meta": {item: title}}``, JSON or plain-data pickle) used as readable text."""
    path = Path(path)
    if path.suffix == ".json":
        raw = json.loads(path.read_text(encoding="utf-8"))
    else:
        with path.open("rb") as f:
            raw = _PlainUnpickler(f).load()
    titles = {int(k): v for k, v in raw["meta"].items()}
    if not titles or any(not isinstance(t, str) or not t.strip() for t in titles.values()):
        raise ValueError("catalog contains empty or non-text titles")
    return titles


# ------------------------------------------------------------------ CLI
def _write_rows(path: Path, rows: list[dict]):
    with path.open("w", newline="", encoding="utf-8") as f:
        wr = csv.DictWriter(f, fieldnames=list(rows[0]), lineterminator="\n")
        wr.writeheader()
        wr.writerows(rows)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("summarize", help="statistics + heat_curves.csv from interaction maps / industrial CSVs")
    s.add_argument("--interactions", type=Path, nargs="*", default=[], help="timestep_map.json files")
    s.add_argument("--industrial", type=Path, nargs="*", default=[], help="users_*.csv files")
    s.add_argument("--output", type=Path, required=True)
    t = sub.add_parser("sample", help="sample request traces from a heat curve")
    t.add_argument("--curve-path", type=Path, help="heat_curves.csv (default: the built-in Zipf curve)")
    t.add_argument("--dataset", default="industrial_10M")
    t.add_argument("--field", default="pv_share")
    t.add_argument("--users", type=int, nargs="+", default=[64, 256, 1024])
    t.add_argument("--requests", type=int, default=4096)
    t.add_argument("--seed", type=int, default=42)
    t.add_argument("--output", type=Path, required=True)
    r = sub.add_parser("reconstruct", help="integer visits histogram from saved curve points")
    r.add_argument("--curve-path", type=Path, required=True)
    r.add_argument("--dataset", required=True)
    r.add_argument("--field", required=True)
    r.add_argument("--users", type=int, required=True)
    r.add_argument("--visits", type=int, required=True)
    r.add_argument("--output", type=Path, required=True)
    a = ap.parse_args(argv)
    a.output.mkdir(parents=True, exist_ok=True)
    if a.cmd == "summarize":
        rows, curves, sources = [], {}, []
        for path in a.interactions:
            row, curve = summarize_weights(interaction_weights(path), path.parent.name, "interaction_count")
            rows.append(row)
            curves[(row["dataset"], row["field"])] = curve
            sources.append(fingerprint(path))
        for path in a.industrial:
            name = "industrial_" + path.stem.removeprefix("users_")
            for field, w in industrial_weights(path).items():
                row, curve = summarize_weights(w, name, field)
                rows.append(row)
                curves[(name, field)] = curve
            sources.append(fingerprint(path))
        if not rows:
            ap.error("give --interactions and/or --industrial files")
        write_heat_artifacts(rows, curves, a.output, sources)
        print(json.dumps({"rows": len(rows), "output": str(a.output)}))
    elif a.cmd == "sample":
        out = []
        for n in a.users:
            pop = HeatPopulation.from_curve(a.curve_path, dataset=a.dataset, field=a.field, num_users=n, seed=a.seed)
            trace, per_user, hist, summary = sample_population(pop, a.requests, ScheduleConfig(seed=a.seed))
            _write_rows(a.output / f"trace_users{n}.csv", trace)
            _write_rows(a.output / f"per_user_users{n}.csv", per_user)
            _write_rows(a.output / f"histogram_users{n}.csv", hist)
            out.append(summary)
        (a.output / "sample_summary.json").write_text(json.dumps(out, indent=2) + "\n")
        print(json.dumps([{k: s[k] for k in ("pool_users", "requests", "revisit_request_fraction")} for s in out]))
    else:
        hist, segments = reconstruct_histogram(read_curve_points(a.curve_path, a.dataset, a.field), a.users, a.visits)
        _write_rows(a.output / "histogram.csv", [{"visits_per_user": k, "users": v} for k, v in sorted(hist.items())])
        _write_rows(a.output / "segments.csv", segments)
        print(json.dumps({"bins": len(hist), "segments": len(segments)}))


if __name__ == "__main__":
    main()
