"""User heat (request weight per user), independent of request text.

Reference semantics (``GR/heat.py:22-207``):

* :meth:`HeatPopulation.from_curve` — synthesise ``N`` users from a ranked
  cumulative-traffic curve ``C(x)`` (fraction of traffic from the hottest
  ``x`` fraction of users, concave, through (0,0) and (1,1)): user ``i`` of
  ``N`` gets ``C(i/N) - C((i-1)/N)`` by piecewise-linear interpolation, and a
  seeded shuffle assigns the weights to IDs ``0..N-1``.  Curves are read from
  a CSV with columns ``dataset, field, user_fraction, traffic_fraction`` (the
  reference's ``heat_curves.csv`` layout works as is).  Without a CSV, a
  built-in analytic curve is used: the cumulative traffic of a Zipf
  population, ``C(x) = H(xM, s) / H(M, s)`` on ``M`` ranks.
* :meth:`HeatPopulation.load` — per-user interaction counts from a JSON
  ``{key: [[user, count], ...]}`` file, or an industrial CSV (``user_id`` +
  one weight field), subsampled uniformly without replacement when asked.
"""

from __future__ import annotations

import csv
import hashlib
import io
import json
import math
import random
from collections import Counter
from dataclasses import dataclass
from pathlib import Path

from .scheduling import _integer

INDUSTRIAL_FIELDS = ("pv_share", "pv_int", "pv_scaled_1_100")


def zipf_curve(ranks: int = 4096, exponent: float = 0.9, points: int = 256) -> list[tuple[float, float]]:
    """Concave cumulative-traffic curve of a Zipf(``exponent``) population of ``ranks`` users."""
    harmonic = [0.0]
    for r in range(1, ranks + 1):
        harmonic.append(harmonic[-1] + r ** -exponent)
    out = []
    for k in range(1, points + 1):
        idx = max(1, round(k * ranks / points))
        out.append((idx / ranks, harmonic[idx] / harmonic[ranks]))
    out[-1] = (1.0, 1.0)
    return out


def _read_curve(raw: bytes, source: str, dataset: str, field: str) -> list[tuple[float, float]]:
    reader = csv.DictReader(io.StringIO(raw.decode("utf-8")))
    needed = {"dataset", "field", "user_fraction", "traffic_fraction"}
    if not needed.issubset(reader.fieldnames or []):
        raise ValueError(f"{source}: missing curve columns {sorted(needed)}")
    pts = []
    for line, row in enumerate(reader, 2):
        if row["dataset"] != dataset or row["field"] != field:
            continue
        try:
            pts.append((float(row["user_fraction"]), float(row["traffic_fraction"])))
        except ValueError as exc:
            raise ValueError(f"{source}:{line}: {exc}") from exc
    if not pts:
        raise ValueError(f"{source}: no curve for {dataset}/{field}")
    return pts


def _validate_curve(pts, source: str) -> list[tuple[float, float]]:
    if pts and pts[0] == (0.0, 0.0):
        pts = pts[1:]
    out = [(0.0, 0.0)]
    slope_prev = math.inf
    for x, y in pts:
        if not (math.isfinite(x) and math.isfinite(y)):
            raise ValueError(f"{source}: curve fractions must be finite")
        px, py = out[-1]
        if not (px < x <= 1 and py < y <= 1):
            raise ValueError(f"{source}: curve fractions must increase strictly within [0, 1]")
        slope = (y - py) / (x - px)
        if slope > slope_prev and not math.isclose(slope, slope_prev, rel_tol=1e-8, abs_tol=1e-10):
            raise ValueError(f"{source}: ranked traffic curve must be concave")
        out.append((x, y))
        slope_prev = slope
    if out[-1] != (1.0, 1.0):
        raise ValueError(f"{source}: curve must end at (1, 1)")
    return out


def _interpolate_weights(curve, n: int) -> list[float]:
    weights, seg, prev = [], 1, 0.0
    for rank in range(1, n + 1):
        x = rank / n
        while curve[seg][0] < x:
            seg += 1
        (x0, y0), (x1, y1) = curve[seg - 1], curve[seg]
        c = y0 + (y1 - y0) * (x - x0) / (x1 - x0)
        w = c - prev
        if not math.isfinite(w) or w <= 0:
            raise ValueError("curve interpolation produced a nonpositive user weight")
        weights.append(w)
        prev = c
    return weights


@dataclass
class HeatPopulation:
    weights: dict
    metadata: dict

    @classmethod
    def from_curve(cls, path: str | Path | None = None, *, dataset: str = "beauty",
                   field: str = "interaction_count", num_users: int = 1000, seed: int = 42) -> "HeatPopulation":
        _integer("num_users", num_users, 1)
        _integer("seed", seed)
        if path is None:
            raw_pts = zipf_curve()
            source, digest = "builtin:zipf(M=4096,s=0.9)", hashlib.sha256(json.dumps(raw_pts).encode()).hexdigest()
        else:
            raw = Path(path).read_bytes()
            source, digest = str(Path(path).resolve()), hashlib.sha256(raw).hexdigest()
            raw_pts = _read_curve(raw, source, dataset, field)
        curve = _validate_curve(raw_pts, source)
        ranked = _interpolate_weights(curve, num_users)
        random.Random(f"{seed}:curve-population").shuffle(ranked)
        weights = dict(enumerate(ranked))
        return cls(weights, {
            "path": source, "sha256": digest, "dataset": dataset, "field": field, "synthetic": True,
            "method": "piecewise_linear_cumulative_increments", "curve_points": len(curve) - 1,
            "selected_users": num_users, "seed": seed, "selection": "synthetic_population",
            "selected_weight_sum": math.fsum(weights.values()),
            "user_identity": "synthetic IDs 0..N-1; seeded shuffle of ranked weights",
        })

    @classmethod
    def uniform(cls, num_users: int) -> "HeatPopulation":
        _integer("num_users", num_users, 1)
        return cls({u: 1.0 for u in range(num_users)}, {
            "source": "explicit_synthetic_ids", "synthetic": True, "selected_users": num_users,
            "selected_weight_sum": float(num_users), "user_identity": "synthetic IDs 0..N-1"})

    @classmethod
    def load(cls, path: Path, *, industrial_field: str | None = None, num_users: int = 1000,
             seed: int = 42) -> "HeatPopulation":
        if num_users < 0:
            raise ValueError("num_users must be nonnegative (0 means all users)")
        path = Path(path)
        rng = random.Random(f"{seed}:heat-population")
        if industrial_field is None:
            counts: Counter = Counter()
            data = json.loads(path.read_text())
            for pairs in data.values():
                for uid, count in pairs:
                    if not isinstance(count, int) or isinstance(count, bool) or count <= 0:
                        raise ValueError(f"{path}: invalid interaction count {count}")
                    counts[int(uid)] += count
            total_users = len(counts)
            users = sorted(counts)
            if num_users and num_users < total_users:
                users = rng.sample(users, num_users)
            rows = [(u, float(counts[u])) for u in users]
        else:
            if industrial_field not in INDUSTRIAL_FIELDS:
                raise ValueError("unsupported industrial heat field")
            rows, total_users = [], 0
            with path.open(newline="", encoding="utf-8") as f:
                reader = csv.DictReader(f)
                if not {"user_id", industrial_field}.issubset(reader.fieldnames or []):
                    raise ValueError(f"{path}: missing user_id or {industrial_field}")
                for line, row in enumerate(reader, 2):
                    try:
                        uid, w = int(row["user_id"]), float(row[industrial_field])
                    except (TypeError, ValueError) as exc:
                        raise ValueError(f"{path}:{line}: {exc}") from exc
                    if uid < 0 or not math.isfinite(w) or w <= 0:
                        raise ValueError(f"{path}:{line}: expected nonnegative ID and finite positive weight")
                    total_users += 1
                    if not num_users or len(rows) < num_users:   # reservoir sampling
                        rows.append((uid, w))
                    else:
                        j = rng.randrange(total_users)
                        if j < num_users:
                            rows[j] = (uid, w)
        if not rows:
            raise ValueError("heat source contains no users")
        if num_users > total_users:
            raise ValueError(f"requested {num_users} users, source has only {total_users}")
        weights = dict(sorted(rows))
        if len(weights) != len(rows):
            raise ValueError("selected heat profiles contain duplicate user IDs")
        return cls(weights, {
            "path": str(path.resolve()), "field": industrial_field or "interaction_count",
            "source_users": total_users, "selected_users": len(weights), "seed": seed,
            "selection": "all" if len(weights) == total_users else "uniform_without_replacement",
            "selected_weight_sum": math.fsum(weights.values()),
            "user_identity": "original heat-source user ID; no text-user mapping",
        })
