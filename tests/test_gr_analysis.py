"""GR analysis tools: heat statistics against independent formulas, sampled
trace invariants, exact curve-point reconstruction and the CLI round trip
(the exported curve file loads back as a heat population)."""

import csv
import json

import numpy as np
import pytest

from cxldsagr_b200.gr.analysis import (load_titles, main, reconstruct_histogram, sample_population,
                                       summarize_weights)
from cxldsagr_b200.gr.heat import HeatPopulation
from cxldsagr_b200.gr.scheduling import ScheduleConfig


def test_summary_statistics():
    row, curve = summarize_weights(np.ones(1000), "d", "f")
    assert abs(row["gini"]) < 1e-12 and row["effective_users"] == pytest.approx(1000)
    assert row["top_10pct_traffic_pct"] == pytest.approx(10.0)
    w = np.random.default_rng(0).pareto(1.5, 5000) + 1
    row, curve = summarize_weights(w, "d", "f")
    mad = np.abs(w[:, None] - w[None, :]).mean()
    assert row["gini"] == pytest.approx(mad / (2 * w.mean()), rel=1e-9)
    assert row["effective_users"] == pytest.approx(w.sum() ** 2 / (w ** 2).sum())
    assert curve["traffic_fraction"][-1] == pytest.approx(1.0) and curve["user_fraction"][-1] == 1.0
    with pytest.raises(ValueError):
        summarize_weights(np.array([1.0, 0.0]), "d", "f")


def test_sample_population_invariants():
    pop = HeatPopulation.from_curve(num_users=64, seed=1)
    trace, per_user, hist, summary = sample_population(pop, 512, ScheduleConfig(seed=1))
    assert len(trace) == 512 == sum(r["visits"] for r in per_user)
    assert sum(h["users"] for h in hist) == 64 and sum(h["requests"] for h in hist) == 512
    assert summary["revisits"] == sum(r["revisits"] for r in per_user)
    assert all(t["is_revisit"] == (t["visit_index"] > 0) for t in trace)


def test_reconstruct_preserves_points():
    pts = [{"user_fraction": "0.1", "traffic_fraction": "0.5"}, {"user_fraction": "1", "traffic_fraction": "1"}]
    hist, segs = reconstruct_histogram(pts, 10, 100)
    assert sum(hist.values()) == 10 and sum(k * v for k, v in hist.items()) == 100
    assert hist == {50: 1, 5: 4, 6: 5}
    assert segs[0]["users"] == 1 and segs[0]["visits"] == 50
    with pytest.raises(ValueError):
        reconstruct_histogram(pts, 10, 99)


def test_cli_round_trip(tmp_path):
    inter = tmp_path / "beauty"
    inter.mkdir()
    (inter / "timestep_map.json").write_text(json.dumps({"1": [[0, 3], [1, 1]], "2": [[0, 2], [2, 5]]}))
    ind = tmp_path / "users_small.csv"
    with ind.open("w", newline="") as f:
        wr = csv.writer(f)
        wr.writerow(["user_id", "pv_share", "pv_int", "pv_scaled_1_100"])
        for u in range(50):
            wr.writerow([u, 1.0 / (u + 1), 100 // (u + 1) + 1, max(1, 100 // (u + 1))])
    out = tmp_path / "out"
    main(["summarize", "--interactions", str(inter / "timestep_map.json"), "--industrial", str(ind),
          "--output", str(out)])
    rows = json.loads((out / "heat_summary.json").read_text())
    assert [r["dataset"] for r in rows] == ["beauty"] + ["industrial_small"] * 3
    pop = HeatPopulation.from_curve(out / "heat_curves.csv", dataset="industrial_small", field="pv_int",
                                    num_users=20)
    assert len(pop.weights) == 20
    main(["sample", "--curve-path", str(out / "heat_curves.csv"), "--dataset", "beauty",
          "--field", "interaction_count", "--users", "8", "--requests", "32", "--output", str(tmp_path / "s")])
    assert (tmp_path / "s" / "trace_users8.csv").exists()


def test_load_titles(tmp_path):
    p = tmp_path / "cat.json"
    p.write_text(json.dumps({"meta": {"3": "A title", "4": "Another"}}))
    assert load_titles(p) == {3: "A title", 4: "Another"}
    p.write_text(json.dumps({"meta": {"3": " "}}))
    with pytest.raises(ValueError):
        load_titles(p)


def test_reconstruct_cli(tmp_path):
    curves = tmp_path / "heat_curves.csv"
    curves.write_text("dataset,field,user_fraction,traffic_fraction,relative_weight\n"
                      "d,f,0.1,0.5,5\nd,f,1,1,1\n")
    main(["reconstruct", "--curve-path", str(curves), "--dataset", "d", "--field", "f", "--users", "10",
          "--visits", "100", "--output", str(tmp_path / "r")])
    rows = (tmp_path / "r" / "histogram.csv").read_text().splitlines()
    assert rows[0] == "visits_per_user,users" and len(rows) == 4
