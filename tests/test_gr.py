"""CPU tests: GR scheduling, heat, exact-budget request generation, workloads."""

import json
import random
from collections import Counter

import pytest

from cxldsagr_b200.gr.heat import HeatPopulation, zipf_curve
from cxldsagr_b200.gr.input_generator import TextConfig, create_input_generator
from cxldsagr_b200.gr.scheduling import FenwickSampler, ScheduleConfig, index_letter, schedule
from cxldsagr_b200.gr.workload import WorkloadConfig, build_workload, token_sha256


def test_index_letters():
    assert [index_letter(i) for i in (0, 25, 26, 27, 701, 702)] == ["A", "Z", "AA", "AB", "ZZ", "AAA"]


def test_fenwick_sampler_matches_weights():
    s = FenwickSampler([1.0, 0.0, 3.0])
    rng = random.Random(0)
    c = Counter(s.draw(rng) for _ in range(20000))
    assert c[1] == 0 and 0.7 < c[2] / 20000 < 0.8
    s.set(2, 0.0)
    assert {s.draw(rng) for _ in range(100)} == {0}


def test_schedule_modes():
    users = [10, 11, 12]
    w = {10: 1.0, 11: 1.0, 12: 8.0}
    seq = list(schedule(users, w, 6, ScheduleConfig(sampling="sequential", arrival="constant", qps=2)))
    assert [u for u, _ in seq] == [10, 11, 12, 10, 11, 12] and [t for _, t in seq] == [0, .5, 1, 1.5, 2, 2.5]
    capped = list(schedule(users, w, 50, ScheduleConfig(max_revisits=1, arrival="poisson")))
    assert len(capped) == 6 and max(Counter(u for u, _ in capped).values()) == 2
    slots = list(schedule(users, w, 9, ScheduleConfig(arrival="timeslot", qps=2)))
    per_slot = Counter(t for _, t in slots)
    assert max(per_slot.values()) <= 2
    with pytest.raises(ValueError):
        ScheduleConfig(arrival="timeslot", sampling="sequential")


def test_heat_from_curve_and_csv(tmp_path):
    pop = HeatPopulation.from_curve(num_users=100, seed=1)
    assert len(pop.weights) == 100 and abs(sum(pop.weights.values()) - 1) < 1e-9
    pts = zipf_curve(ranks=64, points=8)
    csv = tmp_path / "c.csv"
    csv.write_text("dataset,field,user_fraction,traffic_fraction\n" + "".join(f"d,f,{x},{y}\n" for x, y in pts))
    pop2 = HeatPopulation.from_curve(csv, dataset="d", field="f", num_users=10)
    assert len(pop2.weights) == 10 and pop2.metadata["curve_points"] == 8
    bad = tmp_path / "b.csv"
    bad.write_text("dataset,field,user_fraction,traffic_fraction\nd,f,0.5,0.2\nd,f,1,1\n")  # convex
    with pytest.raises(ValueError):
        HeatPopulation.from_curve(bad, dataset="d", field="f", num_users=4)
    counts = tmp_path / "h.json"
    counts.write_text(json.dumps({"a": [[1, 3], [2, 5]], "b": [[1, 2]]}))
    assert HeatPopulation.load(counts, num_users=0).weights == {1: 5.0, 2: 5.0}


def test_generator_exact_budgets_and_stable_prefix():
    gen = create_input_generator(
        num_users=4, text_config=TextConfig(user_lengths=(700,), user_probabilities=(1.0,), item_lengths=(150,),
                                            item_probabilities=(1.0,), max_input_tokens=1000),
        schedule_config=ScheduleConfig(seed=3, sampling="sequential", arrival="constant"))
    rows = list(gen.iter_generate(8))
    for r in rows:
        assert len(r["input_ids"]) == 850
        assert r["stable_prefix_tokens"] == r["instruction_tokens"] + 700
    a, b = rows[0], rows[4]
    assert a["user_id"] == b["user_id"] and b["visit_index"] == 1
    p = a["stable_prefix_tokens"]
    assert a["input_ids"][:p] == b["input_ids"][:p] and a["input_ids"][p:] != b["input_ids"][p:]
    assert b["common_prefix_tokens"] >= p


def test_workload_manifest(tmp_path):
    wl = build_workload(WorkloadConfig("deepseek_v32", 4, 10, history_tokens=400, candidate_tokens=64, seed=7))
    assert wl.manifest["observed"]["requests"] == 10
    ids = [r["input_ids"] for r in wl.requests]
    assert all(len(x) == 464 for x in ids)
    assert wl.requests[0]["input_sha256"] == token_sha256(ids[0])
    again = build_workload(WorkloadConfig("deepseek_v32", 4, 10, history_tokens=400, candidate_tokens=64, seed=7))
    assert again.manifest["workload_sha256"] == wl.manifest["workload_sha256"]
    wl.write(tmp_path)
    with pytest.raises(FileExistsError):
        wl.write(tmp_path)
    assert len((tmp_path / "requests.jsonl").read_text().splitlines()) == 10
