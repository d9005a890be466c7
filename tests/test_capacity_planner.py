"""Static capacity planner: the bisection returns the boundary (selected is
feasible, the next step is not), the ledger adds up, and bad inputs raise."""

import pytest

from cxldsagr_b200.config import v32_config
from cxldsagr_b200.models.deepseek_v32.capacity import CapacityPlanner, allocator_tail


def _planner(**kw):
    args = dict(cfg=v32_config(3), num_layers=3, history_tokens=65536, candidate_tokens=1280, chunk_size=2048,
                total_hbm_bytes=40 << 30, model_hbm_bytes=20 << 30, dram_budget_bytes=64 << 30)
    args.update(kw)
    return CapacityPlanner(**args)


def test_max_host_capacity_is_a_boundary():
    pl = _planner()
    r = pl.max_host_capacity(sparse_pool_tokens=65536)
    assert r["feasible"] and r["selected"]["feasible"] and not r["next_candidate"]["feasible"]
    assert r["max_host_arena_tokens"] == r["max_full_sessions"] * 65536
    assert r["next_candidate"]["host_arena_tokens"] == r["max_host_arena_tokens"] + 65536
    assert r["limiting_constraints"]


def test_max_device_capacity_and_useful_cap():
    pl = _planner()
    r = pl.max_device_capacity(host_arena_tokens=4 * 65536)
    assert r["feasible"]
    assert not r["next_candidate"]["feasible"]
    assert r["useful_max_P"] == min(r["raw_alloc_max_P"], 4 * 65536)
    if r["raw_alloc_max_P"] > 4 * 65536:
        assert r["useful_limiting_constraints"] == ["host_token_capacity"]


def test_ledger_components_add_up():
    e = _planner().estimate(sparse_pool_tokens=8192, host_arena_tokens=2 * 65536)
    hbm = e["hbm"]
    assert hbm["reservation_bytes"] == sum(hbm["components"].values())
    assert hbm["total_bytes"] == hbm["cache_total_bytes"]
    assert e["full_sessions"] == 2 and e["feasible"]
    # more retained sessions cost HBM too (their indexer keys stay resident)
    e4 = _planner().estimate(sparse_pool_tokens=8192, host_arena_tokens=4 * 65536)
    assert e4["hbm"]["components"]["session_private"] == 2 * hbm["components"]["session_private"]


def test_infeasible_and_invalid():
    pl = _planner(total_hbm_bytes=21 << 30)
    r = pl.max_host_capacity(sparse_pool_tokens=65536)
    assert not r["feasible"] and r["selected"] is None and "hbm_budget" in r["limiting_constraints"]
    assert "minimum_device_pool" in pl.estimate(sparse_pool_tokens=64, host_arena_tokens=65536)["violated_constraints"]
    with pytest.raises(ValueError):
        pl.estimate(sparse_pool_tokens=4096, host_arena_tokens=100)
    with pytest.raises(ValueError):
        pl.max_device_capacity(host_arena_tokens=64)
    with pytest.raises(ValueError):
        _planner(scheme="hbm")
    with pytest.raises(ValueError):
        _planner(hbm_fraction=1.5)


def test_allocator_tail():
    assert allocator_tail(0) == 0
    assert allocator_tail(512) == 0 and allocator_tail(513) == 511
    assert allocator_tail(3 << 20) == 1 << 20


def test_capacity_cli(capsys):
    import json

    from cxldsagr_b200.models.deepseek_v32.capacity import main

    main(["--num-layers", "3", "--history", "65536", "--candidate", "1280", "--fixed-p", "65536", "--dram-gib", "64"])
    out = json.loads(capsys.readouterr().out)
    assert out["feasible"] and out["max_full_sessions"] == out["max_host_arena_tokens"] // 65536
    main(["--num-layers", "3", "--history", "65536", "--candidate", "1280", "--fixed-nh", "262144",
          "--total-hbm-gib", "40", "--model-hbm-gib", "20"])
    out = json.loads(capsys.readouterr().out)
    assert out["useful_max_P"] <= 262144
