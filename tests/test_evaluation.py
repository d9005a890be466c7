"""CPU tests: provenance, receipts, cache memory audit, serving comparison."""

import json

import pytest
import torch

from cxldsagr_b200.cache.capacity import CacheFootprint
from cxldsagr_b200.evaluation import cache_memory_audit as audit
from cxldsagr_b200.evaluation import provenance, serving_comparison, validation


def test_source_snapshot_and_verify():
    snap = provenance.source_snapshot()
    assert "bench.py" in snap["files"] and any(p.endswith("gemm_fp8.cuh") for p in snap["files"])
    assert provenance.verify_source_snapshot(snap) == []
    fake = {"files": dict(snap["files"])}
    fake["files"]["bench.py"] = "0" * 64
    assert "bench.py" in provenance.verify_source_snapshot(fake)


def test_numerical_comparison_and_evidence(tmp_path):
    a = torch.arange(6.0).view(2, 3)
    r = provenance.numerical_comparison(a + 1e-6, a, atol=1e-5, rtol=0)
    assert r["ok"] and not r["bitwise"]
    assert not provenance.numerical_comparison(a, a.t(), atol=1, rtol=1)["ok"]
    rec = provenance.save_numerical_evidence(tmp_path, name="x", tensors={"logits": a})
    assert rec["logits"]["shape"] == [2, 3] and (tmp_path / "x.logits.pt").exists()


def test_receipts_bind_identity(tmp_path):
    cfg = {"model": "tiny", "steps": 3}
    validation.write_receipt(tmp_path / "check.json", "check", cfg)
    assert validation.require_receipt(tmp_path / "check.json", "check", cfg)["kind"] == "check"
    with pytest.raises(ValueError):
        validation.require_receipt(tmp_path / "check.json", "check", {"model": "other"})
    with pytest.raises(FileExistsError):
        validation.write_receipt(tmp_path / "check.json", "check", cfg)
    with pytest.raises(FileNotFoundError):
        validation.require_receipt(tmp_path / "bench.json", "bench", cfg)
    assert validation.without_performance({"latency_ms": 1, "hits": 2}) == {"hits": 2}


def test_storage_inventory_counts_storages_once():
    base = torch.zeros(100, dtype=torch.uint8)
    inv = audit.storage_inventory({"shared_pool.a": base, "shared_pool.alias": base[10:], "session.x": torch.zeros(8)})
    assert inv["shared_pool"]["dram"] == 100 and inv["session"]["dram"] == 32
    rep = audit.CacheMemoryAudit({"session": CacheFootprint(0, 16)}).check(inv)
    assert not rep["ok"] and rep["violations"][0]["category"] == "session"


class _FakeAllocator:
    """Caching-allocator counters driven by the test (current, peak, cumulative)."""

    def __init__(self):
        self.cur = self.peak = self.cum = 0

    def alloc(self, n):
        self.cur += n
        self.cum += n
        self.peak = max(self.peak, self.cur)

    def free(self, n):
        self.cur -= n

    def stats(self):
        return {f"{c}.all.{k}": v for c in ("allocated_bytes", "requested_bytes")
                for k, v in (("current", self.cur), ("peak", self.peak), ("allocated", self.cum))}

    def reset(self):
        self.peak = self.cur


def test_scope_memory_tracker_nested_peaks():
    fa = _FakeAllocator()
    tr = audit.ScopeMemoryTracker(stats_fn=fa.stats, reset_fn=fa.reset)
    fa.alloc(1000)                      # live before any scope
    with tr("attention"):
        fa.alloc(100)
        with tr("indexer_select"):
            fa.alloc(500)
            fa.free(500)
        fa.alloc(50)                    # retained by attention
        with tr("sparse_mla"):
            fa.alloc(200)
            fa.free(200)
        fa.free(100)
    with tr("indexer_select"):
        fa.alloc(700)
        fa.free(700)
    rows = tr.summary()
    assert rows["indexer_select"] == {"calls": 2, "peak_transient": 700, "retained": 0, "allocated": 1200,
                                      "block_peak_transient": 700}
    assert rows["sparse_mla"]["peak_transient"] == 200
    # the child's peak (1000 + 100 + 500) counts for the enclosing scope
    assert rows["attention"]["peak_transient"] == 600 and rows["attention"]["retained"] == 50
    al = audit.WorkspaceAllowance(selection=600, attention=10_000, metadata=0)
    rep = audit.audit_scopes(rows, al)
    assert rep["violations"] == ["indexer_select"] and not rep["ok"]
    assert rep["checked"]["sparse_mla"]["component"] == "attention"


def test_workspace_allowance_terms():
    from cxldsagr_b200.config import v32_config

    cfg = v32_config(1)
    fused = audit.WorkspaceAllowance.for_chunk(cfg, queries=2048, context=65536)
    plain = audit.WorkspaceAllowance.for_chunk(cfg, queries=2048, context=65536, fused_select=False)
    cands = 2048 * 8192 * 8
    assert fused.selection - plain.selection >= cands                  # candidate lists dominate
    assert fused.selection < cands + 2048 * 65536 * 4 // 8             # far below a logits buffer
    no_buf = audit.WorkspaceAllowance.for_chunk(cfg, queries=2048, context=65536, logits_preallocated=False)
    assert no_buf.selection - fused.selection == 2048 * 65536 * 4
    split = audit.WorkspaceAllowance.for_chunk(cfg, queries=1, context=65536, splits=8)
    one = audit.WorkspaceAllowance.for_chunk(cfg, queries=1, context=65536)
    assert split.attention - one.attention == 8 * 128 * 512 * 4 + 8 * 128 * 4
    fp8 = audit.WorkspaceAllowance.for_chunk(cfg, queries=128, context=65664, offload=True, kv_format="fp8")
    bf16 = audit.WorkspaceAllowance.for_chunk(cfg, queries=128, context=65664, offload=True)
    assert fp8.attention - bf16.attention == (65664 * 656 + 511) // 512 * 512 and fp8.metadata == 3 * 128 * 2048 * 4
    with pytest.raises(ValueError):
        audit.WorkspaceAllowance.for_chunk(cfg, queries=0, context=10)


def test_allocator_blocks_charge_padding():
    snap = [{"device": 0, "address": 4096, "blocks": [
        {"size": 512, "state": "active_allocated"}, {"size": 1536, "state": "inactive"},
        {"size": 2048, "state": "active_allocated"}]}]
    assert audit.allocator_blocks(snap) == {("cuda:0", 4096): 512, ("cuda:0", 6144): 2048}


def test_model_cache_inventory_and_audit_cli(tmp_path):
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig, tiny_config
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model

    cfg = tiny_config()
    m = DeepSeekV32Model(cfg, StateDictSource(random_state_dict(cfg)), device="cpu",
                         cache=CacheConfig(method="serial_sparse", capacity=256, pool_tokens=128, host_tokens=256))
    inv = audit.storage_inventory(audit.model_cache_tensors(m, [m.session]))
    assert inv["shared_pool"]["dram"] > 0 and inv["session"]["dram"] > 0
    log = tmp_path / "run.jsonl"
    rows = [{"status": "started", "scheme": "hbm", "workload_sha256": "w"},
            {"status": "completed", "metrics": {"request_cache_hbm_bytes": 10, "request_cache_dram_bytes": 5,
                                                "hbm_budget_bytes": 100, "dram_budget_bytes": 100,
                                                "latency_ms": 3.0, "is_revisit": False, "prefix_cache_hit": False,
                                                "evicted_users": []}},
            {"status": "completed", "metrics": {"request_cache_hbm_bytes": 10, "request_cache_dram_bytes": 5,
                                                "hbm_budget_bytes": 100, "dram_budget_bytes": 100,
                                                "latency_ms": 1.0, "is_revisit": True, "prefix_cache_hit": True,
                                                "evicted_users": [3]}}]
    log.write_text("\n".join(json.dumps(r) for r in rows))
    assert audit.main([str(log)]) == 0
    res = serving_comparison.compare([serving_comparison.collect_run(str(log))] * 2)
    assert res["same_workload"] and res["runs"][0]["revisit_ms"]["mean"] == 1.0
    assert "| hbm |" in serving_comparison.markdown(res)


def test_cpu_environment_audit():
    from cxldsagr_b200.evaluation.cpu_environment import (cpu_environment, finish_cpu_environment,
                                                          validate_cpu_environment_record)

    meta = {"cpu_environment": cpu_environment()}
    assert meta["cpu_environment"]["affinity"]
    assert finish_cpu_environment(meta) == {"status": "recorded_and_equal"}
    assert validate_cpu_environment_record(meta)["status"] == "recorded_and_equal"
    changed = dict(meta, cpu_environment=dict(meta["cpu_environment"], torch_num_threads=-1))
    with pytest.raises(ValueError):
        finish_cpu_environment(changed)
    assert changed["cpu_environment_audit"]["status"] == "rejected"
    with pytest.raises(ValueError):
        validate_cpu_environment_record({"cpu_environment_audit": {}})


def test_native_build_identity(tmp_path, monkeypatch):
    """The loader refuses an extension whose sources changed since its build."""
    import json as _json
    import shutil

    from cxldsagr_b200.ops import build_identity as bi

    src = tmp_path / "csrc"
    shutil.copytree(bi.ROOT / "csrc", src)
    before = bi.sources_digest(tmp_path)
    (src / "kernels" / "topk.cu").write_text((src / "kernels" / "topk.cu").read_text() + "\n// edit\n")
    after = bi.sources_digest(tmp_path)
    assert before["sha256"] != after["sha256"]
    assert [k for k in before["files"] if before["files"][k] != after["files"][k]] == ["csrc/kernels/topk.cu"]
    if bi.artifact_path() is None or not bi.RECORD.exists():
        pytest.skip("extension not built here")
    rec = _json.loads(bi.RECORD.read_text())
    rec["sources"]["sha256"] = "0" * 64
    fake = tmp_path / "_C.build.json"
    fake.write_text(_json.dumps(rec))
    monkeypatch.setattr(bi, "RECORD", fake)
    with pytest.raises(RuntimeError, match="stale"):
        bi.verify()


def test_bench_scope_flops():
    """bench.py's per-scope FLOP model: causal indexer pairs, top-2048 MLA keys, achieved TFLOP/s."""
    import importlib.util
    from pathlib import Path

    from cxldsagr_b200.config import v32_config

    spec = importlib.util.spec_from_file_location("bench_mod", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cfg = v32_config(1)
    f = bench.prefill_scope_flops(cfg, 4096, 1)
    keys = sum(min(2048, p + 1) for p in range(2048)) + 2048 * 2048
    assert f["sparse_mla"] == 2.0 * 128 * keys * (576 + 512)
    assert f["indexer"] == 2.0 * 64 * 128 * 4096 * 4097 / 2
    r = bench.scope_rooflines({"indexer": {"ms": 1.0}}, f)
    assert r["indexer"]["tflops"] == round(f["indexer"] / 1e9, 1) and "sparse_mla" not in r


def test_roofline_fraction():
    from cxldsagr_b200.evaluation.kernel_bench import _peaks, roofline

    pk = _peaks()
    r = roofline(2.0, nbytes=pk["hbm_gbs"] * 1e6)            # 1 ms of copy bandwidth in 2 ms
    assert r["bound"] == "memory" and abs(r["frac_of_roofline"] - 0.5) < 1e-9
    r = roofline(1.0, flops=4500e9, fp8=True)                 # 1 ms at nominal FP8 in 1 ms
    assert r["bound"] == "compute" and abs(r["frac_of_roofline"] - 1.0) < 1e-9


def test_shape_matrix_table_and_reference_cells():
    from cxldsagr_b200.evaluation import shape_matrix as sm

    rows = [{"history": 16384, "extend": 128, "method": "hbm", "prefill_ms": 100.0, "extend_ms": 1.5,
             "h200_extend_ms": sm.REFERENCE_H200[(16384, 128)]["hbm"][1], "extend_speedup_vs_h200": 1.75}]
    text = sm.table(rows)
    assert "| 16384 | 128 | hbm | 100.0 | 1.500 | 2.623 | 1.75x |" in text
    assert set(sm.REFERENCE_H200[(65536, 128)]) == set(sm.METHODS)
    assert sm._ints("4096,16384") == [4096, 16384]


def test_shape_matrix_bench_requires_matching_check_receipt(tmp_path):
    from cxldsagr_b200.evaluation import shape_matrix as sm
    from cxldsagr_b200.evaluation import validation as val

    args = ["--histories", "4096", "--extends", "128", "--methods", "hbm,serial_sparse", "--layers", "1"]
    with pytest.raises(SystemExit):
        sm.main(args + ["--mode", "bench"])
    with pytest.raises(FileNotFoundError):
        sm.main(args + ["--mode", "bench", "--receipt", str(tmp_path / "none.json")])
    other = {"harness": "shape_matrix", "histories": [4096], "extends": [128], "methods": ["hbm"], "layers": 1,
             "kv_format": "bf16"}
    val.write_receipt(tmp_path / "r.json", "check", other, {"H4096/A128/hbm": {"equal_to_hbm": True}})
    with pytest.raises(ValueError):  # receipt of another method list
        sm.main(args + ["--receipt", str(tmp_path / "r.json")])
