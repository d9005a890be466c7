"""Host recall dispatch (csrc/host/recall_dispatch.h) on the CPU: each stage's
arguments are validated right before it is enqueued, a failing stage stops
the event (later stages never run) and the error reaches the caller
unchanged; a gather fault is raised after the gather was enqueued."""

import importlib
import subprocess
import sys
import sysconfig
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def probe(tmp_path_factory):
    try:
        return importlib.import_module("cxldsagr_b200.cache._recall_dispatch_probe")
    except ImportError:
        import pybind11

        out = tmp_path_factory.mktemp("probe") / ("_recall_dispatch_probe" + sysconfig.get_config_var("EXT_SUFFIX"))
        subprocess.run(["g++", "-O1", "-std=c++17", "-shared", "-fPIC", f"-I{pybind11.get_include()}",
                        f"-I{sysconfig.get_paths()['include']}", f"-I{ROOT / 'csrc' / 'host'}",
                        str(ROOT / "csrc" / "host" / "recall_dispatch_probe.cpp"), "-o", str(out)], check=True)
        sys.path.insert(0, str(out.parent))
        return importlib.import_module("_recall_dispatch_probe")


def _desc(P=1024, NH=4096, n=2048, dev=0):
    v = lambda dt, k, **kw: {"dtype": dt, "numel": k, "device": dev, **kw}  # noqa: E731
    return {
        "ids": v("i32", n), "page_table": v("i32", NH // 64), "h2d": v("i32", NH), "mark": v("i32", NH),
        "d2h": v("i64", P + 1), "priority": v("i64", P + 1), "meta": v("i64", 144),
        "miss_list": v("i64", P + 1), "victims": v("i64", P + 1), "stats": v("i64", 8), "select_stats": v("i64", 8),
        "host": {"dtype": "bf16", "numel": NH * 576, "ndim": 2, "rows": NH, "row_bytes": 1152, "device": -1,
                 "pinned": True},
        "records": {"dtype": "bf16", "numel": (P + 1) * 576, "ndim": 2, "rows": P + 1, "row_bytes": 1152,
                    "device": dev},
        "hist_end": NH, "k_limit": -1, "count_slot": 1,
    }


def test_stage_order(probe):
    assert probe.run(_desc()) == 123


@pytest.mark.parametrize("stage,trace", [(1, 0), (2, 1), (3, 123)])
def test_fault_injection_stops_later_stages(probe, stage, trace):
    with pytest.raises(RuntimeError, match=f"injected native stage {stage}"):
        probe.run(_desc(), stage)
    assert probe.trace() == trace


@pytest.mark.parametrize("field,change,trace", [
    ("ids", {"dtype": "i64"}, 0),                # classify arguments: nothing launched
    ("mark", {"numel": 7}, 0),
    ("ids", {"device": 1}, 0),
    ("select_stats", {"numel": 2}, 1),           # select arguments: classify already enqueued
    ("host", {"pinned": False}, 12),             # gather arguments: classify + select enqueued
    ("records", {"row_bytes": 1024}, 12),
    ("records", {"rows": 10}, 12),
])
def test_validation_happens_at_the_boundary(probe, field, change, trace):
    d = _desc()
    d[field] = {**d[field], **change}
    with pytest.raises(ValueError, match="recall stage"):
        probe.run(d)
    assert probe.trace() == trace


def test_scalar_checks(probe):
    d = _desc()
    d["hist_end"] = 10**9
    with pytest.raises(ValueError, match="stage 1"):
        probe.validate(d, 1)
    d = _desc()
    d["k_limit"] = -2
    with pytest.raises(ValueError, match="stage 2"):
        probe.validate(d, 2)
    d = _desc()
    d["count_slot"] = 8
    with pytest.raises(ValueError, match="stage 2"):
        probe.validate(d, 2)
    probe.validate(_desc(), 3)
