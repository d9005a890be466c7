"""Rank watchdog on gloo ranks (CPU): a rank that reports a failure, and a rank
whose heartbeat stops, are seen by every other rank on the host before its next
step; healthy ranks never raise."""

import time

import pytest


def _finish(wd, rank, detectors):
    """Rank 0 hosts the store: it leaves only after every detector is done with it."""
    n = wd.store.add(wd.prefix + "/done", 1)
    if rank == 0:
        deadline = time.monotonic() + 10
        while n < detectors and time.monotonic() < deadline:
            time.sleep(0.05)
            n = wd.store.add(wd.prefix + "/done", 0)
    wd.close()

from test_parallel_cpu import _spawn


def _reported(rank, world):
    from cxldsagr_b200.parallel.groups import init_distributed
    from cxldsagr_b200.parallel.watchdog import RankFailure, RankWatchdog

    init_distributed(backend="gloo", timeout_s=30)
    import torch.distributed as dist

    wd = RankWatchdog.for_group(interval_s=0.1, timeout_s=5.0, prefix="t1")
    dist.barrier()
    wd.check()  # everyone healthy
    dist.barrier()  # every rank has checked before rank 1 reports
    if rank == 1:
        try:
            raise ValueError("step failed on rank 1")
        except ValueError as exc:
            wd.report_failure(exc)
        wd.close()
        return None
    deadline = time.monotonic() + 10
    while time.monotonic() < deadline:
        try:
            wd.check()
        except RankFailure as f:
            _finish(wd, rank, world - 1)
            return (f.rank, "step failed" in f.reason)
        time.sleep(0.05)
    wd.close()
    return "not detected"


def _silent(rank, world):
    from cxldsagr_b200.parallel.groups import init_distributed
    from cxldsagr_b200.parallel.watchdog import RankFailure, RankWatchdog

    init_distributed(backend="gloo", timeout_s=30)
    import torch.distributed as dist

    wd = RankWatchdog.for_group(interval_s=0.1, timeout_s=1.0, prefix="t2")
    dist.barrier()
    time.sleep(0.3)
    wd.check()
    if rank == world - 1:
        wd.close()          # the heartbeat stops (a hung or dead host process)
        time.sleep(4.0)     # stay alive so the store outlives the detection
        return None
    deadline = time.monotonic() + 10
    while time.monotonic() < deadline:
        try:
            wd.check()
        except RankFailure as f:
            _finish(wd, rank, world - 1)
            return (f.rank, "no heartbeat" in f.reason)
        time.sleep(0.1)
    wd.close()
    return "not detected"


@pytest.mark.parametrize("world", [3])
def test_reported_failure_reaches_every_rank(world):
    res = dict(_spawn(_reported, world))
    assert res[1] is None
    assert all(res[r] == (1, True) for r in range(world) if r != 1), res


@pytest.mark.parametrize("world", [3])
def test_silent_rank_detected_by_heartbeat(world):
    res = dict(_spawn(_silent, world))
    assert all(res[r] == (world - 1, True) for r in range(world - 1)), res
