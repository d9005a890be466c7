"""CPU tests: capacity types, LRU admission, lifecycle leases, resident caches, staging, host backing."""

import threading

import pytest
import torch

from cxldsagr_b200.cache.capacity import (
    AllocationSpec,
    CacheBudgetExceeded,
    CacheFootprint,
    CapacityPolicy,
    ResourcePlan,
    SessionPlan,
    allocation_footprint,
)
from cxldsagr_b200.cache.host_backing import HostBackingCache
from cxldsagr_b200.cache.indexer_cache import IndexerCache
from cxldsagr_b200.cache.lifecycle import ResourceLifecycle
from cxldsagr_b200.cache.manager import CacheManager, CacheSpec
from cxldsagr_b200.cache.prefix_pool import PrefixSessionPool
from cxldsagr_b200.cache.staging import DoubleBufferStaging


def _alloc(name, nbytes, *, owner="session", device="cuda:0", group=None, phase=None, alias=None):
    return AllocationSpec(name, owner, "uint8", (nbytes,), device, "session", nbytes,
                          0 if alias else nbytes, alias_of=alias, peak_group=group, phase=phase)


def test_footprint_arithmetic_and_fits():
    a, b = CacheFootprint(10, 20), CacheFootprint(5, 1)
    assert a + b == CacheFootprint(15, 21)
    assert a - b == CacheFootprint(5, 19)
    assert b.fits(a) and not a.fits(b)
    with pytest.raises(ValueError):
        CacheFootprint(-1, 0)
    with pytest.raises(ValueError):
        CapacityPolicy("budget")
    assert CapacityPolicy.fixed_pools().budget is None


def test_allocation_footprint_peak_groups_and_aliases():
    allocs = [
        _alloc("records", 100),
        _alloc("host", 300, device="cpu"),
        _alloc("scratch_prefill", 70, group="scratch", phase="prefill"),
        _alloc("scratch_decode", 40, group="scratch", phase="decode"),
        _alloc("view", 50, alias="records"),
    ]
    assert allocation_footprint(allocs) == CacheFootprint(170, 300)
    with pytest.raises(ValueError):
        allocation_footprint([_alloc("a", 1), _alloc("a", 2)])
    with pytest.raises(ValueError):
        allocation_footprint([_alloc("view", 5, alias="missing")])
    with pytest.raises(ValueError):  # a charge below the storage size is rejected
        AllocationSpec("x", "session", "uint8", (8,), "cuda", "s", 8, 4)


def test_plans_validate():
    plan = ResourcePlan(CacheFootprint(100, 0), metadata={"k": [1, 2]})
    assert plan.metadata["k"] == (1, 2)
    with pytest.raises(TypeError):
        plan.metadata["new"] = 1
    with pytest.raises(ValueError):
        ResourcePlan(CacheFootprint(10, 0), allocations=(_alloc("big", 11, owner="shared"),))
    with pytest.raises(ValueError):
        SessionPlan(object(), "h", 100, 50, CacheFootprint())


class _Sessions:
    def __init__(self):
        self.live, self.released = [], []

    def allocate(self, capacity):
        s = {"capacity": capacity}
        self.live.append(s)
        return s

    def release(self, s):
        self.released.append(s)


def _pool(budget=CacheFootprint(1000, 1000), **kw):
    sessions = _Sessions()
    pool = PrefixSessionPool(budget, allocate=sessions.allocate, release=sessions.release,
                             measure=lambda s: CacheFootprint(10, 0), **kw)
    return pool, sessions


def test_prefix_pool_hit_miss_and_lru_eviction():
    pool, sessions = _pool()
    r = CacheFootprint(400, 0)
    a = pool.acquire("a", "sig", 10, r)
    assert not a.hit
    pool.mark_ready(a)
    b = pool.acquire("b", "sig", 10, r)
    pool.mark_ready(b)
    assert pool.acquire("a", "sig", 10, r).hit  # refreshes a
    c = pool.acquire("c", "sig", 10, r)  # evicts b (least recently used)
    assert c.evicted == ("b",) and "b" not in pool and "a" in pool
    assert sessions.released == [b.session]
    # Stale signature replaces the entry.
    d = pool.acquire("a", "other", 10, r)
    assert not d.hit and pool.misses == 4 and pool.hits == 1
    assert pool.audit()["sessions"] == 2


def test_prefix_pool_impossible_request_keeps_users():
    pool, sessions = _pool()
    a = pool.acquire("a", "s", 10, CacheFootprint(400, 0))
    pool.mark_ready(a)
    with pytest.raises(CacheBudgetExceeded):
        pool.acquire("b", "s", 10, CacheFootprint(2000, 0))
    assert "a" in pool and not sessions.released


def test_prefix_pool_fixed_pools_and_unready_lease():
    pool, _ = _pool(budget=None, host_page_capacity=10)
    a = pool.acquire("a", "s", 64, CacheFootprint(), host_pages=6)
    b = pool.acquire("b", "s", 64, CacheFootprint(), host_pages=6)  # evicts a
    assert "a" not in pool
    with pytest.raises(RuntimeError):
        pool.mark_ready(a)
    pool.mark_ready(b)
    with pytest.raises(CacheBudgetExceeded):
        pool.acquire("c", "s", 64, CacheFootprint(), host_pages=11)
    with pytest.raises(ValueError):
        PrefixSessionPool(None, allocate=None, release=None, measure=None)


def test_prefix_pool_audit_detects_overrun():
    sessions = _Sessions()
    pool = PrefixSessionPool(CacheFootprint(1000, 1000), allocate=sessions.allocate, release=sessions.release,
                             measure=lambda s: {"hbm": 500, "dram": 0})
    pool.acquire("a", "s", 1, CacheFootprint(100, 0))
    with pytest.raises(RuntimeError):
        pool.audit()


def test_lifecycle_operation_is_exclusive_and_non_blocking():
    life = ResourceLifecycle("pool")
    entered, release = threading.Event(), threading.Event()
    errors = []

    def hold():
        with life.operation(kind="prefill"):
            entered.set()
            release.wait(5)

    t = threading.Thread(target=hold)
    t.start()
    entered.wait(5)
    try:
        with life.operation(kind="extend"):
            pass
    except RuntimeError as exc:
        errors.append(str(exc))
    release.set()
    t.join()
    assert errors and "prefill" in errors[0]
    with life.operation():
        pass


def test_lifecycle_drain_failure_poisons():
    def bad_drain():
        raise OSError("drain")

    life = ResourceLifecycle("pool", drain=bad_drain)
    with pytest.raises(BaseExceptionGroup):
        with life.operation():
            raise ValueError("step")
    assert life.poisoned
    with pytest.raises(RuntimeError):
        with life.operation():
            pass


def test_lifecycle_owner_and_close_generation():
    life = ResourceLifecycle("pool")
    owner = object()
    life.bind_owner(owner)
    with pytest.raises(RuntimeError):
        life.bind_owner(object())
    reg = life.register("s")
    assert reg.generation == 0 and reg.owner is owner
    life.close()
    assert life.generation == 1 and not life.sessions
    with pytest.raises(RuntimeError):
        life.register("s2")


def test_resident_cache_manager_transactions():
    mgr = CacheManager([CacheSpec("a", (2,), torch.float32, 8), CacheSpec("b", (), torch.int32, 8)], device="cpu")
    rows = mgr.begin(3)
    mgr["a"].write(rows["a"], torch.ones(3, 2))
    with pytest.raises(ValueError):
        mgr["a"].write(slice(2, 5), torch.ones(3, 2))
    mgr.commit()
    assert mgr["a"].view().shape == (3, 2)
    mgr.begin(2)
    mgr.abort()
    assert mgr["a"].length == 3
    mgr["a"].truncate(1)
    with pytest.raises(ValueError):
        mgr["a"].begin(8)
    assert mgr.nbytes() == 8 * 2 * 4 + 8 * 4


def test_indexer_cache_rows_and_snapshot():
    c = IndexerCache(16, 8, device="cpu")
    k, s = c.rows(4, 4)
    assert k.shape == (4, 8) and s.shape == (4,)
    with pytest.raises(ValueError):
        c.rows(14, 4)
    c.commit(8)
    c.offset[0] = 3.0
    snap = c.snapshot()
    c.offset.zero_()
    c.truncate(2)
    c.restore(snap)
    assert c.length == 8 and c.offset[0] == 3.0
    assert c.record_bytes == 12


def test_staging_double_buffer_cpu():
    st = DoubleBufferStaging(8, 4, device="cpu")
    host = torch.arange(32, dtype=torch.bfloat16).reshape(8, 4)
    l0, l1 = st.lease(), st.lease()
    assert (l0.index, l1.index) == (0, 1)
    assert torch.equal(l0.prefetch(host, 5).wait_ready(), host[:5])
    with pytest.raises(ValueError):
        l1.prefetch(torch.zeros(9, 4), 9)
    assert st.lease().index == 0
    assert st.nbytes() == 2 * 8 * 4 * 2


def test_host_backing_window_and_recall():
    c = HostBackingCache(16, 2, device="cpu", dtype=torch.float32, device_rows=4)
    for step in range(4):
        c.begin(3)
        c.append(torch.full((3, 2), float(step)))
        c.commit()
    assert c.length == 12
    assert torch.equal(c.host[:12, 0], torch.arange(4).repeat_interleave(3).float())
    view = c.ensure_resident(0, 4)
    assert torch.equal(view[:, 0], torch.tensor([0.0, 0, 0, 1]))
    with pytest.raises(ValueError):
        c.ensure_resident(0, 5)
    c.begin(2)
    c.rollback()
    assert c.length == 12


def test_fp8_pool_estimate_matches_allocation():
    """The FP8 pool's byte estimate (656-byte host rows + one recall scratch) equals what it allocates."""
    from cxldsagr_b200.cache.sparse_token_pool import SharedSparseTokenPool

    est = SharedSparseTokenPool.estimate_shared_bytes(1024, 576, 3, 256, device="cpu", candidate_slots=16,
                                                      kv_format="fp8")
    pool = SharedSparseTokenPool(1024, 576, 3, 256, device="cpu", candidate_slots=16, kv_format="fp8")
    got = pool.shared_bytes()
    assert pool.layers[0].host.shape == (1024, 656)
    assert est["hbm"] + est["dram"] == got["hbm"] + got["dram"]
