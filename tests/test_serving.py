"""CPU tests: executor contracts, token runtime, DeepSeek serving backend, persistent GR runner."""

from dataclasses import replace

import pytest
import torch

from cxldsagr_b200.cache.capacity import CacheBudgetExceeded, CapacityPolicy, CacheFootprint
from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
from cxldsagr_b200.config import tiny_config
from cxldsagr_b200.executor.contracts import ExecutionLimits, OutputSpec, RequestShape
from cxldsagr_b200.executor.model_executor import run_chunks
from cxldsagr_b200.executor.runtime import TokenRuntime
from cxldsagr_b200.gr.workload import WorkloadConfig, build_workload
from cxldsagr_b200.models.deepseek_v32.serving import DeepSeekServingBackend
from cxldsagr_b200.serving.persistent import PersistentGRRunner, token_digest

HIST, CAND = 384, 48


@pytest.fixture(scope="module")
def tiny3():
    cfg = tiny_config(num_hidden_layers=3, first_k_dense_replace=3)
    return cfg, StateDictSource(random_state_dict(cfg, seed=3))


def _backend(tiny3, scheme, **kw):
    cfg, src = tiny3
    opts = dict(sparse_pool_tokens=256, chunk_size=128, candidate_tokens=64, workspace_query_tokens=128)
    opts.update(kw)
    return DeepSeekServingBackend(source=src, cfg=cfg, scheme=scheme, device="cpu", num_layers=4, **opts)


def _requests(n_users=3, count=6, seed=0):
    wl = build_workload(WorkloadConfig("deepseek_v32", n_users, count, history_tokens=HIST, candidate_tokens=CAND,
                                       seed=seed))
    return list(wl.requests)


LIMITS = {"max_session_capacity": HIST + CAND, "max_history_tokens": HIST, "max_candidate_tokens": CAND}


def test_contract_validation():
    with pytest.raises(ValueError):
        RequestShape(0, 1)
    lim = ExecutionLimits.from_mapping({"max_session_capacity": 100, "max_candidate_tokens": 10}, context=200,
                                       chunk_size=16)
    assert lim.request_tokens == 100 and lim.candidate_tokens == 10 and lim.history_tokens == 100
    with pytest.raises(ValueError):
        lim.validate(RequestShape(95, 10))
    with pytest.raises(ValueError):
        OutputSpec(logits="last")
    assert OutputSpec(logits="last", run_lm_head=True).logits == "last"


class _TinyLM:
    class config:
        max_position_embeddings = 64

    def __call__(self, chunk, cache, return_hidden=False, logits_to_keep=0):
        cache.length += chunk.numel()
        return chunk.float()[:, None] if return_hidden else chunk.float()[-max(logits_to_keep, 1):, None]


def test_run_chunks_feeds_every_token():
    class Cache:
        length, max_seq_len = 0, 64

    c = Cache()
    out = run_chunks(_TinyLM(), torch.arange(10), c, 4)
    assert c.length == 10 and out.shape == (2, 1)
    with pytest.raises(ValueError):
        run_chunks(_TinyLM(), torch.arange(100), Cache(), 4)


def test_backend_prefill_candidate_matches_plain_model(tiny3):
    backend = _backend(tiny3, "serial_sparse")
    runtime = TokenRuntime(backend.runtime_driver(CapacityPolicy.byte_budget(CacheFootprint(1 << 30, 1 << 30))))
    plan = runtime.plan_resources(CapacityPolicy.byte_budget(CacheFootprint(1 << 30, 1 << 30)), LIMITS)
    runtime.allocate_resources(plan)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 150, (HIST + CAND,), generator=g)
    splan = runtime.plan_session(RequestShape(HIST, CAND), "u0")
    s = runtime.create_session(splan)
    runtime.prefill(s, ids[:HIST])
    stages = []
    r1 = runtime.candidate(s, ids[HIST:], observer=stages.append)
    r2 = runtime.candidate(s, ids[HIST:])
    assert stages == ["executed", "cleaned"]
    assert r1.hidden.shape == (CAND, tiny3[0].dim)
    assert torch.equal(r1.hidden, r2.hidden)
    # Same request on the resident scheme gives bitwise identical hidden states.
    hbm = _backend(tiny3, "hbm")
    rt2 = TokenRuntime(hbm.runtime_driver(CapacityPolicy.byte_budget(CacheFootprint(1 << 30, 1 << 30))))
    p2 = rt2.plan_resources(CapacityPolicy.byte_budget(CacheFootprint(1 << 30, 1 << 30)), LIMITS)
    rt2.allocate_resources(p2)
    s2 = rt2.create_session(rt2.plan_session(RequestShape(HIST, CAND), "u0"))
    rt2.prefill(s2, ids[:HIST])
    assert torch.equal(rt2.candidate(s2, ids[HIST:]).hidden, r1.hidden)
    runtime.release_session(s)
    rt2.release_session(s2)


def test_failed_session_cannot_execute(tiny3, monkeypatch):
    backend = _backend(tiny3, "hbm")
    pol = CapacityPolicy.byte_budget(CacheFootprint(1 << 30, 1 << 30))
    rt = TokenRuntime(backend.runtime_driver(pol))
    rt.allocate_resources(rt.plan_resources(pol, LIMITS))
    s = rt.create_session(rt.plan_session(RequestShape(HIST, CAND), "x"))
    ids = torch.randint(0, 150, (HIST + CAND,))
    rt.prefill(s, ids[:HIST])
    block = backend.model.blocks[1]

    def boom(*a, **k):
        raise RuntimeError("injected")

    monkeypatch.setattr(block, "forward", boom)
    with pytest.raises(RuntimeError, match="injected"):
        rt.candidate(s, ids[HIST:])
    monkeypatch.undo()
    assert s.length == HIST  # rolled back
    with pytest.raises(RuntimeError):
        rt.candidate(s, ids[HIST:])
    rt.release_session(s)


@pytest.mark.parametrize("scheme", ["hbm", "serial_sparse", "echo"])
def test_persistent_runner_reuses_prefix_and_matches_across_schemes(tiny3, scheme):
    reqs = _requests()
    outs = {}
    for sch in ("hbm", scheme):
        backend = _backend(tiny3, sch)
        with PersistentGRRunner(backend, hbm_budget_bytes=1 << 30, dram_budget_bytes=1 << 30,
                                resource_limits=LIMITS, native_token_validation=True) as runner:
            results = list(runner.run(reqs))
        outs[sch] = results
    for a, b in zip(outs["hbm"], outs[scheme]):
        assert torch.equal(a.hidden, b.hidden)
    ms = [r.metrics for r in outs[scheme]]
    assert [m["prefix_cache_hit"] for m in ms] == [m["is_revisit"] for m in ms]
    assert all(m["latency_ms"] > 0 and m["candidate_suffix_tokens"] == CAND for m in ms)


def test_persistent_runner_lru_eviction_under_budget(tiny3):
    backend = _backend(tiny3, "hbm")
    # Budget for the shared workspace plus about two sessions.
    probe = _backend(tiny3, "hbm")
    shared = probe.plan_resources(CacheFootprint(1 << 40, 1 << 40), LIMITS).shared
    one = CacheFootprint.from_mapping(probe.estimate_session_bytes(HIST))
    budget = shared + one + one
    reqs = [r for r in _requests(n_users=3, count=12, seed=5)]
    with PersistentGRRunner(backend, hbm_budget_bytes=budget.hbm, dram_budget_bytes=budget.dram + 1,
                            resource_limits=LIMITS) as runner:
        ms = [res.metrics for res in runner.run(reqs)]
    assert max(m["cached_users"] for m in ms) <= 2
    if len({m["user_id"] for m in ms}) == 3:
        assert sum(len(m["evicted_users"]) for m in ms) > 0


def test_runner_rejects_bad_requests(tiny3):
    backend = _backend(tiny3, "hbm")
    with PersistentGRRunner(backend, hbm_budget_bytes=1 << 30, dram_budget_bytes=1 << 30,
                            resource_limits=LIMITS) as runner:
        with pytest.raises(ValueError):
            runner.execute({"user_id": 1, "input_ids": [1, -2, 3], "stable_prefix_tokens": 1})
        with pytest.raises(ValueError):
            runner.execute({"user_id": 1, "input_ids": [1, 2, 3], "stable_prefix_tokens": 3})
        with pytest.raises(TypeError):
            runner.execute({"user_id": True, "input_ids": [1, 2], "stable_prefix_tokens": 1})


def test_fixed_pools_admission(tiny3):
    backend = _backend(tiny3, "serial_sparse", host_arena_tokens=2 * 448)
    reqs = _requests(n_users=3, count=6, seed=2)
    with PersistentGRRunner(backend, resource_limits=LIMITS) as runner:
        ms = [r.metrics for r in runner.run(reqs)]
    assert all(m["resource_mode"] == "fixed_pools" for m in ms)
    assert max(m["cache_host_pages"] for m in ms) <= 2 * 448 // 64
    with pytest.raises(CacheBudgetExceeded):
        PersistentGRRunner(_backend(tiny3, "serial_sparse", host_arena_tokens=64), resource_limits=LIMITS)


def test_token_digest_is_little_endian_int64():
    import hashlib
    import struct

    ids = [1, 2, 2**40]
    assert token_digest(ids) == hashlib.sha256(struct.pack("<3q", *ids)).hexdigest()


def test_borrowed_caches_mutate_only_inside_their_operation(tiny3):
    """A backend session's KV caches refuse mutation outside the backend's operation on that session."""
    backend = _backend(tiny3, "serial_sparse")
    runtime = TokenRuntime(backend.runtime_driver(CapacityPolicy.byte_budget(CacheFootprint(1 << 30, 1 << 30))))
    runtime.allocate_resources(runtime.plan_resources(CapacityPolicy.byte_budget(CacheFootprint(1 << 30, 1 << 30)),
                                                      LIMITS))
    s = runtime.create_session(runtime.plan_session(RequestShape(HIST, CAND), "u0"))
    runtime.prefill(s, torch.randint(0, 150, (HIST,), generator=torch.Generator().manual_seed(1)))
    model_session = next(iter(backend.lifecycle.sessions))
    kv = model_session.layers[0].kv
    with pytest.raises(RuntimeError, match="active operation"):
        kv.begin_step(1)
    with pytest.raises(RuntimeError, match="active operation"):
        kv.truncate(0)
    assert model_session.length == HIST
    runtime.release_session(s)
