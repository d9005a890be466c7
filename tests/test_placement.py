"""Layer placement over several devices of one process: the contiguous
min-max planner and a tiny model placed over two (CPU) devices, which must
give the single-device logits bitwise for the resident and offload methods."""

import pytest
import torch

from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
from cxldsagr_b200.config import CacheConfig, tiny_config
from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model
from cxldsagr_b200.parallel.placement import device_budgets, layer_weight_bytes, plan_layer_devices


def test_planner_balances_contiguous_runs():
    assert plan_layer_devices([1, 1, 8, 8, 8], [0, 1, 2], [3, 16, 8]) == [0, 0, 1, 1, 2]
    assert plan_layer_devices([2, 2], [7], [4]) == [7, 7]
    assert plan_layer_devices([4, 4, 4, 4], ["a", "b"], [100, 100]) == ["a", "a", "b", "b"]
    # every device gets at least one layer
    assert plan_layer_devices([10, 1, 1], [0, 1, 2], [100, 100, 100]) == [0, 1, 2]


def test_planner_rejects_what_does_not_fit():
    with pytest.raises(RuntimeError, match="cannot hold"):
        plan_layer_devices([5, 5, 5], [0, 1], [9, 9])
    with pytest.raises(ValueError):
        plan_layer_devices([1], [0, 1], [9, 9])
    with pytest.raises(ValueError):
        plan_layer_devices([1, 1], [0, 1], [9])


def test_layer_bytes_and_budgets():
    cfg = tiny_config()
    fp8 = layer_weight_bytes(cfg, 0, fp8=True)
    bf16 = layer_weight_bytes(cfg, 0, fp8=False)
    assert 0 < fp8 < bf16
    b = device_budgets([torch.device("cpu"), torch.device("cpu")], 1 << 30, (10, 20))
    assert b[0] == (1 << 62) - 10 and b[1] == (1 << 62) - 20


@pytest.fixture(scope="module")
def tiny():
    cfg = tiny_config()
    return cfg, StateDictSource(random_state_dict(cfg, seed=0))


def _model(cfg, src, method, devices=None, **kw):
    cache = CacheConfig(method=method, capacity=1024 + 64, chunk_size=256, candidate_tokens=16, **kw)
    return DeepSeekV32Model(cfg, src, device="cpu", cache=cache, devices=devices)


@pytest.mark.parametrize("method", ["hbm", "serial_sparse", "echo"])
def test_placed_model_matches_single_device(tiny, method):
    cfg, src = tiny
    kw = {} if method == "hbm" else {"pool_tokens": 256, "host_tokens": 1024 + 64}
    g = torch.Generator().manual_seed(5)
    hist = torch.randint(0, cfg.vocab_size, (768,), generator=g)
    cand = torch.randint(0, cfg.vocab_size, (16,), generator=g)
    one = _model(cfg, src, method, **kw)
    two = _model(cfg, src, method, devices=["cpu:0", "cpu:1"], **kw)
    assert len(set(two.placement)) == 2 and two.placement[0] == torch.device("cpu:0")
    if method != "hbm":
        assert len(two.pools) == 2
        assert sum(p.num_layers for p in two.pools) == len(two.layer_ids)
    assert torch.equal(one.prefill(hist).logits, two.prefill(hist).logits)
    assert torch.equal(one.candidate(cand).logits, two.candidate(cand).logits)
    assert torch.equal(one.extend(cand).logits, two.extend(cand).logits)
    two.session.release()


def test_placement_rejects_unsupported_modes(tiny):
    cfg, src = tiny
    with pytest.raises(ValueError):
        _model(cfg, src, "dense_prefetch", devices=["cpu:0", "cpu:1"], pool_tokens=512, host_tokens=1024 + 64)


@pytest.mark.gpu
def test_placed_model_two_gpus():
    """Layers over two GPUs match one GPU (same kernels, rows handed over between devices)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from cxldsagr_b200.config import v32_config

    cfg = v32_config(2)
    d0, d1 = torch.device("cuda", 0), torch.device("cuda", 1)
    src = StateDictSource(random_state_dict(cfg, layers=[0, 1], seed=0, device=d0))
    g = torch.Generator().manual_seed(0)
    hist = torch.randint(0, cfg.vocab_size, (2048,), generator=g).to(d0)
    ext = torch.randint(0, cfg.vocab_size, (16,), generator=g).to(d0)
    outs = []
    for devices in (None, [d0, d1]):
        cache = CacheConfig(method="serial_sparse", capacity=2048 + 64, chunk_size=1024, candidate_tokens=16,
                            pool_tokens=2048 + 64, host_tokens=2048 + 64)
        m = DeepSeekV32Model(cfg, src, device=d0, cache=cache, devices=devices)
        if devices:
            assert m.placement == [d0, d1] and m.lm_head.device == d1
        outs.append((m.prefill(hist).logits.to(d0), m.extend(ext).logits.to(d0)))
        torch.cuda.synchronize(d0)
        del m
    torch.testing.assert_close(outs[0][0], outs[1][0], rtol=0, atol=0)
    torch.testing.assert_close(outs[0][1], outs[1][1], rtol=0, atol=0)
