"""Fused peer-memory GEMMs on 2+ GPUs against the NCCL baseline.

Runs as child processes (one per GPU, NCCL + CUDA IPC symmetric heap).  Every
device wait in the fused kernels is bounded, so a broken protocol surfaces as
an error word, not a hang.  NVLS stays off (``NCCL_NVLS_ENABLE=0``): the
fused kernels use plain peer stores and the baseline needs no switch reduction.
"""

import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _entry(fn, rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        q.put((rank, fn(rank, world)))
    except BaseException as exc:  # noqa: BLE001
        import traceback

        q.put(f"rank {rank}: {exc!r}\n{traceback.format_exc()}")
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _spawn(fn, world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    errs = [o for o in out if isinstance(o, str)]
    assert not errs, errs[0]
    return dict(out)


def _fused_vs_nccl(rank, world):
    from cxldsagr_b200 import ops
    from cxldsagr_b200.models.deepseek_v32.weights import Linear
    from cxldsagr_b200.ops.native import check_errors
    from cxldsagr_b200.parallel.comm import Comm
    from cxldsagr_b200.parallel.groups import init_distributed
    from cxldsagr_b200.parallel.p2p import P2PComm

    ctx = init_distributed(timeout_s=60, comm="p2p")
    dev = ctx.device
    fused, base = P2PComm(ctx), Comm(ctx)
    g = torch.Generator(device=dev).manual_seed(1234)  # same weights on every rank

    def weight(n, k):
        from cxldsagr_b200.checkpoint import quantize_weight_blocks

        w = torch.randn((n, k), generator=g, device=dev) * 0.05
        q, s = quantize_weight_blocks(w, (128, 128))
        return Linear(q.contiguous(), s.float().contiguous())

    report = {}
    torch.manual_seed(100 + rank)
    T, K = 1024, 7168
    S = T // world
    shapes = [(2304, K), (4608, K), (2304, K), (4608, K), (2304, K)]   # alternate shapes: exercises parity / reuse
    for i, (N, Kd) in enumerate(shapes):
        lin = weight(N, Kd)
        x = torch.randn((S, Kd), device=dev).bfloat16()
        q, s_t = ops.quantize_act(x)
        a = fused.ag_linear(lin, x, (q, s_t), T)
        b = base.ag_linear(lin, x, (q, s_t), T)
        torch.cuda.synchronize()
        check_errors(dev)
        report[f"ag{i}_maxdiff"] = (a.float() - b.float()).abs().max().item()
    for i, N in enumerate([7168, 2304, 7168, 2304, 7168]):
        lin = weight(N, 2304)
        h = torch.randn((T, 2304), device=dev).bfloat16()
        q, s_t = ops.quantize_act(h)
        a = fused.linear_rs(lin, h, (q, s_t))
        b = base.linear_rs(lin, h, (q, s_t))
        torch.cuda.synchronize()
        check_errors(dev)
        report[f"rs{i}_maxdiff"] = (a.float() - b.float()).abs().max().item()
        report[f"rs{i}_scale"] = b.float().abs().max().item()
    report["fused_calls"] = dict(fused.fused_calls)

    # Device time, max over ranks (CUDA events, warm-up first).
    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        import torch.distributed as dist

        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    lin = weight(2304, K)
    x = torch.randn((S, K), device=dev).bfloat16()
    qx = ops.quantize_act(x)
    report["ag_fused_ms"] = timed(lambda: fused.ag_linear(lin, x, qx, T))
    report["ag_nccl_ms"] = timed(lambda: base.ag_linear(lin, x, qx, T))
    lin = weight(7168, 18432 // world)
    h = torch.randn((T, 18432 // world), device=dev).bfloat16()
    qh = ops.quantize_act(h)
    report["rs_fused_ms"] = timed(lambda: fused.linear_rs(lin, h, qh))
    report["rs_nccl_ms"] = timed(lambda: base.linear_rs(lin, h, qh))
    torch.cuda.synchronize()
    check_errors(dev)
    fused.close()
    return report


@pytest.mark.parametrize("world", [2])
def test_fused_ag_rs_match_nccl(world):
    _need(world)
    reports = _spawn(_fused_vs_nccl, world)
    for rank, rep in reports.items():
        print(rank, rep)
        assert rep["fused_calls"] == {"ag": 5, "rs": 5}
        for k, v in rep.items():
            if k.startswith("ag") and k.endswith("maxdiff"):
                assert v == 0.0, (k, v)
            if k.startswith("rs") and k.endswith("maxdiff"):
                assert v <= 1e-2 * max(1.0, rep[k.replace("maxdiff", "scale")]), (k, v)


def _model_backends(rank, world):
    """Layers 0 (dense) and 3 (MoE, reduced expert count) of a V3.2-shaped model:
    the fused peer-memory backend (AG-GEMM, GEMM-RS, EP dispatch/combine) against
    the NCCL baseline, both sequence/expert parallel on the same ranks."""
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig, v32_config
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model
    from cxldsagr_b200.ops.native import check_errors
    from cxldsagr_b200.parallel.groups import ParallelContext, init_distributed

    base = init_distributed(timeout_s=60, comm="torch")
    dev = base.device
    cfg = v32_config(4, n_routed_experts=16, n_group=8, topk_group=4, num_experts_per_tok=4,
                     moe_intermediate_size=512)
    layers = [0, 3]
    per = cfg.n_routed_experts // world
    src = StateDictSource(random_state_dict(cfg, layers=layers, seed=0, device=dev,
                                            experts=range(rank * per, (rank + 1) * per)), cfg)
    cache = CacheConfig(capacity=2048 + 64, chunk_size=1024, candidate_tokens=64)
    fused_ctx = ParallelContext(base.rank, base.world, base.group, dev, backend="p2p")
    m_nccl = DeepSeekV32Model(cfg, src, device=dev, cache=cache, layers=layers, parallel=base)
    m_p2p = DeepSeekV32Model(cfg, src, device=dev, cache=cache, layers=layers, parallel=fused_ctx)
    g = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (2048 + 64,), generator=g, device=dev)
    out = {}
    for name, m in (("nccl", m_nccl), ("p2p", m_p2p)):
        a = m.prefill(ids[:2048]).logits
        b = m.forward(ids[2048:], transient=True, return_hidden=True)
        torch.cuda.synchronize()
        check_errors(dev)
        out[name] = (a.float().cpu(), b.logits.float().cpu(), b.hidden.float().cpu())
    calls = dict(m_p2p.comm.fused_calls)
    m_p2p.comm.close()

    def corr(x, y):
        return torch.corrcoef(torch.stack([x.flatten().double(), y.flatten().double()]))[0, 1].item()

    return {"calls": calls,
            "prefill_maxdiff": (out["nccl"][0] - out["p2p"][0]).abs().max().item(),
            "prefill_scale": out["nccl"][0].abs().max().item(),
            "prefill_corr": corr(out["nccl"][0], out["p2p"][0]),
            "cand_corr": corr(out["nccl"][1], out["p2p"][1]),
            "hidden_corr": corr(out["nccl"][2], out["p2p"][2]),
            "finite": bool(torch.isfinite(out["p2p"][1]).all())}


@pytest.mark.parametrize("world", [2])
def test_model_fused_backend_matches_nccl(world):
    _need(world)
    reports = _spawn(_model_backends, world)
    for rank, rep in reports.items():
        print(rank, rep)
        assert rep["finite"]
        assert rep["calls"].get("ag", 0) > 0 and rep["calls"].get("rs", 0) > 0 and rep["calls"].get("ep", 0) > 0
        assert rep["cand_corr"] > 0.999 and rep["hidden_corr"] > 0.999
        # The fused reduce-scatter sums rank slots in a fixed order, NCCL in its
        # own: the prefill logits agree to BF16 accumulation-order noise.
        assert rep["prefill_corr"] > 0.999
        assert rep["prefill_maxdiff"] <= 5e-2 * rep["prefill_scale"]


def _sp_extend_graph(rank, world):
    """A sequence-parallel extend (AG-GEMM / GEMM-RS, vocabulary-parallel
    embedding and LM head) captured in one CUDA graph per rank: replays give
    the eager extend's logits bit for bit, for the fused peer-memory backend
    (call state in device memory) and for the NCCL baseline."""
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig, v32_config
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model
    from cxldsagr_b200.ops.native import check_errors
    from cxldsagr_b200.parallel.groups import ParallelContext, init_distributed

    base = init_distributed(timeout_s=60, comm="torch")
    dev = base.device
    cfg = v32_config(1)
    src = StateDictSource(random_state_dict(cfg, layers=[0], seed=0, device=dev), cfg)
    cache = CacheConfig(capacity=2048 + 64, chunk_size=1024, candidate_tokens=64)
    g = torch.Generator(device=dev).manual_seed(6)
    ids = torch.randint(0, cfg.vocab_size, (2048 + 64,), generator=g, device=dev)
    out = {}
    for backend in ("p2p", "torch"):
        ctx = base if backend == "torch" else ParallelContext(base.rank, base.world, base.group, dev, backend="p2p")
        m = DeepSeekV32Model(cfg, src, device=dev, cache=cache, layers=[0], parallel=ctx)
        m.prefill(ids[:2048])
        eager = m.extend(ids[2048:]).logits.float().cpu()
        m.session.truncate(2048)
        graph = m.capture_extend(64)
        reps = []
        for _ in range(3):
            reps.append(graph.replay(ids[2048:]).float().cpu())
            graph.rollback()
        torch.cuda.synchronize()
        check_errors(dev)
        del graph
        out[backend] = all(torch.equal(r, eager) for r in reps)
        if hasattr(m.comm, "close"):
            m.comm.close()
        del m
    return out


@pytest.mark.parametrize("world", [2])
def test_sp_extend_cuda_graph(world):
    _need(world)
    reports = _spawn(_sp_extend_graph, world)
    for rank, rep in reports.items():
        print(rank, rep)
        assert rep["p2p"] and rep["torch"]


def _ep_push_vs_pull(rank, world):
    """The expert-parallel combine fused into the down projection (owners push
    rows to the sources' receive slots) equals the pull combine bit for bit."""
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig, v32_config
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model
    from cxldsagr_b200.ops.native import check_errors
    from cxldsagr_b200.parallel.groups import ParallelContext, init_distributed

    base = init_distributed(timeout_s=60, comm="torch")
    dev = base.device
    cfg = v32_config(4, n_routed_experts=16, n_group=8, topk_group=4, num_experts_per_tok=4,
                     moe_intermediate_size=512)
    layers = [0, 3]
    per = cfg.n_routed_experts // world
    src = StateDictSource(random_state_dict(cfg, layers=layers, seed=0, device=dev,
                                            experts=range(rank * per, (rank + 1) * per)), cfg)
    cache = CacheConfig(capacity=2048 + 64, chunk_size=1024, candidate_tokens=64)
    ctx = ParallelContext(base.rank, base.world, base.group, dev, backend="p2p")
    m = DeepSeekV32Model(cfg, src, device=dev, cache=cache, layers=layers, parallel=ctx)
    g = torch.Generator(device=dev).manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (2048 + 64,), generator=g, device=dev)
    out = {}
    for push in (True, False, True):
        m.comm.ep_push = push
        m.reset()
        a = m.prefill(ids[:2048]).logits.float().cpu()
        b = m.extend(ids[2048:]).logits.float().cpu()
        torch.cuda.synchronize()
        check_errors(dev)
        out.setdefault(push, []).append((a, b))
    calls = dict(m.comm.fused_calls)
    m.comm.close()
    pull = out[False][0]
    return {"calls": calls,
            "equal": all(torch.equal(x[0], pull[0]) and torch.equal(x[1], pull[1]) for x in out[True]),
            "finite": bool(torch.isfinite(pull[1]).all())}


@pytest.mark.parametrize("world", [2])
def test_ep_push_combine_matches_pull(world):
    _need(world)
    reports = _spawn(_ep_push_vs_pull, world)
    for rank, rep in reports.items():
        print(rank, rep)
        assert rep["finite"] and rep["calls"].get("ep", 0) > 0
        assert rep["equal"]
