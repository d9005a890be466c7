"""Multi-rank (gloo, CPU) tests of the sequence/expert-parallel model and the row collectives.

Each test spawns ``world`` processes; every rank builds the same seeded tiny
model.  The parallel model (hidden rows sharded, attention AG -> GEMM, dense
MLP AG -> GEMM / GEMM -> RS, MoE all-to-all dispatch/combine) must reproduce
the single-process logits and candidate hidden states.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world, *args):
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    errors = [r for r in results if isinstance(r, str)]
    assert not errors, errors[0]
    return sorted(results, key=lambda r: r[0])


def _entry(fn, rank, world, port, q, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        torch.set_num_threads(2)
        out = fn(rank, world, *args)
        q.put((rank, out))
    except BaseException as exc:  # noqa: BLE001 - reported to the parent
        import traceback

        q.put(f"rank {rank}: {exc!r}\n{traceback.format_exc()}")
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _collectives(rank, world):
    from cxldsagr_b200.parallel import collectives as C
    from cxldsagr_b200.parallel.groups import init_distributed, shard_range

    ctx = init_distributed(backend="gloo", timeout_s=60)
    total = 7
    r0, r1 = shard_range(total, world, rank)
    x = torch.arange(total * 3, dtype=torch.float32).view(total, 3)
    g = C.all_gather_rows(ctx, x[r0:r1], total)
    ok_ag = torch.equal(g, x)
    full = x * (rank + 1)
    rs = C.reduce_scatter_rows(ctx, full)
    ok_rs = torch.allclose(rs, x[r0:r1] * sum(range(1, world + 1)))
    send = torch.full((world + rank, 2), float(rank))
    counts = [1] * world
    counts[0] += rank
    recv, rc = C.all_to_all_rows(ctx, send, counts)
    ok_a2a = rc == [1 + (s if rank == 0 else 0) for s in range(world)]
    back = C.all_to_all_back(ctx, recv, rc, counts)
    return ok_ag and ok_rs and ok_a2a and torch.equal(back, send)


@pytest.mark.parametrize("world", [2, 3])
def test_row_collectives(world):
    assert all(ok for _, ok in _spawn(_collectives, world))


def _tiny_cfg():
    from cxldsagr_b200.config import tiny_config

    return tiny_config(num_hidden_layers=4, first_k_dense_replace=2, n_routed_experts=8, n_group=4,
                       topk_group=2, num_experts_per_tok=4)


def _run_model(rank, world, T_hist, T_cand, method, cp=False):
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model
    from cxldsagr_b200.parallel.groups import init_distributed

    ctx = init_distributed(backend="gloo", timeout_s=120)
    ctx.cp_indexer = cp
    cfg = _tiny_cfg()
    src = StateDictSource(random_state_dict(cfg, seed=0))
    cache = CacheConfig(method=method, capacity=T_hist + T_cand, chunk_size=128, candidate_tokens=T_cand,
                        pool_tokens=192 if method != "hbm" else None, host_tokens=T_hist + T_cand)
    model = DeepSeekV32Model(cfg, src, device="cpu", cache=cache, parallel=ctx)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (T_hist + T_cand,), generator=g)
    a = model.prefill(ids[:T_hist]).logits
    b = model.forward(ids[T_hist:], transient=True, return_hidden=True)
    # numpy copies travel by value through the result queue (tensors would share memory with an exiting child)
    return a.numpy().copy(), b.logits.numpy().copy(), b.hidden.float().numpy().copy()


@pytest.mark.parametrize("world,method,cp", [(2, "hbm", False), (4, "serial_sparse", False), (2, "hbm", True),
                                            (4, "serial_sparse", True)])
def test_sequence_expert_parallel_matches_single(world, method, cp):
    """cp: the indexer split by keys across ranks (context-parallel selection)."""
    single = [torch.from_numpy(x) for x in _spawn(_run_model, 1, 300, 24, method)[0][1]]
    par = _spawn(_run_model, world, 300, 24, method, cp)
    def corr(x, y):
        return torch.corrcoef(torch.stack([x.flatten().double(), y.flatten().double()]))[0, 1].item()

    for _, arrays in par:
        a, b, h = (torch.from_numpy(x) for x in arrays)
        # Row-parallel partial sums are rounded to BF16 before the reduction, so
        # results agree to rounding (amplified where it flips a near-tied
        # indexer selection of the random-init model), not bitwise.
        assert h.shape == single[2].shape
        for got, want in ((a, single[0]), (b, single[1])):
            assert (got - want).abs().max() < 0.15 and corr(got, want) > 0.995
        assert corr(h, single[2]) > 0.99


def test_embed_shards_sum_to_full_table():
    from cxldsagr_b200 import ops

    torch.manual_seed(0)
    table = torch.randn(50, 16)
    ids = torch.randint(0, 50, (30,))
    parts = [ops.embed(ids, table[a:b], row0=a, vocab_total=50) for a, b in ((0, 17), (17, 34), (34, 50))]
    assert torch.equal(sum(p.float() for p in parts).bfloat16(), table[ids].bfloat16())
    with pytest.raises(IndexError):
        ops.embed(torch.tensor([50]), table[:10], row0=0, vocab_total=50)
