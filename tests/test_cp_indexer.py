"""Context-parallel indexer: per-rank key shards, local exact top-k, merge.
The merged selection must equal the single-device exact top-k, ties included."""

import pytest
import torch

from cxldsagr_b200 import ops
from cxldsagr_b200.parallel.cp_indexer import key_shard, local_topk, merge_topk

from test_parallel_cpu import _spawn


def _inputs(Q, N, seed, ties, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    if ties:  # few distinct keys -> many equal logits across shards
        base = torch.randn(40, 128, generator=g)
        pick = torch.randint(0, 40, (N,), generator=g)
        keys = base[pick]
        ks = (torch.rand(40, generator=g) + 0.5)[pick]
    else:
        keys = torch.randn(N, 128, generator=g)
        ks = torch.rand(N, generator=g) + 0.5
    q = torch.randn(Q, 64, 128, generator=g)
    w = torch.randn(Q, 64, generator=g)
    to = dict(device=device)
    return (q.to(torch.float8_e4m3fn).to(**to), keys.to(torch.float8_e4m3fn).to(**to), w.to(**to), ks.to(**to))


def _single(q, keys, w, ks, qpos, k):
    logits = ops.indexer_logits(q, keys, w, ks, qpos)
    return ops.exact_topk(logits, k, causal_start=qpos, n=keys.shape[0])


def _emulated(q, keys, w, ks, qpos, k, world):
    vals, ids = [], []
    for r in range(world):
        k0, k1 = key_shard(keys.shape[0], world, r)
        v, i = local_topk(q, keys[k0:k1], w, ks[k0:k1], k0, qpos, k)
        vals.append(v)
        ids.append(i)
    return merge_topk(torch.cat(vals, 1), torch.cat(ids, 1), k)


@pytest.mark.parametrize("world", [1, 2, 3, 5])
@pytest.mark.parametrize("ties", [False, True])
def test_cp_merge_equals_single_device(world, ties):
    Q, N, k = 24, 700, 64
    q, keys, w, ks = _inputs(Q, N, 1 + world, ties)
    qpos = N - Q                       # a prefill chunk at the end of the context
    v1, i1 = _single(q, keys, w, ks, qpos, k)
    v2, i2 = _emulated(q, keys, w, ks, qpos, k, world)
    assert torch.equal(i1, i2) and torch.equal(v1, v2)
    # queries early in the context: later shards are invisible to some rows
    v1, i1 = _single(q[:8], keys[:200], w[:8], ks[:200], 50, k)
    v2, i2 = _emulated(q[:8], keys[:200], w[:8], ks[:200], 50, k, world)
    assert torch.equal(i1, i2)


def _cp_rank(rank, world):
    from cxldsagr_b200.parallel.cp_indexer import cp_exact_topk
    from cxldsagr_b200.parallel.groups import init_distributed

    ctx = init_distributed(backend="gloo", timeout_s=60)
    q, keys, w, ks = _inputs(16, 500, 7, True)
    k0, k1 = key_shard(500, world, rank)
    v, i = cp_exact_topk(ctx, q, keys[k0:k1], w, ks[k0:k1], k0, 484, 64)
    v1, i1 = _single(q, keys, w, ks, 484, 64)
    return bool(torch.equal(i, i1) and torch.equal(v, v1))


@pytest.mark.parametrize("world", [2, 3])
def test_cp_exact_topk_gloo(world):
    assert all(ok for _, ok in _spawn(_cp_rank, world))


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_cp_merge_on_gpu(world):
    """The sharded indexer / top-k kernels (key shards before, inside and after the
    queries) merged on one GPU equal the single-shard kernels."""
    Q, N, k = 256, 9000, 2048
    q, keys, w, ks = _inputs(Q, N, 11, False, device="cuda")
    qpos = N - Q
    v1, i1 = _single(q, keys, w, ks, qpos, k)
    v2, i2 = _emulated(q, keys, w, ks, qpos, k, world)
    assert torch.equal(i1, i2) and torch.equal(v1, v2)
    ops.check_errors("cuda")
