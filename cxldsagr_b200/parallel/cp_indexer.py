"""Context-parallel lightning indexer: the indexer key cache is split by
sequence over the ranks, each rank scores its key shard and keeps its local
exact top-k, and a merge of the ``R x k`` candidates per query gives the
global exact top-k.

The reference has no parallel indexer (one device scores the whole context:
``operators/deepseek_v32/indexer/echo.py:299-483``); this is the B200 build's
long-context scaling path: with ``R`` ranks every rank stores ``N / R`` FP8
keys (132 B per token per layer) and does ``1 / R`` of the indexer work, and
only ``Q x k`` (score, id) pairs per rank cross NVLink (16 KB per query at
k = 2048).

Exactness.  Shards are contiguous ranges in rank order.  Each rank's list is
ordered by descending score with ties to the smaller id, so in the rank-order
concatenation equal scores appear in ascending global id; the merge selects
by descending score with ties to the smaller position, which is the smaller
id.  The merged selection therefore equals the single-device selection,
ties included (tested against it).
"""

from __future__ import annotations

import torch

from .. import ops
from .groups import ParallelContext, shard_range


def key_shard(total_keys: int, world: int, rank: int) -> tuple[int, int]:
    """The contiguous key range [k0, k1) rank ``rank`` owns."""
    return shard_range(total_keys, world, rank)


def local_topk(q_idx, keys, weights, kscales, k0: int, query_pos: int, k: int):
    """Exact top-k of this rank's key shard with global ids.

    ``keys`` / ``kscales`` hold global positions [k0, k0 + n_local); row r of
    ``q_idx`` is the query at global position ``query_pos + r`` and sees keys
    at positions <= its own.  Returns (values [Q, k] fp32, ids [Q, k] int32),
    value-ordered, padded with (-inf, -1).
    """
    Q, n_local = q_idx.shape[0], keys.shape[0]
    dev = q_idx.device
    values = torch.full((Q, k), -torch.inf, dtype=torch.float32, device=dev)
    ids = torch.full((Q, k), -1, dtype=torch.int32, device=dev)
    # Rows whose position precedes the shard see none of it.
    first = max(0, k0 - query_pos)
    if first >= Q or n_local == 0:
        return values, ids
    rel = query_pos + first - k0                     # shard-relative position of row `first` (>= 0)
    q, w = q_idx[first:], weights[first:]
    logits = ops.indexer_logits(q, keys, w, kscales, rel)
    width = min(k, n_local)
    v, i = ops.exact_topk(logits, k, causal_start=rel, n=n_local)
    values[first:, :width] = v
    ids[first:, :width] = torch.where(i >= 0, i + k0, i)
    return values, ids


def merge_topk(values: torch.Tensor, ids: torch.Tensor, k: int):
    """Global exact top-k from the rank-order concatenation of local lists ([Q, R*k] each)."""
    v, pos = ops.exact_topk(values.contiguous(), k)
    picked = ids.gather(1, pos.clamp_min(0).long())
    picked = torch.where((pos >= 0) & torch.isfinite(v), picked, torch.full_like(picked, -1))
    return v, picked.to(torch.int32)


def cp_exact_topk(ctx: ParallelContext, q_idx, keys, weights, kscales, k0: int, query_pos: int, k: int):
    """Local top-k on this rank's shard, all-gather of the (score, id) lists, merge.

    Every rank passes the same queries (``q_idx``, ``weights``) and its own key
    shard; every rank returns the same global selection.
    """
    values, ids = local_topk(q_idx, keys, weights, kscales, k0, query_pos, k)
    if ctx.world == 1:
        return merge_topk(values, ids, k)
    import torch.distributed as dist

    Q = values.shape[0]
    vs = torch.empty((ctx.world * Q, k), dtype=values.dtype, device=values.device)
    ix = torch.empty((ctx.world * Q, k), dtype=ids.dtype, device=ids.device)
    dist.all_gather_into_tensor(vs, values.contiguous(), group=ctx.group)
    dist.all_gather_into_tensor(ix, ids.contiguous(), group=ctx.group)
    cat = lambda t: t.view(ctx.world, Q, k).permute(1, 0, 2).reshape(Q, ctx.world * k)  # noqa: E731
    return merge_topk(cat(vs), cat(ix), k)
