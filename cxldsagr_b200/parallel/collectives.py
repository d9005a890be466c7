"""Row-sharded collectives over ``torch.distributed`` (the NCCL baseline; gloo on CPU).

Shards may be uneven (``groups.shard_sizes``): every rank pads its rows to
``ceil(T / R)`` so the fixed-size NCCL calls apply, and valid rows are sliced
back out.  FP8 payloads travel as bytes.  These are the reference points the
fused peer-memory kernels (:mod:`.p2p`) are measured against.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .groups import ParallelContext, shard_sizes


def _bytes(x: torch.Tensor) -> torch.Tensor:
    return x.view(torch.uint8) if x.dtype in (torch.float8_e4m3fn, torch.float8_e5m2) else x


def all_gather_rows(ctx: ParallelContext, x: torch.Tensor, total: int, dim: int = 0) -> torch.Tensor:
    """Concatenate every rank's rows (along ``dim``) in rank order."""
    if ctx.world == 1:
        return x
    sizes = shard_sizes(total, ctx.world)
    S = max(sizes)
    xm = x.movedim(dim, 0)
    if xm.shape[0] != sizes[ctx.rank]:
        raise ValueError("local rows differ from this rank's shard size")
    pad = torch.zeros((S, *xm.shape[1:]), dtype=x.dtype, device=x.device)
    pad[: xm.shape[0]] = xm
    out = torch.empty((ctx.world * S, *xm.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(_bytes(out), _bytes(pad), group=ctx.group)
    parts = [out[i * S: i * S + n] for i, n in enumerate(sizes)]
    return torch.cat(parts).movedim(0, dim).contiguous()


def reduce_scatter_rows(ctx: ParallelContext, x: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """Sum ``x`` [T, ...] over ranks and return this rank's rows (fp32 accumulation)."""
    out_dtype = out_dtype or x.dtype
    if ctx.world == 1:
        return x.to(out_dtype)
    T = x.shape[0]
    sizes = shard_sizes(T, ctx.world)
    S = max(sizes)
    buf = torch.zeros((ctx.world, S, *x.shape[1:]), dtype=torch.float32, device=x.device)
    start = 0
    for i, n in enumerate(sizes):
        buf[i, :n] = x[start:start + n]
        start += n
    out = torch.empty((S, *x.shape[1:]), dtype=torch.float32, device=x.device)
    dist.reduce_scatter_tensor(out, buf.reshape(ctx.world * S, *x.shape[1:]), group=ctx.group)
    return out[: sizes[ctx.rank]].to(out_dtype)


def all_reduce(ctx: ParallelContext, x: torch.Tensor) -> torch.Tensor:
    if ctx.world > 1:
        dist.all_reduce(x, group=ctx.group)
    return x


def all_to_all_rows(ctx: ParallelContext, send: torch.Tensor, send_counts: list[int]) -> tuple[torch.Tensor, list[int]]:
    """Send ``send_counts[d]`` consecutive rows to rank ``d``; returns (received rows, counts per source)."""
    if ctx.world == 1:
        return send, list(send_counts)
    counts = torch.tensor(send_counts, dtype=torch.int64, device=send.device)
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=ctx.group)
    rc = recv_counts.tolist()
    recv = torch.empty((sum(rc), *send.shape[1:]), dtype=send.dtype, device=send.device)
    dist.all_to_all_single(_bytes(recv), _bytes(send.contiguous()), output_split_sizes=rc,
                           input_split_sizes=list(send_counts), group=ctx.group)
    return recv, rc


def all_to_all_back(ctx: ParallelContext, send: torch.Tensor, send_counts: list[int],
                    recv_counts: list[int]) -> torch.Tensor:
    """Inverse of :func:`all_to_all_rows` with known counts (no count exchange)."""
    if ctx.world == 1:
        return send
    recv = torch.empty((sum(recv_counts), *send.shape[1:]), dtype=send.dtype, device=send.device)
    dist.all_to_all_single(_bytes(recv), _bytes(send.contiguous()), output_split_sizes=list(recv_counts),
                           input_split_sizes=list(send_counts), group=ctx.group)
    return recv


def broadcast(ctx: ParallelContext, x: torch.Tensor, src: int) -> torch.Tensor:
    if ctx.world > 1:
        dist.broadcast(x, src, group=ctx.group)
    return x
