"""Communication-fused linear ops used by the sequence/expert-parallel model.

Each op is named for the compute it wraps, so a backend can fuse the
collective into the kernel:

* :meth:`Comm.ag_linear`  — all-gather of the row-sharded input, then a linear
  over all rows (AG -> GEMM);
* :meth:`Comm.linear_rs`  — a row-parallel linear whose partial sums are
  reduce-scattered by rows (GEMM -> RS);
* :meth:`Comm.dispatch` / :meth:`Comm.combine` — expert-parallel all-to-all of
  token rows to the expert owners and of expert outputs back.

:class:`Comm` is the baseline over ``torch.distributed`` (NCCL on GPUs, gloo on
CPU): a library collective followed by this package's GEMM.  The fused
peer-memory backend (:mod:`.p2p`) implements the same methods with one kernel
per op.
"""

from __future__ import annotations

from collections import defaultdict
from contextlib import contextmanager

import torch

from .. import ops
from . import collectives as C
from .groups import ParallelContext


class CollectiveTimer:
    """Device time of each communication op (CUDA events on the current stream).

    Attach one to :attr:`Comm.timer`; every ``ag_linear`` / ``linear_rs`` /
    expert-parallel exchange then records a start and end event.  A fused op
    that falls back to the baseline implementation is timed once (only the
    outermost call counts).  :meth:`summary` synchronises and returns
    ``{op: {"calls": n, "ms": total}}``.
    """

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self._spans: dict[str, list] = defaultdict(list)
        self._depth = 0

    @contextmanager
    def span(self, name: str):
        # Not timed inside a CUDA-graph capture (replays are timed as a whole).
        if self._depth or self.device.type != "cuda" or torch.cuda.is_current_stream_capturing():
            yield
            return
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self._depth += 1
        start.record()
        try:
            yield
        finally:
            end.record()
            self._depth -= 1
            self._spans[name].append((start, end))

    def summary(self, *, reset: bool = True) -> dict:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        out = {name: {"calls": len(ev), "ms": sum(a.elapsed_time(b) for a, b in ev)} for name, ev in self._spans.items()}
        if reset:
            self._spans.clear()
        return out


@contextmanager
def _no_span():
    yield


class Comm:
    def __init__(self, ctx: ParallelContext):
        self.ctx = ctx
        self.timer: CollectiveTimer | None = None

    def _span(self, name: str):
        return self.timer.span(name) if self.timer is not None else _no_span()

    @property
    def world(self) -> int:
        return self.ctx.world

    # ------------------------------------------------------------------ AG
    def gather(self, normed, quantized, total: int):
        """Full-chunk input of a column-parallel/replicated linear: FP8 (q, s^T) or BF16 rows."""
        if self.world == 1:
            return quantized if quantized is not None and quantized[0] is not None else normed
        if quantized is not None and quantized[0] is not None:
            q, s_t = quantized
            return C.all_gather_rows(self.ctx, q, total, 0), C.all_gather_rows(self.ctx, s_t, total, 1)
        return C.all_gather_rows(self.ctx, normed, total, 0)

    def ag_linear(self, lin, normed, quantized, total: int) -> torch.Tensor:
        with self._span("ag_gemm"):
            g = self.gather(normed, quantized, total)
            return lin(quantized=g) if isinstance(g, tuple) else lin(g)

    # ------------------------------------------------------------------ RS
    def linear_rs(self, lin, h, quantized) -> torch.Tensor:
        """Row-parallel linear over all rows, reduced and scattered to the row owners."""
        with self._span("gemm_rs"):
            partial = lin(h, quantized=quantized)
            if self.world == 1:
                return partial
            return C.reduce_scatter_rows(self.ctx, partial, out_dtype=torch.bfloat16)

    # -------------------------------------------------------------- EP a2a
    def dispatch(self, rows: torch.Tensor, scales_rows, dest: torch.Tensor, experts: torch.Tensor):
        """Send token rows to expert owners.

        ``rows`` [N, D] are already ordered by destination rank (``dest``
        non-decreasing); ``scales_rows`` [N, D/128] (FP8 rows) or None;
        ``experts`` [N] global expert id per row.  Returns the received rows,
        scales, expert ids and the per-source counts.
        """
        with self._span("ep_dispatch"):
            counts = torch.bincount(dest, minlength=self.world).tolist()
            recv, rc = C.all_to_all_rows(self.ctx, rows, counts)
            rs = C.all_to_all_back(self.ctx, scales_rows, counts, rc) if scales_rows is not None else None
            re = C.all_to_all_back(self.ctx, experts.to(torch.int32), counts, rc)
            return recv, rs, re, counts, rc

    def combine(self, out_rows: torch.Tensor, send_counts, recv_counts) -> torch.Tensor:
        """Return expert outputs to the rows' source ranks (inverse of :meth:`dispatch`)."""
        with self._span("ep_combine"):
            return C.all_to_all_back(self.ctx, out_rows, recv_counts, send_counts)

    # ---------------------------------------------------------------- misc
    def reduce_rows(self, x: torch.Tensor) -> torch.Tensor:
        """Sum [T, D] over ranks and keep this rank's rows (vocabulary-parallel embedding)."""
        if self.world == 1:
            return x
        with self._span("embed_rs"):
            return C.reduce_scatter_rows(self.ctx, x, out_dtype=x.dtype)

    def gather_cols(self, x: torch.Tensor, total: int) -> torch.Tensor:
        """Concatenate every rank's column shard of [R, total] (vocabulary-parallel LM head)."""
        if self.world == 1:
            return x
        with self._span("lm_head_gather"):
            return C.all_gather_rows(self.ctx, x, total, 1)

    def gather_rows(self, x, total: int):
        return x if self.world == 1 else C.all_gather_rows(self.ctx, x, total, 0)

    def broadcast(self, x, src: int):
        return C.broadcast(self.ctx, x, src)


def make_comm(ctx: ParallelContext, *, moe: tuple | None = None, max_rows: int = 1024) -> Comm:
    """``moe=(n_experts, hidden, topk)`` reserves the fused expert-parallel buffers (p2p backend)."""
    if ctx.backend == "p2p" and ctx.world > 1:
        from .p2p import P2PComm

        return P2PComm(ctx, moe=moe, max_rows=max_rows)
    return Comm(ctx)


def quantize_rows(x: torch.Tensor):
    """FP8 rows + per-row scales [N, D/128] (row-major, for row-wise transport)."""
    q, s_t = ops.quantize_act(x)
    return q, s_t.t().contiguous()
