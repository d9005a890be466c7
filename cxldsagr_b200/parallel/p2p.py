"""Fused peer-memory communication backend (NVLink / NVSwitch, one process per GPU).

* :class:`SymmetricHeap` — one ``cudaMalloc`` per rank exported with CUDA IPC
  and opened by every peer, so a (rank, offset) pair addresses the same
  buffer on every GPU.  Sub-regions: the flag block, the double-buffered
  all-gather buffers and the reduce-scatter receive slots.
* :class:`P2PComm` — :class:`~.comm.Comm` whose ``ag_linear`` and ``linear_rs``
  are single fused kernels (``fp8_gemm_ag`` / ``fp8_gemm_rs`` in
  ``csrc/kernels/gemm_p2p.cu``): the GEMM pushes / stores its operands and
  results over NVLink itself while its tensor cores work, instead of a
  library collective before or after.  Shapes the fused kernels do not cover
  (BF16 weights, rows that do not split evenly, buffers too small) fall back
  to the NCCL baseline of the parent class.

Flag counters are cumulative; the host keeps, per op kind, the running
totals that every rank computes identically (same calls, same shapes).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .comm import Comm
from .groups import ParallelContext

FLAG_SLOTS = 64
ALIGN = 256


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class SymmetricHeap:
    """Same-layout device heap on every rank with every peer's base pointer."""

    def __init__(self, ctx: ParallelContext, nbytes: int):
        self.ctx = ctx
        self.lib = ops.lib()
        self.dev = ctx.device.index
        self.nbytes = _align(nbytes)
        self.local = self.lib.symm_alloc(self.dev, self.nbytes)
        handle = self.lib.symm_handle(self.dev, self.local)
        handles = [None] * ctx.world
        dist.all_gather_object(handles, handle, group=ctx.group)
        self.bases = []
        for q, h in enumerate(handles):
            self.bases.append(self.local if q == ctx.rank else self.lib.symm_open(self.dev, h))
        self._next = 0
        self.closed = False

    def region(self, nbytes: int) -> int:
        off = self._next
        self._next = _align(off + nbytes)
        if self._next > self.nbytes:
            raise MemoryError("symmetric heap exhausted")
        return off

    def ptrs(self, offset: int) -> list[int]:
        return [b + offset for b in self.bases]

    def view(self, offset: int, nbytes: int) -> torch.Tensor:
        return self.lib.symm_view(self.dev, self.local + offset, nbytes)

    def close(self):
        if self.closed:
            return
        torch.cuda.synchronize(self.ctx.device)
        dist.barrier(group=self.ctx.group)
        for q, b in enumerate(self.bases):
            if q != self.ctx.rank:
                self.lib.symm_close(self.dev, b)
        self.lib.symm_free(self.dev, self.local)
        self.closed = True


class _Counter:
    """Cumulative targets of one op kind: arrivals incl. this call, reuse = total two calls back."""

    def __init__(self):
        self.calls = 0
        self.arrive = 0
        self.done_history = [0]   # cumulative reader-done counts after each call

    def next(self, arrive_inc: int, done_inc: int) -> tuple[int, int, int]:
        self.calls += 1
        self.arrive += arrive_inc
        reuse = self.done_history[self.calls - 2] if self.calls >= 3 else 0
        self.done_history.append(self.done_history[-1] + done_inc)
        return self.calls, self.arrive, reuse


class P2PComm(Comm):
    def __init__(self, ctx: ParallelContext, *, max_rows: int = 1024, max_k: int = 7168, max_n: int = 7168):
        super().__init__(ctx)
        if ctx.device.type != "cuda" or ctx.world > 8:
            raise ValueError("the p2p backend needs 2-8 GPUs")
        self.max_rows, self.max_k, self.max_n = max_rows, max_k, max_n
        W = ctx.world
        g_bytes = 2 * max_rows * max_k
        gs_bytes = 2 * (max_k // 128) * max_rows * 4
        rb_bytes = 2 * max_rows * max_n * 2
        flags = FLAG_SLOTS * 8
        self.heap = SymmetricHeap(ctx, flags + g_bytes + gs_bytes + rb_bytes + 4 * ALIGN)
        self.off_flags = self.heap.region(flags)
        self.off_g = self.heap.region(g_bytes)
        self.off_gs = self.heap.region(gs_bytes)
        self.off_rb = self.heap.region(rb_bytes)
        self.flag_ptrs = self.heap.ptrs(self.off_flags)
        self.g_ptrs, self.gs_ptrs, self.rb_ptrs = (self.heap.ptrs(o) for o in (self.off_g, self.off_gs, self.off_rb))
        self.ag = _Counter()
        self.rs = _Counter()
        self.barriers = 0
        self.fused_calls = {"ag": 0, "rs": 0}
        self.barrier()  # every peer mapped its neighbours' heaps before any kernel writes to them

    def barrier(self):
        self.barriers += 1
        self.lib().p2p_barrier(self.ctx.device.index, self.ctx.rank, self.world, self.barriers, self.flag_ptrs)

    @staticmethod
    def lib():
        return ops.lib()

    # ------------------------------------------------------------------ AG
    def _ag_ok(self, lin, quantized, total: int) -> bool:
        return (lin.scales is not None and quantized is not None and total % self.world == 0
                and total <= self.max_rows and lin.weight.shape[1] <= self.max_k and lin.weight.shape[1] % 128 == 0)

    def ag_linear(self, lin, normed, quantized, total: int) -> torch.Tensor:
        if not self._ag_ok(lin, quantized, total):
            return super().ag_linear(lin, normed, quantized, total)
        q, s_t = quantized
        N = lin.weight.shape[0]
        out = torch.empty((total, N), dtype=torch.bfloat16, device=q.device)
        grid = self.lib().fp8_gemm_ag_grid(total, N)
        call, arrive, reuse = self.ag.next(grid, grid)
        self.lib().fp8_gemm_ag(q.contiguous(), s_t.contiguous(), lin.weight, lin.scales, out, self.ctx.rank,
                               self.world, call, arrive, reuse, self.flag_ptrs, self.g_ptrs, self.gs_ptrs)
        self.fused_calls["ag"] += 1
        return out

    # ------------------------------------------------------------------ RS
    def _rs_ok(self, lin, quantized, total: int) -> bool:
        N = lin.weight.shape[0]
        return (lin.scales is not None and quantized is not None and quantized[0] is not None
                and total % self.world == 0 and total <= self.max_rows and N <= self.max_n and N % 8 == 0)

    def linear_rs(self, lin, h, quantized) -> torch.Tensor:
        total = h.shape[0]
        if not self._rs_ok(lin, quantized, total):
            return super().linear_rs(lin, h, quantized)
        q, s_t = quantized
        N = lin.weight.shape[0]
        S = total // self.world
        r = self.ctx.rank
        num_n = (N + 127) // 128
        mblocks = (r * S + S - 1) // 128 - (r * S) // 128 + 1
        rgrid = self.lib().rs_reduce_grid(S, N)
        call, arrive, reuse = self.rs.next(num_n * mblocks, rgrid)
        out = torch.empty((S, N), dtype=torch.bfloat16, device=q.device)
        self.lib().fp8_gemm_rs(q, s_t, lin.weight, lin.scales, None, out, r, self.world, call, arrive, reuse,
                               self.flag_ptrs, self.rb_ptrs)
        self.fused_calls["rs"] += 1
        return out

    def close(self):
        self.heap.close()
