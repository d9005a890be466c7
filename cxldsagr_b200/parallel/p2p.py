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

Flag counters are cumulative.  For the fused GEMMs and the barrier, each
rank keeps its op state (calls, arrival and reader-done totals per kind) in a
small block of its own device memory: a call reads its number, parity and
flag targets from it at launch and its last CTA advances it, so the host only
passes the per-call increments, which every rank computes identically from
the shapes.  The same launches therefore replay correctly from a CUDA graph.
The expert-parallel exchange keeps host-side call numbers.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .comm import Comm
from .groups import ParallelContext

FLAG_SLOTS = 128
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
        self.bases = [self.local]
        if ctx.world > 1:
            handle = self.lib.symm_handle(self.dev, self.local)
            handles = [None] * ctx.world
            dist.all_gather_object(handles, handle, group=ctx.group)
            self.bases = [self.local if q == ctx.rank else self.lib.symm_open(self.dev, h)
                          for q, h in enumerate(handles)]
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
        if self.ctx.world > 1:
            dist.barrier(group=self.ctx.group)
        for q, b in enumerate(self.bases):
            if q != self.ctx.rank:
                self.lib.symm_close(self.dev, b)
        self.lib.symm_free(self.dev, self.local)
        self.closed = True


EPOCH_SLOTS = 8                      # u64 per op kind (csrc/common/p2p_args.h kEpochSlots)
EPOCH_AG, EPOCH_RS, EPOCH_BARRIER = 0, 1, 2


class P2PComm(Comm):
    """``moe=(n_experts, hidden, topk)`` also reserves the expert-parallel exchange buffers
    (counts, every owner's grouped FP8 layout and its expert outputs, double-buffered)."""

    def __init__(self, ctx: ParallelContext, *, max_rows: int = 1024, max_k: int = 7168, max_n: int = 7168,
                 moe: tuple | None = None):
        super().__init__(ctx)
        if ctx.device.type != "cuda" or ctx.world > 8:
            raise ValueError("the p2p backend needs 1-8 GPUs (1: single-GPU profiling of the fused kernels)")
        self.max_rows, self.max_k, self.max_n = max_rows, max_k, max_n
        W = ctx.world
        g_bytes = 2 * max_rows * max_k
        gs_bytes = 2 * (max_k // 128) * max_rows * 4
        rb_bytes = 2 * max_rows * max_n * 2
        flags = FLAG_SLOTS * 8
        ep_bytes = 0
        self.moe = moe
        if moe is not None:
            E, D, topk = moe
            # Worst case: every routed row of the chunk lands on one owner, plus per-expert padding.
            self.ep_mpad = (max_rows * topk + (E // W) * 127 + 127) // 128 * 128
            self.ep_shapes = {"cnt": 2 * W * E * 4, "a": 2 * self.ep_mpad * D, "as": 2 * (D // 128) * self.ep_mpad * 4,
                              "y": 2 * self.ep_mpad * D * 2, "rsrc": 2 * self.ep_mpad * 4}
            ep_bytes = sum(self.ep_shapes.values()) + 4 * ALIGN
        self.heap = SymmetricHeap(ctx, flags + g_bytes + gs_bytes + rb_bytes + ep_bytes + 4 * ALIGN)
        self.off_flags = self.heap.region(flags)
        self.off_g = self.heap.region(g_bytes)
        self.off_gs = self.heap.region(gs_bytes)
        self.off_rb = self.heap.region(rb_bytes)
        self.ep_calls = 0
        if moe is not None:
            self.ep_off = {k: self.heap.region(v) for k, v in self.ep_shapes.items()}
            self.ep_ptrs = {k: self.heap.ptrs(o) for k, o in self.ep_off.items()}
            E, D, topk = moe
            dev = ctx.device
            self.ep_blocks = self.ep_mpad // 128
            self.ep_cursor = torch.zeros(E, dtype=torch.int32, device=dev)
            self.ep_block_expert = torch.full((self.ep_blocks,), -1, dtype=torch.int32, device=dev)
            self.ep_block_valid = torch.zeros(self.ep_blocks, dtype=torch.int32, device=dev)
            self.ep_finish = torch.zeros(1, dtype=torch.int32, device=dev)
        # Push mode: the owners' down GEMMs store rows into the sources' receive
        # slots (fused combine); pull mode: sources load the owners' outputs.
        self.ep_push = True
        self.flag_ptrs = self.heap.ptrs(self.off_flags)
        self.g_ptrs, self.gs_ptrs, self.rb_ptrs = (self.heap.ptrs(o) for o in (self.off_g, self.off_gs, self.off_rb))
        # Device-resident op state of the AG, RS and barrier kinds (local memory).
        self.epoch = torch.zeros(3 * EPOCH_SLOTS, dtype=torch.int64, device=ctx.device)
        self.barriers = 0
        self.fused_calls = {"ag": 0, "rs": 0}
        self.barrier()  # every peer mapped its neighbours' heaps before any kernel writes to them

    def barrier(self):
        self.barriers += 1
        self.lib().p2p_barrier(self.ctx.device.index, self.ctx.rank, self.world, 0, self.flag_ptrs,
                               epoch=self._epoch(EPOCH_BARRIER))

    def _epoch(self, kind: int) -> int:
        return self.epoch.data_ptr() + kind * EPOCH_SLOTS * 8

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
        grid = self.lib().fp8_gemm_ag_grid(total, N, q.shape[1])
        with self._span("ag_gemm"):
            # Every CTA of every rank pushes (arrival) and reads (done) once per call.
            self.lib().fp8_gemm_ag(q.contiguous(), s_t.contiguous(), lin.weight, lin.scales, out, self.ctx.rank,
                                   self.world, 0, 0, 0, self.flag_ptrs, self.g_ptrs, self.gs_ptrs,
                                   epoch=self._epoch(EPOCH_AG), arrive_inc=grid, done_inc=grid)
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
        bn = self.lib().fp8_gemm_p2p_bn(total, N, q.shape[1])  # the kernel's tile width
        num_n = (N + bn - 1) // bn
        mblocks = (r * S + S - 1) // 128 - (r * S) // 128 + 1
        rgrid = self.lib().rs_reduce_grid(S, N)
        out = torch.empty((S, N), dtype=torch.bfloat16, device=q.device)
        with self._span("gemm_rs"):
            # Arrivals per source: the tiles covering this rank's rows; done: the owner's reduce CTAs.
            self.lib().fp8_gemm_rs(q, s_t, lin.weight, lin.scales, None, out, r, self.world, 0, 0, 0,
                                   self.flag_ptrs, self.rb_ptrs, epoch=self._epoch(EPOCH_RS),
                                   arrive_inc=num_n * mblocks, done_inc=rgrid)
        self.fused_calls["rs"] += 1
        return out

    # ----------------------------------------------------------------- EP
    def ep_ready(self, n_experts: int, hidden: int, topk: int, tokens: int) -> bool:
        return (self.moe is not None and self.moe == (n_experts, hidden, topk) and tokens <= self.max_rows
                and n_experts % self.world == 0)

    def _ep_views(self, parity: int):
        E, D, topk = self.moe
        M = self.ep_mpad
        a = self.heap.view(self.ep_off["a"], self.ep_shapes["a"]).view(torch.float8_e4m3fn).view(2, M, D)[parity]
        a_s = self.heap.view(self.ep_off["as"], self.ep_shapes["as"]).view(torch.float32).view(2, D // 128, M)[parity]
        y = self.heap.view(self.ep_off["y"], self.ep_shapes["y"]).view(torch.bfloat16).view(2, M, D)[parity]
        return a, a_s, y

    def moe_ep(self, ids, q, s_t, weights, experts_fn):
        """Fused EP MoE: dispatch into owners' grouped layouts, run ``experts_fn(a, a_s, block_expert, y_out)``
        on this rank's experts, combine in k order.  Returns bf16 [T, D]."""
        E, D, topk = self.moe
        T = ids.shape[0]
        self.ep_calls += 1
        call = self.ep_calls
        parity = call & 1
        p = self.ep_ptrs
        pos = torch.full((T * topk,), -1, dtype=torch.int32, device=q.device)
        ids32 = ids.to(torch.int32).contiguous()
        with self._span("ep_dispatch"):
            self.lib().ep_dispatch(ids32, q.contiguous(), s_t, self.ep_cursor, pos, self.ep_block_expert, self.ctx.rank,
                                   self.world, E, self.ep_mpad, call, self.flag_ptrs, p["cnt"], p["a"], p["as"],
                                   p["y"], p["rsrc"], self.ep_block_valid)
        a, a_s, y = self._ep_views(parity)
        if self.ep_push:
            # Receive slots and row-source tables of this call's parity half.
            y_bytes = self.ep_mpad * D * 2
            y = ops.EpPushTarget(p["rsrc"][self.ctx.rank] + parity * self.ep_mpad * 4, self.ep_block_valid,
                                 [b + parity * y_bytes for b in p["y"]], self.flag_ptrs, self.ep_finish,
                                 self.ctx.rank, self.world)
        experts_fn(a, a_s, self.ep_block_expert, y)
        out = torch.empty((T, D), dtype=torch.bfloat16, device=q.device)
        with self._span("ep_combine"):
            self.lib().ep_combine(ids32, pos, weights.contiguous(), out, self.ctx.rank, self.world, E, self.ep_mpad,
                                  call, self.flag_ptrs, p["cnt"], p["a"], p["as"], p["y"], p["rsrc"], self.ep_push)
        self.fused_calls["ep"] = self.fused_calls.get("ep", 0) + 1
        return out

    def close(self):
        self.heap.close()
