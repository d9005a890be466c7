"""Fused peer-memory GEMM collectives against NCCL, device-timed, at world N.

For the tensor-parallel MLP of DeepSeek-V3.2 (gate/up column-parallel after
an all-gather of the sequence shards, down row-parallel before a
reduce-scatter) and one 2048-token chunk, every rank times with CUDA events
(max over ranks):

* ``fused``: ``P2PComm.ag_linear`` / ``linear_rs`` (one kernel pushes or
  stores its operands over NVLink while its tensor cores work);
* ``nccl``: the baseline (``Comm``: NCCL all-gather then GEMM, GEMM then
  NCCL reduce-scatter);
* ``gemm``: the same GEMM alone on local data (the compute floor).

Roofline of a fused op = the slower of the compute floor and the bytes that
must cross NVLink per GPU and direction divided by the measured peer-copy
bandwidth (770 GB/s per direction per GPU on this pool; 900 GB/s nominal):
AG moves (W-1) shards of S x K FP8 (+ scales) into each GPU, RS moves (W-1)
slices of S x N BF16.  ``frac_of_roofline`` = roofline time / fused time.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m cxldsagr_b200.evaluation.collective_bench
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

PEER_GBS = 770.0   # measured peer copy, GB/s per direction per GPU


def _timed(fn, dev, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--tokens", type=int, default=2048, help="rows of the chunk (all ranks together)")
    p.add_argument("--reps", type=int, default=20)
    a = p.parse_args(argv)

    from .. import ops
    from ..checkpoint import quantize_weight_blocks
    from ..config import v32_config
    from ..models.deepseek_v32.weights import Linear
    from ..ops.native import check_errors
    from ..parallel.comm import Comm
    from ..parallel.groups import init_distributed
    from ..parallel.p2p import P2PComm

    ctx = init_distributed(timeout_s=120, comm="p2p")
    dev, W, rank = ctx.device, ctx.world, ctx.rank
    cfg = v32_config(1)
    T, D, I = a.tokens, cfg.dim, cfg.intermediate_size
    S = T // W
    fused = P2PComm(ctx, max_rows=T, max_k=max(D, I // W), max_n=max(D, 2 * I // W))
    base = Comm(ctx)
    g = torch.Generator(device=dev).manual_seed(5)

    def lin(n, k):
        w, s = quantize_weight_blocks(torch.randn((n, k), generator=g, device=dev) * 0.02)
        return Linear(w.contiguous(), s.float().contiguous())

    rows = []
    # AG -> gate/up (column-parallel: this rank's 2I / W output columns).
    w_gu = lin(2 * I // W, D)
    x = torch.randn((S, D), device=dev).bfloat16()
    qx = ops.quantize_act(x)
    gathered = torch.randn((T, D), device=dev).bfloat16()
    qg = ops.quantize_act(gathered)
    ms_f = _timed(lambda: fused.ag_linear(w_gu, x, qx, T), dev, a.reps)
    ms_n = _timed(lambda: base.ag_linear(w_gu, x, qx, T), dev, a.reps)
    ms_g = _timed(lambda: ops.fp8_gemm(qg[0], qg[1], w_gu.weight, w_gu.scales), dev, a.reps)
    link_ms = (W - 1) * S * (D + D // 128 * 4) / (PEER_GBS * 1e6)
    roof = max(ms_g, link_ms)
    rows.append({"op": "ag_gemm", "world": W, "M": T, "N": 2 * I // W, "K": D, "fused_ms": round(ms_f, 4),
                 "nccl_ms": round(ms_n, 4), "gemm_ms": round(ms_g, 4), "link_floor_ms": round(link_ms, 4),
                 "frac_of_roofline": round(roof / ms_f, 3), "fused_vs_nccl": round(ms_n / ms_f, 3)})
    # down -> RS (row-parallel: this rank's I / W input columns, full D outputs).
    w_dn = lin(D, I // W)
    h = torch.randn((T, I // W), device=dev).bfloat16()
    qh = ops.quantize_act(h)
    ms_f = _timed(lambda: fused.linear_rs(w_dn, h, qh), dev, a.reps)
    ms_n = _timed(lambda: base.linear_rs(w_dn, h, qh), dev, a.reps)
    ms_g = _timed(lambda: ops.fp8_gemm(qh[0], qh[1], w_dn.weight, w_dn.scales), dev, a.reps)
    link_ms = (W - 1) * S * D * 2 / (PEER_GBS * 1e6)
    roof = max(ms_g, link_ms)
    rows.append({"op": "gemm_rs", "world": W, "M": T, "N": D, "K": I // W, "fused_ms": round(ms_f, 4),
                 "nccl_ms": round(ms_n, 4), "gemm_ms": round(ms_g, 4), "link_floor_ms": round(link_ms, 4),
                 "frac_of_roofline": round(roof / ms_f, 3), "fused_vs_nccl": round(ms_n / ms_f, 3)})
    torch.cuda.synchronize(dev)
    check_errors(dev)
    fused.close()
    if rank == 0:
        for r in rows:
            print(json.dumps({**r, "timing": "CUDA events, mean of reps after warm-up, max over ranks",
                              "peer_gbs": PEER_GBS}))
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    raise SystemExit(main())
