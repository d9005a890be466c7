"""Per-operator microbenchmarks on one GPU (CUDA-event timing, warm-up,
inputs larger than L2 or an explicit L2 flush between iterations).

    python -m cxldsagr_b200.evaluation.kernel_bench --op sparse_mla --T 256
    python -m cxldsagr_b200.evaluation.kernel_bench --op all

Counterpart of the reference's operator observation harness
(experiments/deepseek_v32_observation): each op reports device time per call,
achieved FLOP/s or bytes/s and the fraction of the measured peaks in
MEASURED_PEAKS.json when present (fallback 6.65 TB/s, 1.59 PFLOP/s bf16).
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from .. import ops
from ..checkpoint import quantize_weight_blocks

_L2_FLUSH = None


def _peaks():
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


FP8_NOMINAL_TFLOPS = 4500.0  # dense FP8 nominal; no measured FP8 denominator exists


def roofline(ms: float, *, flops: float = 0.0, nbytes: float = 0.0, fp8: bool = False) -> dict:
    """Achieved / roofline time, where the roofline is the slower of FLOPs / peak
    (measured BF16 GEMM; nominal 4.5 PF for FP8 work) and bytes / measured copy
    bandwidth.  Values near 1 mean the kernel runs at the bound."""
    pk = _peaks()
    peak = FP8_NOMINAL_TFLOPS if fp8 else pk["bf16_tflops"]
    t_compute = flops / (peak * 1e9) if flops else 0.0      # ms
    t_memory = nbytes / (pk["hbm_gbs"] * 1e6) if nbytes else 0.0
    bound = max(t_compute, t_memory)
    return {"roofline_ms": bound, "frac_of_roofline": bound / ms if ms > 0 else None,
            "bound": "compute" if t_compute >= t_memory else "memory",
            "compute_peak": f"{peak:.0f} TFLOP/s ({'nominal FP8' if fp8 else pk['source'] + ' BF16'})",
            "hbm_gbs": pk["hbm_gbs"]}


def flush_l2(dev):
    global _L2_FLUSH
    if _L2_FLUSH is None:
        _L2_FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    _L2_FLUSH.zero_()


GRAPH = False  # set by --graph: replay each op from a CUDA graph (no host launch cost in the timing)


def time_fn(fn, *, warmup=3, iters=10, flush=True, dev="cuda"):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if GRAPH:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        torch.cuda.synchronize()
        fn = graph.replay
    total = 0.0
    for _ in range(iters):
        if flush:
            flush_l2(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def mla_timeline(q, kv, ids, splits: int) -> dict:
    """Phase clocks (SM cycles) of the first cluster of one cta_group::2 MLA launch
    (kernel debug bit 8): Q landed, each tile's S read and P handed to PV, O ready, exit."""
    ops.sparse_mla(q, kv, ids, 0.1, splits=splits, impl=32 + 8)
    torch.cuda.synchronize()
    tr = ops.lib().sparse_mla_2sm_trace()
    t0 = int(tr[0, 64, 0])
    n = min(64, -(-ids.shape[1] // splits) // 64)
    p_handed = [int(tr[0, i, 5]) - t0 for i in range(n)]
    s_read = [int(tr[0, i, 4]) - t0 for i in range(n)]
    return {"q_landed": int(tr[0, 64, 1]) - t0, "first_s": s_read[0], "first_p": p_handed[0],
            "last_p": p_handed[-1], "cycles_per_tile": (p_handed[-1] - p_handed[0]) / max(1, n - 1),
            "softmax_cycles_per_tile": sum(p - r for p, r in zip(p_handed, s_read)) / n,
            # Softmax phases per tile (mean over tiles, SM cycles): S read -> maxima exchanged
            # (named barrier) -> exponentials and P packed -> P buffer free (PV two tiles back)
            # -> P stored and handed to PV; and the wait for the next S.
            "softmax_phases": {
                "max_exchange": sum(int(tr[0, i, 8]) - int(tr[0, i, 4]) for i in range(n)) / n,
                "exp_pack": sum(int(tr[0, i, 9]) - int(tr[0, i, 8]) for i in range(n)) / n,
                "p_buffer_wait": sum(int(tr[0, i, 10]) - int(tr[0, i, 9]) for i in range(n)) / n,
                "p_store_hand": sum(int(tr[0, i, 5]) - int(tr[0, i, 10]) for i in range(n)) / n,
                "next_s_wait": sum(int(tr[0, i + 1, 4]) - int(tr[0, i, 5]) for i in range(n - 1)) / max(1, n - 1)},
            "o_ready": int(tr[0, 64, 2]) - t0, "exit": int(tr[0, 64, 3]) - t0, "tiles": n, "keys_per_tile": 64}


def bench_sparse_mla(T=256, K=2048, P=65664, splits=1, impl=0, locality=0.0, trace=False, **_):
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    q = (torch.randn(T, 128, 576, device=dev, generator=g) * 0.5).bfloat16()
    kv = (torch.randn(P, 576, device=dev, generator=g) * 0.5).bfloat16()
    ids = torch.randint(0, P, (T, K), device=dev, dtype=torch.int32, generator=g)
    if locality > 0:  # a shared hot set, like correlated top-k of neighbouring queries
        hot = torch.randint(0, P, (K,), device=dev, dtype=torch.int32, generator=g)
        mask = torch.rand(T, K, device=dev, generator=g) < locality
        ids = torch.where(mask, hot[None, :].expand(T, K), ids)
    ms = time_fn(lambda: ops.sparse_mla(q, kv, ids, 0.1, splits=splits, impl=impl))
    timeline = mla_timeline(q, kv, ids, splits) if trace else None
    flops = 2.0 * T * 128 * K * (576 + 512)
    gather = T * K * 1152.0
    pk = _peaks()
    return {"op": "sparse_mla", "T": T, "K": K, "P": P, "splits": splits, "impl": impl, "ms": ms,
            "tflops": flops / ms / 1e9, "frac_bf16_peak": flops / ms / 1e9 / pk["bf16_tflops"],
            "gather_gbs": gather / ms / 1e6, "peaks": pk["source"],
            # distinct KV rows (repeats across queries hit L2) + Q + O
            **roofline(ms, flops=flops, nbytes=int(torch.unique(ids).numel()) * 1152 + T * 128 * (576 + 512) * 2),
            **({"timeline_cycles": timeline} if timeline else {})}


def bench_fp8_gemm(M=1024, N=36864, K=7168, ue8m0=False, pair=False, **_):
    """Power-of-two block scales (the checkpoint convention); ``ue8m0`` picks the
    block-scaled tensor-core path, otherwise the per-K-block FP32 promotion;
    ``pair`` the 2-CTA 256-row tiles."""
    dev = "cuda"
    x = torch.randn(M, K, device=dev).bfloat16()
    w, s = quantize_weight_blocks(torch.randn(N, K, device=dev) * 0.02)
    q, s_t = ops.quantize_act(x)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    ops.lib().set_fp8_gemm_pair_tiles(pair)
    try:
        ms = time_fn(lambda: ops.fp8_gemm(q, s_t, w, s, out=out, ue8m0=ue8m0))
    finally:
        ops.lib().set_fp8_gemm_pair_tiles(False)
    flops = 2.0 * M * N * K
    return {"op": "fp8_gemm", "M": M, "N": N, "K": K, "ue8m0": ue8m0, "pair": pair, "ms": ms,
            "tflops": flops / ms / 1e9,
            "bytes_gbs": (N * K + M * K + M * N * 2) / ms / 1e6,
            **roofline(ms, flops=flops, nbytes=N * K + M * K + M * N * 2, fp8=True)}


def bench_gemm_paths(M=2048, **_):
    """Prefill-chunk FP8 linears of one V3.2 layer on each tile path: 128-row
    tiles with FP32 promotion (default), 128-row block-scaled (UE8M0) tiles,
    and 2-CTA 256-row tiles (promotion).  TFLOP/s per path."""
    from ..config import v32_config

    cfg = v32_config(1)
    dev = "cuda"
    shapes = {
        "fused_a": (cfg.q_lora_rank + 640 + cfg.index_head_dim, cfg.dim),
        "fused_b": (cfg.n_heads * (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
                    + cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank),
        "o_proj": (cfg.dim, cfg.n_heads * cfg.v_head_dim),
        "gate_up": (2 * cfg.intermediate_size, cfg.dim),
        "down": (cfg.dim, cfg.intermediate_size),
    }
    rows = []
    for name, (N, K) in shapes.items():
        x = torch.randn(M, K, device=dev).bfloat16()
        w, s = quantize_weight_blocks(torch.randn(N, K, device=dev) * 0.02)
        q, s_t = ops.quantize_act(x)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ref_out = ops.fp8_gemm(q, s_t, w, s)
        row = {"gemm": name, "M": M, "N": N, "K": K}
        for label, bs, pair in (("promote", False, False), ("block_scaled", True, False), ("pair", False, True)):
            ops.lib().set_fp8_gemm_pair_tiles(pair)
            try:
                ms = time_fn(lambda: ops.fp8_gemm(q, s_t, w, s, out=out, ue8m0=bs))
                ops.fp8_gemm(q, s_t, w, s, out=out, ue8m0=bs)
                diff = (out.float() - ref_out.float()).abs().max().item()
            finally:
                ops.lib().set_fp8_gemm_pair_tiles(False)
            row[f"{label}_us"] = round(ms * 1e3, 1)
            row[f"{label}_tflops"] = round(2.0 * M * N * K / ms / 1e9, 1)
            row[f"{label}_maxdiff"] = diff
        rows.append(row)
    return {"op": "gemm_paths", "rows": rows}


def bench_gemv_ksplit(**_):
    """One-row GEMV of each V3.2 linear with the K split fixed at 1/2/4/8 warps
    per row group (and the heuristic's choice), CUDA-graph replays."""
    from ..config import v32_config

    cfg = v32_config(1)
    dev = "cuda"
    shapes = {"fused_a": (cfg.q_lora_rank + 640 + cfg.index_head_dim, cfg.dim),
              "fused_b": (cfg.n_heads * (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
                          + cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank),
              "o_proj": (cfg.dim, cfg.n_heads * cfg.v_head_dim), "gate_up": (2 * cfg.intermediate_size, cfg.dim),
              "down": (cfg.dim, cfg.intermediate_size)}
    rows = []
    for name, (N, K) in shapes.items():
        w, s = quantize_weight_blocks(torch.randn(N, K, device=dev) * 0.02)
        q, s_t = ops.quantize_act(torch.randn(1, K, device=dev).bfloat16())
        out = torch.empty(1, N, device=dev, dtype=torch.bfloat16)
        row = {"gemm": name, "N": N, "K": K}
        for ks in (0, 1, 2, 4, 8):
            ops.lib().set_gemv_k_split(ks)
            try:
                row[f"ks{ks}_us"] = round(time_fn(lambda: ops.fp8_gemm(q, s_t, w, s, out=out)) * 1e3, 2)
            finally:
                ops.lib().set_gemv_k_split(0)
        rows.append(row)
    return {"op": "gemv_ksplit", "graph": GRAPH, "rows": rows}


def bench_decode_gemms(M=1, **_):
    """The projections of one DeepSeek-V3.2 layer and the LM head at decode row
    counts 1, 2, 4, 8 (up to ``M``): weight bytes streamed per call on the
    GEMV and on the tensor-core tile kernels, against the measured copy
    bandwidth (power-of-two block scales)."""
    from ..config import v32_config

    cfg = v32_config(1)
    dev = "cuda"
    shapes = {  # name: (N, K, fp8)
        "fused_a": (cfg.q_lora_rank + 640 + cfg.index_head_dim, cfg.dim, True),
        "fused_b": (cfg.n_heads * (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
                    + cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank, True),
        "o_proj": (cfg.dim, cfg.n_heads * cfg.v_head_dim, True),
        "gate_up": (2 * cfg.intermediate_size, cfg.dim, True),
        "down": (cfg.dim, cfg.intermediate_size, True),
        "lm_head_bf16": (cfg.vocab_size, cfg.dim, False),
    }
    hbm = _peaks()["hbm_gbs"]
    rows = []
    for name, (N, K, fp8) in shapes.items():
        if fp8:
            w, s = quantize_weight_blocks(torch.randn(N, K, device=dev) * 0.02)
            nbytes = N * K
        else:
            w = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
            nbytes = 2 * N * K
        for m in (1, 2, 4, 8):
            if m > max(M, 1):
                break
            x = torch.randn(m, K, device=dev).bfloat16()
            if fp8:
                q, s_t = ops.quantize_act(x)
                out = torch.empty(m, N, device=dev, dtype=torch.bfloat16)
                fn = lambda: ops.fp8_gemm(q, s_t, w, s, out=out)  # noqa: E731
            else:
                fn = lambda: ops.linear(x, w)  # noqa: E731
            row = {"gemm": name, "M": m, "N": N, "K": K}
            for label, on in (("gemv", True), ("tiles", False)):
                ops.lib().set_decode_gemv(on)
                try:
                    ms = time_fn(fn)
                finally:
                    ops.lib().set_decode_gemv(True)
                row[f"{label}_us"] = round(ms * 1e3, 2)
                row[f"{label}_frac_hbm"] = round(nbytes / ms / 1e6 / hbm, 3)
            rows.append(row)
        del w
    return {"op": "decode_gemms", "graph": GRAPH, "rows": rows}


def bench_indexer(Q=1024, N=65536, **_):
    dev = "cuda"
    q = (torch.randn(Q, 64, 128, device=dev) * 2).to(torch.float8_e4m3fn)
    k = (torch.randn(N, 128, device=dev) * 2).to(torch.float8_e4m3fn)
    w = torch.randn(Q, 64, device=dev)
    ks = torch.rand(N, device=dev)
    out = torch.empty(Q, N, device=dev)
    start = N - Q
    ms = time_fn(lambda: ops.lib().indexer_logits(q, k, w, ks, out, start))
    visible = Q * start + Q * (Q + 1) / 2
    flops = 2.0 * 64 * 128 * visible
    return {"op": "indexer_logits", "Q": Q, "N": N, "ms": ms, "tflops": flops / ms / 1e9,
            **roofline(ms, flops=flops, nbytes=N * 132 + Q * 64 * 132 + visible * 4, fp8=True)}


def bench_indexer_select(Q=1024, N=65536, k=2048, **_):
    """Fused selection (ops.indexer_select) against indexer logits + exact top-k
    (index order), the same causal rows; the outputs are checked equal."""
    dev = "cuda"
    q = (torch.randn(Q, 64, 128, device=dev) * 2).to(torch.float8_e4m3fn)
    kk = (torch.randn(N, 128, device=dev) * 2).to(torch.float8_e4m3fn)
    w = torch.randn(Q, 64, device=dev)
    ks = torch.rand(N, device=dev) + 0.05
    out = torch.empty(Q, N, device=dev)
    start = N - Q

    def separate():
        ops.lib().indexer_logits(q, kk, w, ks, out, start)
        return ops.exact_topk(out, k, causal_start=start, n=N, order="index")

    def fused():
        return ops.indexer_select(q, kk, w, ks, start, k, logits_buf=out, order="index")

    ref_ids = separate()[1]
    diag = torch.zeros(3, dtype=torch.int64, device=dev)
    got_ids = ops.indexer_select(q, kk, w, ks, start, k, logits_buf=out, order="index", diag=diag)[1]
    equal = bool(torch.equal(ref_ids, got_ids))
    redone, kept, most = (int(x) for x in diag.tolist())
    ms_sep = time_fn(separate)
    ms_fused = time_fn(fused)
    return {"op": "indexer_select", "Q": Q, "N": N, "k": k, "ms": ms_fused, "separate_ms": ms_sep,
            "speedup": ms_sep / ms_fused, "ids_equal": equal, "rows_redone": redone,
            "candidates_per_row": kept / Q, "max_candidates": most}


def bench_topk(R=1024, N=65536, k=2048, clustered=False, order="value", causal=False, **_):
    dev = "cuda"
    s = torch.randn(R, N, device=dev)
    if clustered:  # indexer-like: most logits within a narrow band
        s = 10.0 + 0.05 * s
    cs = N - R if causal else None
    ms = time_fn(lambda: ops.exact_topk(s, k, causal_start=cs, order=order))
    return {"op": "topk", "R": R, "N": N, "k": k, "clustered": clustered, "order": order, "causal": causal,
            "ms": ms, "read_gbs": R * N * 4 / ms / 1e6, **roofline(ms, nbytes=R * N * 4 + R * k * 8)}


def _p2p_single():
    """The fused peer-memory GEMMs with world = 1 (self-push through the same
    symmetric-heap protocol): kernel profiling without a multi-rank launch."""
    from ..models.deepseek_v32.weights import Linear
    from ..parallel.groups import single
    from ..parallel.p2p import P2PComm

    return P2PComm(single("cuda")), Linear


def bench_ag_gemm(M=1024, N=2304, Kdim=7168, **_):
    comm, Linear = _p2p_single()
    dev = "cuda"
    w, s = quantize_weight_blocks(torch.randn(N, Kdim, device=dev) * 0.02)
    lin = Linear(w, s)
    x = torch.randn(M, Kdim, device=dev).bfloat16()
    qx = ops.quantize_act(x)
    got, want = comm.ag_linear(lin, x, qx, M), lin(quantized=qx)
    ops.check_errors(dev)
    err = ((got.float() - want.float()).abs().max() / want.float().abs().max()).item()
    ms = time_fn(lambda: comm.ag_linear(lin, x, qx, M))
    ref = time_fn(lambda: lin(quantized=qx))
    flops = 2.0 * M * N * Kdim
    return {"op": "ag_gemm(world=1)", "M": M, "N": N, "K": Kdim, "ms": ms, "plain_gemm_ms": ref,
            "tflops": flops / ms / 1e9, "max_rel_diff_vs_plain": err}


def bench_rs_gemm(M=1024, N=7168, Kdim=2304, **_):
    comm, Linear = _p2p_single()
    dev = "cuda"
    w, s = quantize_weight_blocks(torch.randn(N, Kdim, device=dev) * 0.02)
    lin = Linear(w, s)
    h = torch.randn(M, Kdim, device=dev).bfloat16()
    qh = ops.quantize_act(h)
    ms = time_fn(lambda: comm.linear_rs(lin, h, qh))
    ref = time_fn(lambda: lin(quantized=qh))
    flops = 2.0 * M * N * Kdim
    return {"op": "rs_gemm(world=1)", "M": M, "N": N, "K": Kdim, "ms": ms, "plain_gemm_ms": ref,
            "tflops": flops / ms / 1e9}


def bench_copy_curve(**_):
    """Device-to-device copy time against size (L2 flushed before each call): the
    size-dependent floor of any kernel that streams that many bytes once
    (launch, ramp-up and tail included), to set the decode linears against."""
    dev = "cuda"
    hbm = _peaks()["hbm_gbs"]
    rows = []
    for mb in (8, 16, 32, 64, 128, 256):
        n = mb << 20
        src = torch.empty(n, dtype=torch.uint8, device=dev).fill_(1)
        dst = torch.empty_like(src)
        ms = time_fn(lambda: dst.copy_(src))
        rows.append({"read_mb": mb, "us": round(ms * 1e3, 2), "read_gbs": round(n / ms / 1e6, 1),
                     "rw_frac_of_measured": round(2 * n / ms / 1e6 / hbm, 3)})
        del src, dst
    return {"op": "copy_curve", "graph": GRAPH, "rows": rows}


OPS = {"sparse_mla": bench_sparse_mla, "fp8_gemm": bench_fp8_gemm, "indexer": bench_indexer,
       "indexer_select": bench_indexer_select, "topk": bench_topk, "decode_gemms": bench_decode_gemms,
       "ag_gemm": bench_ag_gemm, "rs_gemm": bench_rs_gemm, "copy_curve": bench_copy_curve,
       "gemm_paths": bench_gemm_paths, "gemv_ksplit": bench_gemv_ksplit}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--op", default="all")
    p.add_argument("--T", type=int, default=256)
    p.add_argument("--K", type=int, default=2048)
    p.add_argument("--P", type=int, default=65664)
    p.add_argument("--splits", type=int, default=1)
    p.add_argument("--impl", type=int, default=0)
    p.add_argument("--locality", type=float, default=0.0)
    p.add_argument("--R", type=int, default=1024)
    p.add_argument("--clustered", action="store_true")
    p.add_argument("--order", default="value", choices=("value", "index"), help="topk: output order")
    p.add_argument("--causal", action="store_true", help="topk: rows end at N - R + r (prefill chunk)")
    p.add_argument("--M", type=int, default=1024)
    p.add_argument("--N", type=int, default=36864)
    p.add_argument("--Kdim", type=int, default=7168)
    p.add_argument("--block-scaled", action="store_true", help="fp8_gemm: block-scaled (UE8M0) tensor-core path")
    p.add_argument("--pair", action="store_true", help="fp8_gemm: 2-CTA 256-row tiles")
    p.add_argument("--trace", action="store_true", help="sparse_mla: phase clocks of the first cluster")
    p.add_argument("--graph", action="store_true", help="time CUDA-graph replays (small, launch-bound ops)")
    a = p.parse_args()
    global GRAPH
    GRAPH = a.graph
    names = list(OPS) if a.op == "all" else a.op.split(",")
    for name in names:
        kw = dict(T=a.T, K=a.K, P=a.P, splits=a.splits, impl=a.impl, locality=a.locality, trace=a.trace)
        if name == "fp8_gemm":
            kw = dict(M=a.M, N=a.N, K=a.Kdim, ue8m0=a.block_scaled, pair=a.pair)
        if name in ("ag_gemm", "rs_gemm"):
            kw = dict(M=a.M, N=a.N, Kdim=a.Kdim)
        if name in ("indexer", "indexer_select"):
            kw = dict(Q=a.R)
        if name in ("decode_gemms", "gemm_paths"):
            kw = dict(M=a.M)
        if name == "topk":
            kw = dict(R=a.R, clustered=a.clustered, order=a.order, causal=a.causal)
        print(json.dumps(OPS[name](**kw)))
    torch.cuda.synchronize()
    ops.check_errors("cuda")


if __name__ == "__main__":
    main()
