"""Shape matrix: prefill and cold-extend latency over history H x candidate A
for every cache method (the reference's MFU shape-matrix experiment,
``experiments/deepseek_v32_mfu/report/shape_matrix/results.md``, whose H200
rows are quoted beside ours).

For each H the model (DeepSeek-V3.2 layers 0-2 + embedding, final norm and
last-token LM head, random-init weights of the real shapes, uniform-random
token ids) is built once; for each method it switches to that cache (P = NH =
H + max A), prefills the H-token history once (timed), then for each A
captures the A-token extend in a CUDA graph (every method) and
times cold replays: before each replay the HBM copies of the history are
dropped (DRAM copies and indexer keys stay), as in the reference's cold
measurement.  Times are CUDA events on the launching stream, minimum over
``--reps`` replays after the capture's warm-up.

    python -m cxldsagr_b200.evaluation.shape_matrix --histories 16384,65536 --extends 128,1024

Check and bench are separate runs (the reference's receipt workflow,
``evaluation/motivation_validation.py:36-231``): ``--mode check`` runs every
cell once, requires each method's cold-extend logits to equal the resident
``hbm`` logits bit for bit, and writes a check receipt bound to the source
tree, the loaded native build and the matrix configuration; ``--mode bench``
(the default when ``--receipt`` is given) refuses to time anything unless
that receipt matches, and publishes no numbers from an unchecked build.
"""

from __future__ import annotations

import argparse
import hashlib
import json

import torch

# H200 (1 GPU) results of the reference's shape matrix, ms:
# (H, A) -> {method: (prefill, extend)}; None where the report has no cell.
REFERENCE_H200 = {
    (16384, 128): {"hbm": (133.099, 2.623), "echo": (134.267, 3.960), "serial_sparse": (133.087, 3.492),
                   "dense_prefetch": (132.410, 3.036)},
    (65536, 128): {"hbm": (644.938, 3.326), "echo": (648.375, 5.716), "serial_sparse": (640.701, 4.265),
                   "dense_prefetch": (645.800, 5.706)},
    (65536, 256): {"hbm": (None, 4.192)},
    (65536, 512): {"hbm": (None, 6.839)},
    (65536, 1024): {"hbm": (None, 12.155), "echo": (None, 17.981), "serial_sparse": (None, 13.231),
                    "dense_prefetch": (None, 12.339)},
}
METHODS = ("hbm", "serial_sparse", "echo", "dense_prefetch")


def _ints(text: str) -> list[int]:
    return [int(x) for x in text.split(",") if x]


def check_history(H: int, extends: list[int], methods, *, layers: int, kv_format: str, dev) -> dict:
    """One cold extend per (method, A): logits digests and bitwise equality with hbm."""
    from ..checkpoint import RandomSource
    from ..config import CacheConfig, v32_config
    from ..models.deepseek_v32.model import DeepSeekV32Model
    cfg = v32_config(layers=layers)
    cap = H + max(extends)
    src = RandomSource(cfg, layers=range(layers), seed=0, device=dev)
    model = DeepSeekV32Model(cfg, src, device=dev,
                             cache=CacheConfig(method="hbm", capacity=cap, chunk_size=2048, candidate_tokens=max(extends),
                                               host_tokens=cap, kv_format=kv_format))
    del src
    g = torch.Generator().manual_seed(H)
    hist = torch.randint(0, cfg.vocab_size, (H,), generator=g).to(dev)
    cands = {A: torch.randint(0, cfg.vocab_size, (A,), generator=g).to(dev) for A in extends}
    out, ref = {}, {}
    for method in ("hbm",) + tuple(m for m in methods if m != "hbm"):
        if method != model.cache_cfg.method:
            model.set_cache_method(method, pool_tokens=cap, host_tokens=cap, kv_format=kv_format)
        model.reset()
        model.prefill(hist)
        for A in extends:
            model.clear_residency()
            logits = model.extend(cands[A]).logits.float().cpu()
            model.session.truncate(H)
            if method == "hbm":
                ref[A] = logits
            key = f"H{H}/A{A}/{method}"
            out[key] = {"logits_sha256": hashlib.sha256(logits.numpy().tobytes()).hexdigest(),
                        "equal_to_hbm": bool(torch.equal(logits, ref[A])),
                        "finite": bool(torch.isfinite(logits).all())}
    del model
    torch.cuda.empty_cache()
    return out


def run_history(H: int, extends: list[int], methods, *, layers: int, kv_format: str, reps: int, dev) -> list[dict]:
    from ..checkpoint import RandomSource
    from ..config import CacheConfig, v32_config
    from ..models.deepseek_v32.model import DeepSeekV32Model

    cfg = v32_config(layers=layers)
    cap = H + max(extends)
    src = RandomSource(cfg, layers=range(layers), seed=0, device=dev)
    model = DeepSeekV32Model(cfg, src, device=dev,
                             cache=CacheConfig(method="hbm", capacity=cap, chunk_size=2048, candidate_tokens=max(extends),
                                               host_tokens=cap, kv_format=kv_format))
    del src
    g = torch.Generator().manual_seed(H)
    hist = torch.randint(0, cfg.vocab_size, (H,), generator=g).to(dev)
    cands = {A: torch.randint(0, cfg.vocab_size, (A,), generator=g).to(dev) for A in extends}
    stream = torch.cuda.current_stream(dev)
    rows = []
    for method in methods:
        if method != model.cache_cfg.method:
            model.set_cache_method(method, pool_tokens=cap, host_tokens=cap, kv_format=kv_format)
        model.reset()
        model.prefill(hist)  # warm-up (kernels, allocator)
        model.reset()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        model.prefill(hist)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        prefill_ms = e0.elapsed_time(e1)
        for A in extends:
            graph = model.capture_extend(A)
            times = []
            for _ in range(reps):
                model.clear_residency()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                if graph is not None:
                    graph.replay(cands[A])
                    b.record(stream)
                    graph.rollback()
                else:
                    model.extend(cands[A])
                    b.record(stream)
                    model.session.truncate(H)
                torch.cuda.synchronize(dev)
                times.append(a.elapsed_time(b))
            del graph
            ref = REFERENCE_H200.get((H, A), {}).get(method, (None, None))
            ext = min(times)
            rows.append({"history": H, "extend": A, "method": method, "kv_format": kv_format,
                         "prefill_ms": round(prefill_ms, 3), "extend_ms": round(ext, 4),
                         "h200_prefill_ms": ref[0], "h200_extend_ms": ref[1],
                         "extend_speedup_vs_h200": round(ref[1] / ext, 3) if ref[1] else None,
                         "prefill_speedup_vs_h200": round(ref[0] / prefill_ms, 3) if ref[0] else None})
    del model
    torch.cuda.empty_cache()
    return rows


def table(rows: list[dict]) -> str:
    lines = ["| H | A | method | prefill ms | extend ms | H200 extend ms | speed-up |", "|---|---|---|---|---|---|---|"]
    for r in rows:
        sp = r["extend_speedup_vs_h200"]
        lines.append(f"| {r['history']} | {r['extend']} | {r['method']} | {r['prefill_ms']:.1f} | {r['extend_ms']:.3f} | "
                     f"{r['h200_extend_ms'] if r['h200_extend_ms'] else '-'} | {f'{sp:.2f}x' if sp else '-'} |")
    return "\n".join(lines)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--histories", default="4096,16384,65536")
    p.add_argument("--extends", default="128,256,512,1024")
    p.add_argument("--methods", default=",".join(METHODS))
    p.add_argument("--layers", type=int, default=3)
    p.add_argument("--kv-format", choices=("bf16", "fp8"), default="bf16")
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--mode", choices=("check", "bench"), default=None,
                   help="check: bitwise method agreement + receipt; bench: timing, requires a check receipt")
    p.add_argument("--receipt", default=None, help="receipt path (written by check, required by bench)")
    a = p.parse_args(argv)
    methods = [m for m in a.methods.split(",") if m]
    for m in methods:
        if m not in METHODS:
            raise SystemExit(f"unknown method {m}")
    from . import validation

    mode = a.mode or ("bench" if a.receipt else None)
    ident = {"harness": "shape_matrix", "histories": _ints(a.histories), "extends": _ints(a.extends),
             "methods": methods, "layers": a.layers, "kv_format": a.kv_format}
    if mode == "bench":
        if not a.receipt:
            raise SystemExit("--mode bench needs the --receipt of a check run")
        validation.require_receipt(a.receipt, "check", ident)   # before any device work
    dev = torch.device(a.device)
    torch.cuda.set_device(dev)
    if mode == "check":
        if not a.receipt:
            raise SystemExit("--mode check needs --receipt PATH to write")
        evidence = {}
        for H in _ints(a.histories):
            evidence.update(check_history(H, _ints(a.extends), methods, layers=a.layers, kv_format=a.kv_format,
                                          dev=dev))
        bad = [k for k, v in evidence.items() if not (v["equal_to_hbm"] and v["finite"])]
        if bad:
            print(json.dumps({"check": "failed", "cells": bad}))
            return 1
        validation.write_receipt(a.receipt, "check", ident, evidence)
        print(json.dumps({"check": "passed", "cells": len(evidence), "receipt": a.receipt}))
        return 0
    rows = []
    for H in _ints(a.histories):
        rows += run_history(H, _ints(a.extends), methods, layers=a.layers, kv_format=a.kv_format, reps=a.reps,
                            dev=dev)
        for r in rows[-len(methods) * len(_ints(a.extends)):]:
            print(json.dumps(r), flush=True)
    print(table(rows))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
