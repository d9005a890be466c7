"""Serve repeated GR users with persistent caches on one B200.

Reference: ``serving/run_multi_user.py:31-312``.  Builds the GR request stream
(heat-weighted users, exact history/candidate token budgets), a DeepSeek-V3.2
serving backend (a checkpoint directory, or ``--random-init`` weights of the
V3.2 architecture) and a :class:`PersistentGRRunner`, then prints one JSON
line per event: ``started``, one ``completed`` per request (its metrics), and
``finished`` (aggregate hit / eviction / latency summary).  There is no
separate warm-up: request latency includes first-use costs (CUDA graph capture
is not used by this path) but excludes weight loading and request generation.

Example::

    python -m cxldsagr_b200.serving.run_multi_user --random-init --scheme echo \\
        --num-users 16 --count 32 --history-tokens 32768 --candidate-tokens 1280 \\
        --resource-mode fixed-pools --sparse-pool-tokens 131072 --host-arena-tokens 524288
"""

from __future__ import annotations

import argparse
import json
import math
from collections import Counter
from pathlib import Path

SCHEMES = ("hbm", "echo", "serial_sparse", "dense_prefetch")


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter,
                                allow_abbrev=False)
    p.add_argument("--scheme", choices=SCHEMES, default="hbm")
    p.add_argument("--model-path", type=Path, help="checkpoint directory (config.json + safetensors)")
    p.add_argument("--random-init", action="store_true", help="random-init V3.2 weights instead of a checkpoint")
    p.add_argument("--num-layers", type=int, default=10, help="physical layers (copies of checkpoint layers 0-2)")
    p.add_argument("--tokenizer", type=Path, help="tokenizer.json (default: the built-in offline tokenizer)")
    p.add_argument("--heat-curves", type=Path, help="ranked traffic curve CSV (default: built-in Zipf curve)")
    p.add_argument("--num-users", type=int, default=8)
    p.add_argument("--count", type=int, default=16)
    p.add_argument("--max-revisits", type=int)
    p.add_argument("--sampling", choices=("weighted", "sequential"), default="weighted",
                   help="user order: heat-weighted draws, or every user in turn (rounds)")
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--history-tokens", type=int, default=16384, help="complete fixed prefix incl. instruction")
    p.add_argument("--candidate-tokens", type=int, default=1024, help="complete changing candidate suffix")
    p.add_argument("--context-limit", type=int)
    p.add_argument("--resource-mode", choices=("budget", "fixed-pools"), default="budget")
    p.add_argument("--hbm-budget-gib", type=float)
    p.add_argument("--dram-budget-gib", type=float)
    p.add_argument("--chunk-size", type=int, default=1024)
    p.add_argument("--sparse-pool-tokens", type=int, default=32768)
    p.add_argument("--host-arena-tokens", type=int)
    p.add_argument("--workspace-query-tokens", type=int)
    p.add_argument("--extend-chunk-size", type=int)
    p.add_argument("--native-token-validation", action="store_true")
    p.add_argument("--kv-format", choices=("bf16", "fp8"), default="bf16",
                   help="KV records: bf16 (1152 bytes) or fp8 (656-byte records in DRAM, dequantized rows in HBM)")
    p.add_argument("--device", default="cuda:0")
    return p


def validate_args(args, parser) -> None:
    for name in ("num_users", "count", "history_tokens", "candidate_tokens", "chunk_size", "sparse_pool_tokens"):
        if getattr(args, name) < 1:
            parser.error(f"--{name.replace('_', '-')} must be positive")
    if args.seed < 0:
        parser.error("--seed must be nonnegative")
    if args.max_revisits is not None and args.max_revisits < 0:
        parser.error("--max-revisits must be nonnegative")
    if args.sampling == "sequential" and args.max_revisits is not None:
        parser.error("--sampling sequential does not take --max-revisits")
    if (args.model_path is None) == (not args.random_init):
        parser.error("give exactly one of --model-path or --random-init")
    if args.resource_mode == "fixed-pools":
        if args.scheme not in ("echo", "serial_sparse"):
            parser.error("fixed-pools requires the echo or serial_sparse scheme")
        if args.host_arena_tokens is None:
            parser.error("fixed-pools requires explicit --host-arena-tokens (NH)")
        if args.hbm_budget_gib is not None or args.dram_budget_gib is not None:
            parser.error("fixed-pools does not accept HBM/DRAM byte sub-budgets")
        args.hbm_budget_bytes = args.dram_budget_bytes = None
    else:
        for name, default in (("hbm_budget_gib", 1.0), ("dram_budget_gib", 16.0)):
            v = getattr(args, name)
            v = default if v is None else v
            if not math.isfinite(v) or v < 0:
                parser.error(f"--{name.replace('_', '-')} must be finite and nonnegative")
            setattr(args, name, v)
        args.hbm_budget_bytes = int(args.hbm_budget_gib * 2**30)
        args.dram_budget_bytes = int(args.dram_budget_gib * 2**30)
        if args.hbm_budget_bytes < 1:
            parser.error("--hbm-budget-gib must allow at least one byte")
    if args.host_arena_tokens is not None and (args.host_arena_tokens < 64 or args.host_arena_tokens % 64):
        parser.error("--host-arena-tokens must be a positive multiple of 64")
    queries = max(args.chunk_size, args.extend_chunk_size or args.candidate_tokens)
    if args.workspace_query_tokens is None:
        args.workspace_query_tokens = queries
    elif args.workspace_query_tokens < queries:
        parser.error("--workspace-query-tokens must cover both prefill and extend batches")


def build_requests(args):
    from ..gr.workload import WorkloadConfig, build_workload

    wl = build_workload(WorkloadConfig(
        "deepseek_v32", args.num_users, args.count, history_tokens=args.history_tokens,
        candidate_tokens=args.candidate_tokens, seed=args.seed, max_revisits=args.max_revisits,
        context_limit=args.context_limit, heat_path=str(args.heat_curves) if args.heat_curves else None,
        sampling=args.sampling),
        tokenizer=args.tokenizer)
    return wl


def build_backend(args):
    import torch

    from ..checkpoint import StateDictSource, random_state_dict
    from ..config import v32_config
    from ..models.deepseek_v32.serving import DeepSeekServingBackend

    device = torch.device(args.device)
    if device.type == "cuda":
        torch.cuda.set_device(device)
    common = dict(scheme=args.scheme, device=device, num_layers=args.num_layers, chunk_size=args.chunk_size,
                  sparse_pool_tokens=args.sparse_pool_tokens, host_arena_tokens=args.host_arena_tokens,
                  workspace_query_tokens=args.workspace_query_tokens, extend_chunk_size=args.extend_chunk_size,
                  candidate_tokens=args.candidate_tokens, kv_format=args.kv_format)
    if args.random_init:
        cfg = v32_config(3)
        src = StateDictSource(random_state_dict(cfg, layers=range(3), seed=args.seed, device=device), cfg)
        return DeepSeekServingBackend(source=src, cfg=cfg, **common)
    return DeepSeekServingBackend(args.model_path, **common)


def _emit(value) -> None:
    print(json.dumps(value, ensure_ascii=False, default=str), flush=True)


def main(argv=None) -> None:
    parser = build_parser()
    args = parser.parse_args(argv)
    validate_args(args, parser)
    from .persistent import PersistentGRRunner

    workload = build_requests(args)
    backend = build_backend(args)
    try:
        _emit({"status": "started", "scheme": args.scheme, "num_users": args.num_users, "count": args.count,
               "history_tokens": args.history_tokens, "candidate_tokens": args.candidate_tokens,
               "resource_mode": args.resource_mode.replace("-", "_"), "hbm_budget_bytes": args.hbm_budget_bytes,
               "dram_budget_bytes": args.dram_budget_bytes, "workload_sha256": workload.manifest["workload_sha256"],
               "timing": "no separate warmup; excludes weight loading and request generation",
               "heat": workload.manifest["heat"], "backend": backend.describe()})
        done = revisits = hits = evicted = 0
        per_user = Counter()
        total_ms = revisit_ms = 0.0
        limits = {"max_session_capacity": args.history_tokens + args.candidate_tokens,
                  "max_history_tokens": args.history_tokens, "max_candidate_tokens": args.candidate_tokens}
        with PersistentGRRunner(backend, hbm_budget_bytes=args.hbm_budget_bytes,
                                dram_budget_bytes=args.dram_budget_bytes, resource_limits=limits,
                                native_token_validation=args.native_token_validation) as runner:
            for result in runner.run(workload.requests):
                m = result.metrics
                _emit({"status": "completed", "metrics": m, "hidden_shape": list(result.hidden.shape),
                       "hidden_dtype": str(result.hidden.dtype), "hidden_device": str(result.hidden.device)})
                done += 1
                per_user[m["user_id"]] += 1
                revisits += m["is_revisit"]
                hits += m["prefix_cache_hit"]
                evicted += len(m["evicted_users"])
                total_ms += m["latency_ms"]
                revisit_ms += m["latency_ms"] if m["is_revisit"] else 0.0
        _emit({"status": "finished", "requests": done, "first_visits": done - revisits, "revisits": revisits,
               "returning_users": sum(c > 1 for c in per_user.values()), "prefix_cache_hits": hits,
               "evicted_users": evicted, "mean_latency_ms": total_ms / done if done else None,
               "revisit_mean_latency_ms": revisit_ms / revisits if revisits else None, "separate_warmup": False})
    except BaseException as exec_error:
        try:
            backend.close()
        except BaseException as close_error:  # noqa: BLE001 - keep both failures
            raise BaseExceptionGroup("serving execution and backend close failed", [exec_error, close_error]) from None
        raise
    else:
        backend.close()


if __name__ == "__main__":
    main()
