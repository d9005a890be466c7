"""Sparse KV fetch microbenchmark (the reference's cache-manager fetch path,
``experiments/cache_manager_performance``; recall through
``cache/sparse_token_cache.py:502-569`` and ``operators/common/kv_transfer.py:21``).

One "layer" on one GPU: FP8 lightning-indexer logits of Q queries over an
N-token context (random BF16 queries/keys quantised to E4M3), exact
top-2048, the exact recall of the selected rows that are not resident in the
HBM pool from pinned DRAM (576-wide BF16 MLA records, 1,152 B), and sparse
MLA over the pool.  ``--hit`` sets the fraction of the selected rows made
resident before each timed step.  Each phase is timed with CUDA events on
the launching stream; the fetch is also run overlapped with another layer's
sparse MLA (a second cache, its recall on a side stream), which is how the
offload methods hide it across layers.  The PCIe roofline is a pinned
host-to-device copy measured in the same process.

Run on 1..8 GPUs with torchrun (one independent fetch per GPU; rank 0 prints
the max time over ranks and the summed bandwidth)::

    python -m cxldsagr_b200.evaluation.kv_fetch_bench --context 65536 --hit 0.5
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m cxldsagr_b200.evaluation.kv_fetch_bench ...

``--cp`` (with torchrun): one context shared by all ranks; the indexer and
top-k are split by keys (every rank scores all queries against its key shard,
the (score, id) lists are all-gathered and merged, ``parallel.cp_indexer``),
and each rank then fetches and attends for its share of the queries.
``--kv-format fp8``: 656-byte FP8 records in pinned DRAM (1,152-byte BF16
otherwise).
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from .. import ops
from ..cache.sparse_token_cache import SparseTokenCache
from ..parallel import cp_indexer
from ..parallel.groups import ParallelContext, shard_range

WIDTH = 576
TOPK = 2048


def _ev():
    return torch.cuda.Event(enable_timing=True)


def pcie_h2d_gbs(dev, nbytes=256 << 20, reps=5) -> float:
    host = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    buf.copy_(host, non_blocking=True)
    torch.cuda.synchronize(dev)
    a, b = _ev(), _ev()
    a.record()
    for _ in range(reps):
        buf.copy_(host, non_blocking=True)
    b.record()
    b.synchronize()
    return nbytes * reps / (a.elapsed_time(b) * 1e-3) / 1e9


class Layer:
    """A context of N records in a pool of N slots, backed by pinned host memory."""

    def __init__(self, N: int, Q: int, dev, seed: int, kv_format: str = "bf16", cp=None):
        g = torch.Generator(device=dev).manual_seed(seed)
        self.cache = SparseTokenCache(N, WIDTH, device=dev, slots=N, kv_format=kv_format)
        self.cp = cp  # ParallelContext for the context-parallel selection, or None
        for s in range(0, N, 8192):
            n = min(8192, N - s)
            self.cache.begin_step(n)
            self.cache.append(torch.randn(n, WIDTH, device=dev, generator=g).bfloat16())
            self.cache.commit()
        self.q8 = (torch.randn(Q, 64, 128, device=dev, generator=g) * 2).to(torch.float8_e4m3fn)
        self.k8 = (torch.randn(N, 128, device=dev, generator=g) * 2).to(torch.float8_e4m3fn)
        self.w = torch.randn(Q, 64, device=dev, generator=g)
        self.ks = torch.rand(N, device=dev, generator=g)
        self.qa = (torch.randn(Q, 128, WIDTH, device=dev, generator=g) * 0.5).bfloat16()
        self.N, self.Q = N, Q
        self.rows = (0, Q) if cp is None else shard_range(Q, cp.world, cp.rank)
        self.logits = torch.empty(Q, N, device=dev) if cp is None else None
        self.ids = None

    def select(self):
        if self.cp is None:
            ops.lib().indexer_logits(self.q8, self.k8, self.w, self.ks, self.logits, self.N - self.Q)

    def topk(self):
        if self.cp is None:
            _, self.ids = ops.exact_topk(self.logits, TOPK, causal_start=self.N - self.Q, n=self.N)
            return
        k0, k1 = cp_indexer.key_shard(self.N, self.cp.world, self.cp.rank)
        _, ids = cp_indexer.cp_exact_topk(self.cp, self.q8, self.k8[k0:k1], self.w, self.ks[k0:k1], k0,
                                          self.N - self.Q, TOPK)
        self.ids = ids[self.rows[0]:self.rows[1]].contiguous()

    def set_residency(self, hit: float, gen: torch.Generator):
        """Drop every HBM copy, then make a random ``hit`` fraction of the selected rows resident."""
        pool = self.cache._pool
        pool.drain()
        pool.release_ids(0, self.cache.session.global_ids())
        uniq = torch.unique(self.ids[self.ids >= 0])
        keep = uniq[torch.rand(uniq.numel(), device=uniq.device, generator=gen) < hit]
        if keep.numel():
            self.cache.ensure(keep.view(1, -1).int())
        return int(uniq.numel())

    def fetch(self):
        return self.cache.ensure(self.ids)

    def mla(self, phys):
        return ops.sparse_mla(self.qa[self.rows[0]:self.rows[1]], self.cache.records, phys, 0.0723)

    def recalled(self) -> int:
        return int(self.cache.stats.recalled_records)


def run(N: int, Q: int, hit: float, reps: int, dev, kv_format: str = "bf16", cp=None) -> dict:
    a, b = Layer(N, Q, dev, 1, kv_format, cp), Layer(N, Q, dev, 2, kv_format, cp)
    for L in (a, b):
        L.select()
        L.topk()
    gen = torch.Generator(device=dev).manual_seed(3)
    phases = {"indexer": [], "topk": [], "fetch": [], "mla": [], "serial": [], "overlapped": []}
    rows = []
    side = torch.cuda.Stream(dev)
    for rep in range(reps + 2):  # two warm-up steps
        uniq = a.set_residency(hit, gen)
        b.set_residency(hit, gen)
        torch.cuda.synchronize(dev)
        before = a.recalled()
        e = [_ev() for _ in range(5)]
        e[0].record()
        a.select()
        e[1].record()
        a.topk()
        e[2].record()
        phys = a.fetch()
        e[3].record()
        a.mla(phys)
        e[4].record()
        torch.cuda.synchronize(dev)
        recalled = a.recalled() - before
        # Overlapped: layer b's fetch on a side stream while layer a's MLA runs.
        a.set_residency(1.0, gen)
        phys_a = a.fetch()
        b_before = b.recalled()
        torch.cuda.synchronize(dev)
        o0, o1 = _ev(), _ev()
        main = torch.cuda.current_stream(dev)
        o0.record()
        side.wait_stream(main)
        with torch.cuda.stream(side):
            phys_b = b.fetch()
        a.mla(phys_a)
        main.wait_stream(side)
        o1.record()
        torch.cuda.synchronize(dev)
        del phys_b
        if rep < 2:
            continue
        t = [e[i].elapsed_time(e[i + 1]) for i in range(4)]
        for k, v in zip(("indexer", "topk", "fetch", "mla"), t):
            phases[k].append(v)
        phases["serial"].append(sum(t))
        phases["overlapped"].append(o0.elapsed_time(o1))
        rows.append((uniq, recalled, b.recalled() - b_before))
    med = {k: sorted(v)[len(v) // 2] for k, v in phases.items()}
    uniq, recalled, _ = rows[len(rows) // 2]
    return {"ms": med, "selected_unique_rows": uniq, "recalled_rows": recalled,
            "fetch_bytes": recalled * a.cache.record_bytes, "record_bytes": a.cache.record_bytes}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--context", type=int, default=65536)
    p.add_argument("--queries", type=int, default=128)
    p.add_argument("--hit", type=float, default=0.0)
    p.add_argument("--reps", type=int, default=5)
    p.add_argument("--kv-format", choices=("bf16", "fp8"), default="bf16")
    p.add_argument("--cp", action="store_true", help="one shared context, indexer split by keys across ranks")
    a = p.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
    cp = None
    if a.cp:
        import torch.distributed as dist

        cp = ParallelContext(rank, world, dist.group.WORLD if world > 1 else None, dev)
    pcie = pcie_h2d_gbs(dev)
    r = run(a.context, a.queries, a.hit, a.reps, dev, a.kv_format, cp)
    fetch_gbs = r["fetch_bytes"] / (r["ms"]["fetch"] * 1e-3) / 1e9 if r["ms"]["fetch"] > 0 else 0.0
    if world > 1:
        import torch.distributed as dist

        names = ("indexer", "topk", "fetch", "mla", "serial", "overlapped")
        t = torch.tensor([r["ms"][k] for k in names], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        bw = torch.tensor([fetch_gbs, pcie], device=dev)
        dist.all_reduce(bw)
        r["ms"] = dict(zip(names, t.tolist()))
        fetch_gbs, pcie = bw.tolist()
        dist.destroy_process_group()
    if rank == 0:
        out = {"op": "kv_fetch", "gpus": world, "context": a.context, "queries": a.queries, "topk": TOPK,
               "hit": a.hit, "kv_format": a.kv_format, "context_parallel_selection": a.cp,
               **r, "fetch_gbs": fetch_gbs, "pcie_h2d_gbs": pcie,
               "fetch_frac_of_pcie": fetch_gbs / pcie if pcie else None,
               "timing": "CUDA events, median of reps after 2 warm-up steps; max over ranks"}
        print(json.dumps(out))


if __name__ == "__main__":
    main()
