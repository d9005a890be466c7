"""Process-group layout for multi-GPU serving (one process per GPU).

The reference runs single-process with sequential layer placement
(``models/deepseek_v32/model.py:34-60,874-894``); it has no collectives.  The
B200 framework adds the layouts a DeepSeek-V3.2 box needs:

* ``sp`` (sequence parallel): the hidden stream of a chunk is sharded by
  tokens across the ``R`` ranks; attention projections start with an
  all-gather (AG -> GEMM), the attention core runs on the rank's own queries
  with all 128 heads, the dense MLP is column/row parallel (AG -> GEMM,
  GEMM -> reduce-scatter);
* ``ep`` (expert parallel): the 256 routed experts are split evenly, tokens
  are dispatched to the owners and combined back (all-to-all);
* ``dp`` (data parallel): independent replicas serve different requests.

``ParallelContext`` holds the group and this rank's coordinates and the
communication backend (``torch`` = NCCL/gloo collectives, the baseline;
``p2p`` = this package's fused peer-memory kernels, GPU only).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


def shard_sizes(total: int, parts: int) -> list[int]:
    """Balanced split: the first ``total % parts`` shards get one extra row."""
    base, extra = divmod(total, parts)
    return [base + (i < extra) for i in range(parts)]


def shard_range(total: int, parts: int, index: int) -> tuple[int, int]:
    sizes = shard_sizes(total, parts)
    start = sum(sizes[:index])
    return start, start + sizes[index]


@dataclass
class ParallelContext:
    rank: int
    world: int
    group: object | None
    device: torch.device
    backend: str = "torch"          # "torch" (NCCL/gloo collectives) or "p2p" (fused peer-memory kernels)
    ep: bool = True                 # experts sharded across the group
    vocab_parallel: bool = True     # embedding table and LM head split by vocabulary rows
    cp_indexer: bool = False        # indexer split by keys across ranks (every query scored on every rank's shard)

    @property
    def is_parallel(self) -> bool:
        return self.world > 1

    def expert_range(self, n_experts: int) -> range:
        if not self.ep or self.world == 1:
            return range(n_experts)
        if n_experts % self.world:
            raise ValueError("routed experts must divide evenly across ranks")
        per = n_experts // self.world
        return range(self.rank * per, (self.rank + 1) * per)

    def token_range(self, total: int) -> tuple[int, int]:
        return shard_range(total, self.world, self.rank)


def single(device) -> ParallelContext:
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    return ParallelContext(0, 1, None, dev)


def init_distributed(*, backend: str | None = None, timeout_s: float = 120.0, comm: str = "torch",
                     ep: bool = True) -> ParallelContext:
    """Initialise from torchrun's env (RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT).

    NCCL on GPUs (one device per local rank), gloo on CPU.  The short timeout
    makes a rank that never joins, or dies between steps, end the others'
    next collective with an error instead of a hang.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    use_cuda = torch.cuda.is_available() and backend != "gloo"
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    if world == 1:
        return ParallelContext(0, 1, None, device, backend=comm, ep=ep)
    if not dist.is_initialized():
        kw = {"device_id": device} if use_cuda else {}
        dist.init_process_group(backend or ("nccl" if use_cuda else "gloo"), timeout=timedelta(seconds=timeout_s), **kw)
    if comm == "p2p" and not use_cuda:
        raise ValueError("the p2p backend needs GPUs")
    return ParallelContext(rank, world, dist.group.WORLD, device, backend=comm, ep=ep)
