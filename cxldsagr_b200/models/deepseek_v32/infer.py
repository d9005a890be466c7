"""Standalone DeepSeek-V3.2 prefill + extend from a token-id file.

Reference: ``models/deepseek_v32/infer.py:14-46``.  Reads a JSON list of token
ids, prefills the first ``--history`` of them and extends with the rest, then
prints ``{"length": ..., "next_token_id": ...}``.  ``--random-init`` runs the
V3.2 architecture with random weights (no checkpoint needed).

    python -m cxldsagr_b200.models.deepseek_v32.infer --model ckpt/ --input-ids ids.json --history 65536
    python -m cxldsagr_b200.models.deepseek_v32.infer --model ckpt/ --devices 0,1,2,3 ...   # layers over 4 GPUs
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", type=Path, help="checkpoint directory")
    p.add_argument("--random-init", action="store_true")
    p.add_argument("--input-ids", type=Path, required=True, help="JSON token id list")
    p.add_argument("--history", type=int, default=65536)
    p.add_argument("--method", choices=("hbm", "echo", "serial_sparse", "dense_prefetch"), default="hbm")
    p.add_argument("--offload", action="store_true", help="shorthand for --method serial_sparse")
    p.add_argument("--sparse-pool-tokens", "--slots", dest="slots", type=int, default=16384)
    p.add_argument("--host-arena-tokens", type=int)
    p.add_argument("--chunk-size", type=int, default=2048)
    p.add_argument("--num-layers", type=int, help="run only the first N checkpoint layers")
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--devices", help="comma-separated GPU indices: place the layers over these GPUs "
                   "(contiguous runs by weight bytes; the reference's multi-GPU mode)")
    a = p.parse_args(argv)
    if (a.model is None) == (not a.random_init):
        p.error("give exactly one of --model or --random-init")
    import torch

    from ...checkpoint import CheckpointReader, StateDictSource, random_state_dict
    from ...config import CacheConfig, v32_config
    from .inputs import prepare_token_ids
    from .model import DeepSeekV32Model

    ids = json.loads(a.input_ids.read_text())
    if not 0 < a.history < len(ids):
        p.error("--history must leave a nonempty extension")
    devices = [torch.device("cuda", int(x)) for x in a.devices.split(",")] if a.devices else None
    dev = devices[0] if devices else torch.device(a.device)
    if a.random_init:
        cfg = v32_config(a.num_layers or 3)
        src = StateDictSource(random_state_dict(cfg, layers=range(cfg.num_hidden_layers), device=dev), cfg)
    else:
        src = CheckpointReader(a.model)
        cfg = src.config
    layers = list(range(a.num_layers)) if a.num_layers else None
    method = "serial_sparse" if a.offload else a.method
    cache = CacheConfig(method=method, capacity=len(ids), pool_tokens=a.slots if method != "hbm" else None,
                        host_tokens=a.host_arena_tokens, chunk_size=a.chunk_size,
                        candidate_tokens=len(ids) - a.history)
    model = DeepSeekV32Model(cfg, src, device=dev, cache=cache, layers=layers, devices=devices)
    tokens = prepare_token_ids(ids, device=dev, vocab_size=cfg.vocab_size, max_tokens=len(ids))
    model.prefill(tokens[: a.history])
    result = model.extend(tokens[a.history:])
    print(json.dumps({"length": model.length, "next_token_id": int(result.logits.argmax(-1))}))


if __name__ == "__main__":
    main()
