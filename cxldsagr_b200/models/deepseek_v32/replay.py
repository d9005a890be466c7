"""Replay workload over physical copies of checkpoint layers 0, 1 and 2.

Reference semantics (``models/deepseek_v32/replay.py:12-97``): a model of
``L >= 3`` physical blocks whose block ``l`` holds its own copy of checkpoint
layer ``l % 3``.  Blocks 0-2 run as a normal sequential model; every later
block receives a private clone of the input (hidden, residual) that its source
block received in the same chunk.  This gives the memory footprint and the
per-layer work of an ``L``-layer model from a three-layer checkpoint; it is a
workload, not a trained model.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

_ENDPOINTS = ("model.embed_tokens.weight", "model.norm.weight", "lm_head.weight")


def _check_layers(n):
    if type(n) is not int or n < 3:
        raise ValueError("the replay model requires at least three physical layers")


def replay_parameter_count(reader, num_layers: int) -> dict:
    """Parameter counts (FP8 scale tensors excluded) of an ``num_layers`` replay model."""
    _check_layers(num_layers)
    meta = reader.tensor_metadata
    per_source = []
    for src in range(3):
        prefix = f"model.layers.{src}."
        names = [n for n in meta if n.startswith(prefix)]
        if not names:
            raise ValueError(f"checkpoint is missing source layer {src}")
        per_source.append(sum(math.prod(meta[n]["shape"]) for n in names if not n.endswith(".weight_scale_inv")))
    endpoints = sum(math.prod(meta[n]["shape"]) for n in _ENDPOINTS)
    backbone = sum(per_source[layer % 3] for layer in range(num_layers))
    return {
        "source_layer_parameters": per_source,
        "backbone_parameters": backbone,
        "endpoint_parameters": endpoints,
        "total_parameters": endpoints + backbone,
    }


@dataclass(frozen=True)
class ReplayLayout:
    source_layers: tuple

    @classmethod
    def repeated_sources(cls, physical_layers: int) -> "ReplayLayout":
        _check_layers(physical_layers)
        return cls(tuple(layer % 3 for layer in range(physical_layers)))

    def __post_init__(self):
        n = len(self.source_layers)
        if n < 3 or tuple(self.source_layers) != tuple(i % 3 for i in range(n)):
            raise ValueError("replay requires checkpoint sources 0, 1, 2 in repeating order")

    def begin_chunk(self) -> "ReplayInputs":
        return ReplayInputs(self)


@dataclass
class ReplayInputs:
    """Per-chunk record of the source blocks' inputs."""

    layout: ReplayLayout
    sources: list = field(default_factory=list)

    def for_layer(self, layer: int, hidden, residual, *, scope=None, copy_source: bool = True):
        if layer < 3:
            self.sources.append((hidden, residual))
            return hidden, residual
        src_hidden, src_residual = self.sources[self.layout.source_layers[layer]]
        if not copy_source:
            return src_hidden, src_residual
        return src_hidden.clone(), (None if src_residual is None else src_residual.clone())
