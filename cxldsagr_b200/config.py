"""Model, cache and parallel configuration.

``ModelConfig`` carries the DeepSeek-V3.2 dimensions, YaRN rotary parameters,
quantisation format and MoE routing constants.  It reads the same
``config.json`` keys as the upstream checkpoint (reference:
``models/deepseek_v32/config.py:12-143``) so a real checkpoint directory and the
random-init writer in :mod:`cxldsagr_b200.checkpoint` are interchangeable.
"""

from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass, field, replace
from pathlib import Path


@dataclass(frozen=True)
class ModelConfig:
    dim: int = 7168
    n_heads: int = 128
    q_lora_rank: int = 1536
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    index_n_heads: int = 64
    index_head_dim: int = 128
    index_topk: int = 2048
    num_hidden_layers: int = 61
    vocab_size: int = 129280
    norm_eps: float = 1e-6
    max_seq_len: int = 163840
    original_seq_len: int = 4096
    rope_theta: float = 10000.0
    rope_factor: float = 40.0
    beta_fast: float = 32.0
    beta_slow: float = 1.0
    mscale: float = 1.0
    scale_fmt: str | None = "ue8m0"
    weight_block_size: tuple[int, int] = (128, 128)
    intermediate_size: int = 18432
    moe_intermediate_size: int = 2048
    n_routed_experts: int = 256
    n_shared_experts: int = 1
    num_experts_per_tok: int = 8
    n_group: int = 8
    topk_group: int = 4
    first_k_dense_replace: int = 3
    norm_topk_prob: bool = True
    scoring_func: str = "sigmoid"
    routed_scaling_factor: float = 2.5
    # "fp8" keeps checkpoint FP8 weights with 128x128 block scales, "bf16"
    # stores dense BF16 weights (used by the CPU tiny model).
    weight_dtype: str = "fp8"
    raw: dict = field(default_factory=dict, repr=False, compare=False)

    # ------------------------------------------------------------------ io
    _JSON_RENAMES = {
        "dim": "hidden_size",
        "n_heads": "num_attention_heads",
        "norm_eps": "rms_norm_eps",
        "max_seq_len": "max_position_embeddings",
    }
    _JSON_FIELDS = (
        "q_lora_rank", "kv_lora_rank", "qk_nope_head_dim", "qk_rope_head_dim",
        "v_head_dim", "index_n_heads", "index_head_dim", "index_topk",
        "num_hidden_layers", "vocab_size", "rope_theta", "intermediate_size",
        "moe_intermediate_size", "n_routed_experts", "n_shared_experts",
        "num_experts_per_tok", "n_group", "topk_group", "first_k_dense_replace",
        "norm_topk_prob", "scoring_func", "routed_scaling_factor",
    )
    _ROPE_FIELDS = (
        ("original_seq_len", "original_max_position_embeddings"),
        ("rope_factor", "factor"),
        ("beta_fast", "beta_fast"),
        ("beta_slow", "beta_slow"),
        ("mscale", "mscale"),
    )

    @classmethod
    def from_json(cls, raw: dict) -> "ModelConfig":
        rope = raw.get("rope_scaling") or {}
        if rope and rope.get("rope_type", rope.get("type", "yarn")) != "yarn":
            raise ValueError("only YaRN rotary scaling is supported")
        quant = raw.get("quantization_config")
        if quant is not None and quant.get("quant_method", "fp8") != "fp8":
            raise ValueError("weights must be BF16 or block-FP8")
        values = {dst: raw[src] for dst, src in cls._JSON_RENAMES.items() if src in raw}
        values.update({name: raw[name] for name in cls._JSON_FIELDS if name in raw})
        for dst, src in cls._ROPE_FIELDS:
            if src in rope:
                values[dst] = rope[src]
        if quant is not None:
            values["scale_fmt"] = quant.get("scale_fmt")
            values["weight_block_size"] = tuple(quant.get("weight_block_size", (128, 128)))
            values["weight_dtype"] = "fp8"
        else:
            values["weight_dtype"] = "bf16"
            values["scale_fmt"] = raw.get("index_scale_fmt", "ue8m0")
        values["raw"] = raw
        return cls(**values)

    @classmethod
    def from_checkpoint(cls, path: Path | str) -> "ModelConfig":
        path = Path(path)
        raw = json.loads((path / "config.json" if path.is_dir() else path).read_text())
        return cls.from_json(raw)

    def to_json(self) -> dict:
        out = {src: getattr(self, dst) for dst, src in self._JSON_RENAMES.items()}
        out.update({name: getattr(self, name) for name in self._JSON_FIELDS})
        out["rope_scaling"] = {"type": "yarn", "rope_type": "yarn"}
        for dst, src in self._ROPE_FIELDS:
            out["rope_scaling"][src] = getattr(self, dst)
        out["architectures"] = ["DeepseekV32ForCausalLM"]
        out["model_type"] = "deepseek_v32"
        if self.weight_dtype == "fp8":
            out["quantization_config"] = {
                "quant_method": "fp8",
                "fmt": "e4m3",
                "activation_scheme": "dynamic",
                "scale_fmt": self.scale_fmt,
                "weight_block_size": list(self.weight_block_size),
            }
        else:
            out["index_scale_fmt"] = self.scale_fmt
        return out

    def __post_init__(self):
        dims = (
            self.dim, self.n_heads, self.q_lora_rank, self.kv_lora_rank,
            self.qk_nope_head_dim, self.qk_rope_head_dim, self.v_head_dim,
            self.index_n_heads, self.index_head_dim, self.index_topk,
            self.num_hidden_layers, self.vocab_size, self.max_seq_len,
            self.original_seq_len,
        )
        if any(not isinstance(x, int) or isinstance(x, bool) or x <= 0 for x in dims):
            raise ValueError("model dimensions and context lengths must be positive integers")
        if self.qk_rope_head_dim % 2 or self.qk_rope_head_dim > self.index_head_dim:
            raise ValueError("RoPE dimension must be even and fit the indexer head")
        if self.scale_fmt not in (None, "ue8m0"):
            raise ValueError("unsupported indexer scale format")
        if self.weight_dtype not in ("fp8", "bf16"):
            raise ValueError("weight_dtype must be fp8 or bf16")

    # ------------------------------------------------------------ derived
    @property
    def qk_head_dim(self) -> int:
        """Width of an absorbed MLA query / latent KV record (512 + 64 = 576)."""
        return self.kv_lora_rank + self.qk_rope_head_dim

    @property
    def attention_scale(self) -> float:
        """Softmax scale: (nope+rope)^-1/2, times the YaRN mscale^2 correction."""
        scale = (self.qk_nope_head_dim + self.qk_rope_head_dim) ** -0.5
        if self.max_seq_len > self.original_seq_len:
            scale *= (1 + 0.1 * self.mscale * math.log(self.rope_factor)) ** 2
        return scale

    @property
    def hidden_size(self) -> int:
        return self.dim

    def is_moe_layer(self, layer: int) -> bool:
        return layer >= self.first_k_dense_replace

    def with_layers(self, n: int) -> "ModelConfig":
        return replace(self, num_hidden_layers=n)

    def asdict(self) -> dict:
        d = asdict(self)
        d.pop("raw", None)
        return d


def tiny_config(**overrides) -> ModelConfig:
    """The CPU tiny DSA model: 2 layers, hidden 256, 4 MLA heads, indexer 4x32 top-64."""
    base = dict(
        dim=256, n_heads=4, q_lora_rank=128, kv_lora_rank=64, qk_nope_head_dim=32,
        qk_rope_head_dim=16, v_head_dim=32, index_n_heads=4, index_head_dim=32,
        index_topk=64, num_hidden_layers=2, vocab_size=1024, intermediate_size=512,
        moe_intermediate_size=128, n_routed_experts=8, n_shared_experts=1,
        num_experts_per_tok=2, n_group=2, topk_group=1, first_k_dense_replace=2,
        max_seq_len=163840, weight_dtype="bf16",
    )
    base.update(overrides)
    return ModelConfig(**base)


def v32_config(layers: int = 61, **overrides) -> ModelConfig:
    """Full DeepSeek-V3.2 dimensions with ``layers`` hidden layers."""
    return ModelConfig(num_hidden_layers=layers, **overrides)


@dataclass(frozen=True)
class CacheConfig:
    """KV storage for one model instance.

    ``method``: "hbm" (resident main KV), "echo" (indexer-fused prefetch then
    exact recall), "serial_sparse" (recall after exact top-k) or
    "dense_prefetch" (next-layer whole-history DMA).  ``pool_tokens`` is the
    finite HBM pool P per layer; ``host_tokens`` the pinned DRAM arena NH.
    """

    method: str = "hbm"
    capacity: int = 65536 + 1024
    pool_tokens: int | None = None
    host_tokens: int | None = None
    candidate_tokens: int = 0
    page_size: int = 64
    chunk_size: int = 2048
    # "bf16": 1152-byte KV records everywhere.  "fp8": every KV row is quantized
    # once (per 128 latent dims, E4M3 + FP32 scale); HBM rows hold the exact
    # dequantized BF16 values and the pinned-DRAM arena the 656-byte records, so
    # recalls move 43 % fewer bytes over PCIe and resident and offloaded caches
    # stay bitwise equal.
    kv_format: str = "bf16"

    METHODS = ("hbm", "echo", "serial_sparse", "dense_prefetch")

    def __post_init__(self):
        if self.method not in self.METHODS:
            raise ValueError(f"cache method must be one of {self.METHODS}")
        if self.capacity < 1 or self.chunk_size < 1:
            raise ValueError("capacity and chunk_size must be positive")
        if self.method != "hbm" and self.pool_tokens is not None and self.pool_tokens < 1:
            raise ValueError("pool_tokens must be positive")
        if self.kv_format not in ("bf16", "fp8"):
            raise ValueError("kv_format must be 'bf16' or 'fp8'")

    @property
    def offload(self) -> bool:
        return self.method != "hbm"


@dataclass(frozen=True)
class ParallelConfig:
    """Process-group layout: tp (heads / columns), ep (experts), dp (requests), cp (indexer keys)."""

    tp: int = 1
    ep: int = 1
    dp: int = 1
    cp: int = 1
    pp: int = 1

    def __post_init__(self):
        for name in ("tp", "ep", "dp", "cp", "pp"):
            v = getattr(self, name)
            if type(v) is not int or v < 1:
                raise ValueError(f"{name} must be a positive integer")

    @property
    def world_size(self) -> int:
        return self.tp * self.dp * self.pp

    def label(self) -> str:
        parts = [f"{n}{getattr(self, n)}" for n in ("tp", "ep", "dp", "cp", "pp") if getattr(self, n) > 1]
        return "+".join(parts) or "single"
