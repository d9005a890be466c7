"""DeepSeek-V3.2 safetensors layout: lazy reader, random-init writer, FP8 helpers.

The tensor names and the FP8 ``weight`` + ``weight_scale_inv`` (one FP32 scale
per 128x128 block) layout are those of the public checkpoint, so a real
checkpoint directory loads through the same code path as a random one.
Reference parity: ``models/deepseek_v32/checkpoint.py:14-113`` (header scan,
lazy reads, block dequant) and the expert stacking in
``models/deepseek_v32/layers.py:141-168``.

No checkpoint is reachable offline, so :func:`random_state_dict` produces the
same names, shapes and dtypes from a seed, either on the host (to write a
directory with :func:`write_checkpoint`) or directly on a GPU for benchmarks.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Iterable

import torch

from .config import ModelConfig

FP8_MAX = 448.0
FP8 = torch.float8_e4m3fn


# ----------------------------------------------------------------- names
def layer_prefix(layer: int) -> str:
    return f"model.layers.{layer}."


def attention_linears(cfg: ModelConfig) -> dict[str, tuple[int, int]]:
    """Checkpoint linear weights of one attention block, name -> (out, in)."""
    h = cfg.n_heads
    return {
        "self_attn.q_a_proj": (cfg.q_lora_rank, cfg.dim),
        "self_attn.q_b_proj": (h * (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim), cfg.q_lora_rank),
        "self_attn.kv_a_proj_with_mqa": (cfg.kv_lora_rank + cfg.qk_rope_head_dim, cfg.dim),
        "self_attn.kv_b_proj": (h * (cfg.qk_nope_head_dim + cfg.v_head_dim), cfg.kv_lora_rank),
        "self_attn.o_proj": (cfg.dim, h * cfg.v_head_dim),
        "self_attn.indexer.wq_b": (cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank),
        "self_attn.indexer.wk": (cfg.index_head_dim, cfg.dim),
    }


def mlp_linears(cfg: ModelConfig, stem: str, inter: int) -> dict[str, tuple[int, int]]:
    return {
        f"{stem}.gate_proj": (inter, cfg.dim),
        f"{stem}.up_proj": (inter, cfg.dim),
        f"{stem}.down_proj": (cfg.dim, inter),
    }


def layer_tensor_specs(cfg: ModelConfig, layer: int) -> dict[str, tuple[tuple[int, ...], str]]:
    """name -> (shape, kind) for one layer; kind in {linear, norm, bias, fp32}."""
    p = layer_prefix(layer)
    specs: dict[str, tuple[tuple[int, ...], str]] = {
        p + "input_layernorm.weight": ((cfg.dim,), "norm"),
        p + "post_attention_layernorm.weight": ((cfg.dim,), "norm"),
        p + "self_attn.q_a_layernorm.weight": ((cfg.q_lora_rank,), "norm"),
        p + "self_attn.kv_a_layernorm.weight": ((cfg.kv_lora_rank,), "norm"),
        p + "self_attn.indexer.k_norm.weight": ((cfg.index_head_dim,), "norm"),
        p + "self_attn.indexer.k_norm.bias": ((cfg.index_head_dim,), "bias"),
        p + "self_attn.indexer.weights_proj.weight": ((cfg.index_n_heads, cfg.dim), "fp32"),
    }
    for name, shape in attention_linears(cfg).items():
        specs[p + name + ".weight"] = (shape, "linear")
    if cfg.is_moe_layer(layer):
        specs[p + "mlp.gate.weight"] = ((cfg.n_routed_experts, cfg.dim), "fp32")
        specs[p + "mlp.gate.e_score_correction_bias"] = ((cfg.n_routed_experts,), "bias")
        for e in range(cfg.n_routed_experts):
            for name, shape in mlp_linears(cfg, f"mlp.experts.{e}", cfg.moe_intermediate_size).items():
                specs[p + name + ".weight"] = (shape, "linear")
        if cfg.n_shared_experts:
            inter = cfg.moe_intermediate_size * cfg.n_shared_experts
            for name, shape in mlp_linears(cfg, "mlp.shared_experts", inter).items():
                specs[p + name + ".weight"] = (shape, "linear")
    else:
        for name, shape in mlp_linears(cfg, "mlp", cfg.intermediate_size).items():
            specs[p + name + ".weight"] = (shape, "linear")
    return specs


def model_tensor_specs(cfg: ModelConfig, layers: Iterable[int] | None = None):
    layers = range(cfg.num_hidden_layers) if layers is None else layers
    specs = {
        "model.embed_tokens.weight": ((cfg.vocab_size, cfg.dim), "embed"),
        "model.norm.weight": ((cfg.dim,), "norm"),
        "lm_head.weight": ((cfg.vocab_size, cfg.dim), "embed"),
    }
    for layer in layers:
        specs.update(layer_tensor_specs(cfg, layer))
    return specs


# ------------------------------------------------------------ fp8 blocks
def _cdiv(a: int, b: int) -> int:
    return (a + b - 1) // b


def quantize_weight_blocks(w: torch.Tensor, block=(128, 128), pow2_scales=True):
    """Quantise a 2-D weight to E4M3 with one FP32 scale per block.

    ``pow2_scales`` rounds each block scale up to a power of two (the UE8M0
    convention); otherwise the scale is amax/448 exactly.
    Returns (fp8 weight, scales[ceil(N/bn), ceil(K/bk)]) with dequant
    ``w ~= fp8 * scale`` (the checkpoint calls this ``weight_scale_inv``).
    """
    n, k = w.shape
    bn, bk = block
    gn, gk = _cdiv(n, bn), _cdiv(k, bk)
    padded = torch.zeros((gn * bn, gk * bk), dtype=torch.float32, device=w.device)
    padded[:n, :k] = w.float()
    blocks = padded.reshape(gn, bn, gk, bk)
    amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    scale = amax / FP8_MAX
    if pow2_scales:
        scale = torch.exp2(torch.ceil(torch.log2(scale)))
    q = (blocks / scale[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(FP8)
    q = q.reshape(gn * bn, gk * bk)[:n, :k].contiguous()
    return q, scale.contiguous()


def dequantize_weight_blocks(w: torch.Tensor, scales: torch.Tensor, block=(128, 128)) -> torch.Tensor:
    """FP32 dequantisation of an FP8 block-scaled weight (works for partial edge blocks)."""
    bn, bk = block
    expanded = scales.float().repeat_interleave(bn, -2).repeat_interleave(bk, -1)
    return w.float() * expanded[..., : w.shape[-2], : w.shape[-1]]


# ------------------------------------------------------------- random init
def _random_tensors(name: str, shape, kind: str, cfg: ModelConfig, gen, *, seed: int, std: float, device,
                    pow2_scales: bool) -> dict[str, torch.Tensor]:
    """The tensor(s) named ``name`` (an FP8 linear also yields its ``weight_scale_inv``)."""
    import zlib

    gen.manual_seed((seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF)
    if kind == "norm":
        return {name: torch.ones(shape, dtype=torch.float32 if "k_norm" in name else torch.bfloat16, device=device)}
    if kind == "bias":
        return {name: torch.zeros(shape, dtype=torch.float32, device=device)}
    if kind == "fp32":
        return {name: torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std}
    if kind == "embed":
        return {name: (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).bfloat16()}
    w = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std
    if cfg.weight_dtype == "fp8":
        q, sc = quantize_weight_blocks(w, cfg.weight_block_size, pow2_scales)
        return {name: q, name[: -len(".weight")] + ".weight_scale_inv": sc}
    return {name: w.bfloat16()}


def _expert_of(name: str):
    if ".mlp.experts." not in name:
        return None
    return int(name.split(".mlp.experts.")[1].split(".")[0])


def random_state_dict(
    cfg: ModelConfig,
    layers: Iterable[int] | None = None,
    *,
    seed: int = 0,
    std: float = 0.02,
    device="cpu",
    pow2_scales: bool = True,
    include_embeddings: bool = True,
    experts: Iterable[int] | None = None,
) -> dict[str, torch.Tensor]:
    """Seeded random weights with the checkpoint's names, shapes and dtypes.

    Linear weights are N(0, std); with ``cfg.weight_dtype == "fp8"`` they are
    stored as E4M3 plus ``weight_scale_inv`` block scales, otherwise BF16.
    Norm weights are one, biases zero; the indexer head weights and the MoE
    gate are FP32 like the checkpoint.  Tensors are generated one at a time on
    ``device`` (a GPU makes the 3-layer / 671B benchmark models fast to build).
    Every tensor has its own seed (from ``seed`` and its name), so a rank that
    generates only its own routed ``experts`` gets the same replicated tensors
    as every other rank.
    """
    gen = torch.Generator(device=device)
    keep = None if experts is None else set(experts)
    out: dict[str, torch.Tensor] = {}
    for name, (shape, kind) in model_tensor_specs(cfg, layers).items():
        if not include_embeddings and kind == "embed":
            continue
        e = _expert_of(name)
        if keep is not None and e is not None and e not in keep:
            continue
        out.update(_random_tensors(name, shape, kind, cfg, gen, seed=seed, std=std, device=device,
                                   pow2_scales=pow2_scales))
    return out


class RandomSource:
    """Lazily generated random weights (same values as :func:`random_state_dict`).

    Each tensor is created when the model loader asks for it, so a 61-layer
    671B model can be built rank by rank without ever holding a full state
    dict next to the loaded weights.
    """

    def __init__(self, cfg: ModelConfig, layers: Iterable[int] | None = None, *, seed: int = 0, std: float = 0.02,
                 device="cpu", pow2_scales: bool = True):
        self.cfg = cfg
        self.config = cfg
        self.device = device
        self.seed, self.std, self.pow2 = seed, std, pow2_scales
        self.specs = model_tensor_specs(cfg, layers)
        self._scale_of = {n[: -len(".weight")] + ".weight_scale_inv": n for n, (_, k) in self.specs.items()
                          if k not in ("norm", "bias", "fp32", "embed") and cfg.weight_dtype == "fp8"}
        self._gen = torch.Generator(device=device)
        self._cache: dict[str, torch.Tensor] = {}

    def __contains__(self, name):
        return name in self.specs or name in self._scale_of

    def keys(self):
        return list(self.specs) + list(self._scale_of)

    @property
    def tensor_metadata(self) -> dict:
        meta = {n: {"shape": list(shape)} for n, (shape, _) in self.specs.items()}
        for sname, wname in self._scale_of.items():
            n, k = self.specs[wname][0]
            bn, bk = self.cfg.weight_block_size
            meta[sname] = {"shape": [_cdiv(n, bn), _cdiv(k, bk)]}
        return meta

    def get_tensor(self, name: str) -> torch.Tensor:
        if name in self._cache:
            return self._cache.pop(name)
        base = self._scale_of.get(name, name)
        if base not in self.specs:
            raise KeyError(f"required tensor {name!r} is absent")
        shape, kind = self.specs[base]
        made = _random_tensors(base, shape, kind, self.cfg, self._gen, seed=self.seed, std=self.std,
                               device=self.device, pow2_scales=self.pow2)
        out = made.pop(name)
        self._cache.update(made)  # the partner (weight or its scales), asked for next by the loader
        return out


# --------------------------------------------------------------- writer
_SAFETENSORS_DTYPES = {
    torch.float32: "F32",
    torch.bfloat16: "BF16",
    torch.float16: "F16",
    FP8: "F8_E4M3",
    torch.int32: "I32",
    torch.int64: "I64",
}


def write_checkpoint(path, cfg: ModelConfig, tensors: dict[str, torch.Tensor], *, shard_bytes=2 << 30):
    """Write ``config.json`` plus ``model-XXXXX-of-YYYYY.safetensors`` shards and an index."""
    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(cfg.to_json(), indent=2))
    shards: list[dict[str, torch.Tensor]] = [{}]
    size = 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        nbytes = t.numel() * t.element_size()
        if shards[-1] and size + nbytes > shard_bytes:
            shards.append({})
            size = 0
        shards[-1][name] = t
        size += nbytes
    weight_map = {}
    for i, shard in enumerate(shards):
        fname = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(shard, str(path / fname), metadata={"format": "pt"})
        weight_map.update({name: fname for name in shard})
    (path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}, indent=1))
    return path


# --------------------------------------------------------------- reader
class CheckpointReader:
    """Locate tensors by scanning every shard header; data is read only on ``get_tensor``.

    Missing unrelated shards are tolerated (partial checkpoints for a few
    layers); a requested missing tensor raises ``KeyError``.  The header size
    is bounded and duplicate names are rejected.
    """

    MAX_HEADER = 100_000_000

    def __init__(self, model_path):
        self.model_path = Path(model_path)
        self.tensor_files: dict[str, Path] = {}
        self.tensor_metadata: dict[str, dict] = {}
        for path in sorted(self.model_path.glob("*.safetensors")):
            with path.open("rb") as handle:
                prefix = handle.read(8)
                if len(prefix) != 8:
                    raise ValueError(f"incomplete safetensors header: {path}")
                size = struct.unpack("<Q", prefix)[0]
                if not 0 < size <= min(path.stat().st_size - 8, self.MAX_HEADER):
                    raise ValueError(f"invalid safetensors header size: {path}")
                header = json.loads(handle.read(size))
            for name, meta in header.items():
                if name == "__metadata__":
                    continue
                if name in self.tensor_files:
                    raise ValueError(f"duplicate checkpoint tensor {name}")
                self.tensor_files[name] = path
                self.tensor_metadata[name] = meta
        if not self.tensor_files:
            raise FileNotFoundError(f"no safetensors weights found in {self.model_path}")
        self.config = ModelConfig.from_checkpoint(self.model_path) if (self.model_path / "config.json").exists() else None

    def __contains__(self, name: str) -> bool:
        return name in self.tensor_files

    def keys(self):
        return self.tensor_files.keys()

    def get_tensor(self, name: str) -> torch.Tensor:
        from safetensors import safe_open

        try:
            path = self.tensor_files[name]
        except KeyError as exc:
            raise KeyError(f"required tensor {name!r} is absent from {self.model_path}") from exc
        with safe_open(str(path), framework="pt", device="cpu") as handle:
            return handle.get_tensor(name)


class StateDictSource:
    """Wrap an in-memory tensor dict (e.g. random GPU weights) with the reader API."""

    def __init__(self, tensors: dict[str, torch.Tensor], config: ModelConfig | None = None):
        self.tensors = tensors
        self.config = config

    def __contains__(self, name):
        return name in self.tensors

    def keys(self):
        return self.tensors.keys()

    @property
    def tensor_metadata(self) -> dict:
        return {n: {"shape": list(t.shape), "dtype": str(t.dtype).removeprefix("torch.")} for n, t in self.tensors.items()}

    def get_tensor(self, name: str) -> torch.Tensor:
        try:
            return self.tensors[name]
        except KeyError as exc:
            raise KeyError(f"required tensor {name!r} is absent") from exc


def linear_weight_bf16(source, stem: str, *, device, block=(128, 128)) -> torch.Tensor:
    """Dense BF16 weight of a linear (dequantising FP8 blocks; partial blocks allowed)."""
    data = source.get_tensor(stem + ".weight").to(device)
    if data.ndim != 2:
        raise ValueError(f"linear weight must be a matrix: {stem}")
    if data.dtype == FP8:
        scales = source.get_tensor(stem + ".weight_scale_inv").to(device)
        expected = tuple(_cdiv(n, b) for n, b in zip(data.shape, block))
        if tuple(scales.shape) != expected:
            raise ValueError(f"invalid FP8 scale shape for {stem}: expected {expected}")
        data = dequantize_weight_blocks(data, scales, block)
    elif data.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError(f"unsupported checkpoint weight dtype {data.dtype}: {stem}")
    return data.to(torch.bfloat16).contiguous()
