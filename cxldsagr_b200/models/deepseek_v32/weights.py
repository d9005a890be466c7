"""Per-layer weights in the layout the sm_100a kernels consume.

Checkpoint linears that read the same activation are packed into one GEMM:

* ``fused_a`` = [q_a_proj (1536); kv_a_proj_with_mqa (576, zero-padded to 640);
  indexer.wk (128)] -> one FP8 GEMM on the normalised input (reference runs
  three linears, ``models/deepseek_v32/projections.py:195-250``);
* ``fused_b`` = [q_b_proj (128*192); indexer.wq_b (64*128)] on the normalised
  q latent;
* dense / shared MLP ``gate_up`` = [gate_proj; up_proj] whose output feeds the
  fused SiLU*up + FP8 quantisation kernel.

Padding rows keep every 128-row block scale of the FP8 checkpoint aligned with
one output block.  ``kv_b_proj`` is dequantised to BF16 and split into the
absorbed ``W_UK^T`` [H, 512, 128] and ``W_UV`` [H, 128, 512] (reference:
``projections.py:79-85``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ...checkpoint import FP8, _cdiv, linear_weight_bf16
from ...config import ModelConfig
from ... import ops


@dataclass
class Linear:
    """FP8 block-scaled (``scales`` set) or BF16 linear weight [N, K]."""

    weight: torch.Tensor
    scales: torch.Tensor | None = None
    # Power-of-two block scales may take the block-scaled tensor-core MMA
    # (ops.fp8_gemm ue8m0=True).  Off by default: on B200 it measured at parity
    # with the FP32-promotion kernel for 128 x 224 tiles and slower for 128 x 256
    # tiles with short K (one TMEM accumulator), both being operand-feed bound.
    ue8m0: bool = False

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    def __call__(self, x=None, *, quantized=None, residual=None, out=None):
        if self.scales is None:
            if x is None:
                raise ValueError("a BF16 linear needs its BF16 input")
            y = ops.linear(x, self.weight)
            return y if residual is None else (y.float() + residual.float()).bfloat16()
        if quantized is not None:
            q, s_t = quantized
            return ops.fp8_gemm(q, s_t, self.weight, self.scales, out=out, residual=residual, ue8m0=self.ue8m0)
        return ops.fp8_linear(x, self.weight, self.scales, out=out, residual=residual, ue8m0=self.ue8m0)


def load_linear(source, stem: str, *, device, dtype: str) -> Linear:
    w = source.get_tensor(stem + ".weight")
    if w.dtype == FP8 and dtype == "fp8":
        s = source.get_tensor(stem + ".weight_scale_inv")
        return Linear(w.to(device).contiguous(), s.to(device=device, dtype=torch.float32).contiguous())
    return Linear(linear_weight_bf16(source, stem, device=device))


def pack_linears(parts: list[Linear], *, pad_to: int = 128) -> tuple[Linear, list[tuple[int, int]]]:
    """Stack linears along N, zero-padding each part to a multiple of ``pad_to`` rows.

    Returns the packed linear and each part's (start, rows) in the output.
    """
    fp8 = parts[0].scales is not None
    if any((p.scales is not None) != fp8 for p in parts):
        raise ValueError("cannot pack FP8 and BF16 linears together")
    K = parts[0].weight.shape[1]
    spans, weights, scales, offset = [], [], [], 0
    for p in parts:
        n = p.weight.shape[0]
        padded = _cdiv(n, pad_to) * pad_to if fp8 else n
        spans.append((offset, n))
        w = p.weight
        if padded != n:
            pad = torch.zeros((padded - n, K), dtype=torch.uint8, device=w.device).view(w.dtype)
            w = torch.cat((w, pad))
        weights.append(w)
        if fp8:
            s = p.scales
            blocks = padded // 128
            if s.shape[0] < blocks:
                s = torch.cat((s, torch.ones((blocks - s.shape[0], s.shape[1]), dtype=s.dtype, device=s.device)))
            scales.append(s[:blocks])
        offset += padded
    packed = Linear(torch.cat(weights).contiguous(), torch.cat(scales).contiguous() if fp8 else None)
    return packed, spans


@dataclass
class AttentionWeights:
    input_norm: torch.Tensor       # fp32 [D]
    q_norm: torch.Tensor           # fp32 [q_lora]
    kv_norm: torch.Tensor          # fp32 [kv_lora]
    index_norm_w: torch.Tensor     # fp32 [128]
    index_norm_b: torch.Tensor     # fp32 [128]
    index_head: torch.Tensor       # fp32 [64, D]
    index_head_split: torch.Tensor  # bf16 [128, D]: hi || lo of index_head
    fused_a: Linear
    spans_a: list
    fused_b: Linear
    spans_b: list
    wk_b_t: torch.Tensor           # bf16 [H, kv_lora, nope]
    wv_b: torch.Tensor             # bf16 [H, v, kv_lora]
    wo: Linear


@dataclass
class MLPWeights:
    gate_up: Linear
    down: Linear
    inter: int


@dataclass
class MoEWeights:
    gate: torch.Tensor             # fp32 [E, D]
    bias: torch.Tensor             # fp32 [E]
    w_gate_up: torch.Tensor        # fp8 [E, 2I, D] (or bf16)
    s_gate_up: torch.Tensor | None
    w_down: torch.Tensor           # fp8 [E, D, I]
    s_down: torch.Tensor | None
    shared: MLPWeights | None
    experts: range                 # global expert ids resident here (EP shard)
    gate_split: torch.Tensor | None = None  # bf16 [2E, D]: hi || lo of the fp32 gate (tensor-core GEMV)


def _f32(source, name, device):
    return source.get_tensor(name).to(device=device, dtype=torch.float32).contiguous()


def load_attention(source, cfg: ModelConfig, layer: int, *, device) -> AttentionWeights:
    p = f"model.layers.{layer}."
    a = p + "self_attn."
    dt = cfg.weight_dtype

    def lin(name):
        return load_linear(source, a + name, device=device, dtype=dt)

    fused_a, spans_a = pack_linears([lin("q_a_proj"), lin("kv_a_proj_with_mqa"), lin("indexer.wk")])
    fused_b, spans_b = pack_linears([lin("q_b_proj"), lin("indexer.wq_b")])
    wkv_b = linear_weight_bf16(source, a + "kv_b_proj", device=device, block=cfg.weight_block_size)
    wkv_b = wkv_b.reshape(cfg.n_heads, cfg.qk_nope_head_dim + cfg.v_head_dim, cfg.kv_lora_rank)
    wk_b = wkv_b[:, : cfg.qk_nope_head_dim]                 # [H, nope, L]
    wv_b = wkv_b[:, cfg.qk_nope_head_dim :].contiguous()    # [H, v, L]
    return AttentionWeights(
        input_norm=_f32(source, p + "input_layernorm.weight", device),
        q_norm=_f32(source, a + "q_a_layernorm.weight", device),
        kv_norm=_f32(source, a + "kv_a_layernorm.weight", device),
        index_norm_w=_f32(source, a + "indexer.k_norm.weight", device),
        index_norm_b=_f32(source, a + "indexer.k_norm.bias", device),
        index_head=(ih := _f32(source, a + "indexer.weights_proj.weight", device)),
        index_head_split=ops.split_bf16(ih),
        fused_a=fused_a,
        spans_a=spans_a,
        fused_b=fused_b,
        spans_b=spans_b,
        wk_b_t=wk_b.transpose(1, 2).contiguous(),
        wv_b=wv_b,
        wo=lin("o_proj"),
    )


def _slice_rows(lin: Linear, r0: int, r1: int) -> Linear:
    if lin.scales is None:
        return Linear(lin.weight[r0:r1].contiguous())
    if r0 % 128 or r1 % 128:
        raise ValueError("FP8 row shards must align to the 128-row scale blocks")
    return Linear(lin.weight[r0:r1].contiguous(), lin.scales[r0 // 128:r1 // 128].contiguous())


def _slice_cols(lin: Linear, c0: int, c1: int) -> Linear:
    if lin.scales is None:
        return Linear(lin.weight[:, c0:c1].contiguous())
    if c0 % 128 or c1 % 128:
        raise ValueError("FP8 column shards must align to the 128-column scale blocks")
    return Linear(lin.weight[:, c0:c1].contiguous(), lin.scales[:, c0 // 128:c1 // 128].contiguous())


def load_mlp(source, cfg: ModelConfig, stem: str, *, device, shard: tuple[int, int] = (0, 1)) -> MLPWeights:
    """Dense SwiGLU MLP; ``shard=(rank, world)`` keeps a column slice of gate/up and
    the matching row slice (input columns) of down (tensor parallel)."""
    dt = cfg.weight_dtype
    gate = load_linear(source, stem + ".gate_proj", device=device, dtype=dt)
    up = load_linear(source, stem + ".up_proj", device=device, dtype=dt)
    down = load_linear(source, stem + ".down_proj", device=device, dtype=dt)
    rank, world = shard
    if world > 1:
        inter = gate.out_features
        if inter % world:
            raise ValueError("intermediate size must divide across ranks")
        c0, c1 = rank * inter // world, (rank + 1) * inter // world
        gate, up, down = _slice_rows(gate, c0, c1), _slice_rows(up, c0, c1), _slice_cols(down, c0, c1)
    gate_up, _ = pack_linears([gate, up])
    return MLPWeights(gate_up, down, gate.out_features)


def load_moe(source, cfg: ModelConfig, layer: int, *, device, experts: range | None = None) -> MoEWeights:
    p = f"model.layers.{layer}.mlp."
    experts = range(cfg.n_routed_experts) if experts is None else experts
    I, D = cfg.moe_intermediate_size, cfg.dim
    fp8 = cfg.weight_dtype == "fp8"
    wdt = FP8 if fp8 else torch.bfloat16
    n = len(experts)
    w_gu = torch.empty((n, 2 * I, D), dtype=wdt, device=device)
    w_d = torch.empty((n, D, I), dtype=wdt, device=device)
    s_gu = torch.empty((n, _cdiv(2 * I, 128), _cdiv(D, 128)), dtype=torch.float32, device=device) if fp8 else None
    s_d = torch.empty((n, _cdiv(D, 128), _cdiv(I, 128)), dtype=torch.float32, device=device) if fp8 else None
    for j, e in enumerate(experts):
        stem = f"{p}experts.{e}."
        for k, name in enumerate(("gate_proj", "up_proj")):
            lin = load_linear(source, stem + name, device=device, dtype=cfg.weight_dtype)
            w_gu[j, k * I : (k + 1) * I].copy_(lin.weight)
            if fp8:
                nb = _cdiv(I, 128)
                s_gu[j, k * nb : (k + 1) * nb].copy_(lin.scales)
        lin = load_linear(source, stem + "down_proj", device=device, dtype=cfg.weight_dtype)
        w_d[j].copy_(lin.weight)
        if fp8:
            s_d[j].copy_(lin.scales)
    shared = load_mlp(source, cfg, p + "shared_experts", device=device) if cfg.n_shared_experts else None
    gate = _f32(source, p + "gate.weight", device)
    return MoEWeights(
        gate=gate,
        bias=_f32(source, p + "gate.e_score_correction_bias", device),
        w_gate_up=w_gu, s_gate_up=s_gu, w_down=w_d, s_down=s_d, shared=shared, experts=experts,
        gate_split=ops.split_bf16(gate) if torch.device(device).type == "cuda" else None,
    )
