"""Plain-PyTorch FP32 oracles for every hot op.

These restate the reference math and never load native code, so they run on
the CPU (the tiny model, cache tests) and serve as the numerics baseline for
the sm_100a kernels in ``csrc/``.  Reference math:

* RMSNorm / fused residual RMSNorm: ``models/deepseek_v32/nonmatrix.py:21-57``
  (FP32 accumulation, the residual sum is normalised *unrounded* and returned
  separately rounded).
* YaRN frequencies and the two RoPE pairings: ``models/deepseek_v32/rotary.py:26-56``.
* Indexer ue8m0 quantisation: ``operators/deepseek_v32/indexer/quantization.py:12-24``.
* 1x128 activation quantisation and FP8 block linear:
  ``operators/deepseek_v32/linear/fp8.py:63-102``.
* Indexer logits ``kscale[t] * sum_h relu(q_h . k_t) * w[q,h]`` with causal
  -inf: ``operators/deepseek_v32/indexer/csrc/echo_logits.cuh`` (epilogue) and
  ``echo.py:299``.
* Exact top-k (descending, ties -> smaller index, -1 for non-finite):
  ``operators/deepseek_v32/indexer/selection.py:62-113``.
* Sparse MLA: ``operators/deepseek_v32/attention/reference/torch.py:14-28``.
* MoE routing: ``models/deepseek_v32/layers.py:22-51``.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0


# ------------------------------------------------------------------ norms
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * weight.float()).to(x.dtype)


def residual_rms_norm(x, residual, weight, eps):
    """Return (rmsnorm(x + residual) in x.dtype, (x + residual) rounded to x.dtype).

    With ``residual is None`` this is a plain RMSNorm and the residual output is ``x``.
    """
    if residual is None:
        return rms_norm(x, weight, eps), x
    summed = x.float() + residual.float()
    normed = summed * torch.rsqrt(summed.square().mean(-1, keepdim=True) + eps) * weight.float()
    return normed.to(x.dtype), summed.to(x.dtype)


def layer_norm(x, weight, bias, eps):
    return F.layer_norm(x.float(), (x.shape[-1],), weight.float(), bias.float(), eps)


def silu_mul(gate, up):
    return (F.silu(gate.float()) * up.float()).to(torch.bfloat16)


# ------------------------------------------------------------------ rope
# ------------------------------------------------------------ FP8 KV records
FP8_RECORD_BYTES = 656  # V3.2 (L = 512, R = 64): 512 E4M3 latent + 4 FP32 block scales + 64 BF16 RoPE


def _fp8_blocks(L: int) -> int:
    """Latent quantization blocks: 128 dims each (one block when L < 128)."""
    if L < 128:
        return 1
    if L % 128:
        raise ValueError("FP8 KV records need a latent width that is a multiple of 128 (or below 128)")
    return L // 128


def fp8_record_bytes(L: int, R: int) -> int:
    return L + 4 * _fp8_blocks(L) + 2 * R


def fp8_kv_quantize(latent: torch.Tensor):
    """Per-block E4M3 quantization of BF16-valued latents [T, L] (128-dim blocks):
    scale = amax / 448 (FP32), q = e4m3(x / scale); returns (q [T, L], scales
    [T, blocks], dequantized BF16 rows bf16(float(q) * scale))."""
    T, L = latent.shape
    nb = _fp8_blocks(L)
    x = latent.float().reshape(T, nb, L // nb)
    scale = x.abs().amax(-1) / 448.0
    safe = torch.where(scale > 0, scale, torch.ones_like(scale))
    q = torch.where(scale[..., None] > 0, x / safe[..., None], torch.zeros_like(x)).to(torch.float8_e4m3fn)
    deq = (q.float() * scale[..., None]).bfloat16()
    return q.reshape(T, L), scale, deq.reshape(T, L)


def fp8_kv_pack(q: torch.Tensor, scale: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
    """Packed records: [L E4M3 | blocks FP32 scales | R BF16 RoPE] (656 bytes for V3.2)."""
    T = q.shape[0]
    return torch.cat((q.contiguous().view(torch.uint8).reshape(T, -1),
                      scale.float().contiguous().view(torch.uint8).reshape(T, -1),
                      rope.bfloat16().contiguous().view(torch.uint8).reshape(T, -1)), -1)


def fp8_kv_unpack(packed: torch.Tensor, L: int = 512) -> torch.Tensor:
    """Packed records -> BF16 rows [T, L + R] (bitwise the rows kv_finish stored)."""
    T = packed.shape[0]
    nb = _fp8_blocks(L)
    p = packed.contiguous()
    q = p[:, :L].contiguous().view(torch.float8_e4m3fn).reshape(T, nb, L // nb)
    scale = p[:, L:L + 4 * nb].contiguous().view(torch.float32).reshape(T, nb)
    rope = p[:, L + 4 * nb:].contiguous().view(torch.bfloat16).reshape(T, -1)
    lat = (q.float() * scale[..., None]).bfloat16().reshape(T, L)
    return torch.cat((lat, rope), -1)


def embed_shard(ids: torch.Tensor, table: torch.Tensor, row0: int, vocab_total: int) -> torch.Tensor:
    """Rows of a vocabulary shard (rows [row0, row0 + len(table))); ids outside the shard give zeros."""
    ids = ids.long().reshape(-1)
    if ((ids < 0) | (ids >= vocab_total)).any():
        raise IndexError("token id outside the vocabulary")
    local = ids - row0
    inside = (local >= 0) & (local < table.shape[0])
    out = torch.zeros((ids.numel(), table.shape[1]), dtype=torch.bfloat16, device=table.device)
    out[inside] = table[local[inside]].bfloat16()
    return out


def rotary_frequencies(cfg, device="cpu") -> torch.Tensor:
    """YaRN-corrected inverse frequencies, length rope_dim / 2."""
    dim = cfg.qk_rope_head_dim
    freq = cfg.rope_theta ** (-torch.arange(0, dim, 2, device=device).float() / dim)
    if cfg.max_seq_len > cfg.original_seq_len:

        def correction(rotations):
            return dim * math.log(cfg.original_seq_len / (rotations * 2 * math.pi)) / (2 * math.log(cfg.rope_theta))

        low = max(math.floor(correction(cfg.beta_fast)), 0)
        high = min(math.ceil(correction(cfg.beta_slow)), dim - 1)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(dim // 2, device=device).float() - low) / (high - low)).clamp(0, 1)
        freq = freq * (1 - ramp) + freq / cfg.rope_factor * ramp
    return freq


def apply_rope(x: torch.Tensor, angles: torch.Tensor, *, interleaved: bool) -> torch.Tensor:
    """Rotate the leading 2*len(freq) dims of the last axis.

    ``interleaved`` pairs (2i, 2i+1) (MLA); otherwise (i, i + d/2) (indexer).
    ``angles`` is [tokens, d/2]; x is [tokens, ..., width].
    """
    width = angles.shape[-1] * 2
    rot, rest = x[..., :width], x[..., width:]
    cos = angles.cos().reshape(angles.shape[0], *([1] * (x.ndim - 2)), -1)
    sin = angles.sin().reshape_as(cos)
    xf = rot.float()
    if interleaved:
        a, b = xf[..., ::2], xf[..., 1::2]
    else:
        a, b = xf.chunk(2, -1)
    real, imag = a * cos - b * sin, b * cos + a * sin
    out = torch.stack((real, imag), -1).flatten(-2) if interleaved else torch.cat((real, imag), -1)
    return torch.cat((out.to(x.dtype), rest), -1) if rest.shape[-1] else out.to(x.dtype)


# ---------------------------------------------------------- quantisation
def ue8m0_round(scale: torch.Tensor) -> torch.Tensor:
    """Round a positive FP32 scale up to the next power of two (exponent-only UE8M0)."""
    return torch.exp2(torch.ceil(torch.log2(scale)))


def quantize_index(x: torch.Tensor, scale_fmt: str | None = "ue8m0"):
    """Per-row (last axis) E4M3 quantisation with amax/448 scale (optionally UE8M0).

    Returns (fp8 tensor, fp32 scale with a trailing singleton axis).
    """
    amax = x.float().abs().amax(-1, keepdim=True).clamp_min(1e-4)
    scale = amax / FP8_MAX
    if scale_fmt == "ue8m0":
        scale = ue8m0_round(scale)
    q = (x.float() / scale).clamp(-FP8_MAX, FP8_MAX).to(FP8)
    return q.contiguous(), scale.contiguous()


def quantize_act(x: torch.Tensor):
    """1x128 UE8M0 activation quantisation: returns (fp8 [M,K], fp32 scales [M, ceil(K/128)])."""
    rows, cols = x.shape
    groups = (cols + 127) // 128
    blocks = F.pad(x.float(), (0, groups * 128 - cols)).reshape(rows, groups, 128)
    scale = ue8m0_round(blocks.abs().amax(-1).clamp_min(1e-4) / FP8_MAX)
    q = (blocks / scale[..., None]).clamp(-FP8_MAX, FP8_MAX).to(FP8)
    return q.reshape(rows, groups * 128)[:, :cols].contiguous(), scale.contiguous()


def dequantize_act(q, scales):
    return q.float() * scales.repeat_interleave(128, -1)[:, : q.shape[-1]]


def dequantize_weight(w, scales):
    expanded = scales.float().repeat_interleave(128, -2).repeat_interleave(128, -1)
    return w.float() * expanded[..., : w.shape[-2], : w.shape[-1]]


def fp8_linear(x: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """FP32 product of the 1x128-quantised activation and the block-dequantised weight -> BF16."""
    x2 = x.reshape(-1, x.shape[-1])
    a = dequantize_act(*quantize_act(x2))
    out = a @ dequantize_weight(weight, scales).T
    return out.reshape(*x.shape[:-1], weight.shape[0]).to(torch.bfloat16)


def linear(x, weight, scales=None):
    """BF16 or FP8-block linear oracle, output BF16."""
    if scales is not None:
        return fp8_linear(x, weight, scales)
    return (x.float() @ weight.float().T).to(torch.bfloat16)


# --------------------------------------------------------------- indexer
def indexer_logits(q, k, weights, kscale, query_start: int, *, causal: bool = True):
    """FP32 logits[Q, N] = kscale[t] * sum_h relu(q[h] . k[t]) * w[q, h].

    q: fp8 [Q, H, D]; k: fp8 [N, D]; weights fp32 [Q, H] (already includes the
    query quantisation scale and head scaling); kscale fp32 [N].
    Column t is visible to row i iff t <= query_start + i (else -inf).
    """
    qf, kf = q.float(), k.float()
    scores = torch.einsum("qhd,nd->qhn", qf, kf).relu()
    logits = torch.einsum("qhn,qh->qn", scores, weights.float()) * kscale.float()[None, :]
    if causal:
        rows = torch.arange(q.shape[0], device=q.device)[:, None]
        cols = torch.arange(k.shape[0], device=q.device)[None, :]
        logits = logits.masked_fill(cols > query_start + rows, -torch.inf)
    return logits


def exact_topk(scores: torch.Tensor, k: int):
    """Descending top-k with ties broken towards the smaller index; -1 for non-finite."""
    count = min(k, scores.shape[1])
    values, order = torch.sort(scores, dim=-1, descending=True, stable=True)
    values, order = values[:, :count].contiguous(), order[:, :count]
    ids = torch.where(torch.isfinite(values), order, -1).to(torch.int32)
    return values, ids.contiguous()


# ------------------------------------------------------------- attention
def sparse_mla(q, kv, indices, scale, value_dim=512):
    """q [Q,H,Dqk], kv [N,Dqk] (values = first value_dim), indices [Q,K]; -1/out-of-range = padding.

    Duplicate ids participate independently; all-padding rows give zero.
    """
    out = torch.zeros((*q.shape[:2], value_dim), dtype=q.dtype, device=q.device)
    for row in range(q.shape[0]):
        sel = indices[row]
        sel = sel[(sel >= 0) & (sel < kv.shape[0])].long()
        if not sel.numel():
            continue
        rec = kv[sel].float()
        logits = q[row].float() @ rec.T * scale
        out[row] = (logits.softmax(-1) @ rec[:, :value_dim]).to(q.dtype)
    return out


def sparse_mla_lse(q, kv, indices, scale, value_dim=512):
    """Like :func:`sparse_mla` but also returns the natural-log LSE per (query, head)."""
    out = torch.zeros((*q.shape[:2], value_dim), dtype=torch.float32, device=q.device)
    lse = torch.full(q.shape[:2], -torch.inf, dtype=torch.float32, device=q.device)
    for row in range(q.shape[0]):
        sel = indices[row]
        sel = sel[(sel >= 0) & (sel < kv.shape[0])].long()
        if not sel.numel():
            continue
        rec = kv[sel].float()
        logits = q[row].float() @ rec.T * scale
        lse[row] = torch.logsumexp(logits, -1)
        out[row] = logits.softmax(-1) @ rec[:, :value_dim]
    return out, lse


# ------------------------------------------------------------------- moe
def route_experts(hidden, gate_weight, correction_bias, cfg):
    """Sigmoid scores; bias-corrected group choice (top-2 sum per group, top groups), top-k experts.

    Weights use the *uncorrected* scores, normalised, times routed_scaling_factor.
    Returns (expert_ids int64 [T, k], weights fp32 [T, k]).
    """
    experts = cfg.n_routed_experts
    scores = F.linear(hidden.float(), gate_weight.float()).sigmoid()
    corrected = scores + correction_bias.float()
    grouped = corrected.reshape(len(hidden), cfg.n_group, experts // cfg.n_group)
    group_scores = grouped.topk(2, dim=-1).values.sum(-1)
    groups = group_scores.topk(cfg.topk_group, dim=-1).indices
    keep = torch.zeros_like(group_scores, dtype=torch.bool).scatter_(1, groups, True)
    corrected = grouped.masked_fill(~keep[..., None], -torch.inf).flatten(1)
    ids = corrected.topk(cfg.num_experts_per_tok, dim=-1).indices
    weights = scores.gather(1, ids)
    if cfg.norm_topk_prob:
        weights = weights / weights.sum(-1, keepdim=True).clamp_min(torch.finfo(torch.float32).tiny)
    return ids, (weights * cfg.routed_scaling_factor).contiguous()


def moe_experts(hidden, ids, weights, w_gate, w_up, w_down, s_gate=None, s_up=None, s_down=None):
    """Reference routed-expert SwiGLU: sum_j weights[t,j] * expert_{ids[t,j]}(x_t)."""
    out = torch.zeros(hidden.shape, dtype=torch.float32, device=hidden.device)
    for e in ids.unique().tolist():
        rows, slot = (ids == e).nonzero(as_tuple=True)
        x = hidden[rows]
        g = linear(x, w_gate[e], None if s_gate is None else s_gate[e])
        u = linear(x, w_up[e], None if s_up is None else s_up[e])
        y = linear(silu_mul(g, u), w_down[e], None if s_down is None else s_down[e])
        out.index_add_(0, rows, y.float() * weights[rows, slot, None])
    return out


# ---------------------------------------------------------------- hints
def prefetch_hint(scores: torch.Tensor) -> torch.Tensor:
    """Mean of finite scores in the last min(4, Q) rows (the ECHO offset[0] hint)."""
    tail = scores[-4:]
    finite = torch.isfinite(tail)
    return tail.masked_fill(~finite, 0).sum() / finite.sum().clamp_min(1)


def decode_hint(previous: torch.Tensor, kth_value: torch.Tensor) -> torch.Tensor:
    """offset[1] EMA: 0.5 * previous + 0.5 * kth exact score."""
    return previous * 0.5 + kth_value * 0.5
