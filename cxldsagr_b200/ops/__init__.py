"""Operator API: sm_100a kernels for CUDA tensors, FP32 oracles for CPU tensors.

Each function accepts tensors on either device.  CUDA inputs always run the
native kernels of ``csrc/`` (no silent PyTorch fallback); CPU inputs run the
restated reference math of :mod:`.reference`.
"""

from __future__ import annotations

import math

import torch

from . import reference
from .native import check_errors, error_word, lib  # noqa: F401

FP8 = torch.float8_e4m3fn


def _cuda(t: torch.Tensor) -> bool:
    return t.is_cuda


# ------------------------------------------------------------------- norms
def rms_norm(x, weight, eps, *, out=None):
    if not _cuda(x):
        return reference.rms_norm(x, weight, eps)
    x2 = x.reshape(-1, x.shape[-1])
    out = torch.empty_like(x2) if out is None else out
    lib().rms_norm(x2, None, weight.float().contiguous(), eps, out, None, None, None)
    return out.reshape(x.shape)


def residual_rms_norm(x, residual, weight, eps):
    """(rmsnorm(x + residual), x + residual rounded); residual None -> (rmsnorm(x), x)."""
    if not _cuda(x):
        return reference.residual_rms_norm(x, residual, weight, eps)
    if residual is None:
        return rms_norm(x, weight, eps), x
    out, summed = torch.empty_like(x), torch.empty_like(x)
    lib().rms_norm(x, residual, weight.float().contiguous(), eps, out, summed, None, None)
    return out, summed


def norm_quant(x, residual, weight, eps, *, want_out=True):
    """Fused (residual) RMSNorm + 1x128 FP8 quantisation of the normalised rows.

    Returns (normed bf16 or None, summed bf16 (or x), q fp8 [M,D], scales_t fp32 [D/128, M]).
    """
    M, D = x.shape
    if not _cuda(x):
        normed, summed = reference.residual_rms_norm(x, residual, weight, eps)
        q, s = reference.quantize_act(normed)
        return normed, summed, q, s.t().contiguous()
    out = torch.empty_like(x) if want_out else None
    summed = torch.empty_like(x) if residual is not None else x
    q = torch.empty((M, D), dtype=FP8, device=x.device)
    s_t = torch.empty((D // 128, M), dtype=torch.float32, device=x.device)
    lib().rms_norm(x, residual, weight, eps, out, summed if residual is not None else None, q, s_t)
    return out, summed, q, s_t


# ---------------------------------------------------------------- quant
def quantize_act(x):
    """1x128 UE8M0 quantisation -> (fp8 [M,K], scales_t fp32 [K/128, M])."""
    if not _cuda(x):
        q, s = reference.quantize_act(x)
        return q, s.t().contiguous()
    M, K = x.shape
    q = torch.empty((M, K), dtype=FP8, device=x.device)
    s_t = torch.empty((K // 128, M), dtype=torch.float32, device=x.device)
    lib().quant_act(x, q, s_t)
    return q, s_t


def quantize_index(x, scale_fmt="ue8m0"):
    return reference.quantize_index(x, scale_fmt)


# ----------------------------------------------------------------- gemms
def is_ue8m0(scales) -> bool:
    """True when every scale is a positive power of two (UE8M0-representable)."""
    s = scales.float()
    return bool(torch.all(s > 0) and torch.equal(s, torch.exp2(torch.round(torch.log2(s)))))


def fp8_gemm(q, s_t, weight, w_scales, *, out=None, residual=None, ue8m0: bool = False):
    """BF16 [M,N] = dequant(q, s_t) @ dequant(weight, w_scales)^T (+ residual).

    ``ue8m0``: the weight scales are powers of two (``is_ue8m0``); the
    activation scales always are (``quantize_act``).  The tensor core then
    applies both scales itself (block-scaled MMA) instead of the kernel
    promoting every 128-wide K block in FP32.
    """
    if not _cuda(q):
        a = reference.dequantize_act(q, s_t.t())
        res = a @ reference.dequantize_weight(weight, w_scales).T
        if residual is not None:
            res = res + residual.float()
        return res.to(torch.bfloat16)
    M, N = q.shape[0], weight.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=q.device) if out is None else out
    lib().fp8_gemm(q, s_t, weight, w_scales, out, residual, bool(ue8m0))
    return out


def fp8_linear(x, weight, w_scales, *, out=None, residual=None, ue8m0: bool = False):
    """Checkpoint FP8 linear: quantise x 1x128 (UE8M0), block-scaled GEMM -> BF16."""
    x2 = x.reshape(-1, x.shape[-1])
    if not _cuda(x):
        res = reference.fp8_linear(x2, weight, w_scales)
        if residual is not None:
            res = (res.float() + residual.float()).bfloat16()
        return res.reshape(*x.shape[:-1], weight.shape[0])
    q, s_t = quantize_act(x2.contiguous())
    return fp8_gemm(q, s_t, weight, w_scales, out=out, residual=residual,
                    ue8m0=ue8m0).reshape(*x.shape[:-1], weight.shape[0])


def linear(x, weight, scales=None):
    """FP8-block (``scales`` given) or BF16 linear -> BF16."""
    if scales is not None:
        return fp8_linear(x, weight, scales)
    if not _cuda(x):
        return reference.linear(x, weight)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    M, K = x2.shape
    N = weight.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    lib().bf16_gemm(x2, 0, K, 0, weight.contiguous(), 0, K, 0, out, 0, N, 0, M, N, K, 1)
    return out.reshape(*x.shape[:-1], N)


def bmm_nt(a, b, out=None, *, out_dtype=torch.bfloat16):
    """Batched out[g] = a[g] @ b[g]^T for a [G,M,K], b [G,N,K] (contiguous views)."""
    if not _cuda(a):
        return torch.bmm(a.float(), b.float().transpose(1, 2)).to(out_dtype)
    G, M, K = a.shape
    N = b.shape[1]
    a, b = a.contiguous(), b.contiguous()
    out = torch.empty((G, M, N), dtype=out_dtype, device=a.device) if out is None else out
    lib().bf16_gemm(a, 0, K, M * K, b, 0, K, N * K, out, 0, N, M * N, M, N, K, G)
    return out


def linear_f32(x, weight):
    """FP32 x @ weight^T with a BF16 x and an FP32 weight -> FP32 (SIMT kernel)."""
    if not _cuda(x):
        return x.float() @ weight.float().T
    out = torch.empty((x.shape[0], weight.shape[0]), dtype=torch.float32, device=x.device)
    lib().linear_f32(x.contiguous(), weight.contiguous(), out)
    return out


def split_bf16(weight: torch.Tensor) -> torch.Tensor:
    """[N, K] FP32 -> [2N, K] BF16 = [hi; lo] with hi + lo ~= weight (~16 mantissa bits)."""
    hi = weight.float().bfloat16()
    lo = (weight.float() - hi.float()).bfloat16()
    return torch.cat((hi, lo)).contiguous()


def linear_split(x, w_split):
    """Tensor-core x @ [hi; lo]^T for a BF16 x -> FP32 [M, 2N] partials (hi || lo).

    hi + lo reproduces an FP32 weight to ~2^-17 relative, so summing the two
    halves (done by the consumer) matches an FP32 GEMV to FP32 accumulation noise.
    """
    if not _cuda(x):
        return x.float() @ w_split.float().T
    x2 = x.contiguous()
    M, K = x2.shape
    N = w_split.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    lib().bf16_gemm(x2, 0, K, 0, w_split, 0, K, 0, out, 0, N, 0, M, N, K, 1)
    return out


def silu_mul(gate, up):
    if not _cuda(gate):
        return reference.silu_mul(gate, up)
    packed = torch.cat((gate, up), -1).contiguous()
    h = torch.empty_like(gate)
    lib().silu_mul_quant(packed, h, None, None)
    return h


def silu_mul_quant(packed):
    """packed [M, 2I] (gate|up) -> (h bf16 [M,I], q fp8 [M,I], scales_t [I/128, M])."""
    M, I2 = packed.shape
    I = I2 // 2
    if not _cuda(packed):
        h = reference.silu_mul(packed[:, :I], packed[:, I:])
        q, s = reference.quantize_act(h)
        return h, q, s.t().contiguous()
    h = torch.empty((M, I), dtype=torch.bfloat16, device=packed.device)
    q = torch.empty((M, I), dtype=FP8, device=packed.device)
    s_t = torch.empty((I // 128, M), dtype=torch.float32, device=packed.device)
    lib().silu_mul_quant(packed, h, q, s_t)
    return h, q, s_t


# --------------------------------------------------------------- indexer
def indexer_logits(q, k, weights, kscale, query_start: int, *, out=None):
    """Causal FP32 logits [Q, N] (masked columns -inf)."""
    if not _cuda(q):
        return reference.indexer_logits(q, k, weights, kscale, query_start)
    Q, N = q.shape[0], k.shape[0]
    if out is None:
        out = torch.full((Q, N), -torch.inf, dtype=torch.float32, device=q.device)
    lib().indexer_logits(q, k, weights, kscale, out, query_start)
    return out


def indexer_select(q, keys, weights, kscale, query_start: int, k: int, *, logits_buf=None, order: str = "index",
                   sample_stride: int = 32, cand_cap: int = 8192, diag=None):
    """Fused indexer + exact top-k: ``exact_topk(indexer_logits(...), k, causal_start=query_start,
    n=len(keys), order=order)`` without the full FP32 logits in HBM.

    On CUDA a 1/``sample_stride`` sampling pass of the indexer sets a per-row
    threshold, the selection pass keeps only logits at or above it (at most
    ``cand_cap`` per row) and an exact top-k runs over those candidates; rows
    whose candidates cannot decide the top-k are redone from full logits in
    ``logits_buf`` (allocated when not given).  Returns (values, ids), width
    min(k, len(keys)).  ``diag`` (int64 [3], CUDA) receives the rows redone
    from full logits, the candidates kept and the largest per-row count.
    """
    if order not in ("value", "index"):
        raise ValueError("order must be 'value' or 'index'")
    N = keys.shape[0]
    if not _cuda(q):
        logits = reference.indexer_logits(q, keys, weights, kscale, query_start)
        return exact_topk(logits, k, causal_start=query_start, n=N, order=order)
    Q = q.shape[0]
    width = min(k, N)
    if logits_buf is None or logits_buf.shape[0] < Q or logits_buf.shape[1] < N:
        logits_buf = torch.empty((Q, max(4, (N + 3) // 4 * 4)), dtype=torch.float32, device=q.device)
    values = torch.empty((Q, width), dtype=torch.float32, device=q.device)
    ids = torch.empty((Q, width), dtype=torch.int32, device=q.device)
    lib().indexer_select(q, keys, weights, kscale, logits_buf, query_start, k, values, ids, order == "index",
                         sample_stride, max(cand_cap, 2 * k), diag)
    return values, ids


def exact_topk(scores, k: int, *, causal_start: int | None = None, n: int | None = None, algo: int = 0,
               order: str = "value", out=None):
    """Exact top-k (ties -> smaller index), -1 ids for non-finite/empty slots.

    ``causal_start`` restricts row r to columns [0, causal_start + r + 1).
    Output width is min(k, n) like the reference selection API.
    ``order="value"`` lists the selection by descending value; ``order="index"``
    lists the same selection by ascending index (padding last), which skips the
    kernel's final sort -- for consumers that need the set in a deterministic
    order, not its ranking (rows with one value shared by more than 6,144 keys
    are finished by the multi-pass kernel and stay value-ordered).
    """
    if order not in ("value", "index"):
        raise ValueError("order must be 'value' or 'index'")
    n = scores.shape[1] if n is None else n
    count = min(k, n)
    if not _cuda(scores):
        s = scores[:, :n]
        if causal_start is not None:
            rows = torch.arange(s.shape[0])[:, None]
            cols = torch.arange(n)[None, :]
            s = s.masked_fill(cols > causal_start + rows, -torch.inf)
        values, ids = reference.exact_topk(s, count)
        if order == "index":
            key = torch.where(ids >= 0, ids.long(), torch.iinfo(torch.int64).max)
            perm = key.argsort(dim=-1, stable=True)
            values, ids = values.gather(1, perm).contiguous(), ids.gather(1, perm).contiguous()
        return values, ids
    if order == "index" and algo == 0:
        algo = 2
    R = scores.shape[0]
    if out is not None:  # caller-owned [R, count] outputs (row slices of a larger result)
        values, ids = out
    else:
        values = torch.empty((R, count), dtype=torch.float32, device=scores.device)
        ids = torch.empty((R, count), dtype=torch.int32, device=scores.device)
    lib().topk(scores, n, count, -1 if causal_start is None else causal_start, values, ids, algo)
    return values, ids


# ------------------------------------------------------------------- MoE
def moe_route(logits, bias, cfg, *, split: bool = False):
    """Routing from gate logits [T, E] (or [T, 2E] hi||lo halves when ``split``).

    Returns (ids int32 [T, k], weights fp32 [T, k]); same rule as
    :func:`reference.route_experts` (ties -> smaller index)."""
    T = logits.shape[0]
    K = cfg.num_experts_per_tok
    ids = torch.empty((T, K), dtype=torch.int32, device=logits.device)
    w = torch.empty((T, K), dtype=torch.float32, device=logits.device)
    lib().moe_route(logits, split, bias, cfg.n_routed_experts, cfg.n_group, cfg.topk_group, K, cfg.norm_topk_prob,
                    cfg.routed_scaling_factor, ids, w)
    return ids, w


class MoELayout:
    """Padded contiguous grouped-GEMM layout built on the device (no host sync)."""

    def __init__(self, rows: int, e0: int, n_local: int, K: int, device):
        self.max_blocks = (rows + n_local * 127 + 127) // 128
        self.M_pad = self.max_blocks * 128
        self.e0, self.n_local = e0, n_local
        self.row_pos = torch.empty(rows, dtype=torch.int32, device=device)
        self.block_expert = torch.empty(self.max_blocks, dtype=torch.int32, device=device)
        self.cursor = torch.empty(n_local, dtype=torch.int32, device=device)
        self.total = torch.zeros(1, dtype=torch.int32, device=device)
        self.a = torch.zeros((self.M_pad, K), dtype=FP8, device=device)
        self.a_s = torch.zeros((K // 128, self.M_pad), dtype=torch.float32, device=device)

    def build(self, ids, q, s_t, topk: int):
        """Lay out ``ids`` (<= the workspace's row capacity) for the grouped GEMM; ``row_pos`` covers them."""
        n = ids.numel()
        if n > self.row_pos.numel():
            raise ValueError("more routed rows than the layout workspace holds")
        self.rows = n
        lib().moe_layout(ids.reshape(-1), self.e0, self.n_local, self.max_blocks, self.row_pos[:n], self.block_expert,
                         self.cursor, self.total)
        lib().moe_gather(q, s_t, topk, self.row_pos[:n], self.a, self.a_s)
        return self

    @property
    def positions(self):
        return self.row_pos[: self.rows]


class EpPushTarget:
    """Destination of an expert-parallel down projection that pushes its rows
    to their source ranks (``out=`` of :func:`fp8_gemm_grouped`): the owner's
    row-source table and block validity, every rank's receive slots and flag
    block (call parity half), and a local CTA finish counter."""

    def __init__(self, row_src: int, block_valid, dst: list, flags: list, finish, rank: int, world: int):
        self.row_src, self.block_valid, self.dst, self.flags = row_src, block_valid, dst, flags
        self.finish, self.rank, self.world = finish, rank, world


def fp8_gemm_grouped(a, a_s, w, w_s, block_expert, out=None):
    """Grouped FP8 GEMM over a padded layout: out[m] = a[m] . w[expert(m // 128)]^T.

    With ``out`` an :class:`EpPushTarget` the rows go to their source ranks
    over NVLink instead (returns None)."""
    if isinstance(out, EpPushTarget):
        lib().fp8_gemm_grouped_push(a, a_s, w, w_s, block_expert, out.block_valid, out.row_src, out.dst, out.flags,
                                    out.finish, out.rank, out.world)
        return None
    if out is None:
        out = torch.empty((a.shape[0], w.shape[1]), dtype=torch.bfloat16, device=a.device)
    lib().fp8_gemm_grouped(a, a_s, w, w_s, block_expert, out)
    return out


def moe_combine(y, row_pos, weights, T: int):
    out = torch.empty((T, y.shape[1]), dtype=torch.bfloat16, device=y.device)
    lib().moe_combine(y, row_pos, weights.contiguous(), weights.shape[1], out)
    return out


# ------------------------------------------------------------- attention
def sparse_mla(q, kv, ids, scale, *, splits: int = 1, return_lse: bool = False, value_dim: int = 512,
               impl: int = 0):
    """Sparse MLA: q [T,H,576], kv [P,576], ids [T,K] -> [T,H,512] (BF16)."""
    if not _cuda(q):
        if return_lse:
            o, lse = reference.sparse_mla_lse(q, kv, ids, scale, value_dim)
            return o.to(q.dtype), lse
        return reference.sparse_mla(q, kv, ids, scale, value_dim)
    if value_dim != 512 or q.shape[-1] != 576:
        raise ValueError("the sm_100a sparse MLA kernel covers the V3.2 shape (576 / 512)")
    T, H, _ = q.shape
    out = torch.empty((T, H, 512), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((T, H), dtype=torch.float32, device=q.device) if return_lse else None
    scratch = None
    if splits > 1:
        nbytes = lib().sparse_mla_scratch_bytes(T, H, splits)
        scratch = torch.empty(nbytes // 4, dtype=torch.float32, device=q.device)
    lib().sparse_mla(q.contiguous(), kv, ids.contiguous(), float(scale), out, lse, splits, scratch, impl)
    return (out, lse) if return_lse else out


def mla_splits(T: int, K: int = 2048, *, clusters: int = 74) -> int:
    """Split-K factor for the 2-CTA sparse MLA: few queries (decode, short
    extends) leave most of the 74 cluster slots (148 SMs) idle, so split each
    query's selection over more clusters, keeping >= 256 keys (four 64-key
    pair tiles) per split: each split reloads the query (~5K cycles), pays its
    pipeline fill and writes a 256 KB FP32 partial (head-minor, ~4.4K
    cycles), and the LSE combine reads every split.  Measured on B200 at
    K = 2048, cold L2, CUDA graph replays: T = 1 takes 39.5 / 29.5 / 24.9 us
    with 2 / 4 / 8 splits; T = 128 is faster unsplit."""
    if T >= clusters:
        return 1
    return max(1, min(32, clusters // max(T, 1), K // 256))


def sparse_mla_decode(q, kv, ids, scale, splits: int = 16):
    """Single-query decode: split the selection over ``splits`` CTAs and LSE-merge."""
    return sparse_mla(q, kv, ids, scale, splits=splits)


# -------------------------------------------------------------- transfer
def gather_host_records(host, records, host_ids, slots, *, device_count=None, fp8_scratch=None, latent_dim=512):
    """records[slots[i]] = host[host_ids[i]] (SM gather from pinned host memory on CUDA).

    ``fp8_scratch`` ([>= n, 656] uint8 on the device): the host holds 656-byte
    FP8 records; they cross PCIe into the scratch and are dequantized into
    ``records[slots]``."""
    if fp8_scratch is not None:
        n = host_ids.numel()
        if not records.is_cuda:
            records[slots.long()] = reference.fp8_kv_unpack(host[host_ids.long()], latent_dim).to(records.dtype)
            return records
        if n:
            lib().gather_rows(host, fp8_scratch, host_ids.long().contiguous(), None, n, device_count)
            lib().dequant_kv_rows(fp8_scratch, records, slots.long().contiguous(), n, device_count)
        return records
    if not records.is_cuda:
        records[slots.long()] = host[host_ids.long()].to(records.dtype)
        return records
    n = host_ids.numel()
    if n:
        lib().gather_rows(host, records, host_ids.long().contiguous(), slots.long().contiguous(), n, device_count)
    return records


_ARANGE_CACHE: dict = {}
_ARANGE_MAX_LEN, _ARANGE_MAX_ENTRIES = 256, 64


def arange_cached(start: int, end: int, *, device, dtype=torch.int64):
    """``torch.arange(start, end)`` for short CUDA ranges, kept on the device.

    Decode and extend steps ask for the same small index ranges (token
    positions, the rows a chunk's records go to) on every call; a captured
    CUDA graph then reads the kept tensor instead of running an arange kernel
    in each replay.  Callers must not write to the result.  Entries are never
    freed (a graph may still read them), so at most 64 ranges of at most 256
    elements are kept; other requests, and misses inside a stream capture,
    get a fresh ``torch.arange``."""
    device = torch.device(device)
    if device.type != "cuda" or end - start > _ARANGE_MAX_LEN:
        return torch.arange(start, end, device=device, dtype=dtype)
    key = (device, start, end, dtype)
    t = _ARANGE_CACHE.get(key)
    if t is None:
        if len(_ARANGE_CACHE) >= _ARANGE_MAX_ENTRIES or torch.cuda.is_current_stream_capturing():
            return torch.arange(start, end, device=device, dtype=dtype)
        t = torch.arange(start, end, device=device, dtype=dtype)
        torch.cuda.current_stream(device).synchronize()  # ready for any stream that reads it later
        _ARANGE_CACHE[key] = t
    return t


def l2_prefetch(t, nbytes: int | None = None):
    """Start pulling ``t`` (contiguous, not written while in flight) into L2; no-op off CUDA."""
    if _cuda(t):
        lib().l2_prefetch(t, -1 if nbytes is None else int(nbytes))


def embed(ids, table, *, row0: int = 0, vocab_total: int | None = None):
    """Embedding rows of ``ids``.  ``table`` may be a vocabulary shard holding
    rows [row0, row0 + len(table)) of a ``vocab_total``-row table; ids outside
    the shard give zero rows (sum the shards' outputs across ranks)."""
    total = table.shape[0] if vocab_total is None else vocab_total
    if not table.is_cuda:
        return reference.embed_shard(ids, table, row0, total)
    out = torch.empty((ids.numel(), table.shape[1]), dtype=torch.bfloat16, device=table.device)
    lib().embed(ids.long().contiguous(), table, out, row0, total)
    return out


route_experts = reference.route_experts


def attention_scale_log2(scale: float) -> float:
    return scale * math.log2(math.e)


# ------------------------------------------------- projection epilogues
def _angles(freqs, positions):
    return positions.float()[:, None] * freqs[None, :].float()


def mla_q_rope(b, H, nope, rope, freqs, positions, q_proj, latent):
    """q_proj[:, h, latent:] = interleaved-RoPE(b[:, h*(nope+rope)+nope : ...])."""
    T = q_proj.shape[0]
    if not _cuda(b):
        qpe = b[:, : H * (nope + rope)].reshape(T, H, nope + rope)[..., nope:]
        q_proj[..., latent:] = reference.apply_rope(qpe, _angles(freqs, positions), interleaved=True)
        return
    lib().mla_q_rope(b, b.stride(0), T, H, nope, rope, freqs, positions, q_proj, q_proj.stride(0), q_proj.stride(1), latent)


def kv_finish(kv, L, R, norm_w, eps, freqs, positions, records, rows, *, packed=None):
    """records[rows] = [rmsnorm(kv[:, :L]) || interleaved-RoPE(kv[:, L:L+R])].

    ``packed`` ([>= T, 656] uint8): FP8 records.  The latent is quantized per
    128 dims (E4M3, FP32 scale amax / 448), ``packed[:T]`` receives the 656-byte
    records and ``records[rows]`` their exact dequantized values."""
    if not _cuda(kv):
        lat = reference.rms_norm(kv[:, :L], norm_w, eps)
        pe = reference.apply_rope(kv[:, L:L + R], _angles(freqs, positions), interleaved=True).bfloat16()
        if packed is not None:
            q, scale, lat = reference.fp8_kv_quantize(lat.bfloat16())
            packed[: kv.shape[0]] = reference.fp8_kv_pack(q, scale, pe)
        records[rows.long()] = torch.cat((lat.to(records.dtype), pe.to(records.dtype)), -1)
        return
    lib().kv_finish(kv, L, R, norm_w, eps, freqs, positions, records, rows.long(), packed)


def fp8_kv_records(rows: torch.Tensor, latent_dim: int = 512):
    """(dequantized BF16 rows, packed FP8 records) of BF16 KV rows [T, L + R]: the
    generic append path (records that did not come from kv_finish); same
    arithmetic as kv_finish's FP8 path, in torch ops on either device."""
    q, scale, lat = reference.fp8_kv_quantize(rows[:, :latent_dim])
    pe = rows[:, latent_dim:].bfloat16()
    return torch.cat((lat, pe), -1), reference.fp8_kv_pack(q, scale, pe)


def dequant_kv_rows(packed, records, slots=None, *, count=None, device_count=None, latent_dim: int = 512):
    """records[slots[i]] = BF16 row of the packed FP8 record packed[i] (i < count)."""
    n = packed.shape[0] if count is None else count
    if not _cuda(records):
        rows = reference.fp8_kv_unpack(packed[:n], latent_dim)
        idx = torch.arange(n) if slots is None else slots[:n].long()
        records[idx] = rows.to(records.dtype)
        return records
    if n:
        lib().dequant_kv_rows(packed, records, None if slots is None else slots.long().contiguous(), n, device_count)
    return records


def index_k(ik, R, ln_w, ln_b, eps, freqs, positions, k_out, s_out):
    """Indexer key: LayerNorm(+bias) -> BF16 -> split-half RoPE -> UE8M0 FP8 (into k_out/s_out)."""
    if not _cuda(ik):
        k = reference.layer_norm(ik, ln_w, ln_b, eps).bfloat16()
        k = reference.apply_rope(k, _angles(freqs, positions), interleaved=False)
        q, s = reference.quantize_index(k)
        k_out.copy_(q)
        s_out.copy_(s[:, 0])
        return
    lib().index_k(ik, R, ln_w, ln_b, eps, freqs, positions, k_out, s_out)


def kv_finish_index_k(kv, L, R, norm_w, eps, freqs, positions, records, rows, ik, ln_w, ln_b, ln_eps, k_out, s_out,
                      *, packed=None):
    """:func:`kv_finish` then :func:`index_k` (both read the fused_a output); one launch on CUDA."""
    if not _cuda(kv):
        kv_finish(kv, L, R, norm_w, eps, freqs, positions, records, rows, packed=packed)
        index_k(ik, R, ln_w, ln_b, ln_eps, freqs, positions, k_out, s_out)
        return
    lib().kv_finish_index_k(kv, L, R, norm_w, eps, records, rows.long(), packed, ik, R, ln_w, ln_b, ln_eps, k_out,
                            s_out, freqs, positions)


def index_q(iq, heads, dim, R, freqs, positions, w_raw, head_scale):
    """Indexer query: split-half RoPE + per-head UE8M0 FP8; weights = raw * head_scale * q_scale.

    ``w_raw`` is [T, heads] or the [T, 2*heads] hi || lo partials of :func:`linear_split`.
    """
    T = iq.shape[0]
    if w_raw.shape[-1] == 2 * heads and not _cuda(iq):
        w_raw = w_raw[:, :heads] + w_raw[:, heads:]
    if not _cuda(iq):
        q = reference.apply_rope(iq[:, : heads * dim].reshape(T, heads, dim), _angles(freqs, positions), interleaved=False)
        qq, qs = reference.quantize_index(q)
        return qq, (w_raw * head_scale * qs[..., 0]).contiguous()
    qq = torch.empty((T, heads, dim), dtype=FP8, device=iq.device)
    qs = torch.empty((T, heads), dtype=torch.float32, device=iq.device)
    w = torch.empty((T, heads), dtype=torch.float32, device=iq.device)
    lib().index_q(iq, iq.stride(0), T, heads, dim, R, freqs, positions, qq, qs, w_raw.contiguous(), head_scale, w)
    return qq, w


def mla_q_rope_index_q(b, H, nope, rope, freqs, positions, q_proj, latent, iq, heads, dim, R, w_raw, head_scale):
    """:func:`mla_q_rope` then :func:`index_q` (returns its (q, weights)); one launch on CUDA."""
    if not _cuda(b):
        mla_q_rope(b, H, nope, rope, freqs, positions, q_proj, latent)
        return index_q(iq, heads, dim, R, freqs, positions, w_raw, head_scale)
    T = iq.shape[0]
    qq = torch.empty((T, heads, dim), dtype=FP8, device=iq.device)
    qs = torch.empty((T, heads), dtype=torch.float32, device=iq.device)
    w = torch.empty((T, heads), dtype=torch.float32, device=iq.device)
    lib().q_rope_index_q(b, b.stride(0), T, H, nope, rope, q_proj, q_proj.stride(0), q_proj.stride(1), latent,
                         iq, iq.stride(0), heads, dim, R, qq, qs, w_raw.contiguous(), head_scale, w, freqs, positions)
    return qq, w


def mla_absorb(b, H, nope, rope, wk_b_t, q_proj):
    """q_proj[:, h, :L] = b_nope[:, h] @ wk_b_t[h]^T  (W_UK absorption, BF16 GEMM per head)."""
    T = q_proj.shape[0]
    L = wk_b_t.shape[1]
    if not _cuda(b):
        qn = b[:, : H * (nope + rope)].reshape(T, H, nope + rope)[..., :nope].float()
        q_proj[..., :L] = torch.einsum("thn,hln->thl", qn, wk_b_t.float()).to(q_proj.dtype)
        return
    if not b.is_contiguous():
        raise ValueError("absorb input must be the contiguous projection output")
    lib().bf16_gemm(b, 0, b.stride(0), nope + rope, wk_b_t, 0, nope, L * nope,
                    q_proj, 0, q_proj.stride(0), q_proj.stride(1), T, L, nope, H)


def mla_expand(attn, wv_b):
    """out[:, h] = attn[:, h] @ wv_b[h]^T : [T,H,L] x [H,V,L] -> [T,H,V] (BF16)."""
    T, H, L = attn.shape
    V = wv_b.shape[1]
    if not _cuda(attn):
        return torch.einsum("thl,hvl->thv", attn.float(), wv_b.float()).to(torch.bfloat16)
    out = torch.empty((T, H, V), dtype=torch.bfloat16, device=attn.device)
    attn = attn.contiguous()
    lib().bf16_gemm(attn, 0, H * L, L, wv_b, 0, L, V * L, out, 0, H * V, V, T, V, L, H)
    return out
