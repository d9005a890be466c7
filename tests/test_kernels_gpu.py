"""Numerics of every sm_100a kernel against the plain-PyTorch FP32 oracle."""

import math

import pytest
import torch

from cxldsagr_b200 import ops
from cxldsagr_b200.checkpoint import quantize_weight_blocks
from cxldsagr_b200.config import v32_config
from cxldsagr_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


@pytest.fixture(autouse=True)
def _check_device_errors():
    yield
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        ops.check_errors(DEV)


# ------------------------------------------------------------------ norms
@pytest.mark.parametrize("rows,D", [(1, 7168), (37, 1536), (130, 512)])
def test_rms_norm(rows, D):
    torch.manual_seed(0)
    x = torch.randn(rows, D, device=DEV).bfloat16()
    r = torch.randn(rows, D, device=DEV).bfloat16()
    w = torch.rand(D, device=DEV) + 0.5
    got = ops.rms_norm(x, w, 1e-6)
    want = ref.rms_norm(x.cpu(), w.cpu(), 1e-6)
    assert rel_err(got.cpu(), want) < 1e-2
    n, s = ops.residual_rms_norm(x, r, w, 1e-6)
    wn, ws = ref.residual_rms_norm(x.cpu(), r.cpu(), w.cpu(), 1e-6)
    assert torch.equal(s.cpu(), ws)
    assert rel_err(n.cpu(), wn) < 1e-2


@pytest.mark.parametrize("rows,D", [(64, 7168), (1, 7168), (3, 1536), (5, 512)])
def test_norm_quant_matches_quantize(rows, D):
    torch.manual_seed(1)
    x = torch.randn(rows, D, device=DEV).bfloat16()
    w = torch.rand(D, device=DEV) + 0.5
    n, _, q, s_t = ops.norm_quant(x, None, w, 1e-6)
    q2, s2 = ops.quantize_act(n)
    assert torch.equal(q.view(torch.uint8), q2.view(torch.uint8))
    assert torch.equal(s_t, s2)


@pytest.mark.parametrize("M,K", [(1, 128), (33, 7168), (256, 18432)])
def test_quant_act_bitwise(M, K):
    torch.manual_seed(2)
    x = (torch.randn(M, K, device=DEV) * 3).bfloat16()
    q, s_t = ops.quantize_act(x)
    rq, rs = ref.quantize_act(x.cpu())
    assert torch.equal(s_t.cpu(), rs.t())
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


def test_silu_mul_quant():
    torch.manual_seed(3)
    packed = torch.randn(17, 2 * 2048, device=DEV).bfloat16()
    h, q, s_t = ops.silu_mul_quant(packed)
    rh = ref.silu_mul(packed[:, :2048].cpu(), packed[:, 2048:].cpu())
    assert rel_err(h.cpu(), rh) < 1e-2
    rq, rs = ref.quantize_act(h.cpu())
    assert torch.equal(s_t.cpu(), rs.t())


# ------------------------------------------------------------------ gemms
@pytest.mark.parametrize("M,N,K", [(1, 576, 7168), (128, 1536, 7168), (200, 7168, 2048), (1024, 2240, 7168), (77, 130, 256),
                                   (128, 7168, 18432), (1024, 36864, 1024), (1024, 7168, 4096), (640, 7168, 2048)])
def test_fp8_gemm(M, N, K):
    """Includes N = 7168 shapes that take the 224-wide tiles (scale blocks straddle a warp's columns)."""
    torch.manual_seed(4)
    x = torch.randn(M, K, device=DEV).bfloat16()
    w, s = quantize_weight_blocks(torch.randn(N, K, device=DEV) * 0.02, pow2_scales=False)
    got = ops.fp8_linear(x, w, s)
    want = ref.fp8_linear(x.cpu(), w.cpu(), s.cpu())
    assert rel_err(got.cpu(), want) < 2e-2


@pytest.mark.parametrize("M,N,K", [(1, 576, 7168), (128, 1536, 7168), (200, 7168, 2048), (1024, 2240, 7168),
                                   (77, 130, 256), (128, 7168, 18432), (1024, 36864, 1024), (1024, 7168, 4096),
                                   (640, 7168, 2048), (1024, 18432, 7168)])
def test_fp8_gemm_block_scaled(M, N, K):
    """Power-of-two scales through the block-scaled MMA (tcgen05 kind::mxf8f6f4.block_scale):
    every tile width (256 with one accumulator, 224 and 128 with two) and split-K."""
    torch.manual_seed(6)
    x = torch.randn(M, K, device=DEV).bfloat16()
    w, s = quantize_weight_blocks(torch.randn(N, K, device=DEV) * 0.02)
    assert ops.is_ue8m0(s)
    res = torch.randn(M, N, device=DEV).bfloat16()
    got = ops.fp8_linear(x, w, s, residual=res, ue8m0=True)
    want = ref.fp8_linear(x.cpu(), w.cpu(), s.cpu()).float() + res.cpu().float()
    assert rel_err(got.cpu(), want) < 2e-2
    promoted = ops.fp8_linear(x, w, s, residual=res)
    assert rel_err(got.cpu(), promoted.cpu().float()) < 5e-3


@pytest.mark.parametrize("M,N,K", [(130, 384, 1024), (128, 7168, 16384), (1024, 7168, 2048)])
def test_fp8_gemm_residual(M, N, K):
    """Residual fused in the epilogue (no split) and in the split-K reduce."""
    torch.manual_seed(5)
    x = torch.randn(M, K, device=DEV).bfloat16()
    res = torch.randn(M, N, device=DEV).bfloat16()
    w, s = quantize_weight_blocks(torch.randn(N, K, device=DEV) * 0.05)
    got = ops.fp8_linear(x, w, s, residual=res)
    want = ref.fp8_linear(x.cpu(), w.cpu(), s.cpu()).float() + res.cpu().float()
    assert rel_err(got.cpu(), want) < 2e-2


@pytest.mark.parametrize("M,N,K", [(256, 7168, 2048), (300, 2304, 7168), (1000, 7168, 4096), (2048, 2048, 1024),
                                   (512, 18432, 2048), (384, 640, 512)])
def test_fp8_gemm_pair_tiles_match_single(M, N, K):
    """256-row pair tiles (2-CTA cta_group::2) against the FP32 oracle and the 128-row kernel:
    every tile width, an M that is not a multiple of 256, a residual."""
    torch.manual_seed(8)
    x = torch.randn(M, K, device=DEV).bfloat16()
    w, s = quantize_weight_blocks(torch.randn(N, K, device=DEV) * 0.02, pow2_scales=False)
    res = torch.randn(M, N, device=DEV).bfloat16()
    ops.lib().set_fp8_gemm_pair_tiles(True)
    try:
        got = ops.fp8_linear(x, w, s, residual=res)
    finally:
        ops.lib().set_fp8_gemm_pair_tiles(False)
    want = ref.fp8_linear(x.cpu(), w.cpu(), s.cpu()).float() + res.cpu().float()
    assert rel_err(got.cpu(), want) < 2e-2
    single = ops.fp8_linear(x, w, s, residual=res)
    torch.cuda.synchronize()
    # Same per-128-K promotion order per output: the two kernels agree to BF16 rounding.
    assert rel_err(got.cpu(), single.cpu().float()) < 5e-3
    ops.check_errors(DEV)


@pytest.mark.parametrize("G,M,N,K", [(1, 1, 1000, 7168), (4, 130, 512, 128), (3, 64, 128, 512)])
def test_bf16_bmm(G, M, N, K):
    torch.manual_seed(6)
    a = torch.randn(G, M, K, device=DEV).bfloat16()
    b = torch.randn(G, N, K, device=DEV).bfloat16()
    got = ops.bmm_nt(a, b, out_dtype=torch.float32)
    want = torch.bmm(a.float().cpu(), b.float().cpu().transpose(1, 2))
    assert rel_err(got.cpu(), want) < 1e-3


# ------------------------------------------------------------- indexer
@pytest.mark.parametrize("Q,N,start", [(1, 700, 699), (1, 130, 129), (1, 65537, 65536), (7, 300, 200),
                                       (64, 4096, 4032), (130, 2000, 0)])
def test_indexer_logits(Q, N, start):
    torch.manual_seed(7)
    N = max(N, start + Q)
    q = (torch.randn(Q, 64, 128, device=DEV) * 2).to(torch.float8_e4m3fn)
    k = (torch.randn(N, 128, device=DEV) * 2).to(torch.float8_e4m3fn)
    w = torch.randn(Q, 64, device=DEV)
    ks = torch.rand(N, device=DEV) + 0.1
    got = ops.indexer_logits(q, k, w, ks, start)
    want = ref.indexer_logits(q.cpu(), k.cpu(), w.cpu(), ks.cpu(), start)
    fin = torch.isfinite(want)
    assert torch.equal(torch.isfinite(got.cpu()), fin)
    assert rel_err(got.cpu()[fin], want[fin]) < 1e-4
    if Q == 1 and start > 0:
        # The single-query layout (four key tiles per accumulator) gives the
        # same bits as the query's row of a multi-query launch.
        pair = ops.indexer_logits(torch.cat([q, q]), k, torch.cat([w, w]), ks, start - 1)
        assert torch.equal(pair[1, :start + 1], got[0, :start + 1])


# ------------------------------------------------- fused indexer selection
@pytest.mark.parametrize("order", ["index", "value"])
@pytest.mark.parametrize("Q,N,start", [(7, 300, 200), (64, 20000, 19936), (130, 12000, 0), (256, 65536, 65280),
                                       (1, 70000, 69999), (40, 9000, 3000)])
def test_indexer_select_matches_logits_topk(Q, N, start, order):
    """The fused selection (sampled threshold, candidate lists, candidate top-k,
    fallback) equals exact_topk over the kernel's full logits, bit for bit."""
    torch.manual_seed(31)
    N = max(N, start + Q)
    q = (torch.randn(Q, 64, 128, device=DEV) * 2).to(torch.float8_e4m3fn)
    k = (torch.randn(N, 128, device=DEV) * 2).to(torch.float8_e4m3fn)
    w = torch.randn(Q, 64, device=DEV)
    ks = torch.rand(N, device=DEV) + 0.1
    logits = ops.indexer_logits(q, k, w, ks, start)
    rv, ri = ops.exact_topk(logits, 2048, causal_start=start, n=N, order=order)
    v, i = ops.indexer_select(q, k, w, ks, start, 2048, order=order)
    ops.check_errors(DEV)
    assert torch.equal(i, ri)
    assert torch.equal(v, rv)


@pytest.mark.parametrize("Q", [48, 1])
@pytest.mark.parametrize("kind", ["equal_keys", "banded"])
def test_indexer_select_fallback_rows(kind, Q):
    """Rows the candidate lists cannot decide (one value shared by every key:
    the threshold keeps them all and overflows the list) are redone from full
    logits; the result still equals the plain path (one query: the
    single-query indexer layout in every pass)."""
    torch.manual_seed(32)
    N = 30000
    start = N - Q
    q = (torch.randn(Q, 64, 128, device=DEV) * 2).to(torch.float8_e4m3fn)
    if kind == "equal_keys":
        k = (torch.randn(1, 128, device=DEV) * 2).expand(N, 128).contiguous().to(torch.float8_e4m3fn)
        ks = torch.full((N,), 0.5, device=DEV)
    else:  # few distinct keys: large tie groups around the threshold
        k = (torch.randn(7, 128, device=DEV) * 2)[torch.randint(0, 7, (N,), device=DEV)].to(torch.float8_e4m3fn)
        ks = torch.full((N,), 0.5, device=DEV)
    w = torch.randn(Q, 64, device=DEV)
    w[: Q // 2] = w[: Q // 2].abs()
    logits = ops.indexer_logits(q, k, w, ks, start)
    rv, ri = ops.exact_topk(logits, 2048, causal_start=start, n=N, order="index")
    v, i = ops.indexer_select(q, k, w, ks, start, 2048, order="index")
    ops.check_errors(DEV)
    assert torch.equal(i, ri)
    assert torch.equal(v, rv)


# ----------------------------------------------------------------- topk
@pytest.mark.parametrize("algo", [0, 1], ids=["two_pass", "multi_pass"])
@pytest.mark.parametrize("R,N,k", [(3, 100, 64), (5, 5000, 2048), (2, 70000, 2048), (4, 1500, 2048), (300, 65536, 2048)])
def test_topk(R, N, k, algo):
    torch.manual_seed(8)
    s = torch.randn(R, N, device=DEV)
    v, i = ops.exact_topk(s, k, algo=algo)
    rv, ri = ref.exact_topk(s.cpu(), k)
    assert torch.equal(i.cpu(), ri)
    assert torch.equal(v.cpu(), rv)


@pytest.mark.parametrize("algo", [0, 1])
def test_topk_ties_and_causal(algo):
    """Heavy ties overflow the two-pass kernel's threshold bin -> multi-pass fallback."""
    torch.manual_seed(9)
    s = torch.randint(0, 5, (6, 3000), device=DEV).float()
    v, i = ops.exact_topk(s, 2048, causal_start=1000, algo=algo)
    rows = torch.arange(6)[:, None]
    cols = torch.arange(3000)[None, :]
    masked = s.cpu().masked_fill(cols > 1000 + rows, -torch.inf)
    rv, ri = ref.exact_topk(masked, 2048)
    assert torch.equal(i.cpu(), ri)


def test_topk_moderate_ties_two_pass():
    """Coarse values with a threshold bin that fits in shared memory."""
    torch.manual_seed(14)
    s = (torch.randn(8, 20000, device=DEV) * 4).round() / 4
    v, i = ops.exact_topk(s, 2048, causal_start=15000)
    rows = torch.arange(8)[:, None]
    cols = torch.arange(20000)[None, :]
    masked = s.cpu().masked_fill(cols > 15000 + rows, -torch.inf)
    rv, ri = ref.exact_topk(masked, 2048)
    assert torch.equal(i.cpu(), ri) and torch.equal(v.cpu(), rv)


@pytest.mark.parametrize("ld_pad", [0, 3])
def test_topk_indexer_like_rows(ld_pad):
    """Narrow-band logits (threshold decided inside the staged bin by the index
    bits for equal values), unaligned row starts, short rows that take every
    element, -inf entries."""
    torch.manual_seed(15)
    R, N = 40, 9000
    base = torch.randn(R, N + ld_pad, device=DEV)
    s = (10.0 + 0.01 * base).half().float()  # many exact duplicates near the threshold
    s[:, 7] = -torch.inf
    view = s[:, ld_pad:] if ld_pad else s
    v, i = ops.exact_topk(view, 2048, causal_start=1000)
    rows = torch.arange(R)[:, None]
    cols = torch.arange(N)[None, :]
    masked = view.cpu().masked_fill(cols > 1000 + rows, -torch.inf)
    rv, ri = ref.exact_topk(masked, 2048)
    assert torch.equal(i.cpu(), ri)
    fin = torch.isfinite(rv)
    assert torch.equal(v.cpu()[fin], rv[fin])


# ------------------------------------------------------------ sparse MLA
@pytest.mark.parametrize("impl", [0, 1, 4], ids=["tcgen05_pair", "mma_sync", "tcgen05_exchange"])
@pytest.mark.parametrize("T,K,P,splits", [(2, 2048, 5000, 1), (3, 256, 300, 1), (1, 2048, 9000, 16), (5, 100, 64, 4),
                                          (300, 2048, 70000, 1)])
def test_sparse_mla(T, K, P, splits, impl):
    torch.manual_seed(10)
    H = 128
    q = (torch.randn(T, H, 576, device=DEV) * 0.5).bfloat16()
    kv = (torch.randn(P, 576, device=DEV) * 0.5).bfloat16()
    ids = torch.randint(0, P, (T, K), device=DEV, dtype=torch.int32)
    ids[:, -7:] = -1
    ids[0, :3] = P + 5  # out of range = padding
    scale = v32_config().attention_scale
    got, lse = ops.sparse_mla(q, kv, ids, scale, splits=splits, return_lse=True, impl=impl)
    if T > 8:  # oracle on a subset of rows
        rows = torch.tensor([0, 1, T // 2, T - 1])
        want, wlse = ref.sparse_mla_lse(q[rows].cpu(), kv.cpu(), ids[rows].cpu(), scale)
        got, lse = got[rows.to(DEV)], lse[rows.to(DEV)]
    else:
        want, wlse = ref.sparse_mla_lse(q.cpu(), kv.cpu(), ids.cpu(), scale)
    assert rel_err(got.cpu(), want) < 2e-2
    assert torch.allclose(lse.cpu(), wlse, atol=2e-2, rtol=1e-3)


@pytest.mark.parametrize("impl", [0, 1, 4])
def test_sparse_mla_all_padding_is_zero(impl):
    q = torch.randn(2, 128, 576, device=DEV).bfloat16()
    kv = torch.randn(10, 576, device=DEV).bfloat16()
    ids = torch.full((2, 64), -1, dtype=torch.int32, device=DEV)
    out = ops.sparse_mla(q, kv, ids, 0.1, impl=impl)
    assert torch.count_nonzero(out) == 0


def test_sparse_mla_large_logit_range_rescale():
    """Scores growing by far more than 2^8 across tiles exercise the lazy O rescale."""
    torch.manual_seed(13)
    T, K, P = 2, 512, 600
    q = torch.randn(T, 128, 576, device=DEV).bfloat16()
    kv = torch.randn(P, 576, device=DEV)
    kv *= torch.linspace(0.1, 4.0, P, device=DEV)[:, None]
    kv = kv.bfloat16()
    ids = torch.arange(K, device=DEV, dtype=torch.int32).repeat(T, 1)
    got = ops.sparse_mla(q, kv, ids, 0.2)
    want = ref.sparse_mla(q.cpu(), kv.cpu(), ids.cpu(), 0.2)
    assert rel_err(got.cpu(), want) < 2e-2


# ---------------------------------------------------------- elementwise
def test_projection_epilogues():
    torch.manual_seed(11)
    cfg = v32_config(3)
    T = 19
    freqs = ref.rotary_frequencies(cfg).to(DEV)
    pos = torch.arange(100, 100 + T, device=DEV).float()
    angles = (pos[:, None] * freqs[None, :]).cpu()
    L = ops.lib()
    # MLA q rope
    q = torch.randn(T, 128 * 192, device=DEV).bfloat16()
    out = torch.zeros(T, 128, 576, device=DEV).bfloat16()
    L.mla_q_rope(q, q.stride(0), T, 128, 128, 64, freqs, pos, out, 128 * 576, 576, 512)
    want = ref.apply_rope(q.cpu().reshape(T, 128, 192)[..., 128:], angles, interleaved=True)
    assert rel_err(out[..., 512:].cpu(), want) < 1e-2
    # kv finish
    kv = torch.randn(T, 576, device=DEV).bfloat16()
    nw = torch.rand(512, device=DEV) + 0.5
    rec = torch.empty(T, 576, device=DEV).bfloat16()
    L.kv_finish(kv, 512, 64, nw, 1e-6, freqs, pos, rec, None)
    lat = ref.rms_norm(kv.cpu()[:, :512], nw.cpu(), 1e-6)
    pe = ref.apply_rope(kv.cpu()[:, 512:], angles, interleaved=True)
    assert rel_err(rec[:, :512].cpu(), lat) < 1e-2 and rel_err(rec[:, 512:].cpu(), pe) < 1e-2
    # index k
    k = torch.randn(T, 128, device=DEV).bfloat16()
    lw, lb = torch.rand(128, device=DEV) + 0.5, torch.randn(128, device=DEV) * 0.1
    kq = torch.empty(T, 128, device=DEV, dtype=torch.float8_e4m3fn)
    ksc = torch.empty(T, device=DEV)
    L.index_k(k, 64, lw, lb, 1e-6, freqs, pos, kq, ksc)
    kk = ref.layer_norm(k.cpu(), lw.cpu(), lb.cpu(), 1e-6).bfloat16()
    kk = ref.apply_rope(kk, angles, interleaved=False)
    rq, rs = ref.quantize_index(kk)
    assert torch.allclose(ksc.cpu(), rs[:, 0])
    assert rel_err(kq.cpu().float() * ksc.cpu()[:, None], rq.float() * rs) < 0.07  # one e4m3 step
    # index q
    iq = torch.randn(T, 64 * 128, device=DEV).bfloat16()
    wraw = torch.randn(T, 64, device=DEV)
    qq = torch.empty(T, 64, 128, device=DEV, dtype=torch.float8_e4m3fn)
    qs = torch.empty(T, 64, device=DEV)
    wts = torch.empty(T, 64, device=DEV)
    L.index_q(iq, iq.stride(0), T, 64, 128, 64, freqs, pos, qq, qs, wraw, 0.125, wts)
    rq2 = ref.apply_rope(iq.cpu().reshape(T, 64, 128), angles, interleaved=False)
    _, rqs = ref.quantize_index(rq2)
    assert torch.allclose(qs.cpu(), rqs[..., 0])
    assert torch.allclose(wts.cpu(), wraw.cpu() * 0.125 * rqs[..., 0])


def test_linear_f32_and_embed():
    torch.manual_seed(12)
    x = torch.randn(40, 7168, device=DEV).bfloat16()
    W = torch.randn(64, 7168, device=DEV)
    got = ops.linear_f32(x, W)
    want = x.cpu().float() @ W.cpu().T
    assert rel_err(got.cpu(), want) < 1e-5
    parts = ops.linear_split(x, ops.split_bf16(W))
    assert rel_err((parts[:, :64] + parts[:, 64:]).cpu(), want) < 1e-5
    table = torch.randn(1000, 256, device=DEV).bfloat16()
    ids = torch.tensor([5, 0, 999, 17], device=DEV)
    assert torch.equal(ops.embed(ids, table), table[ids])


def test_gather_rows_from_pinned_host():
    host = torch.randn(256, 576).bfloat16().pin_memory()
    records = torch.zeros(65, 576, device=DEV).bfloat16()
    hid = torch.tensor([3, 100, 255, 7], device=DEV)
    slots = torch.tensor([1, 64, 2, 30], device=DEV)
    ops.gather_host_records(host, records, hid, slots)
    assert torch.equal(records[slots].cpu(), host[hid.cpu()])


# ------------------------------------------------------------------- MoE
class _MoECfg:
    n_routed_experts = 64
    n_group = 8
    topk_group = 4
    num_experts_per_tok = 8
    norm_topk_prob = True
    routed_scaling_factor = 2.5


@pytest.mark.parametrize("T", [1, 37, 300])
def test_moe_route_matches_reference(T):
    torch.manual_seed(11)
    cfg = _MoECfg
    E, D = cfg.n_routed_experts, 256
    x = torch.randn(T, D, device=DEV).bfloat16()
    gate = torch.randn(E, D, device=DEV) * 0.05
    bias = torch.randn(E, device=DEV) * 0.1
    logits = ops.linear_split(x, ops.split_bf16(gate))
    ids, w = ops.moe_route(logits, bias, cfg, split=True)
    want_ids, want_w = ref.route_experts(x.cpu(), gate.cpu(), bias.cpu(), cfg)
    for t in range(T):
        a = sorted(zip(ids[t].cpu().tolist(), w[t].cpu().tolist()))
        b = sorted(zip(want_ids[t].tolist(), want_w[t].tolist()))
        assert [i for i, _ in a] == [i for i, _ in b]
        assert max(abs(p - q) for (_, p), (_, q) in zip(a, b)) < 1e-4


@pytest.mark.parametrize("T,E,e0,n_local", [(64, 16, 0, 16), (200, 32, 8, 8)])
def test_grouped_moe_matches_reference(T, E, e0, n_local):
    """Device layout + grouped FP8 GEMMs + combine vs the FP32 reference over the local experts."""
    torch.manual_seed(12)
    D, I, K = 256, 256, 4
    x = torch.randn(T, D, device=DEV).bfloat16()
    q, s_t = ops.quantize_act(x)
    ids = torch.randint(0, E, (T, K), device=DEV, dtype=torch.int32)
    w = torch.rand(T, K, device=DEV)
    wg = [quantize_weight_blocks(torch.randn(2 * I, D, device=DEV) * 0.05, pow2_scales=False) for _ in range(n_local)]
    wd = [quantize_weight_blocks(torch.randn(D, I, device=DEV) * 0.05, pow2_scales=False) for _ in range(n_local)]
    w_gu = torch.stack([a for a, _ in wg]).contiguous()
    s_gu = torch.stack([b for _, b in wg]).float().contiguous()
    w_d = torch.stack([a for a, _ in wd]).contiguous()
    s_d = torch.stack([b for _, b in wd]).float().contiguous()
    lay = ops.MoELayout(T * K, e0, n_local, D, DEV).build(ids, q, s_t, K)
    gu = ops.fp8_gemm_grouped(lay.a, lay.a_s, w_gu, s_gu, lay.block_expert)
    _, hq, hs = ops.silu_mul_quant(gu)
    y = ops.fp8_gemm_grouped(hq, hs, w_d, s_d, lay.block_expert)
    got = ops.moe_combine(y, lay.positions, w, T).float().cpu()
    ops.check_errors(DEV)
    # reference: only local experts contribute
    want = torch.zeros(T, D)
    for t in range(T):
        for k in range(K):
            e = int(ids[t, k]) - e0
            if not 0 <= e < n_local:
                continue
            g = ref.fp8_linear(x[t:t + 1].cpu(), wg[e][0].cpu(), wg[e][1].cpu()).float()
            h = ref.silu_mul(g[:, :I], g[:, I:])
            yk = ref.fp8_linear(h.bfloat16(), wd[e][0].cpu(), wd[e][1].cpu()).float()
            want[t] += float(w[t, k]) * yk[0]
    assert rel_err(got, want) < 3e-2
    rows = (lay.positions >= 0).sum().item()
    assert rows == int(((ids >= e0) & (ids < e0 + n_local)).sum())


# ------------------------------------------------------- pool metadata (native)
@pytest.mark.parametrize("slots", [96, 256])
def test_native_pool_recall_matches_resident(slots):
    """Appends, exact recall and transient tails through the device-side pool
    metadata give the resident rows bit for bit, including under eviction."""
    from cxldsagr_b200.cache.sparse_token_cache import SparseTokenCache

    torch.manual_seed(21)
    width, cap, cand = 576, 640, 32
    res = SparseTokenCache(cap + cand, width, device=DEV, candidate_slots=cand)
    off = SparseTokenCache(cap + cand, width, device=DEV, slots=slots, candidate_slots=cand)
    assert off.native
    for step in range(10):
        n = 64
        recs = torch.randn(n, width, device=DEV).bfloat16()
        for c in (res, off):
            c.begin_step(n)
            c.append(recs)
            c.commit()
        hist = res.length
        q = 8 if slots >= 96 else 1
        ids = torch.randint(-1, hist, (q, 12), device=DEV, dtype=torch.int32)
        phys_r = res.ensure(ids)
        phys_o = off.ensure(ids)
        valid = ids >= 0
        assert torch.equal(res.records[phys_r[valid].long()], off.records[phys_o[valid].long()])
        assert bool((phys_o[~valid] == -1).all())
    # transient candidate tail
    crec = torch.randn(cand, width, device=DEV).bfloat16()
    for c in (res, off):
        c.begin_transient(cand)
        c.append(crec)
    ids = torch.cat([torch.randint(0, res.length, (4, 8), device=DEV),
                     res.length + torch.randint(0, cand, (4, 4), device=DEV)], 1).int()
    a, b = res.ensure(ids), off.ensure(ids)
    assert torch.equal(res.records[a.long()], off.records[b.long()])
    for c in (res, off):
        c.discard_transient()
    ops.check_errors(DEV)
    st = off.stats
    assert st.recalled_records > 0 and st.evicted_records > 0 and st.selection_records > 0


@pytest.mark.parametrize("rows,hist,k", [(1, 5000, 2048), (16, 3000, 64), (4, 70000, 2048)])
def test_echo_predictor_matches_reference(rows, hist, k):
    """Device ECHO predictor = the histogram-threshold rule of the Python predictor."""
    from cxldsagr_b200.models.deepseek_v32.attention import _order_bins

    torch.manual_seed(23)
    logits = torch.randn(rows, hist + 7, device=DEV) * 3
    logits[:, 5] = -torch.inf
    offset = torch.tensor([0.25] + [0.0] * 15, device=DEV)
    pred = torch.full((hist,), -1, dtype=torch.int32, device=DEV)
    ops.lib().echo_predict(logits, rows, hist, offset, k, pred)
    key = _order_bins(logits[:, :hist] - offset[0])
    counts = torch.zeros((rows, 257), dtype=torch.int64, device=DEV)
    counts.scatter_add_(1, key.long(), torch.ones_like(key, dtype=torch.int64))
    above = counts.flip(1).cumsum(1).flip(1)
    thr = (above[:, 1:] > k).sum(1)
    want = torch.nonzero((key > thr[:, None]).any(0)).flatten()
    got = torch.nonzero(pred >= 0).flatten()
    assert torch.equal(got, want)
    assert bool((pred[got] == got.int()).all())


@pytest.mark.parametrize("rows,cols", [(1, 700), (3, 5000), (16, 70000)])
def test_echo_hint_matches_reference(rows, cols):
    """Device ECHO offset[0] hint = mean of the finite logits of the last min(4, Q) rows."""
    torch.manual_seed(24)
    logits = torch.randn(rows, cols + 9, device=DEV) * 2 + 1
    logits[:, 3] = -torch.inf
    logits[-1, 7] = torch.nan
    offset = torch.zeros(16, device=DEV)
    ops.lib().echo_hint(logits, rows, cols, offset)
    want = ref.prefetch_hint(logits[:, :cols].cpu())
    assert abs(float(offset[0]) - float(want)) < 1e-4 * max(1.0, abs(float(want)))


@pytest.mark.parametrize("R,N,k,cs,pad,ties", [(3, 100, 64, None, 0, False), (5, 5000, 2048, None, 0, False),
                                               (300, 65536, 2048, None, 0, False), (40, 9000, 2048, 1000, 3, True),
                                               (6, 3000, 2048, 1000, 0, True), (4, 1500, 2048, None, 0, False)])
def test_topk_index_order(R, N, k, cs, pad, ties):
    """order="index": the exact selection of the value-ordered kernel, listed by ascending index."""
    torch.manual_seed(21)
    base = torch.randn(R, N + pad, device=DEV)
    s = (10.0 + 0.01 * base).half().float() if ties else base
    view = s[:, pad:] if pad else s
    v, i = ops.exact_topk(view, k, causal_start=cs, order="index")
    rows = torch.arange(R)[:, None]
    cols = torch.arange(N)[None, :]
    masked = view.cpu() if cs is None else view.cpu().masked_fill(cols > cs + rows, -torch.inf)
    rv, ri = ref.exact_topk(masked, k)
    got = i.cpu()
    assert torch.equal(torch.sort(got, dim=1).values, torch.sort(ri, dim=1).values)
    valid = got >= 0
    big = torch.where(valid, got, torch.iinfo(torch.int32).max)
    assert torch.equal(big, torch.sort(big, dim=1).values)  # ascending, padding last
    assert torch.equal(v.cpu()[valid], masked.gather(1, got.clamp_min(0).long())[valid])


@pytest.mark.parametrize("method", ["hbm", "serial_sparse"])
def test_indexer_topk_rounds_match_whole_chunk(method):
    """Running the indexer + top-k in L2-sized row rounds (an option) gives the whole-chunk result bit for bit."""
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig, v32_config
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model

    cfg = v32_config(1)
    src = StateDictSource(random_state_dict(cfg, layers=[0], seed=0, device=DEV))
    g = torch.Generator().manual_seed(3)
    hist = torch.randint(0, cfg.vocab_size, (3000,), generator=g).to(DEV)
    ext = torch.randint(0, cfg.vocab_size, (16,), generator=g).to(DEV)
    outs = []
    for rows in (0, 296):
        kw = {} if method == "hbm" else {"pool_tokens": 3072 + 16, "host_tokens": 3072 + 16}
        cache = CacheConfig(method=method, capacity=3072 + 16, chunk_size=1024, candidate_tokens=16, **kw)
        m = DeepSeekV32Model(cfg, src, device=DEV, cache=cache)
        m.blocks[0].attention.select_rows = rows
        outs.append((m.prefill(hist).logits, m.extend(ext).logits, m.blocks[0].attention.last_indices.clone()))
        del m
    ops.check_errors(DEV)
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_model_replay_is_deterministic():
    """The same request twice (reset in between) gives bitwise equal logits: no
    order-dependent atomics reach the results (top-k, MoE layout, split-K)."""
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig, v32_config
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model

    cfg = v32_config(1)
    src = StateDictSource(random_state_dict(cfg, layers=[0], seed=1, device=DEV))
    g = torch.Generator().manual_seed(4)
    hist = torch.randint(0, cfg.vocab_size, (2500,), generator=g).to(DEV)
    ext = torch.randint(0, cfg.vocab_size, (1,), generator=g).to(DEV)
    cache = CacheConfig(method="serial_sparse", capacity=2560, chunk_size=1024, candidate_tokens=1,
                        pool_tokens=2560, host_tokens=2560)
    m = DeepSeekV32Model(cfg, src, device=DEV, cache=cache)
    runs = []
    for _ in range(2):
        m.reset()
        runs.append((m.prefill(hist).logits.clone(), m.extend(ext).logits.clone()))
    ops.check_errors(DEV)
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])


# ------------------------------------------------------- bounded failures
def test_peer_flag_wait_times_out_and_reports():
    """A flag barrier whose arrival target no rank reaches gives up after its
    budget: the kernel returns, the error word holds the peer-flag timeout and
    check_errors raises; the context stays usable."""
    from cxldsagr_b200.ops import native

    dev = torch.device(DEV, torch.cuda.current_device())
    flags = torch.zeros(128, dtype=torch.int64, device=dev)  # one rank's flag block
    ops.check_errors(dev)
    # call=5: the barrier bumps its own slot to 1 and waits for 5 (never reached).
    ops.lib().p2p_barrier(dev.index, 0, 1, 5, [flags.data_ptr()], wait_ns=10_000_000)
    torch.cuda.synchronize()
    assert int(native.error_word(dev).item()) == 5  # kErrTimeoutPeerFlag
    with pytest.raises(native.DeviceError, match="peer"):
        ops.check_errors(dev)
    ops.check_errors(dev)  # reset by the raise above
    assert torch.ones(4, device=dev).sum().item() == 4.0


def test_kv_gather_rejects_out_of_range_rows():
    """An out-of-range host row or pool slot is skipped and reported as a bad index."""
    from cxldsagr_b200.ops import native

    dev = torch.device(DEV, torch.cuda.current_device())
    host = torch.randn(64, 576).bfloat16().pin_memory()
    records = torch.zeros(32, 576, dtype=torch.bfloat16, device=dev)
    ops.check_errors(dev)
    ops.gather_host_records(host, records, torch.tensor([3, 64], device=dev), torch.tensor([1, 2], device=dev))
    torch.cuda.synchronize()
    with pytest.raises(native.DeviceError, match="index"):
        ops.check_errors(dev)
    assert torch.equal(records[1].cpu(), host[3])  # the valid row still landed
    assert torch.count_nonzero(records[2]) == 0


def test_embed_vocab_shard_matches_reference():
    """A vocabulary shard embeds its own rows and zeros elsewhere; shards sum to the full table's rows."""
    torch.manual_seed(3)
    V, D = 1000, 256
    table = torch.randn(V, D).bfloat16()
    ids = torch.randint(0, V, (77,))
    total = torch.zeros(77, D, dtype=torch.float32)
    for r0, r1 in ((0, 334), (334, 667), (667, 1000)):
        got = ops.embed(ids.to(DEV), table[r0:r1].to(DEV), row0=r0, vocab_total=V)
        want = ref.embed_shard(ids, table[r0:r1], r0, V)
        assert torch.equal(got.cpu(), want)
        total += got.float().cpu()
    assert torch.equal(total.bfloat16(), table[ids])
    ops.check_errors(DEV)


# ------------------------------------------------------- FP8 KV records
def test_kv_finish_fp8_records_match_reference():
    """kv_finish's FP8 path: packed 656-byte records and dequantized rows equal
    the CPU oracle bit for bit; dequant_kv_rows reproduces the rows from the records."""
    torch.manual_seed(30)
    cfg = v32_config()
    T, L, R = 70, 512, 64
    kv = (torch.randn(T, L + R, device=DEV) * 2).bfloat16()
    kv[5, :128] = 0  # an all-zero latent block (scale 0)
    norm_w = torch.rand(L, device=DEV) + 0.5
    freqs = ref.rotary_frequencies(cfg, device=DEV)
    pos = torch.arange(100, 100 + T, device=DEV, dtype=torch.float32)
    rows = torch.randperm(200, device=DEV)[:T]
    recs = torch.zeros(200, L + R, dtype=torch.bfloat16, device=DEV)
    packed = torch.zeros(T, 656, dtype=torch.uint8, device=DEV)
    ops.kv_finish(kv, L, R, norm_w, cfg.norm_eps, freqs, pos, recs, rows, packed=packed)
    want_recs = torch.zeros(200, L + R, dtype=torch.bfloat16)
    want_packed = torch.zeros(T, 656, dtype=torch.uint8)
    ops.kv_finish(kv.cpu(), L, R, norm_w.cpu(), cfg.norm_eps, freqs.cpu(), pos.cpu(), want_recs, rows.cpu(),
                  packed=want_packed)
    torch.cuda.synchronize()
    assert torch.equal(packed.cpu(), want_packed)
    assert torch.equal(recs.cpu(), want_recs)
    out = torch.zeros(300, L + R, dtype=torch.bfloat16, device=DEV)
    slots = torch.randperm(300, device=DEV)[:T]
    ops.dequant_kv_rows(packed, out, slots)
    torch.cuda.synchronize()
    assert torch.equal(out[slots].cpu(), recs[rows].cpu())
    ops.check_errors(DEV)


@pytest.mark.parametrize("slots", [96, 256])
def test_native_pool_recall_fp8_records(slots):
    """FP8 host records: recalls through the native dispatch (gather into the
    scratch + dequant) give the resident rows bit for bit under eviction."""
    from cxldsagr_b200.cache.sparse_token_cache import SparseTokenCache

    torch.manual_seed(31)
    width, cap = 576, 640
    res = SparseTokenCache(cap, width, device=DEV, kv_format="fp8")
    off = SparseTokenCache(cap, width, device=DEV, slots=slots, kv_format="fp8")
    assert off.native and off.record_bytes == 656
    for step in range(8):
        recs = (torch.randn(64, width, device=DEV) * 3).bfloat16()
        for c in (res, off):
            c.begin_step(64)
            c.append(recs)
            c.commit()
        ids = torch.randint(-1, res.length, (8, 12), device=DEV, dtype=torch.int32)
        a, b = res.ensure(ids), off.ensure(ids)
        valid = ids >= 0
        assert torch.equal(res.records[a[valid].long()], off.records[b[valid].long()])
    ops.check_errors(DEV)
    st = off.stats
    assert st.recalled_records > 0 and st.host_to_device_bytes == (st.recalled_records + st.prefetched_records) * 656


@pytest.mark.parametrize("method", ["serial_sparse", "echo", "dense_prefetch"])
def test_model_fp8_records_offload_matches_resident(method):
    """One V3.2 layer with FP8 KV records: every offload method (finite pool,
    656-byte host records) gives the resident model's logits bit for bit."""
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model

    cfg = v32_config(1)
    src = StateDictSource(random_state_dict(cfg, layers=[0], seed=2, device=DEV))
    g = torch.Generator().manual_seed(5)
    hist = torch.randint(0, cfg.vocab_size, (3000,), generator=g).to(DEV)
    ext = torch.randint(0, cfg.vocab_size, (16,), generator=g).to(DEV)
    out = {}
    for m_name in ("hbm", method):
        # P = NH: every history row recalled after clear_residency (a smaller
        # pool would split the selection into rounds, a different schedule).
        kw = {} if m_name == "hbm" else {"pool_tokens": 3072 + 16, "host_tokens": 3072 + 16}
        cache = CacheConfig(method=m_name, capacity=3072 + 16, chunk_size=1024, candidate_tokens=16, kv_format="fp8",
                            **kw)
        m = DeepSeekV32Model(cfg, src, device=DEV, cache=cache)
        a = m.prefill(hist).logits.clone()
        if m_name != "hbm":
            m.clear_residency()
        out[m_name] = (a, m.extend(ext).logits.clone())
        del m
    ops.check_errors(DEV)
    assert torch.equal(out["hbm"][0], out[method][0]) and torch.equal(out["hbm"][1], out[method][1])


@pytest.mark.parametrize("method,kv_format", [("hbm", "bf16"), ("serial_sparse", "fp8"), ("dense_prefetch", "bf16"),
                                              ("dense_prefetch", "fp8")])
def test_extend_graph_matches_eager(method, kv_format):
    """A captured extend (dense_prefetch included: its staging copies become
    graph nodes) gives the eager extend's logits bit for bit, on two replays."""
    from cxldsagr_b200.checkpoint import StateDictSource, random_state_dict
    from cxldsagr_b200.config import CacheConfig
    from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model

    cfg = v32_config(1)
    src = StateDictSource(random_state_dict(cfg, layers=[0], seed=3, device=DEV))
    g = torch.Generator().manual_seed(6)
    H, A = 3000, 16
    hist = torch.randint(0, cfg.vocab_size, (H,), generator=g).to(DEV)
    ext = torch.randint(0, cfg.vocab_size, (A,), generator=g).to(DEV)
    kw = {} if method == "hbm" else {"pool_tokens": H + A, "host_tokens": H + A}
    cache = CacheConfig(method=method, capacity=H + A, chunk_size=1024, candidate_tokens=A, kv_format=kv_format, **kw)
    m = DeepSeekV32Model(cfg, src, device=DEV, cache=cache)
    m.prefill(hist)
    eager = m.extend(ext).logits.clone()
    m.session.truncate(H)
    graph = m.capture_extend(A)
    for _ in range(2):
        got = graph.replay(ext).clone()
        graph.rollback()
        torch.cuda.synchronize()
        assert torch.equal(got, eager)
    del graph
    ops.check_errors(DEV)


@pytest.mark.parametrize("method,kv_format", [("hbm", "bf16"), ("serial_sparse", "fp8")])
def test_cache_memory_audit_model(method, kv_format, capsys):
    """Per-scope transient memory of a real prefill + extend stays inside the
    workspace allowance of the selection and attention paths."""
    import argparse
    import json

    from cxldsagr_b200.evaluation import cache_memory_audit as audit

    a = argparse.Namespace(history=4096, extend=64, chunk=2048, layers=1, method=method, kv_format=kv_format,
                           device=DEV)
    rc = audit.audit_model(a)
    rep = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    for phase in ("prefill", "extend"):
        checked = rep[phase]["audit"]["checked"]
        assert "sparse_mla" in checked and ("indexer_select" in checked or "indexer" in checked), checked
    assert rc == 0, {p: {k: (v["peak_transient"], v["allowance"]) for k, v in rep[p]["audit"]["checked"].items()}
                     for p in ("prefill", "extend")}
    assert rep["fixed"]["total"]["hbm"] > 0


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("N,K", [(2304, 7168), (7168, 16384), (1000, 1536)])
def test_decode_gemv_fp8(M, N, K):
    """Decode-size FP8 linears run on the weight-streaming GEMV: FP32-oracle
    accuracy, and agreement with the tensor-core tile kernel."""
    torch.manual_seed(41)
    x = torch.randn(M, K, device=DEV).bfloat16()
    w, s = quantize_weight_blocks(torch.randn(N, K, device=DEV) * 0.02)
    q, s_t = ops.quantize_act(x)
    res = torch.randn(M, N, device=DEV).bfloat16()
    got = ops.fp8_gemm(q, s_t, w, s, residual=res)
    ops.lib().set_decode_gemv(False)
    try:
        tiles = ops.fp8_gemm(q, s_t, w, s, residual=res)
    finally:
        ops.lib().set_decode_gemv(True)
    a = ref.dequantize_act(q.cpu(), s_t.t().cpu())
    want = a @ ref.dequantize_weight(w.cpu(), s.cpu()).T + res.float().cpu()
    assert rel_err(got.float().cpu(), want) < 1e-2
    assert rel_err(got.float().cpu(), tiles.float().cpu()) < 1e-2


@pytest.mark.parametrize("fp8", [False, True])
def test_kv_finish_index_k_fused_matches_separate(fp8):
    """The one-launch KV record finish + indexer key gives the bits of the two
    separate kernels (BF16 and FP8 records, decode and prefill row counts)."""
    cfg = v32_config(1)
    L, R = cfg.kv_lora_rank, cfg.qk_rope_head_dim
    freqs = torch.rand(R // 2, device=DEV) * 0.1
    nw = torch.rand(L, device=DEV) + 0.5
    lw, lb = torch.rand(128, device=DEV) + 0.5, torch.randn(128, device=DEV) * 0.1
    for T in (1, 5, 300):
        torch.manual_seed(47 + T)
        a = torch.randn(T, 2304, device=DEV).bfloat16()
        kv, ik = a[:, 1536:1536 + L + R], a[:, 1536 + L + R:1536 + L + R + 128]
        pos = torch.arange(2000, 2000 + T, device=DEV, dtype=torch.float32)
        rows = torch.randperm(512, device=DEV)[:T]
        outs = []
        for fused in (False, True):
            rec = torch.zeros(512, L + R, device=DEV).bfloat16()
            packed = torch.zeros(T, 656, dtype=torch.uint8, device=DEV) if fp8 else None
            kq = torch.zeros(T, 128, device=DEV).to(torch.float8_e4m3fn)
            ks = torch.zeros(T, device=DEV)
            if fused:
                ops.kv_finish_index_k(kv, L, R, nw, 1e-6, freqs, pos, rec, rows, ik, lw, lb, 1e-6, kq, ks,
                                      packed=packed)
            else:
                ops.kv_finish(kv, L, R, nw, 1e-6, freqs, pos, rec, rows, packed=packed)
                ops.index_k(ik, R, lw, lb, 1e-6, freqs, pos, kq, ks)
            outs.append((rec, packed, kq.view(torch.uint8), ks))
        ops.check_errors(torch.device(DEV))
        for x, y in zip(outs[0], outs[1]):
            assert (x is None and y is None) or torch.equal(x, y)


def test_q_rope_index_q_fused_matches_separate():
    """The one-launch MLA query RoPE + indexer query gives the bits of the two
    separate kernels (decode and prefill row counts)."""
    cfg = v32_config(1)
    H, nope, rope, L = cfg.n_heads, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.kv_lora_rank
    IH, ID = cfg.index_n_heads, cfg.index_head_dim
    freqs = torch.rand(rope // 2, device=DEV) * 0.1
    for T in (1, 37, 300):
        torch.manual_seed(46 + T)
        b = torch.randn(T, H * (nope + rope) + IH * ID, device=DEV).bfloat16()
        pos = torch.arange(1000, 1000 + T, device=DEV, dtype=torch.float32)
        w_raw = torch.randn(T, 2 * IH, device=DEV)
        iq = b[:, H * (nope + rope):]
        q1 = torch.zeros(T, H, L + rope, device=DEV).bfloat16()
        q2 = torch.zeros_like(q1)
        ops.mla_q_rope(b, H, nope, rope, freqs, pos, q1, L)
        qa, wa = ops.index_q(iq, IH, ID, rope, freqs, pos, w_raw, 0.01)
        qb, wb = ops.mla_q_rope_index_q(b, H, nope, rope, freqs, pos, q2, L, iq, IH, ID, rope, w_raw, 0.01)
        ops.check_errors(torch.device(DEV))
        assert torch.equal(q1, q2)
        assert torch.equal(qa.view(torch.uint8), qb.view(torch.uint8))
        assert torch.equal(wa, wb)


def test_l2_prefetch_leaves_data():
    """The bulk L2 prefetch runs on ragged sizes and changes nothing it touches."""
    x = torch.randint(0, 255, (3 * (1 << 16) + 48,), dtype=torch.uint8, device=DEV)
    before = x.clone()
    ops.l2_prefetch(x)
    ops.l2_prefetch(x, 1000)
    torch.cuda.synchronize()
    ops.check_errors(torch.device(DEV))
    assert torch.equal(x, before)


def test_pdl_switch_same_bits():
    """Programmatic dependent launch changes launch overlap only: a decode-size
    norm -> GEMV -> norm chain gives the same bits with it on and off."""
    torch.manual_seed(45)
    D, N = 7168, 2304
    x = torch.randn(1, D, device=DEV).bfloat16()
    res = torch.randn(1, D, device=DEV).bfloat16()
    nw = torch.rand(D, device=DEV) + 0.5
    w, s = quantize_weight_blocks(torch.randn(N, D, device=DEV) * 0.02)

    def chain():
        normed, summed, q, s_t = ops.norm_quant(x, res, nw, 1e-6)
        y = ops.fp8_gemm(q, s_t, w, s)
        return normed, summed, q.view(torch.uint8), s_t, y

    on = chain()
    ops.lib().set_pdl(False)
    try:
        off = chain()
    finally:
        ops.lib().set_pdl(True)
    for a, b in zip(on, off):
        assert torch.equal(a, b)


@pytest.mark.parametrize("M", [1, 2, 8])
def test_decode_gemv_bf16(M):
    torch.manual_seed(42)
    x = torch.randn(M, 7168, device=DEV).bfloat16()
    w = (torch.randn(4100, 7168, device=DEV) * 0.02).bfloat16()
    got = ops.linear(x, w)
    want = x.float().cpu() @ w.float().cpu().T
    assert rel_err(got.float().cpu(), want) < 1e-2


def test_decode_gemv_bf16_fp32_out():
    """The LM head's FP32-output BF16 GEMM at one row (the decode head) uses the GEMV."""
    torch.manual_seed(43)
    x = torch.randn(1, 7168, device=DEV).bfloat16()
    w = (torch.randn(3000, 7168, device=DEV) * 0.02).bfloat16()
    out = torch.empty(1, 3000, device=DEV, dtype=torch.float32)
    ops.lib().bf16_gemm(x, 0, 7168, 0, w, 0, 7168, 0, out, 0, 3000, 0, 1, 3000, 7168, 1)
    want = x.float().cpu() @ w.float().cpu().T
    assert rel_err(out.cpu(), want) < 1e-3


def test_ag_gemm_world1_matches_plain_gemm():
    """The AG-GEMM on one rank (its own rows come straight from the local input)
    against the plain FP8 GEMM of the same rows."""
    from cxldsagr_b200.models.deepseek_v32.weights import Linear
    from cxldsagr_b200.parallel.groups import single
    from cxldsagr_b200.parallel.p2p import P2PComm

    torch.manual_seed(44)
    comm = P2PComm(single("cuda"))
    try:
        w, s = quantize_weight_blocks(torch.randn(2304, 7168, device=DEV) * 0.02)
        lin = Linear(w, s)
        for M in (1024, 256):
            x = torch.randn(M, 7168, device=DEV).bfloat16()
            qx = ops.quantize_act(x)
            for _ in range(3):  # both parity halves and the reuse guard
                got = comm.ag_linear(lin, x, qx, M)
            want = lin(quantized=qx)
            ops.check_errors(DEV)
            assert rel_err(got.float().cpu(), want.float().cpu()) < 1e-2
    finally:
        comm.close()


@pytest.mark.parametrize("T", [1, 3])
def test_decode_gemv_batched_absorb_expand(T):
    """Per-head absorb / expand products at decode row counts run on the batched
    GEMV; they match an FP32 oracle and the tile kernels."""
    torch.manual_seed(45)
    H, nope, rope, L, V = 128, 128, 64, 512, 128
    b = torch.randn(T, H * (nope + rope) + 8192, device=DEV).bfloat16()
    wk_b_t = (torch.randn(H, L, nope, device=DEV) * 0.05).bfloat16()
    q_proj = torch.zeros(T, H, L + rope, device=DEV, dtype=torch.bfloat16)
    ops.mla_absorb(b, H, nope, rope, wk_b_t, q_proj)
    qn = b[:, : H * (nope + rope)].reshape(T, H, nope + rope)[..., :nope].float().cpu()
    want = torch.einsum("thn,hln->thl", qn, wk_b_t.float().cpu())
    assert rel_err(q_proj[..., :L].float().cpu(), want) < 1e-2
    attn = torch.randn(T, H, L, device=DEV).bfloat16()
    wv_b = (torch.randn(H, V, L, device=DEV) * 0.05).bfloat16()
    got = ops.mla_expand(attn, wv_b)
    ops.lib().set_decode_gemv(False)
    try:
        tiles = ops.mla_expand(attn, wv_b)
    finally:
        ops.lib().set_decode_gemv(True)
    want = torch.einsum("thl,hvl->thv", attn.float().cpu(), wv_b.float().cpu())
    assert rel_err(got.float().cpu(), want) < 1e-2
    assert rel_err(got.float().cpu(), tiles.float().cpu()) < 1e-2
