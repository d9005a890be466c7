"""BASELINE config 1 on the CPU: the tiny DSA model, resident KV vs a finite
HBM pool (256 tokens) with pinned-host backing must give identical logits."""

import pytest
import torch

from cxldsagr_b200.checkpoint import CheckpointReader, StateDictSource, random_state_dict, write_checkpoint
from cxldsagr_b200.config import CacheConfig, tiny_config
from cxldsagr_b200.models.deepseek_v32.model import DeepSeekV32Model


@pytest.fixture(scope="module")
def tiny():
    cfg = tiny_config()
    return cfg, StateDictSource(random_state_dict(cfg, seed=0))


def _model(cfg, src, method, **kw):
    cache = CacheConfig(method=method, capacity=1024 + 64, chunk_size=256, candidate_tokens=16, **kw)
    return DeepSeekV32Model(cfg, src, device="cpu", cache=cache)


def test_resident_vs_pool_offload_identical(tiny):
    cfg, src = tiny
    g = torch.Generator().manual_seed(0)
    hist = torch.randint(0, cfg.vocab_size, (1024,), generator=g)
    cand = torch.randint(0, cfg.vocab_size, (16,), generator=g)
    ref = _model(cfg, src, "hbm")
    off = _model(cfg, src, "serial_sparse", pool_tokens=256, host_tokens=1024 + 64)
    r1 = ref.prefill(hist).logits
    o1 = off.prefill(hist).logits
    assert torch.equal(r1, o1)
    r2 = ref.extend(cand).logits
    o2 = off.extend(cand).logits
    assert torch.equal(r2, o2)
    stats = [c.stats for c in off.caches]
    assert sum(s.recalled_records for s in stats) > 0
    assert sum(s.evicted_records for s in stats) > 0


def test_echo_and_transient_candidates(tiny):
    cfg, src = tiny
    g = torch.Generator().manual_seed(1)
    hist = torch.randint(0, cfg.vocab_size, (512,), generator=g)
    cand = torch.randint(0, cfg.vocab_size, (16,), generator=g)
    ref = _model(cfg, src, "hbm")
    echo = _model(cfg, src, "echo", pool_tokens=256, host_tokens=1024 + 64)
    ref.prefill(hist)
    echo.prefill(hist)
    a = ref.candidate(cand).logits
    b = echo.candidate(cand).logits
    assert torch.equal(a, b)
    assert echo.length == 512 and all(c.length == 512 for c in echo.caches)
    # a second candidate batch against the same history gives the same answer
    assert torch.equal(echo.candidate(cand).logits, b)


def test_checkpoint_roundtrip(tmp_path, tiny):
    cfg, src = tiny
    write_checkpoint(tmp_path, cfg, src.tensors)
    reader = CheckpointReader(tmp_path)
    assert reader.config.dim == cfg.dim
    name = "model.layers.0.self_attn.q_a_proj.weight"
    assert torch.equal(reader.get_tensor(name), src.get_tensor(name))
    m1 = DeepSeekV32Model(cfg, reader, device="cpu", cache=CacheConfig(capacity=128))
    m2 = DeepSeekV32Model(cfg, src, device="cpu", cache=CacheConfig(capacity=128))
    ids = torch.arange(40) % cfg.vocab_size
    assert torch.equal(m1.prefill(ids).logits, m2.prefill(ids).logits)


@pytest.mark.parametrize("method", ["dense_prefetch", "echo"])
def test_offload_methods_match_resident(tiny, method):
    """Whole-history staging (dense_prefetch) and predicted prefetch + exact recall (echo)
    give the resident results bitwise: prefill, a transient candidate batch, a committed extend."""
    cfg, src = tiny
    g = torch.Generator().manual_seed(3)
    hist = torch.randint(0, cfg.vocab_size, (1024,), generator=g)
    cand = torch.randint(0, cfg.vocab_size, (16,), generator=g)
    ref = _model(cfg, src, "hbm")
    off = _model(cfg, src, method, pool_tokens=512 if method == "dense_prefetch" else 256, host_tokens=1024 + 64)
    assert torch.equal(ref.prefill(hist).logits, off.prefill(hist).logits)
    assert torch.equal(ref.candidate(cand).logits, off.candidate(cand).logits)
    assert torch.equal(ref.extend(cand).logits, off.extend(cand).logits)


@pytest.mark.parametrize("method", ["hbm", "serial_sparse"])
def test_snapshot_restore_prefix(tiny, method):
    """Rewinding to a snapshot and replaying the same extend gives the same logits."""
    cfg, src = tiny
    g = torch.Generator().manual_seed(7)
    hist = torch.randint(0, cfg.vocab_size, (512,), generator=g)
    a = torch.randint(0, cfg.vocab_size, (16,), generator=g)
    b = torch.randint(0, cfg.vocab_size, (16,), generator=g)
    kw = {} if method == "hbm" else {"pool_tokens": 256, "host_tokens": 1024 + 64}
    m = _model(cfg, src, method, **kw)
    m.prefill(hist)
    snap = m.snapshot_prefix()
    first = m.extend(a).logits
    m.extend(b)
    m.restore_prefix(snap)
    assert m.length == 512
    assert torch.equal(m.extend(a).logits, first)
    other = _model(cfg, src, method, **kw)
    with pytest.raises(ValueError):
        other.restore_prefix(snap)


def test_set_cache_method(tiny):
    """Switching methods gives a fresh empty cache with the new method's results."""
    cfg, src = tiny
    g = torch.Generator().manual_seed(8)
    hist = torch.randint(0, cfg.vocab_size, (512,), generator=g)
    ref = _model(cfg, src, "hbm")
    want = ref.prefill(hist).logits
    m = _model(cfg, src, "hbm")
    m.prefill(hist[:100])
    m.set_cache_method("echo", pool_tokens=256, host_tokens=1024 + 64)
    assert m.length == 0 and m.pool is not None
    assert torch.equal(m.prefill(hist).logits, want)
    m.set_cache_method("hbm")
    assert m.pool is None and torch.equal(m.prefill(hist).logits, want)
    with pytest.raises(ValueError):
        m.set_cache_method("bogus")


def test_mla_split_policy():
    """Few queries split the selection (>= 256 keys per split, <= 32 splits); 74+ run unsplit."""
    from cxldsagr_b200 import ops

    assert ops.mla_splits(1) == 8 and ops.mla_splits(16) == 4 and ops.mla_splits(37) == 2
    assert ops.mla_splits(74) == 1 and ops.mla_splits(2048) == 1
    assert ops.mla_splits(1, K=512) == 2 and ops.mla_splits(1, K=1024) == 4
    assert all(2048 // ops.mla_splits(T) >= 256 for T in range(1, 200))


@pytest.mark.parametrize("method", ["serial_sparse", "echo", "dense_prefetch"])
def test_fp8_records_resident_vs_offload_identical(tiny, method):
    """FP8 KV records: the resident rows hold the dequantized values, the host
    arena the packed records; recalls (or whole-history staging) reproduce the
    resident rows bitwise, so logits match exactly."""
    cfg, src = tiny
    g = torch.Generator().manual_seed(2)
    hist = torch.randint(0, cfg.vocab_size, (1024,), generator=g)
    cand = torch.randint(0, cfg.vocab_size, (16,), generator=g)
    ref = _model(cfg, src, "hbm", kv_format="fp8")
    pool = 1024 + 64 if method == "dense_prefetch" else 256
    off = _model(cfg, src, method, pool_tokens=pool, host_tokens=1024 + 64, kv_format="fp8")
    assert torch.equal(ref.prefill(hist).logits, off.prefill(hist).logits)
    assert torch.equal(ref.extend(cand).logits, off.extend(cand).logits)
    if method != "dense_prefetch":
        assert sum(c.stats.recalled_records for c in off.caches) > 0
        host = off.pool.layers[0].host
        assert host.dtype == torch.uint8 and host.shape[1] == off.caches[0].record_bytes
    # FP8 records change the values (quantization), so BF16 and FP8 models differ.
    bf16 = _model(cfg, src, "hbm")
    ref.reset()
    assert not torch.equal(bf16.prefill(hist).logits, ref.prefill(hist).logits)


def test_fp8_record_pack_roundtrip():
    from cxldsagr_b200.ops import reference as R

    torch.manual_seed(0)
    for L, Rd in ((512, 64), (64, 16)):
        rows = (torch.randn(33, L + Rd) * 3).bfloat16()
        rows[3, :L] = 0  # an all-zero latent block keeps scale 0
        q, s, deq = R.fp8_kv_quantize(rows[:, :L])
        packed = R.fp8_kv_pack(q, s, rows[:, L:])
        assert packed.shape[1] == R.fp8_record_bytes(L, Rd)
        back = R.fp8_kv_unpack(packed, L)
        assert torch.equal(back[:, :L], deq) and torch.equal(back[:, L:], rows[:, L:])
        assert torch.count_nonzero(back[3, :L]) == 0
        # within E4M3's relative precision of each block's scale
        err = (back[:, :L].float() - rows[:, :L].float()).abs().reshape(33, -1, min(L, 128)).amax(-1)
        amax = rows[:, :L].float().abs().reshape(33, -1, min(L, 128)).amax(-1)
        assert bool((err <= amax * 0.07 + 1e-6).all())
    assert R.fp8_record_bytes(512, 64) == R.FP8_RECORD_BYTES == 656
