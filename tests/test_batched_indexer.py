"""Batched resident indexer: one query per independent sequence equals the
per-sequence indexer; lengths mask the tail."""

import pytest
import torch

from cxldsagr_b200.ops import batched, reference


def test_paged_logits_match_single_sequences():
    g = torch.Generator().manual_seed(0)
    B, N = 3, 200
    keys = torch.randn(B, N, 128, generator=g).to(torch.float8_e4m3fn)
    scales = torch.rand(B, N, generator=g) + 0.5
    q = torch.randn(B, 64, 128, generator=g).to(torch.float8_e4m3fn)
    w = torch.randn(B, 64, generator=g)
    prep = batched.prepare_keys(keys, scales, lengths=[200, 150, 7])
    out = batched.paged_logits(prep, q, w)
    for b, n in enumerate((200, 150, 7)):
        want = reference.indexer_logits(q[b:b + 1], keys[b, :n], w[b:b + 1], scales[b, :n], n - 1)[0]
        assert torch.equal(out[b, :n], want)
        assert bool(torch.isinf(out[b, n:]).all())
    m = torch.zeros(2, 5)
    batched.mask_causal_(m, [3, 5])
    assert bool(torch.isinf(m[0, 3:]).all()) and bool(torch.isfinite(m[1]).all())
    with pytest.raises(ValueError):
        batched.prepare_keys(keys, scales, lengths=[0, 1, 2])
