"""The allocation-free C entry point of the split-K sparse MLA decode.

Hosts that embed these kernels but may not allocate device memory (all HBM
reserved up front, allocator owned by another framework, no allocation in a
latency-critical loop) call ``cxld_sparse_mla_split_noalloc`` through its C
symbol; it takes its split-K scratch from a fixed array in the library.  This
test calls that symbol with ctypes, twice in a row, and checks each result
against the FP32 oracle and the regular entry point (which gets the same
scratch from the torch allocator), that the call's device error word reads 0
and that no device memory is allocated by the call.  The file name makes
pytest collect it last.
"""

import ctypes

import pytest
import torch

from cxldsagr_b200 import ops
from cxldsagr_b200.config import v32_config
from cxldsagr_b200.ops import reference as ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _symbol():
    from cxldsagr_b200 import _C

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.cxld_sparse_mla_split_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.cxld_sparse_mla_noalloc_max_rows.restype = ctypes.c_int
    lib.cxld_noalloc_error_string.restype = ctypes.c_char_p
    lib.cxld_noalloc_error_string.argtypes = [ctypes.c_int]
    lib.cxld_sparse_mla_noalloc_error.restype = ctypes.c_int
    lib.cxld_sparse_mla_noalloc_error.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    return lib, fn


def _device_error(lib, stream):
    code = ctypes.c_int(-1)
    rc = lib.cxld_sparse_mla_noalloc_error(ctypes.byref(code), stream)
    assert rc == 0, lib.cxld_noalloc_error_string(rc).decode()
    return code.value


def _rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def _case(seed, T, K, P):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = (torch.randn(T, 128, 576, device=DEV, generator=g) * 0.5).bfloat16()
    kv = (torch.randn(P, 576, device=DEV, generator=g) * 0.5).bfloat16()
    ids = torch.randint(0, P, (T, K), device=DEV, dtype=torch.int32, generator=g)
    ids[:, -5:] = -1
    return q, kv, ids


def test_noalloc_matches_regular_entry_point_twice():
    lib, fn = _symbol()
    scale = v32_config().attention_scale
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row (the second reuses the scratch the first one left).
    for seed, (T, K, P, splits) in enumerate([(2, 2048, 9000, 16), (1, 2048, 70000, 16)]):
        q, kv, ids = _case(seed, T, K, P)
        out = torch.empty(T, 128, 512, device=DEV, dtype=torch.bfloat16)
        lse = torch.empty(T, 128, device=DEV, dtype=torch.float32)
        torch.cuda.synchronize()
        allocated = torch.cuda.memory_allocated()
        free_before = torch.cuda.mem_get_info()[0]
        rc = fn(q.data_ptr(), kv.data_ptr(), ids.data_ptr(), T, K, P, scale, splits, out.data_ptr(),
                lse.data_ptr(), stream)
        assert rc == 0, lib.cxld_noalloc_error_string(rc).decode()
        assert _device_error(lib, stream) == 0
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == allocated
        if seed > 0:  # the first call on a device may load the library's device image
            assert torch.cuda.mem_get_info()[0] == free_before
        want, want_lse = ref.sparse_mla_lse(q.cpu(), kv.cpu(), ids.cpu(), scale)
        assert _rel_err(out.cpu(), want) < 2e-2
        assert torch.allclose(lse.cpu(), want_lse.float(), atol=2e-2, rtol=1e-3)
        got, got_lse = ops.sparse_mla(q, kv, ids, scale, splits=splits, return_lse=True)
        torch.cuda.synchronize()
        assert _rel_err(out, got) < 2e-2
        assert torch.allclose(lse, got_lse, atol=2e-2, rtol=1e-3)
    ops.check_errors(DEV)


def test_noalloc_rejects_oversized_request():
    lib, fn = _symbol()
    max_rows = lib.cxld_sparse_mla_noalloc_max_rows()
    T, splits = max_rows, 2  # splits * T above the fixed scratch capacity
    q = torch.zeros(T, 128, 576, device=DEV, dtype=torch.bfloat16)
    kv = torch.zeros(16, 576, device=DEV, dtype=torch.bfloat16)
    ids = torch.zeros(T, 64, device=DEV, dtype=torch.int32)
    out = torch.empty(T, 128, 512, device=DEV, dtype=torch.bfloat16)
    rc = fn(q.data_ptr(), kv.data_ptr(), ids.data_ptr(), T, 64, 16, 0.1, splits, out.data_ptr(), None,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 2, lib.cxld_noalloc_error_string(rc).decode()
