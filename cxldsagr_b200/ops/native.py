"""Loader of the in-tree sm_100a extension (``cxldsagr_b200/_C*.so``).

CUDA tensors always go through the native kernels; if the extension is missing
or was built for another architecture the call fails loudly instead of falling
back to PyTorch.  CPU tensors use :mod:`cxldsagr_b200.ops.reference`.
"""

from __future__ import annotations

import functools

import torch


class NativeUnavailable(RuntimeError):
    pass


# Entry points that launch more than one kernel per call.
_MULTI_LAUNCH = {
    "sparse_mla": lambda args: 2 if len(args) > 6 and int(args[6]) > 1 else 1,  # + LSE combine
    "topk": lambda args: 3 if len(args) > 6 and int(args[6]) in (0, 2) else 1,  # zero + select + fallback
}


def _fp8_gemm_launches(mod, args):
    q, w = args[0], args[2]
    ue8m0 = bool(args[6]) if len(args) > 6 else False
    return 2 if mod.fp8_gemm_splits(q.shape[0], w.shape[0], q.shape[1], ue8m0) > 1 else 1  # + split-K reduce
_NO_LAUNCH = {"error_word", "sparse_mla_scratch_bytes", "fp8_gemm_splits", "set_decode_gemv", "set_gemv_k_split", "set_pdl",
              "pdl_enabled"}


class _CountingLib:
    """Proxy of the extension that counts kernel launches issued from Python.

    ``launches`` counts every native kernel launch (a CUDA-graph replay
    re-issues the launches recorded while it was captured).
    """

    def __init__(self, mod):
        self._mod = mod
        self.launches = 0

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if name in _NO_LAUNCH or not callable(fn):
            return fn
        multi = _MULTI_LAUNCH.get(name)
        if name == "fp8_gemm":
            multi = lambda args: _fp8_gemm_launches(self._mod, args)  # noqa: E731

        def call(*args, **kwargs):
            self.launches += multi(args) if multi else 1
            return fn(*args, **kwargs)

        return call


@functools.cache
def lib():
    from . import build_identity

    try:
        from .. import _C  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - depends on the build
        raise NativeUnavailable(
            "the sm_100a extension is not built; run `python setup.py build_ext --inplace`"
        ) from exc
    try:
        build_identity.verify()
    except RuntimeError as exc:
        raise NativeUnavailable(str(exc)) from exc
    return _CountingLib(_C)


def native_info() -> dict:
    """Build record of the loaded extension (sources, flags, compiler, artifact digests), re-verified."""
    from . import build_identity

    lib()
    return build_identity.verify()


def launch_count() -> int:
    return lib().launches


def available() -> bool:
    try:
        lib()
        return True
    except NativeUnavailable:
        return False


def require_sm100(device: torch.device):
    major, minor = torch.cuda.get_device_capability(device)
    if (major, minor) != (10, 0):
        raise NativeUnavailable(f"kernels are built for sm_100a; device {device} is sm_{major}{minor}")


def error_word(device) -> torch.Tensor:
    """Per-device int32 error word written by kernels (0 = no error)."""
    device = torch.device(device)
    return lib().error_word(device.index if device.index is not None else torch.cuda.current_device())


ERROR_NAMES = {
    1: "TMA load wait timed out",
    2: "shared-memory stage release wait timed out",
    3: "TMEM accumulator wait timed out",
    4: "TMEM release wait timed out",
    5: "peer flag wait timed out",
    6: "index out of range",
    7: "bounded wait timed out",
    8: "pool overflow",
}


class DeviceError(RuntimeError):
    pass


def check_errors(device, *, reset: bool = True):
    """Raise if any kernel on ``device`` recorded an error (synchronises the stream)."""
    word = error_word(device)
    code = int(word.item())
    if code:
        if reset:
            word.zero_()
        raise DeviceError(f"device kernel error {code}: {ERROR_NAMES.get(code, 'unknown')}")
