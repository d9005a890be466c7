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


@functools.cache
def lib():
    try:
        from .. import _C  # noqa: PLC0415
    except ImportError as exc:  # pragma: no cover - depends on the build
        raise NativeUnavailable(
            "the sm_100a extension is not built; run `python setup.py build_ext --inplace`"
        ) from exc
    return _C


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
