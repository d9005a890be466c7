"""Request token-id validation: a Python scan and a native CPython scan.

Reference: ``serving/token_validation.py:29-199``.  Both predicates answer
"is this an exact, nonempty list of non-negative builtin ints".  The native
one is the in-tree extension ``cxldsagr_b200.serving._token_validation``
(built with the package by ``setup.py build_ext --inplace``); its identity
(path + SHA-256 of the loaded binary and of its source) is recorded so a
benchmark receipt can name exactly what validated its inputs.
"""

from __future__ import annotations

import copy
import hashlib
import threading
from pathlib import Path

_LOCK = threading.Lock()
_predicate = None
_runtime = None
_SOURCE = Path(__file__).resolve().parents[2] / "csrc" / "host" / "token_validation.cpp"


def reference(snapshot: list) -> bool:
    """Python predicate (also the fallback on systems without the extension)."""
    if type(snapshot) is not list:
        raise TypeError("expected an exact list snapshot")
    return bool(snapshot) and all(type(v) is int for v in snapshot) and min(snapshot) >= 0


def _sha256(path: Path) -> str | None:
    try:
        with path.open("rb") as f:
            return hashlib.file_digest(f, "sha256").hexdigest()
    except OSError:
        return None


def prepare():
    """Load the native predicate once; errors propagate before the runner takes ownership."""
    global _predicate, _runtime
    with _LOCK:
        if _predicate is None:
            from . import _token_validation as native

            binary = Path(native.__file__).resolve()
            _predicate = native.nonnegative_builtin_ints
            _runtime = {
                "backend": "cpython_native",
                "fallback_reason": None,
                "loaded_binary_path": str(binary),
                "loaded_binary_sha256": _sha256(binary),
                "source_sha256": _sha256(_SOURCE),
            }
        return _predicate


def runtime_info() -> dict | None:
    """The identity recorded by :func:`prepare` (no loading, no I/O)."""
    return copy.deepcopy(_runtime)
