"""Host CPU environment of a measurement: affinity, thread pools and NUMA
memory policy, read without changing any of them.

Reference: ``evaluation/cpu_environment.py:11-122``.  A benchmark records the
environment when it starts (:func:`cpu_environment`) and checks it again when
it ends (:func:`finish_cpu_environment`); a changed affinity, thread count or
memory policy rejects the run, since host-side stages (pinned copies, Python
launch loops, token validation) depend on them.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import os
from pathlib import Path

_POLICY_NAMES = {0: "default", 1: "preferred", 2: "bind", 3: "interleave", 4: "local", 5: "preferred_many",
                 6: "weighted_interleave"}
_ENV_KEYS = ("OMP_NUM_THREADS", "MKL_NUM_THREADS", "OPENBLAS_NUM_THREADS", "OMP_PROC_BIND", "OMP_PLACES",
             "KMP_AFFINITY", "GOMP_CPU_AFFINITY", "PYTORCH_CUDA_ALLOC_CONF", "PYTORCH_ALLOC_CONF",
             "CUDA_VISIBLE_DEVICES")


def numa_policy() -> dict:
    """The calling thread's default memory policy through libnuma's ``get_mempolicy`` (if present)."""
    name = ctypes.util.find_library("numa")
    if name is None:
        return {"available": False, "reason": "libnuma not found"}
    try:
        lib = ctypes.CDLL(name, use_errno=True)
        fn = lib.get_mempolicy
        fn.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_ulong), ctypes.c_ulong,
                       ctypes.c_void_p, ctypes.c_ulong]
        fn.restype = ctypes.c_int
        nodes = 1024
        bits = ctypes.sizeof(ctypes.c_ulong) * 8
        mask = (ctypes.c_ulong * (nodes // bits))()
        mode = ctypes.c_int()
        if fn(ctypes.byref(mode), mask, nodes, None, 0) != 0:
            err = ctypes.get_errno()
            return {"available": False, "errno": err, "reason": os.strerror(err)}
        return {"available": True, "mode_raw": mode.value, "mode": _POLICY_NAMES.get(mode.value & 0x7FFF, "unknown"),
                "nodes": [n for n in range(nodes) if mask[n // bits] >> (n % bits) & 1]}
    except (AttributeError, OSError) as exc:
        return {"available": False, "reason": str(exc)}


def cpu_environment(torch=None) -> dict:
    if torch is None:
        import torch
    allowed = {}
    status = Path("/proc/self/status")
    if status.exists():
        for line in status.read_text().splitlines():
            key, _, value = line.partition(":")
            if key in ("Cpus_allowed_list", "Mems_allowed_list"):
                allowed[key] = value.strip()
    return {"schema": "cpu-environment-v1", "affinity": sorted(os.sched_getaffinity(0)), "allowed": allowed,
            "torch_num_threads": torch.get_num_threads(),
            "torch_num_interop_threads": torch.get_num_interop_threads(),
            "numa_policy": numa_policy(), "environment": {k: os.environ.get(k) for k in _ENV_KEYS}}


def require_matching(actual: dict | None, reference: dict | None) -> dict:
    if actual is None and reference is None:
        return {"status": "not_recorded"}
    if actual is None or reference is None or actual != reference:
        raise ValueError("CPU affinity, thread configuration or NUMA policy differs or is unrecorded")
    return {"status": "recorded_and_equal"}


def finish_cpu_environment(metadata: dict, torch=None) -> dict:
    """Record the end-of-run environment in ``metadata`` and reject a change since ``metadata["cpu_environment"]``."""
    final = cpu_environment(torch)
    metadata["cpu_environment_final"] = final
    try:
        audit = require_matching(final, metadata.get("cpu_environment"))
    except ValueError as exc:
        metadata["cpu_environment_audit"] = {"status": "rejected", "reason": str(exc)}
        raise
    metadata["cpu_environment_audit"] = audit
    return audit


def validate_cpu_environment_record(metadata: dict) -> dict:
    """Re-check a saved record: the stored audit must follow from its start and end entries."""
    start, end = metadata.get("cpu_environment"), metadata.get("cpu_environment_final")
    if start is None and end is None:
        if "cpu_environment_audit" in metadata:
            raise ValueError("a record without environments cannot claim an audit")
        return {"status": "not_recorded"}
    audit = require_matching(end, start)
    if metadata.get("cpu_environment_audit") != audit:
        raise ValueError("saved CPU environment audit differs from the start/end evidence")
    return audit
