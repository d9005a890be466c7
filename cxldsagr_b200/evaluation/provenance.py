"""Source, backend and numerical provenance of a benchmark or validation run.

Reference: ``evaluation/provenance.py:31-225`` and ``native_provenance.py:10-62``.
A run records (a) a snapshot of the source identity (SHA-256 of every source
file of the package, the native sources and the benchmark driver, plus the git
commit when available), (b) the backend (torch, CUDA, NCCL, driver, GPU), (c)
which native libraries the process actually loaded (read from the process's
memory map: path + SHA-256), and (d) numerical evidence (digests and small
tensors) that a later run can be compared against.  Provenance uses source
hashes and tool-reported versions only; it never reads compiled artifacts
beyond hashing their bytes.
"""

from __future__ import annotations

import hashlib
import json
import os
import platform
import subprocess
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
SOURCE_GLOBS = ("cxldsagr_b200/**/*.py", "csrc/**/*.cu", "csrc/**/*.cuh", "csrc/**/*.h", "csrc/**/*.cpp",
                "bench.py", "setup.py", "__graft_entry__.py")


def digest(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def identity_digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":"), default=str).encode()).hexdigest()


def _git(*args) -> str | None:
    try:
        out = subprocess.run(["git", *args], cwd=ROOT, capture_output=True, text=True, timeout=10, check=False)
    except OSError:
        return None
    return out.stdout.strip() if out.returncode == 0 else None


def source_snapshot(root: Path = ROOT) -> dict:
    files = {}
    for pattern in SOURCE_GLOBS:
        for p in sorted(root.glob(pattern)):
            if p.is_file() and "_work" not in p.parts and "build" not in p.parts:
                files[str(p.relative_to(root))] = digest(p)
    return {
        "files": files,
        "tree_sha256": identity_digest(files),
        "git_commit": _git("rev-parse", "HEAD"),
        "git_dirty": bool(_git("status", "--porcelain")),
    }


def verify_source_snapshot(snapshot: dict, root: Path = ROOT) -> list[str]:
    """Paths whose current content differs from ``snapshot`` (empty list = identical)."""
    now = source_snapshot(root)["files"]
    changed = [p for p, d in snapshot["files"].items() if now.get(p) != d]
    return changed + [p for p in now if p not in snapshot["files"]]


def backend_provenance() -> dict:
    info = {
        "python": platform.python_version(),
        "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda,
        "platform": platform.platform(),
    }
    try:
        info["nccl"] = ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None
    except (AttributeError, RuntimeError):
        info["nccl"] = None
    if torch.cuda.is_available():
        i = torch.cuda.current_device()
        p = torch.cuda.get_device_properties(i)
        info.update(gpu=p.name, capability=f"{p.major}.{p.minor}", sms=p.multi_processor_count,
                    memory_gb=round(p.total_memory / 2**30, 1))
    return info


def loaded_native_artifacts(maps_path: str = "/proc/self/maps", roots=(ROOT,)) -> dict:
    """Shared objects of this repository mapped into the process: {path: sha256}."""
    paths = set()
    try:
        with open(maps_path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 6 and parts[-1].endswith(".so"):
                    paths.add(parts[-1])
    except OSError:
        return {}
    out = {}
    for p in sorted(paths):
        rp = Path(p)
        if any(str(rp).startswith(str(r)) for r in roots) and rp.exists():
            out[str(rp.relative_to(ROOT)) if str(rp).startswith(str(ROOT)) else str(rp)] = digest(rp)
    return out


def built_native_artifacts(root: Path = ROOT) -> dict:
    """The repository's built shared objects on disk: {path: sha256} (what a run
    will load, independent of which of them this process has loaded yet)."""
    out = {}
    for p in sorted((root / "cxldsagr_b200").rglob("*.so")):
        out[str(p.relative_to(root))] = digest(p)
    return out


def verify_native_artifacts(expected: dict, *, allow_additions: bool = False) -> None:
    got = loaded_native_artifacts()
    for path, d in expected.items():
        if got.get(path) != d:
            raise RuntimeError(f"native artifact {path} differs from the recorded build")
    if not allow_additions:
        extra = sorted(set(got) - set(expected))
        if extra:
            raise RuntimeError(f"unexpected native artifacts loaded: {extra}")


def save_numerical_evidence(output: Path, *, name: str, tensors: dict) -> dict:
    """Store small tensors (CPU copies) and their digests for later comparison."""
    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    record = {}
    for key, t in tensors.items():
        cpu = t.detach().float().cpu().contiguous()
        torch.save(cpu, output / f"{name}.{key}.pt")
        record[key] = {"shape": list(cpu.shape), "sha256": hashlib.sha256(cpu.numpy().tobytes()).hexdigest()}
    (output / f"{name}.json").write_text(json.dumps(record, indent=2))
    return record


def numerical_comparison(actual: torch.Tensor, expected: torch.Tensor, *, atol: float, rtol: float) -> dict:
    a, e = actual.detach().float().cpu(), expected.detach().float().cpu()
    if a.shape != e.shape:
        return {"ok": False, "reason": f"shape {tuple(a.shape)} != {tuple(e.shape)}"}
    diff = (a - e).abs()
    bound = atol + rtol * e.abs()
    return {"ok": bool((diff <= bound).all()), "max_abs": float(diff.max()) if diff.numel() else 0.0,
            "bitwise": bool(torch.equal(a, e))}


def run_record(**extra) -> dict:
    """Everything a published number needs next to it."""
    from ..ops import native as _native
    from .cpu_environment import cpu_environment

    try:
        build = _native.native_info()
        build = {k: v for k, v in build.items() if k != "sources"} | {"sources_sha256": build["sources"]["sha256"]}
    except _native.NativeUnavailable as exc:
        build = {"unavailable": str(exc)}
    return {"source": source_snapshot(), "backend": backend_provenance(), "native": loaded_native_artifacts(),
            "native_build": build, "cpu_environment": cpu_environment(),
            "environment": {k: v for k, v in os.environ.items() if k.startswith(("NCCL_", "CUDA_", "PYTORCH_"))},
            **extra}
