"""Source-bound identity of the in-tree native build.

Reference: ``operators/deepseek_v32/indexer/_native_cache.py:104-198`` binds
each native artifact to the exact sources, flags and toolchain it was built
from and refuses a mismatching one.  Here the extension is built in-tree by
``setup.py``, which writes ``cxldsagr_b200/_C.build.json`` next to the shared
object: the SHA-256 of every file under ``csrc/``, the compiler flags, the
``nvcc`` version line and the artifact's own SHA-256.  The loader
(:func:`cxldsagr_b200.ops.native.lib`) recomputes both digests and fails
loudly on a stale or replaced extension instead of running kernels that no
longer match their sources.
"""

from __future__ import annotations

import hashlib
import json
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
PACKAGE = ROOT / "cxldsagr_b200"
RECORD = PACKAGE / "_C.build.json"
SOURCE_SUFFIXES = (".cu", ".cuh", ".h", ".cpp")


def _sha256(path: Path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def sources_digest(root: Path = ROOT) -> dict:
    files = sorted(p for p in (root / "csrc").rglob("*") if p.is_file() and p.suffix in SOURCE_SUFFIXES)
    per_file = {str(p.relative_to(root)): _sha256(p) for p in files}
    total = hashlib.sha256(json.dumps(per_file, sort_keys=True).encode()).hexdigest()
    return {"files": per_file, "sha256": total}


def nvcc_version(nvcc: str = "nvcc") -> str:
    try:
        out = subprocess.check_output([nvcc, "--version"], text=True)
    except (OSError, subprocess.CalledProcessError):
        return "unavailable"
    return out.strip().splitlines()[-1]


def artifact_path() -> Path | None:
    found = sorted(PACKAGE.glob("_C*.so"))
    return found[0] if found else None


def write_record(flags: list[str], nvcc: str = "nvcc") -> dict:
    so = artifact_path()
    if so is None:
        raise FileNotFoundError("no built extension to record")
    record = {"schema": 1, "sources": sources_digest(), "nvcc_flags": list(flags), "nvcc": nvcc_version(nvcc),
              "artifact": so.name, "artifact_sha256": _sha256(so)}
    RECORD.write_text(json.dumps(record, indent=1, sort_keys=True) + "\n")
    return record


def verify() -> dict:
    """The build record, after checking it against the sources and the shared object on disk.

    Raises ``RuntimeError`` naming what differs.
    """
    if not RECORD.exists():
        raise RuntimeError("the extension has no build record; rebuild with `python setup.py build_ext --inplace`")
    record = json.loads(RECORD.read_text())
    so = artifact_path()
    if so is None or so.name != record.get("artifact"):
        raise RuntimeError("the built extension is missing or differs from its build record")
    if _sha256(so) != record["artifact_sha256"]:
        raise RuntimeError("the extension on disk is not the one its build record describes; rebuild")
    now = sources_digest()
    if now["sha256"] != record["sources"]["sha256"]:
        changed = sorted(k for k in set(now["files"]) | set(record["sources"]["files"])
                         if now["files"].get(k) != record["sources"]["files"].get(k))
        raise RuntimeError(f"the extension is stale (sources changed since the build: {', '.join(changed[:8])}); "
                           "rebuild with `python setup.py build_ext --inplace`")
    return record
