"""Check -> bench -> profile receipts.

Reference: ``evaluation/validation.py`` and ``motivation_validation.py:121-231``.
A benchmark is only published against a *check* run of the same identity:
the check writes a receipt (source tree hash, backend, native artifacts, the
run's configuration and its numerical evidence digest); the bench refuses to
run unless a receipt for an identical identity exists, and the profile run
records which bench it explains.
"""

from __future__ import annotations

import json
from pathlib import Path

from .provenance import built_native_artifacts, identity_digest, source_snapshot


def run_identity(config: dict) -> dict:
    """The part of a run that must match between check, bench and profile: the
    configuration, the source tree and the built native artifacts on disk (a
    check and a bench of the same build agree whatever each has loaded so far)."""
    snap = source_snapshot()
    return {"config": config, "source_tree": snap["tree_sha256"], "native": built_native_artifacts()}


def write_receipt(path: Path, kind: str, config: dict, evidence: dict | None = None) -> dict:
    if kind not in ("check", "bench", "profile"):
        raise ValueError("receipt kind must be check, bench or profile")
    ident = run_identity(config)
    receipt = {"kind": kind, "identity": ident, "identity_sha256": identity_digest(ident), "evidence": evidence or {}}
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    if path.exists():
        raise FileExistsError(f"{path} exists; receipts are never replaced")
    path.write_text(json.dumps(receipt, indent=2, sort_keys=True))
    return receipt


def require_receipt(path: Path, kind: str, config: dict) -> dict:
    """Load the receipt of a prior ``kind`` run and insist it has this run's identity."""
    path = Path(path)
    if not path.exists():
        raise FileNotFoundError(f"no {kind} receipt at {path}: run the {kind} step first")
    receipt = json.loads(path.read_text())
    if receipt.get("kind") != kind:
        raise ValueError(f"{path} is a {receipt.get('kind')} receipt, expected {kind}")
    want = identity_digest(run_identity(config))
    if receipt.get("identity_sha256") != want:
        raise ValueError(f"{kind} receipt identity differs from this run (source, native build or configuration)")
    return receipt


def without_performance(metrics: dict) -> dict:
    """Drop timing fields so two runs' functional outputs can be compared."""
    drop = ("_ms", "_s", "latency", "timestamp", "clocks")
    return {k: v for k, v in metrics.items() if not any(d in k for d in drop)}
