"""Deterministic multi-user GR workloads shared by every cache scheme.

Reference semantics (``GR/workload.py:41-377``): ``history_tokens`` is the
complete stable prefix (instruction + user history) and ``candidate_tokens``
the complete changing suffix — both are exact KV boundaries.  ``weighted``
sampling draws users by normalised heat (with replacement); ``sequential``
cycles through synthetic IDs.  The manifest signs every request's token ids
(SHA-256 of the canonical JSON list) so that runs of different schemes can be
shown to have served byte-identical requests.

CLI: ``python -m cxldsagr_b200.gr.workload --num-users 16 --requests 32
--history-tokens 32768 --candidate-tokens 1280 --output-dir out/``
"""

from __future__ import annotations

import argparse
import hashlib
import json
from collections import Counter
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any

from .heat import HeatPopulation
from .input_generator import INSTRUCTION, MODEL_FORMATS, InputGenerator, TextConfig, create_input_generator
from .scheduling import ScheduleConfig
from .tokenizer import load_tokenizer


def _check(name, value, minimum=1):
    if isinstance(value, bool) or not isinstance(value, int) or value < minimum:
        raise ValueError(f"{name} must be an integer >= {minimum}")


def _canonical(value: Any) -> str:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=False)


def token_sha256(ids) -> str:
    """Signature of exact token ids, independent of tensor dtype, device or hash seed."""
    return hashlib.sha256(_canonical(list(ids)).encode()).hexdigest()


@dataclass(frozen=True)
class WorkloadConfig:
    model: str
    num_users: int
    requests: int
    history_tokens: int = 8192
    candidate_tokens: int = 1024
    seed: int = 42
    heat_dataset: str | None = "beauty"
    heat_field: str | None = None
    heat_path: str | None = None
    max_revisits: int | None = None
    context_limit: int | None = None
    sampling: str = "weighted"

    def __post_init__(self):
        if self.model not in MODEL_FORMATS:
            raise ValueError("model must be deepseek_v32")
        for name in ("num_users", "requests", "history_tokens", "candidate_tokens"):
            _check(name, getattr(self, name))
        _check("seed", self.seed, 0)
        if self.sampling not in ("weighted", "sequential"):
            raise ValueError("sampling must be weighted or sequential")
        if self.max_revisits is not None:
            _check("max_revisits", self.max_revisits, 0)
        if self.sampling == "sequential":
            if self.max_revisits is not None:
                raise ValueError("sequential sampling does not support max_revisits")
            object.__setattr__(self, "heat_dataset", None)
            object.__setattr__(self, "heat_field", None)
        else:
            if not isinstance(self.heat_dataset, str) or not self.heat_dataset:
                raise ValueError("heat_dataset must be a nonempty curve dataset name")
            if self.heat_field is None:
                object.__setattr__(self, "heat_field", "pv_share" if self.heat_dataset.startswith("industrial_")
                                   else "interaction_count")
        limit = MODEL_FORMATS[self.model].MAX_INPUT_TOKENS
        if self.context_limit is not None:
            _check("context_limit", self.context_limit)
            if self.context_limit > limit:
                raise ValueError(f"context_limit exceeds the {limit}-token backend limit")
            limit = self.context_limit
        if self.history_tokens + self.candidate_tokens > limit:
            raise ValueError("history + candidate tokens exceeds model context")


@dataclass(frozen=True)
class Workload:
    requests: tuple
    manifest: dict

    def write(self, output_dir: str | Path) -> None:
        """Write ``requests.jsonl`` + ``workload.json``; never replaces an existing workload."""
        out = Path(output_dir)
        out.mkdir(parents=True, exist_ok=True)
        req, man = out / "requests.jsonl", out / "workload.json"
        if req.exists() or man.exists():
            raise FileExistsError("requests.jsonl or workload.json already exists")
        with req.open("x", encoding="utf-8") as f:
            for row in self.requests:
                f.write(_canonical(row) + "\n")
        man.write_text(json.dumps(self.manifest, indent=2, ensure_ascii=False) + "\n")


_TRACE_KEYS = ("request_id", "user_id", "visit_index", "previous_request_id", "timestamp")
_IDENTITY_KEYS = ("request_id", "user_id", "visit_index", "visit_number", "is_revisit", "timestamp",
                  "stable_prefix_tokens", "candidate_suffix_tokens", "prefix_sha256", "candidate_sha256",
                  "input_sha256")


def build_workload(config: WorkloadConfig, *, tokenizer=None) -> Workload:
    tokenizer_path = None
    if tokenizer is None or isinstance(tokenizer, (str, Path)):
        tokenizer_path = None if tokenizer is None else Path(tokenizer)
        tokenizer = load_tokenizer(tokenizer_path)
    tokenizer.no_padding()
    tokenizer.no_truncation()
    fmt = MODEL_FORMATS[config.model]
    instruction = len(tokenizer.encode(fmt.prefix(INSTRUCTION), add_special_tokens=False).ids)
    if config.history_tokens <= instruction:
        raise ValueError("history_tokens must leave room for history after the fixed instruction")
    opts = dict(
        model=config.model, tokenizer=tokenizer, context_limit=config.context_limit,
        text_config=TextConfig(
            user_lengths=(config.history_tokens - instruction,), user_probabilities=(1.0,),
            item_lengths=(config.candidate_tokens + instruction,), item_probabilities=(1.0,),
            max_input_tokens=config.history_tokens + config.candidate_tokens,
            history_cache_users=min(config.num_users, config.requests)),
        schedule_config=ScheduleConfig(seed=config.seed, sampling=config.sampling, arrival="constant", qps=1,
                                       max_revisits=config.max_revisits),
    )
    if config.sampling == "sequential":
        gen = InputGenerator(HeatPopulation.uniform(config.num_users), **opts)
    else:
        gen = create_input_generator(**opts, heat_source="curve", heat_path=config.heat_path,
                                     curve_dataset=config.heat_dataset, curve_field=config.heat_field,
                                     num_users=config.num_users)
    prefixes, last_candidate, counts = {}, {}, Counter()
    requests, identities, trace = [], [], []
    for request_id, row in enumerate(gen.iter_generate(config.requests)):
        user, ids = row["user_id"], row["input_ids"]
        prefix, candidate = tuple(ids[:config.history_tokens]), tuple(ids[config.history_tokens:])
        if row["stable_prefix_tokens"] != config.history_tokens or row["candidate_suffix_tokens"] != config.candidate_tokens:
            raise ValueError("GR generator did not preserve the requested KV boundaries")
        if prefixes.setdefault(user, prefix) != prefix:
            raise ValueError(f"user {user}: stable prefix changed across visits")
        if last_candidate.get(user) == candidate:
            raise ValueError(f"user {user}: candidate did not change across visits")
        if row["visit_index"] != counts[user]:
            raise ValueError(f"user {user}: noncontiguous visit indices")
        row.update(request_id=request_id, visit_number=counts[user] + 1, is_revisit=counts[user] > 0,
                   prefix_sha256=token_sha256(prefix), candidate_sha256=token_sha256(candidate),
                   input_sha256=token_sha256(ids))
        counts[user] += 1
        last_candidate[user] = candidate
        requests.append(row)
        trace.append({k: row[k] for k in _TRACE_KEYS})
        identities.append({k: row[k] for k in _IDENTITY_KEYS})
    identity = {
        "config": asdict(config),
        "heat_sha256": gen.population.metadata.get("sha256"),
        "tokenizer_sha256": hashlib.sha256(tokenizer.to_str().encode()).hexdigest(),
        "requests": identities,
    }
    weight_sum = gen.population.metadata["selected_weight_sum"]
    manifest = {
        "schema_version": 1, **identity,
        "workload_sha256": hashlib.sha256(_canonical(identity).encode()).hexdigest(),
        "access_trace_sha256": hashlib.sha256(_canonical(trace).encode()).hexdigest(),
        "tokenizer_path": str(tokenizer_path.resolve()) if tokenizer_path else "builtin:synthetic-word-level",
        "heat": gen.population.metadata,
        "schedule": asdict(gen.schedule_config),
        "context": {"format_default_tokens": fmt.MAX_INPUT_TOKENS, "effective_limit_tokens": gen.context_limit,
                    "override_explicit": config.context_limit is not None},
        "text_config": json.loads(_canonical(asdict(gen.text_config))),
        "measurement_policy": {
            "request_execution": "serial; synthetic timestamps do not cause wall-clock sleeps",
            "revisit": "visit_index > 0, independent of cache residency or hit status",
            "history_tokens": "complete stable prefix including fixed instruction",
            "candidate_tokens": "complete changing suffix",
            "sampling": config.sampling,
        },
        "observed": {
            "requests": len(requests), "unique_users": len(counts),
            "returning_users": sum(c > 1 for c in counts.values()), "first_visits": len(counts),
            "revisits": sum(c - 1 for c in counts.values()), "max_visits": max(counts.values(), default=0),
            "max_revisits": max((c - 1 for c in counts.values()), default=0),
        },
        "users": [
            {"user_id": u, "weight": w,
             "probability": None if config.sampling == "sequential" else w / weight_sum,
             "visits": counts[u], "revisits": max(counts[u] - 1, 0),
             "prefix_sha256": token_sha256(prefixes[u]) if u in prefixes else None}
            for u, w in gen.population.weights.items()
        ],
    }
    return Workload(tuple(requests), manifest)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model", choices=tuple(MODEL_FORMATS), default="deepseek_v32")
    p.add_argument("--num-users", type=int, required=True)
    p.add_argument("--requests", type=int, default=128)
    p.add_argument("--max-revisits", type=int)
    p.add_argument("--history-tokens", type=int, default=8192)
    p.add_argument("--candidate-tokens", type=int, default=1024)
    p.add_argument("--context-limit", type=int)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--sampling", choices=("weighted", "sequential"), default="weighted")
    p.add_argument("--heat-dataset", default="beauty")
    p.add_argument("--heat-field")
    p.add_argument("--heat-curves", help="CSV of ranked traffic curves (default: built-in Zipf curve)")
    p.add_argument("--tokenizer", type=Path)
    p.add_argument("--output-dir", type=Path, required=True)
    a = p.parse_args(argv)
    try:
        wl = build_workload(WorkloadConfig(
            model=a.model, num_users=a.num_users, requests=a.requests, history_tokens=a.history_tokens,
            candidate_tokens=a.candidate_tokens, seed=a.seed, heat_dataset=a.heat_dataset, heat_field=a.heat_field,
            heat_path=a.heat_curves, sampling=a.sampling, max_revisits=a.max_revisits,
            context_limit=a.context_limit), tokenizer=a.tokenizer)
        wl.write(a.output_dir)
    except (ValueError, OSError) as exc:
        p.error(str(exc))
    print(json.dumps({"workload_sha256": wl.manifest["workload_sha256"], **wl.manifest["observed"]}))


if __name__ == "__main__":
    main()
