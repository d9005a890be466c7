"""Readable GR requests with exact token budgets, user heat and arrival times.

Reference semantics (``GR/input_generator.py:71-645``).  A request for user
``u`` on visit ``v`` is::

    chat prefix (instruction)  |  user history block  |  candidate block + ending
    <------------- stable prefix (fixed per user) ----->|<--- changes per visit -->

Budgets are exact token counts: the history block holds ``user_length``
tokens and the candidate block ``item_length - len(prefix)`` tokens.  Blocks
are built from whole synthetic records (history: "Record i: Viewed P123,
blue lamp. Preference: ...", candidates: a lettered candidate pool plus
detail lines); the residual budget after the last whole record is closed with
short whole sentences chosen by an exact-sum search over their measured token
increments, so no id padding or partial token is ever used.  Every random
choice comes from a stream seeded by ``(seed, purpose, user, visit)``, so a
user's history is identical on every visit and across cache schemes.
"""

from __future__ import annotations

import hashlib
import math
import random
from collections import Counter
from dataclasses import dataclass
from functools import lru_cache
from pathlib import Path

from ..models.deepseek_v32 import request_format as deepseek_format
from .heat import HeatPopulation
from .scheduling import ScheduleConfig, _integer, index_letter, schedule
from .tokenizer import load_tokenizer

MODEL_FORMATS = {"deepseek_v32": deepseek_format}
INSTRUCTION = "Recommend one item from the candidate pool based on the user history. Output its index letter."
ATTRIBUTES = ("easy to clean", "comfortable to use", "compact and lightweight", "suitable for daily use",
              "simple to store", "designed for travel")
PRODUCTS = ("travel bag", "desk lamp", "water bottle", "running shoes", "wireless headphones", "coffee maker",
            "notebook", "storage box", "cotton shirt", "face moisturizer")
COLORS = ("blue", "green", "black", "white", "silver", "red")
ACTIONS = ("Viewed", "Compared", "Saved", "Purchased")
TAILS = ("Looks good.\n", "Quality is good.\n", "The design is practical.\n", "The finish is smooth.\n",
         "The size is convenient.\n", "Checked.\n")


def _probabilities_ok(p) -> bool:
    return all(math.isfinite(x) and x >= 0 for x in p) and math.isclose(sum(p), 1)


@dataclass(frozen=True)
class TextConfig:
    user_lengths: tuple = deepseek_format.USER_LENGTHS
    user_probabilities: tuple = (1 / len(deepseek_format.USER_LENGTHS),) * len(deepseek_format.USER_LENGTHS)
    item_lengths: tuple = deepseek_format.ITEM_LENGTHS
    item_probabilities: tuple = (1 / len(deepseek_format.ITEM_LENGTHS),) * len(deepseek_format.ITEM_LENGTHS)
    candidate_count: int = 20
    max_input_tokens: int = deepseek_format.MAX_INPUT_TOKENS
    history_cache_users: int = 8

    def __post_init__(self):
        for kind in ("user", "item"):
            lengths, probs = getattr(self, f"{kind}_lengths"), getattr(self, f"{kind}_probabilities")
            if not lengths or len(lengths) != len(probs):
                raise ValueError(f"{kind}: lengths and probabilities must be nonempty and equally sized")
            for n in lengths:
                _integer(f"{kind}_length", n, 1)
            if not _probabilities_ok(probs):
                raise ValueError(f"{kind}: probabilities must be finite, nonnegative and sum to 1")
        _integer("candidate_count", self.candidate_count, 1)
        _integer("max_input_tokens", self.max_input_tokens, 1)
        _integer("history_cache_users", self.history_cache_users)
        if max(self.user_lengths) + max(self.item_lengths) > self.max_input_tokens:
            raise ValueError("user + item length exceeds max_input_tokens")


class InputGenerator:
    def __init__(self, population: HeatPopulation, tokenizer, *, model: str = "deepseek_v32",
                 text_config: TextConfig | None = None, schedule_config: ScheduleConfig | None = None,
                 titles: dict | None = None, context_limit: int | None = None):
        if model not in MODEL_FORMATS:
            raise ValueError(f"unsupported model: {model}")
        fmt = MODEL_FORMATS[model]
        self.model, self.request_format = model, fmt
        if context_limit is not None:
            _integer("context_limit", context_limit, 1)
        self.context_limit = fmt.MAX_INPUT_TOKENS if context_limit is None else context_limit
        self.text_config = text_config or TextConfig()
        if max(self.text_config.user_lengths) + max(self.text_config.item_lengths) > self.context_limit:
            raise ValueError(f"{model} request exceeds the configured {self.context_limit}-token context")
        self.schedule_config = schedule_config or ScheduleConfig(sampling="weighted")
        self.seed = self.schedule_config.seed
        self.population = population
        self.users = sorted(population.weights)
        if not self.users:
            raise ValueError("population must not be empty")
        self.tokenizer = tokenizer
        tokenizer.no_padding()
        tokenizer.no_truncation()
        for special in fmt.SPECIAL_TOKENS:
            if tokenizer.token_to_id(special) is None:
                raise ValueError(f"tokenizer lacks {model} token {special}")
        if titles is not None and not titles:
            raise ValueError("text catalog is empty")
        self.titles = titles
        self.catalog = sorted(titles) if titles is not None else range(1_000_000)
        if len(self.catalog) < self.text_config.candidate_count:
            raise ValueError("candidate_count exceeds catalog size")
        self.prefix = fmt.prefix(INSTRUCTION)
        self.ending = fmt.ENDING
        self.prefix_ids = self.encode(self.prefix)
        self._title = lru_cache(maxsize=16384)(self._make_title)
        self._history = lru_cache(maxsize=max(1, self.text_config.history_cache_users))(self._make_history)

    # ------------------------------------------------------------------ text
    def encode(self, text: str) -> list:
        return self.tokenizer.encode(text, add_special_tokens=False).ids

    def _count(self, text: str) -> int:
        return len(self.encode(text))

    def _make_title(self, item: int) -> str:
        if self.titles is not None:
            words = self.titles[item].split()[:24]
            while words and self._count(" ".join(words)) > 24:
                words.pop()
            return " ".join(words) if words else f"Catalog product P{item}"
        rng = random.Random(f"{self.seed}:product:{item}")
        return f"{rng.choice(COLORS)} {rng.choice(PRODUCTS)}"

    def lengths_for_user(self, uid) -> tuple:
        cfg = self.text_config
        h = random.Random(f"{self.seed}:history-length:{uid}").choices(cfg.user_lengths, cfg.user_probabilities)[0]
        n = random.Random(f"{self.seed}:non-history-length:{uid}").choices(cfg.item_lengths, cfg.item_probabilities)[0]
        return h, n

    def _fit(self, heading: str, records, target: int, ending: str = "") -> str:
        """Whole records, then whole tail sentences that close the budget exactly."""
        if self._count(heading + ending) > target:
            raise ValueError(f"mandatory text does not fit {target} tokens")
        lines, used = [], self._count(heading + ending)
        while used < target + 64:                      # overshoot, then cut back exactly
            line = next(records)
            lines.append(line)
            used += max(1, self._count(line))
        lo, hi = 0, len(lines)
        while lo < hi:                                 # longest record prefix that fits
            mid = (lo + hi + 1) // 2
            if self._count(heading + "".join(lines[:mid]) + ending) <= target:
                lo = mid
            else:
                hi = mid - 1
        for keep in range(lo, max(-1, lo - 4), -1):
            body = heading + "".join(lines[:keep])
            base = self._count(body + ending)
            gap = target - base
            incs = [self._count(body + t + ending) - base for t in TAILS]
            best = {0: ()}                              # exact-sum search over tail increments
            for total in range(1, gap + 1):
                for tail, inc in zip(TAILS, incs):
                    if inc > 0 and total - inc in best:
                        best[total] = best[total - inc] + (tail,)
                        break
            if gap in best:
                text = body + "".join(best[gap]) + ending
                if self._count(text) == target:
                    return text
        raise ValueError(f"cannot fit a readable block to {target} tokens with this tokenizer")

    def _make_history(self, uid):
        h, _ = self.lengths_for_user(uid)
        rng = random.Random(f"{self.seed}:history:{uid}")

        def records():
            i = 0
            while True:
                i += 1
                item = rng.choice(self.catalog)
                yield (f"Record {i}: {rng.choice(ACTIONS)} P{item}, {self._title(item)}. "
                       f"Preference: {rng.choice(ATTRIBUTES)}.\n")

        text = self._fit(f"User profile U{uid}.\n", records(), h)
        return text, tuple(self.encode(text))

    def _candidates(self, uid, visit: int, item_variant: int | None = None):
        _, n = self.lengths_for_user(uid)
        budget = n - len(self.prefix_ids)
        limit = budget - self.request_format.TAIL_RESERVE_TOKENS
        key = f"{uid}:{visit}" if item_variant is None else f"shared:{item_variant}:{visit}"
        rng = random.Random(f"{self.seed}:candidates:{key}")
        items = rng.sample(self.catalog, self.text_config.candidate_count)
        title = f"Candidate pool for visit {visit}:\n"
        lines = [f"({index_letter(i)}) P{item}: {self._title(item)}.\n" for i, item in enumerate(items)]
        while len(items) > 1 and self._count(title + "".join(lines) + self.ending) > limit:
            items.pop()
            lines.pop()
        if len(items) == 1 and self._count(title + lines[0] + self.ending) > limit:
            words = self._title(items[0]).split()
            while len(words) > 1 and self._count(title + lines[0] + self.ending) > limit:
                words.pop()
                lines[0] = f"(A) P{items[0]}: {' '.join(words)}.\n"
            if self._count(title + lines[0] + self.ending) > limit:
                lines[0] = f"(A) P{items[0]}: Catalog product.\n"

        def details():
            while True:
                i = rng.randrange(len(items))
                yield f"Details for ({index_letter(i)}): {rng.choice(ATTRIBUTES)}.\n"

        return self._fit(title + "".join(lines), details(), budget, self.ending), items

    # -------------------------------------------------------------- requests
    def for_user(self, uid, *, visit_index: int = 0, item_variant: int | None = None) -> dict:
        if uid not in self.population.weights:
            raise KeyError(uid)
        _integer("visit_index", visit_index)
        history, history_ids = self._history(uid)
        suffix, items = self._candidates(uid, visit_index, item_variant)
        suffix_ids = self.encode(suffix)
        prompt = self.prefix + history + suffix
        ids = self.encode(prompt)
        if ids != self.prefix_ids + list(history_ids) + suffix_ids:
            raise ValueError("tokenizer merges across section boundaries; cannot guarantee exact budgets")
        h, n = self.lengths_for_user(uid)
        if len(ids) != h + n:
            raise ValueError("full prompt length does not match configured budgets")
        start = len(self.prefix_ids)
        return {
            "model": self.model, "user_id": uid, "visit_index": visit_index, "prompt": prompt,
            "input_ids": ids, "attention_mask": [1] * len(ids),
            "user_heat_weight": self.population.weights[uid], "user_tokens": h, "item_tokens": n,
            "instruction_tokens": start, "candidate_suffix_tokens": len(suffix_ids),
            "total_input_tokens": len(ids), "stable_prefix_tokens": start + h,
            "history_sha256": hashlib.sha256(history.encode()).hexdigest(),
            "history_token_span": [start, start + h], "candidate_token_span": [start + h, len(ids)],
            "candidate_item_ids": items, "item_content_variant": item_variant,
            "content_is_synthetic": True, "target_item_id": None,
        }

    def iter_generate(self, count: int):
        _integer("count", count)
        visits: Counter = Counter()
        last: dict = {}
        for task_id, (uid, ts) in enumerate(schedule(self.users, self.population.weights, count,
                                                      self.schedule_config)):
            visit = visits[uid]
            row = self.for_user(uid, visit_index=visit)
            prev = last.get(uid)
            row.update(task_id=task_id, timestamp=ts, previous_request_id=prev[0] if prev else None,
                       revisit_interval_s=ts - prev[1] if prev else None, common_prefix_tokens=0)
            if prev:
                old = self.encode(self._candidates(uid, visit - 1)[0])
                new = row["input_ids"][row["stable_prefix_tokens"]:]
                shared = next((i for i, (a, b) in enumerate(zip(old, new)) if a != b), min(len(old), len(new)))
                row["common_prefix_tokens"] = row["stable_prefix_tokens"] + shared
            last[uid] = (task_id, ts)
            visits[uid] += 1
            yield row


def create_input_generator(*, model: str = "deepseek_v32", heat_source: str = "curve",
                           heat_path: str | Path | None = None, curve_dataset: str = "beauty",
                           curve_field: str | None = None, industrial_heat_field: str = "pv_share",
                           num_users: int = 1000, tokenizer=None, text_config: TextConfig | None = None,
                           schedule_config: ScheduleConfig | None = None, context_limit: int | None = None,
                           titles: dict | None = None, text_material: str = "synthetic") -> InputGenerator:
    """A reusable in-memory request generator (no files written, nothing sent)."""
    if model not in MODEL_FORMATS:
        raise ValueError(f"unsupported model: {model}")
    if text_material not in ("catalog", "synthetic"):
        raise ValueError(f"unsupported text_material: {text_material}")
    if text_material == "catalog" and not titles:
        raise ValueError("catalog text needs a titles mapping")
    seed = (schedule_config or ScheduleConfig()).seed
    if heat_source == "curve":
        field = curve_field or ("pv_share" if curve_dataset.startswith("industrial") else "interaction_count")
        population = HeatPopulation.from_curve(heat_path, dataset=curve_dataset, field=field,
                                               num_users=num_users, seed=seed)
    elif heat_source == "industrial":
        population = HeatPopulation.load(Path(heat_path), industrial_field=industrial_heat_field,
                                         num_users=num_users, seed=seed)
    elif heat_source == "counts":
        population = HeatPopulation.load(Path(heat_path), num_users=num_users, seed=seed)
    elif heat_source == "uniform":
        population = HeatPopulation.uniform(num_users)
    else:
        raise ValueError(f"unsupported heat_source: {heat_source}")
    if tokenizer is None or isinstance(tokenizer, (str, Path)):
        tokenizer = load_tokenizer(tokenizer)
    return InputGenerator(population, tokenizer, model=model, text_config=text_config,
                          schedule_config=schedule_config, context_limit=context_limit,
                          titles=titles if text_material == "catalog" else None)
