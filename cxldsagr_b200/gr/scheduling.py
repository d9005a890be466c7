"""User sampling and request arrival schedules of the GR workload.

Reference semantics (``GR/scheduling.py:32-176``):

* ``sampling``: ``weighted`` (draw users by heat), ``uniform`` or
  ``sequential`` (cycle through users in order);
* ``arrival``: ``poisson`` (exponential gaps at ``qps``), ``constant``
  (``order / qps``) or ``timeslot`` (``qps`` draws per one-second slot, each
  drawn user cools down for a per-user gap drawn from a fixed table before it
  can be drawn again);
* ``max_revisits``: optional cap on visits per user (a capped user leaves
  the draw; the stream ends once every user is exhausted).

The weighted draw uses a binary indexed (Fenwick) tree of weights so that a
draw and a weight update are ``O(log users)`` — the standard structure from
Fenwick, "A new data structure for cumulative frequency tables" (1994).
"""

from __future__ import annotations

import heapq
import math
import random
from collections.abc import Iterator
from dataclasses import dataclass

# Cool-down gap table (seconds) and its weights for the timeslot arrival.
GAP_SECONDS = (5, 15, 25, 35, 45, 55, 65)
GAP_WEIGHTS = (18, 12, 8, 5, 3, 2, 52)


def _integer(name: str, value, minimum: int = 0) -> None:
    if isinstance(value, bool) or not isinstance(value, int) or value < minimum:
        raise ValueError(f"{name} must be an integer >= {minimum}, got {value!r}")


def index_letter(index: int) -> str:
    """0 -> A, 25 -> Z, 26 -> AA, ... (bijective base 26)."""
    _integer("index", index)
    letters = []
    n = index + 1
    while n > 0:
        n, rem = divmod(n - 1, 26)
        letters.append(chr(ord("A") + rem))
    return "".join(reversed(letters))


@dataclass(frozen=True)
class ScheduleConfig:
    seed: int = 42
    qps: int = 100
    arrival: str = "poisson"
    sampling: str = "weighted"
    start_timestamp: float = 0.0
    max_revisits: int | None = None

    def __post_init__(self):
        _integer("seed", self.seed)
        _integer("qps", self.qps, 1)
        if self.max_revisits is not None:
            _integer("max_revisits", self.max_revisits)
        if self.arrival not in ("poisson", "constant", "timeslot"):
            raise ValueError("arrival must be poisson, constant, or timeslot")
        if self.sampling not in ("weighted", "uniform", "sequential"):
            raise ValueError("sampling must be weighted, uniform, or sequential")
        if self.arrival == "timeslot" and self.sampling == "sequential":
            raise ValueError("timeslot requires weighted or uniform sampling")
        if not math.isfinite(self.start_timestamp) or self.start_timestamp < 0:
            raise ValueError("start_timestamp must be finite and nonnegative")


class FenwickSampler:
    """Weighted draws with O(log n) weight updates (prefix sums in a Fenwick tree)."""

    def __init__(self, weights):
        self.n = len(weights)
        self.weights = [float(w) for w in weights]
        self.tree = [0.0] * (self.n + 1)
        for i, w in enumerate(self.weights):
            self._add(i, w)
        self._top = 1 << max(self.n.bit_length() - 1, 0)

    def _add(self, index: int, delta: float):
        i = index + 1
        while i <= self.n:
            self.tree[i] += delta
            i += i & -i

    def total(self) -> float:
        s, i = 0.0, self.n
        while i > 0:
            s += self.tree[i]
            i -= i & -i
        return s

    def set(self, index: int, weight: float) -> None:
        self._add(index, weight - self.weights[index])
        self.weights[index] = weight

    def draw(self, rng: random.Random) -> int:
        """Index i with probability weight[i] / total (descends the implicit tree)."""
        target = rng.random() * self.total()
        pos, step = 0, self._top
        while step:
            nxt = pos + step
            if nxt <= self.n and self.tree[nxt] <= target:
                target -= self.tree[nxt]
                pos = nxt
            step >>= 1
        return min(pos, self.n - 1)


def schedule(users: list, weights: dict, count: int, cfg: ScheduleConfig) -> Iterator[tuple]:
    """Yield ``(user_id, timestamp)`` for up to ``count`` requests."""
    _integer("count", count)
    rng = random.Random(cfg.seed)
    clock = random.Random(f"{cfg.seed}:clock")
    gap_rng = random.Random(f"{cfg.seed}:gap")
    base = [float(weights[u]) if cfg.sampling == "weighted" else 1.0 for u in users]
    sampler = FenwickSampler(base)
    cooldown = gap_rng.choices(GAP_SECONDS, weights=GAP_WEIGHTS, k=len(users))
    cap = None if cfg.max_revisits is None else cfg.max_revisits + 1
    visits = [0] * len(users)
    exhausted = 0
    waiting: list[tuple[int, int]] = []   # (slot when eligible again, index)
    eligible = len(users)
    slot, used_in_slot = 0, 0
    t = cfg.start_timestamp
    for order in range(count):
        if exhausted == len(users):
            return
        if cfg.arrival == "timeslot":
            if used_in_slot == cfg.qps:
                slot, used_in_slot = slot + 1, 0
            while True:
                while waiting and waiting[0][0] <= slot:
                    _, i = heapq.heappop(waiting)
                    sampler.set(i, base[i])
                    eligible += 1
                if eligible:
                    break
                slot, used_in_slot = waiting[0][0], 0
            i = sampler.draw(rng)
            t = cfg.start_timestamp + slot
            sampler.set(i, 0.0)
            eligible -= 1
            if cap is None or visits[i] + 1 < cap:
                heapq.heappush(waiting, (slot + cooldown[i], i))
            used_in_slot += 1
        else:
            i = order % len(users) if cfg.sampling == "sequential" else sampler.draw(rng)
            t = t + clock.expovariate(cfg.qps) if cfg.arrival == "poisson" else cfg.start_timestamp + order / cfg.qps
        if cap is not None:
            visits[i] += 1
            if visits[i] == cap:
                exhausted += 1
                if cfg.arrival != "timeslot":
                    sampler.set(i, 0.0)
        yield users[i], t
