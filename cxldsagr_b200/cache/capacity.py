"""Capacity declarations: byte footprints, admission policies and plans.

Model- and allocator-independent types used by planning, admission and
audits (reference: ``cache/capacity.py:84-295``):

* :class:`CacheFootprint` — HBM + DRAM bytes, additive, ``fits`` a budget;
* :class:`CapacityPolicy` — a byte budget, or fixed pools (host pages / HBM tokens);
* :class:`AllocationSpec` — one named storage with its allocator charge;
  allocations in one ``peak_group`` are mutually exclusive phases (only the
  largest phase counts); aliases charge nothing;
* :class:`ResourcePlan` — shared reservations + quotas, immutable metadata;
* :class:`SessionPlan` — one admission decision for one user history;
* :class:`ResourceUsage` — measured bytes / pages / tokens of a session.
"""

from __future__ import annotations

from collections.abc import Hashable, Mapping
from dataclasses import dataclass, field
from math import prod
from types import MappingProxyType
from typing import Any, Literal

DTYPE_BYTES = {
    "bool": 1, "uint8": 1, "int8": 1, "float8_e4m3fn": 1, "float8_e5m2": 1,
    "uint16": 2, "int16": 2, "float16": 2, "bfloat16": 2,
    "uint32": 4, "int32": 4, "float32": 4,
    "uint64": 8, "int64": 8, "float64": 8,
}


class CacheBudgetExceeded(ValueError):
    """An admission or shared reservation does not fit the configured budget."""


def _nonneg(value, name):
    if type(value) is not int or value < 0:
        raise ValueError(f"{name} must be a nonnegative integer")


def _freeze(value):
    if isinstance(value, (str, int, float, bool, type(None))):
        return value
    if isinstance(value, Mapping):
        if any(not isinstance(k, str) for k in value):
            raise TypeError("plan metadata keys must be strings")
        return MappingProxyType({k: _freeze(v) for k, v in value.items()})
    if isinstance(value, (list, tuple)):
        return tuple(_freeze(v) for v in value)
    raise TypeError("plan metadata must be plain immutable data")


@dataclass(frozen=True)
class CacheFootprint:
    hbm: int = 0
    dram: int = 0

    def __post_init__(self):
        _nonneg(self.hbm, "hbm bytes")
        _nonneg(self.dram, "dram bytes")

    @classmethod
    def from_mapping(cls, m: Mapping[str, int]) -> "CacheFootprint":
        return cls(hbm=int(m["hbm"]), dram=int(m["dram"]))

    def fits(self, budget: "CacheFootprint") -> bool:
        return self.hbm <= budget.hbm and self.dram <= budget.dram

    def __add__(self, other: "CacheFootprint") -> "CacheFootprint":
        return CacheFootprint(self.hbm + other.hbm, self.dram + other.dram)

    def __sub__(self, other: "CacheFootprint") -> "CacheFootprint":
        return CacheFootprint(max(0, self.hbm - other.hbm), max(0, self.dram - other.dram))


@dataclass(frozen=True)
class CapacityPolicy:
    mode: Literal["budget", "fixed_pools"]
    budget: CacheFootprint | None = None

    def __post_init__(self):
        if self.mode not in ("budget", "fixed_pools"):
            raise ValueError("unknown capacity policy")
        if (self.mode == "budget") != isinstance(self.budget, CacheFootprint):
            raise ValueError("a byte-budget policy needs a CacheFootprint; fixed pools carry none")

    @classmethod
    def byte_budget(cls, budget: CacheFootprint) -> "CapacityPolicy":
        return cls("budget", budget)

    @classmethod
    def fixed_pools(cls) -> "CapacityPolicy":
        return cls("fixed_pools")


@dataclass(frozen=True)
class AllocationSpec:
    name: str
    owner: Literal["shared", "session"]
    dtype: str
    shape: tuple[int, ...]
    device: str
    lifetime: str
    storage_bytes: int
    charged_bytes: int
    alias_of: str | None = None
    peak_group: str | None = None
    phase: str | None = None

    def __post_init__(self):
        if not (self.name and self.dtype and self.device and self.lifetime):
            raise ValueError("allocation name, dtype, device and lifetime must be explicit")
        if self.owner not in ("shared", "session"):
            raise ValueError("allocation owner must be shared or session")
        if self.dtype.removeprefix("torch.") not in DTYPE_BYTES:
            raise ValueError("allocation dtype needs a known element size")
        if self.device.split(":", 1)[0] not in ("cpu", "cuda"):
            raise ValueError("allocation device must be cpu or cuda")
        if self.phase is not None and not self.peak_group:
            raise ValueError("an allocation phase needs a peak group")
        if not isinstance(self.shape, tuple):
            raise TypeError("allocation shape must be a tuple")
        for d in self.shape:
            _nonneg(d, "allocation dimension")
        _nonneg(self.storage_bytes, "storage_bytes")
        _nonneg(self.charged_bytes, "charged_bytes")
        if self.logical_bytes > self.storage_bytes:
            raise ValueError("allocation storage cannot hold its dtype and shape")
        if self.alias_of == self.name:
            raise ValueError("an allocation cannot alias itself")
        if self.alias_of is not None and self.charged_bytes:
            raise ValueError("an alias must not charge its owner again")
        if self.alias_of is None and self.charged_bytes < self.storage_bytes:
            raise ValueError("the allocator charge must cover the storage")

    @property
    def logical_bytes(self) -> int:
        return prod(self.shape) * DTYPE_BYTES[self.dtype.removeprefix("torch.")]

    @property
    def tier(self) -> str:
        return "hbm" if self.device.startswith("cuda") else "dram"


def allocation_footprint(allocations) -> CacheFootprint:
    """Total charge: independent items add; per peak group only the largest phase counts."""
    by_name = {a.name: a for a in allocations}
    if len(by_name) != len(allocations):
        raise ValueError("allocation names must be unique")
    totals = {"hbm": 0, "dram": 0}
    groups: dict = {}
    for a in allocations:
        if a.alias_of is not None:
            target = by_name.get(a.alias_of)
            if target is None or target.alias_of is not None:
                raise ValueError("an alias must name an owning storage")
            if target.device != a.device or a.storage_bytes > target.storage_bytes:
                raise ValueError("an alias must stay within its owner's storage")
            continue
        if a.peak_group is None:
            totals[a.tier] += a.charged_bytes
        else:
            g = groups.setdefault((a.tier, a.owner, a.device, a.peak_group), {})
            ph = a.phase or a.name
            g[ph] = g.get(ph, 0) + a.charged_bytes
    for (tier, *_), g in groups.items():
        totals[tier] += max(g.values())
    return CacheFootprint(**totals)


@dataclass(frozen=True)
class ResourcePlan:
    shared: CacheFootprint = field(default_factory=CacheFootprint)
    host_pages: int = 0
    page_size: int = 64
    metadata: Mapping[str, Any] = field(default_factory=dict)
    hbm_tokens: int = 0
    allocations: tuple = ()
    policy: CapacityPolicy | None = None
    limits: Any = None

    def __post_init__(self):
        object.__setattr__(self, "metadata", _freeze(dict(self.metadata)))
        _nonneg(self.host_pages, "host_pages")
        _nonneg(self.hbm_tokens, "hbm_tokens")
        if type(self.page_size) is not int or self.page_size <= 0:
            raise ValueError("page_size must be positive")
        if any(a.owner != "shared" for a in self.allocations):
            raise ValueError("a resource plan holds only shared allocations")
        if self.allocations and not allocation_footprint(self.allocations).fits(self.shared):
            raise ValueError("shared allocations exceed their reservation")


@dataclass(frozen=True)
class SessionPlan:
    resource_identity: object
    history_identity: Hashable
    history_tokens: int
    retained_capacity: int
    reservation: CacheFootprint
    host_pages: int = 0
    hbm_tokens: int = 0
    allocations: tuple = ()
    model_plan: Any = None

    def __post_init__(self):
        if type(self.history_tokens) is not int or self.history_tokens <= 0:
            raise ValueError("history_tokens must be positive")
        if type(self.retained_capacity) is not int or self.retained_capacity < self.history_tokens:
            raise ValueError("retained capacity must cover the history")
        hash(self.history_identity)
        _nonneg(self.host_pages, "session host_pages")
        _nonneg(self.hbm_tokens, "session hbm_tokens")


@dataclass(frozen=True)
class ResourceUsage:
    bytes: CacheFootprint = field(default_factory=CacheFootprint)
    host_pages: int = 0
    hbm_tokens: int = 0
    owner: str = "session"

    def as_mapping(self) -> dict:
        return {"hbm": self.bytes.hbm, "dram": self.bytes.dram}

    @classmethod
    def coerce(cls, value) -> "ResourceUsage":
        if isinstance(value, ResourceUsage):
            return value
        if isinstance(value, CacheFootprint):
            return cls(value)
        return cls(CacheFootprint.from_mapping(value))
