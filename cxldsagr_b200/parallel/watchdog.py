"""Host-side rank watchdog: ranks learn of a failed or vanished peer before
their next launch, not by hanging in a collective.

Each rank's background thread writes a heartbeat (a counter) into the process
group's key-value store every ``interval_s``.  A rank whose step raised calls
:meth:`RankWatchdog.report_failure`, which records the failure in the store.
Before every step the loop calls :meth:`RankWatchdog.check`; it raises
:class:`RankFailure` if any peer reported a failure or if a peer's heartbeat
has not advanced for ``timeout_s`` (a process that died or hung outside the
GPU).  Nothing here touches a GPU: the failure is detected on the host
between steps, and the process group's own short timeout remains the last
bound for a collective already in flight.

The reference has no multi-rank code (errors propagate within one process);
this is the multi-GPU counterpart of its transactional failure handling.
"""

from __future__ import annotations

import threading
import time

import torch.distributed as dist


class RankFailure(RuntimeError):
    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank}: {reason}")
        self.rank = rank
        self.reason = reason


class RankWatchdog:
    def __init__(self, rank: int, world: int, store=None, *, interval_s: float = 0.5, timeout_s: float = 10.0,
                 prefix: str = "cxld_watchdog"):
        if store is None:
            from torch.distributed import distributed_c10d

            store = distributed_c10d._get_default_store()
        self.rank, self.world, self.store = rank, world, store
        self.interval_s, self.timeout_s, self.prefix = interval_s, timeout_s, prefix
        self._beat = 0
        self._stop = threading.Event()
        self._seen: dict[int, tuple[int, float]] = {}
        self._key_hb = lambda r: f"{prefix}/hb/{r}"
        self._key_fail = lambda r: f"{prefix}/fail/{r}"
        self.store.set(self._key_hb(rank), "0")
        self._thread = threading.Thread(target=self._run, name=f"watchdog-{rank}", daemon=True)
        self._thread.start()

    @classmethod
    def for_group(cls, **kw) -> "RankWatchdog":
        return cls(dist.get_rank(), dist.get_world_size(), **kw)

    def _run(self):
        while not self._stop.wait(self.interval_s):
            self._beat += 1
            try:
                self.store.set(self._key_hb(self.rank), str(self._beat))
            except Exception:  # noqa: BLE001 - the store went away: peers see a stale heartbeat
                return

    def report_failure(self, exc: BaseException | str):
        """Record this rank's failure so every peer's next :meth:`check` raises."""
        self.store.set(self._key_fail(self.rank), repr(exc)[:512])

    def check(self):
        """Raise :class:`RankFailure` for the first failed or silent peer (call between steps)."""
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank:
                continue
            if self.store.check([self._key_fail(r)]):
                raise RankFailure(r, "reported failure: " + self.store.get(self._key_fail(r)).decode())
            try:
                beat = int(self.store.get(self._key_hb(r)).decode()) if self.store.check([self._key_hb(r)]) else -1
            except Exception as exc:  # noqa: BLE001
                raise RankFailure(r, f"heartbeat unreadable ({exc!r})") from exc
            last = self._seen.get(r)
            if last is None or beat != last[0]:
                self._seen[r] = (beat, now)
            elif now - last[1] > self.timeout_s:
                raise RankFailure(r, f"no heartbeat for {now - last[1]:.1f} s")

    def close(self):
        self._stop.set()
        self._thread.join(timeout=2 * self.interval_s + 1)
