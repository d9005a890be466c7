"""Resource generations, admission owners and exclusive operations.

Reference semantics (``cache/lifecycle.py:17-243``): one admission owner per
resource generation; at most one active operation at a time, acquired
without blocking (a concurrent caller gets an error rather than waiting);
an operation that fails *and* whose completion (drain) could not be
confirmed poisons the resources, because storage might still be in use by
the device.  ``close`` ends the generation after draining.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass
from threading import Lock


@dataclass(frozen=True)
class SessionRegistration:
    identity: object
    generation: int
    owner: object | None


class ResourceLifecycle:
    def __init__(self, label: str, *, drain=None):
        self.label = label
        self.identity = object()
        self.generation = 0
        self.sessions: set = set()
        self.admission_owner = None
        self.active_session = None
        self.active_kind = None
        self.poisoned = False
        self.closed = False
        self.failure = None
        self._drain = drain
        self._lock = Lock()

    def poison(self, error=None):
        self.poisoned = True
        if error is not None:
            self.failure = error

    def check_access(self, owner=None, *, allow_closed=False):
        if self.poisoned:
            raise RuntimeError(f"{self.label} resources are poisoned")
        if self.closed and not allow_closed:
            raise RuntimeError(f"{self.label} resource generation is closed")
        if owner is not self.admission_owner:
            raise RuntimeError(f"{self.label} resources belong to another admission owner")

    def check_active(self, session):
        """Borrowed session caches mutate only inside their own session's operation.

        Reference: ``models/deepseek_v32/cache/session.py:12-84`` (``ServingCacheGuard``).
        """
        if self.poisoned:
            raise RuntimeError(f"{self.label} resources are poisoned")
        if session not in self.sessions:
            raise RuntimeError(f"{self.label}: the session is released or belongs to another generation")
        if self.active_session is not session:
            raise RuntimeError(f"{self.label}: session cache mutation requires the session's active operation")

    def bind_owner(self, owner):
        if self.admission_owner is not None and self.admission_owner is not owner:
            raise RuntimeError(f"{self.label} already has an admission owner")
        self.admission_owner = owner
        self.closed = False

    def unbind_owner(self, owner):
        if self.admission_owner is owner:
            self.admission_owner = None

    def register(self, session) -> SessionRegistration:
        self.check_access(self.admission_owner)
        self.sessions.add(session)
        return SessionRegistration(self.identity, self.generation, self.admission_owner)

    def release(self, session):
        self.sessions.discard(session)

    @contextmanager
    def operation(self, session=None, kind="execute", owner=None):
        """Exclusive, non-blocking operation scope over these resources."""
        self.check_access(owner if owner is not None else self.admission_owner)
        if not self._lock.acquire(blocking=False):
            raise RuntimeError(f"{self.label} already runs an operation ({self.active_kind})")
        self.active_session, self.active_kind = session, kind
        try:
            yield
        except BaseException as primary:
            if self._drain is not None:
                try:
                    self._drain()
                except BaseException as cleanup:  # noqa: BLE001 - unconfirmed completion
                    self.poison(cleanup)
                    raise BaseExceptionGroup(f"{self.label} operation and drain failed", [primary, cleanup]) from None
            raise
        finally:
            self.active_session = self.active_kind = None
            self._lock.release()

    def close(self):
        if self.closed:
            return
        if self._drain is not None:
            try:
                self._drain()
            except BaseException as exc:
                self.poison(exc)
                raise
        self.closed = True
        self.generation += 1
        self.sessions.clear()
