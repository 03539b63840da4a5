"""Host-side liveness of the ranks of a one-process-per-GPU run (sequence-sharded replicas).

The step itself has no collective, so a rank that exits or stops between steps is invisible
to the others until their next collective times out. `PeerGuard` makes it visible earlier and
by name: before each step every rank publishes that it reached the step in the process
group's key-value store and waits, with a short limit, for the others; a rank that leaves
between steps says so first. Nothing here touches the GPU, so a lost rank is found on the
host with no kernel or collective in flight.
"""

from __future__ import annotations

import datetime


class RankFailure(RuntimeError):
    """A peer rank left or did not reach a step in time."""

    def __init__(self, step: int, missing: list[int], left: dict[int, int]):
        self.step, self.missing, self.left = step, missing, left
        parts = []
        if left:
            parts.append(", ".join(f"rank {r} left after step {s}" for r, s in sorted(left.items())))
        late = [r for r in missing if r not in left]
        if late:
            parts.append(f"rank(s) {late} did not reach step {step}")
        super().__init__("; ".join(parts) or f"peer failure at step {step}")


class PeerGuard:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "qsp"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.prefix = prefix

    def _key(self, *parts) -> str:
        return "/".join((self.prefix,) + tuple(str(p) for p in parts))

    def _left(self) -> dict[int, int]:
        out = {}
        for r in range(self.world):
            if r != self.rank and self.store.check([self._key("left", r)]):
                out[r] = int(self.store.get(self._key("left", r)))
        return out

    def checkpoint(self, step: int):
        """Publish that this rank reached `step`, then wait for every peer to reach it. Raises
        RankFailure naming the ranks that left (announced) or did not arrive in time."""
        self.store.set(self._key("at", step, self.rank), "1")
        left = self._left()
        if left:
            raise RankFailure(step, sorted(left), left)
        keys = [self._key("at", step, r) for r in range(self.world)]
        try:
            self.store.wait(keys, self.timeout)
        except Exception:  # noqa: BLE001 - the store raises its own timeout type
            missing = [r for r in range(self.world) if not self.store.check([self._key("at", step, r)])]
            raise RankFailure(step, missing, self._left()) from None

    def leave(self, last_step: int):
        """Announce that this rank stops after `last_step` (call between steps, with none of its
        kernels or collectives in flight)."""
        self.store.set(self._key("left", self.rank), str(last_step))
