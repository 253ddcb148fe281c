"""Host-side liveness of the expert-parallel ranks.

The device side bounds every wait on the communicator and aborts it when a
peer stops answering (the guarded waits behind k3xb_ep_init_config). A rank
that leaves between steps should not be found out that way, by a collective
running into its deadline: the others should learn of it on the host before
they launch the next step. PeerWatch does that over any torch.distributed
key-value store (TCPStore, FileStore, the process group's own store):
before step i every rank posts "step i" and waits, with a bound, until all
ranks have posted it; a rank that announced it is leaving, or that has not
posted by the bound, ends the wait with PeerLost naming the missing ranks.
No GPU work is in flight at that point, so the caller can tear the
communicator down (k3xb_ep_finalize) and re-form the group.

The reference runs one process on one GPU and has no counterpart; its
single-rank failure convention (a status, never a hang; runtime/include/
k3x/status.hpp:9-76) is what this extends to several ranks.
"""
from __future__ import annotations

import time
from datetime import timedelta


class PeerLost(RuntimeError):
    """Ranks that did not reach a step (announced departures first)."""

    def __init__(self, step: int, missing: list, departed: list):
        self.step = step
        self.missing = sorted(set(missing) | set(departed))
        self.departed = sorted(departed)
        what = "left" if departed and set(departed) >= set(missing) else "did not reach the step"
        super().__init__(f"expert parallelism: rank(s) {self.missing} {what} (step {step})")


class PeerWatch:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "k3xb/ep",
                 poll_s: float = 0.005):
        if not 0 <= rank < world:
            raise ValueError("rank must be in [0, world)")
        if timeout_s <= 0 or poll_s <= 0:
            raise ValueError("timeout_s and poll_s must be positive")
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix, self.poll_s = timeout_s, prefix, poll_s
        self._left = False

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/step/{step}/{rank}"

    def _leave_key(self, rank: int) -> str:
        return f"{self.prefix}/leave/{rank}"

    def departed(self) -> list:
        """Ranks that announced they are leaving (does not wait)."""
        return [g for g in range(self.world) if self.store.check([self._leave_key(g)])]

    def step(self, step: int) -> None:
        """Posts `step` for this rank and returns once every rank has posted
        it; raises PeerLost (bounded by timeout_s) otherwise."""
        if self._left:
            raise RuntimeError("this rank has left the group")
        self.store.set(self._key(step, self.rank), b"1")
        pending = [g for g in range(self.world) if g != self.rank]
        deadline = time.monotonic() + self.timeout_s
        while True:
            pending = [g for g in pending if not self.store.check([self._key(step, g)])]
            if not pending:
                break
            gone = [g for g in pending if self.store.check([self._leave_key(g)])]
            if gone or time.monotonic() >= deadline:
                raise PeerLost(step, pending, gone)
            time.sleep(self.poll_s)
        if step >= 2:   # every rank has posted `step`, so all are past step - 1's wait
            try:
                self.store.delete_key(self._key(step - 2, self.rank))
            except (RuntimeError, NotImplementedError):   # stores without deletion keep the key
                pass

    def leave(self) -> None:
        """Announces an orderly departure between steps: the other ranks'
        next step() raises PeerLost at once instead of at the bound."""
        self.store.set(self._leave_key(self.rank), b"1")
        self._left = True


def make_store(rank: int, world: int, host: str = "127.0.0.1", port: int = 29400,
               timeout_s: float = 30.0):
    """A TCPStore for PeerWatch, served by rank 0."""
    from torch.distributed import TCPStore

    return TCPStore(host, port, world, is_master=rank == 0, timeout=timedelta(seconds=timeout_s),
                    wait_for_workers=False)
