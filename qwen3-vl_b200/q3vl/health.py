"""Host-side liveness of tensor-parallel ranks.

The in-kernel all-reduce waits for peers with a bounded spin and reports
Q3_ERR_TIMEOUT through the device error word when a peer never writes, but a
rank should not launch a step whose peers are already gone.  RankHealth keeps
one heartbeat key per rank in a torch.distributed store: each rank records
the step it finished, and before its next launch waits (bounded) until every
peer has finished the previous step.  A rank that fails on the host records
the reason, and the others raise RankFailure naming it instead of waiting.
"""
from __future__ import annotations

import time


class RankFailure(RuntimeError):
    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank}: {reason}")
        self.rank, self.reason = rank, reason


class RankHealth:
    def __init__(self, store, rank: int, world: int, prefix: str = "q3vl/health"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix
        self._step = -1
        self.beat(-1)

    def tick(self) -> int:
        """Record the next step of a sequence that only grows (across calls of
        whatever loop uses it) and return its number; every rank ticks the
        same number of times."""
        self._step += 1
        self.beat(self._step)
        return self._step

    def _key(self, r: int, what: str) -> str:
        return f"{self.prefix}/{r}/{what}"

    def beat(self, step: int) -> None:
        """This rank finished `step`."""
        self.store.set(self._key(self.rank, "step"), str(int(step)))

    def fail(self, reason: str) -> None:
        """Tell the peers this rank stops (called from its error path)."""
        self.store.set(self._key(self.rank, "failed"), reason)

    def _failed(self, r: int):
        key = self._key(r, "failed")
        return self.store.get(key).decode() if self.store.check([key]) else None

    def wait_for_peers(self, step: int, timeout_s: float = 10.0, poll_s: float = 0.01) -> None:
        """Return once every peer has finished `step`; raise RankFailure for a
        peer that declared failure or has not got there within timeout_s."""
        t0 = time.monotonic()
        pending = [r for r in range(self.world) if r != self.rank]
        while pending:
            still = []
            for r in pending:
                reason = self._failed(r)
                if reason is not None:
                    raise RankFailure(r, f"failed: {reason}")
                key = self._key(r, "step")
                done = int(self.store.get(key).decode()) if self.store.check([key]) else -2
                if done < step:
                    still.append(r)
            pending = still
            if pending:
                if time.monotonic() - t0 > timeout_s:
                    raise RankFailure(pending[0], f"no heartbeat for step {step} within "
                                                  f"{timeout_s:.1f} s")
                time.sleep(poll_s)
