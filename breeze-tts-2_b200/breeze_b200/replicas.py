"""Host-side coordination of independent decode replicas, one process per GPU.

A single decode stream does not shard profitably, so several GPUs run full,
independent copies of the decode step (replicas) with no traffic between
them: no collective on the data path and no NCCL. The ranks only meet at the
edges of a timed region -- a start line, a finish line, and one gather of
their results -- and they meet through a TCP key-value store
(torch.distributed.TCPStore) with a deadline at every meeting. A rank that
has not arrived when the deadline passes (it crashed, exited or hung) is
reported as failed; the ranks that did arrive carry on and finish, so one
lost replica never takes the others down with it.

Under torchrun the ranks use the launcher's own store (MASTER_ADDR /
MASTER_PORT, ``TORCHELASTIC_USE_AGENT_STORE``); otherwise rank 0 hosts one on
MASTER_PORT. Keys carry a per-run prefix.
"""

from __future__ import annotations

import json
import os
import time
from datetime import timedelta


class ReplicaGroup:
    """Meeting points of ``world`` replica processes.

    ``meet(name)`` returns the sorted ranks that reached meeting ``name``
    before its deadline (always including this rank); ``gather(name, value)``
    does the same and hands rank 0 every arrived rank's JSON-serialisable
    ``value``. Meeting names must be unique per run and used in the same
    order by every rank."""

    def __init__(self, rank: int, world: int, addr: str = "127.0.0.1", port: int | None = None,
                 timeout_s: float = 60.0, prefix: str | None = None):
        from torch.distributed import TCPStore

        self.rank, self.world, self.timeout_s = rank, world, timeout_s
        self.failed: set[int] = set()
        self.hosting = False
        run = prefix or os.environ.get("TORCHELASTIC_RUN_ID", "bq")
        restart = os.environ.get("TORCHELASTIC_RESTART_COUNT", "0")
        self.prefix = f"bq_replicas/{run}/{restart}/"
        port = int(port if port is not None else os.environ.get("MASTER_PORT", 29500))
        agent = os.environ.get("TORCHELASTIC_USE_AGENT_STORE", "").lower() == "true"
        host = agent is False and rank == 0
        self.hosting = host
        # the store's own timeout covers connecting while the other processes start up
        self.store = TCPStore(addr, port, world_size=None if agent else world, is_master=host,
                              timeout=timedelta(seconds=max(timeout_s, 120.0)), wait_for_workers=False)

    def _key(self, name: str, what: str) -> str:
        return f"{self.prefix}{name}/{what}"

    def _lost_store(self) -> list[int]:
        # the store's host is gone: nobody else can be reached, so this rank
        # carries on alone and reports every other rank as failed
        self.failed |= set(range(self.world)) - {self.rank}
        return [self.rank]

    def meet(self, name: str, timeout_s: float | None = None) -> list[int]:
        """Arrive at meeting ``name``; wait until every rank that has not
        already failed has arrived, or the deadline passes."""
        try:
            return self._meet(name, timeout_s)
        except (RuntimeError, OSError):  # DistNetworkError derives from RuntimeError
            return self._lost_store()

    def _meet(self, name: str, timeout_s: float | None) -> list[int]:
        self.store.set(self._key(name, f"rank{self.rank}"), "1")
        expected = self.world - len(self.failed)
        self.store.add(self._key(name, "count"), 1)
        deadline = time.monotonic() + (self.timeout_s if timeout_s is None else timeout_s)
        pause = 1e-4
        while True:
            if self.store.add(self._key(name, "count"), 0) >= expected:
                break
            if time.monotonic() > deadline:
                break
            time.sleep(pause)
            pause = min(pause * 2, 0.01)
        keys = [self._key(name, f"rank{r}") for r in range(self.world)]
        arrived = [r for r, k in enumerate(keys) if r == self.rank or self.store.check([k])]
        self.failed |= set(range(self.world)) - set(arrived)
        return arrived

    def gather(self, name: str, value, timeout_s: float | None = None) -> dict[int, object] | None:
        """Publish ``value`` and meet; rank 0 receives {rank: value} of the
        ranks that arrived, the others None."""
        try:
            self.store.set(self._key(name, f"value{self.rank}"), json.dumps(value))
        except (RuntimeError, OSError):
            self._lost_store()
            return {self.rank: value} if self.rank == 0 else None
        arrived = self.meet(name, timeout_s)
        if self.rank != 0:
            return None
        return {r: json.loads(self.store.get(self._key(name, f"value{r}"))) for r in arrived}

    def close(self, timeout_s: float = 30.0) -> None:
        """Leave the group. The rank hosting the store waits (up to
        ``timeout_s``) until every rank still counted alive has left, so no
        rank loses the store while it is still using it."""
        try:
            if not self.hosting:
                self.store.set(self._key("close", f"left{self.rank}"), "1")
                return
            deadline = time.monotonic() + timeout_s
            others = [r for r in range(self.world) if r != self.rank and r not in self.failed]
            while others and time.monotonic() < deadline:
                others = [r for r in others if not self.store.check([self._key("close", f"left{r}")])]
                time.sleep(0.001)
        except (RuntimeError, OSError):
            pass
