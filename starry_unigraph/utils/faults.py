"""Host-side failure injection and detection (the reference has none: failures
surface as Python exceptions, and a rank that leaves blocks the others in the
next collective forever).

* ``FaultInjector``: ``SU_FAULT="rank:step:kind[,rank:step:kind...]"`` makes the
  named rank fail at the start of the named step. Kinds: ``raise`` (Python
  exception), ``exit`` (the process ends without cleanup), ``hang`` (the rank
  stops taking steps: it sleeps ``SU_FAULT_HANG_S`` seconds, default 3600), and
  ``delay:<seconds>``. Faults act between steps only, never inside a kernel or
  a collective.
* ``Heartbeat``: every rank stamps ``su_hb/<rank>`` in the process group's store;
  ``check()`` raises ``PeerFailure`` naming the ranks whose stamp is older than
  the timeout, so survivors stop before their next collective instead of
  waiting in it.
* Collective timeouts: ``dist.timeout_s`` bounds every process-group call, so a
  rank stuck in a collective with a dead peer gets an error.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass
from typing import Any


class InjectedFault(RuntimeError):
    pass


class PeerFailure(RuntimeError):
    pass


@dataclass
class _Fault:
    rank: int
    step: int
    kind: str


class FaultInjector:
    def __init__(self, faults: list[_Fault]):
        self.faults = faults

    @classmethod
    def from_env(cls, var: str = "SU_FAULT") -> "FaultInjector":
        spec = os.environ.get(var, "").strip()
        faults: list[_Fault] = []
        for item in filter(None, (x.strip() for x in spec.split(","))):
            parts = item.split(":")
            if len(parts) < 3:
                raise ValueError(f"bad {var} entry {item!r}; expected rank:step:kind")
            faults.append(_Fault(int(parts[0]), int(parts[1]), ":".join(parts[2:])))
        return cls(faults)

    def __bool__(self) -> bool:
        return bool(self.faults)

    def maybe_inject(self, rank: int, step: int) -> None:
        for f in self.faults:
            if f.rank != rank or f.step != step:
                continue
            if f.kind == "raise":
                raise InjectedFault(f"injected failure on rank {rank} at step {step}")
            if f.kind == "exit":
                os._exit(17)
            if f.kind == "hang":
                time.sleep(float(os.environ.get("SU_FAULT_HANG_S", "3600")))
            elif f.kind.startswith("delay:"):
                time.sleep(float(f.kind.split(":", 1)[1]))
            else:
                raise ValueError(f"unknown fault kind {f.kind!r}")


class Heartbeat:
    def __init__(self, store: Any, rank: int, world_size: int, timeout_s: float = 30.0, prefix: str = "su_hb"):
        self.store, self.rank, self.world, self.timeout = store, int(rank), int(world_size), float(timeout_s)
        self.prefix = prefix
        self._started = time.time()

    def beat(self, step: int) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", f"{time.time():.6f}:{int(step)}")

    def check(self) -> None:
        now = time.time()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                stamp = self.store.get(f"{self.prefix}/{r}").decode()
                t = float(stamp.split(":")[0])
            except Exception:
                t = self._started  # never beat yet: count from our own start
            if now - t > self.timeout:
                dead.append(r)
        if dead:
            raise PeerFailure(f"no heartbeat from rank(s) {dead} for more than {self.timeout:.1f} s")
