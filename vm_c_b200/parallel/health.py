"""Failure detection for multi-rank serving: rank heartbeats, a step watchdog and host-side fault
injection.

The reference has none of this (no timeouts; a failed step is logged and retried after 100 ms,
src/main.cpp:829-832). Here:

* ``Heartbeats``: every rank's thread publishes (wall time, engine step) into the process group's
  key-value store every ``interval_s``; ``check()`` raises :class:`RankFailure` when a peer's entry
  is older than ``timeout_s`` (the peer process is gone) — the driver calls it before each control
  collective, so the survivors stop before their next launch instead of waiting in a collective.
  A peer that is alive but stuck (its step number does not move) is reported by ``stalled()``;
  the control group's short timeout ends the collective that waits for it.
* ``StepWatchdog``: a thread that flags an engine step running longer than ``timeout_s`` and calls
  a handler (the server fails the in-flight requests; a launcher may exit). It cannot interrupt
  device work: device-side waits are bounded in the kernels themselves and report through the
  device error word.
* ``FaultPlan``: ``VMC_FAULT="kind:rank:step[,...]"`` injects a failure on the host at a step
  boundary (never inside a step, so no kernel or collective is in flight): ``raise`` (the step
  raises), ``exit`` (the process exits with status 3), ``hang`` (the main thread stops taking
  steps; its heartbeat thread keeps running, so peers see a stall, not a death).
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass
from typing import Callable, Optional

from ..utils.logging import get_logger

log = get_logger("health")


class RankFailure(RuntimeError):
    def __init__(self, rank: int, what: str):
        super().__init__(f"rank {rank} {what}")
        self.rank = rank


class InjectedFault(RuntimeError):
    pass


# ------------------------------------------------------------------------------------------------
@dataclass
class Fault:
    kind: str
    rank: int
    step: int


class FaultPlan:
    KINDS = ("raise", "exit", "hang")

    def __init__(self, faults: list[Fault]):
        self.faults = faults

    @staticmethod
    def parse(spec: str) -> "FaultPlan":
        faults = []
        for part in filter(None, (p.strip() for p in (spec or "").split(","))):
            kind, rank, step = part.split(":")
            if kind not in FaultPlan.KINDS:
                raise ValueError(f"VMC_FAULT: unknown kind {kind!r} (one of {FaultPlan.KINDS})")
            faults.append(Fault(kind, int(rank), int(step)))
        return FaultPlan(faults)

    @staticmethod
    def from_env() -> Optional["FaultPlan"]:
        spec = os.environ.get("VMC_FAULT", "")
        return FaultPlan.parse(spec) if spec else None

    def due(self, rank: int, step: int) -> Optional[Fault]:
        for f in self.faults:
            if f.rank == rank and f.step == step:
                return f
        return None

    def fire(self, rank: int, step: int, hang_s: float = 3600.0) -> None:
        """Called by the driver between steps."""
        f = self.due(rank, step)
        if f is None:
            return
        log.error("injecting fault %s on rank %d at step %d", f.kind, rank, step)
        if f.kind == "raise":
            raise InjectedFault(f"injected fault on rank {rank} at step {step}")
        if f.kind == "exit":
            os._exit(3)
        time.sleep(hang_s)  # hang


# ------------------------------------------------------------------------------------------------
class Heartbeats:
    def __init__(self, store, rank: int, world: int, interval_s: float = 0.2, timeout_s: float = 5.0,
                 progress: Callable[[], int] = lambda: 0, prefix: str = "vmc/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval_s, self.timeout_s = interval_s, timeout_s
        self.progress = progress
        self.prefix = prefix
        self._stop = threading.Event()
        self._seen: dict[int, tuple[float, int, float]] = {}  # peer -> (their time, step, when step last moved)
        self._publish()
        self._thread = threading.Thread(target=self._run, daemon=True, name=f"heartbeat-{rank}")
        self._thread.start()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _publish(self) -> None:
        self.store.set(self._key(self.rank), f"{time.time():.6f} {int(self.progress())}")

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            try:
                self._publish()
            except Exception:  # the store went away with the job
                return

    def read(self, r: int) -> Optional[tuple[float, int]]:
        try:
            t, s = self.store.get(self._key(r)).decode().split()
            return float(t), int(s)
        except Exception:
            return None

    def check(self) -> None:
        """Raise RankFailure if a peer's heartbeat is older than the timeout (its process is gone)."""
        now = time.time()
        for r in range(self.world):
            if r == self.rank:
                continue
            hb = self.read(r)
            if hb is None:
                raise RankFailure(r, "has no heartbeat")
            age = now - hb[0]
            if age > self.timeout_s:
                raise RankFailure(r, f"heartbeat is {age:.1f} s old (timeout {self.timeout_s:.1f} s)")

    def stalled(self, for_s: float) -> list[int]:
        """Peers whose step number has not moved for `for_s` seconds while their heartbeat is live."""
        now = time.time()
        out = []
        for r in range(self.world):
            if r == self.rank:
                continue
            hb = self.read(r)
            if hb is None:
                continue
            prev = self._seen.get(r)
            if prev is None or prev[1] != hb[1]:
                self._seen[r] = (hb[0], hb[1], now)
            elif now - prev[2] > for_s and now - hb[0] <= self.timeout_s:
                out.append(r)
        return out

    def stop(self) -> None:
        self._stop.set()


# ------------------------------------------------------------------------------------------------
class StepWatchdog:
    """Flags an engine step that runs longer than `timeout_s` (checked every `poll_s`)."""

    def __init__(self, timeout_s: float, on_timeout: Callable[[int, float], None], poll_s: float = 0.5):
        self.timeout_s, self.on_timeout, self.poll_s = timeout_s, on_timeout, poll_s
        self._lock = threading.Lock()
        self._step: Optional[int] = None
        self._t0 = 0.0
        self._fired: Optional[int] = None
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True, name="step-watchdog")
        self._thread.start()

    def begin(self, step: int) -> None:
        with self._lock:
            self._step, self._t0 = step, time.monotonic()

    def end(self) -> None:
        with self._lock:
            self._step = None

    def _run(self) -> None:
        while not self._stop.wait(self.poll_s):
            with self._lock:
                step, t0 = self._step, self._t0
            if step is None or step == self._fired:
                continue
            dt = time.monotonic() - t0
            if dt > self.timeout_s:
                self._fired = step
                log.error("engine step %d has run for %.1f s (watchdog timeout %.1f s)", step, dt, self.timeout_s)
                try:
                    self.on_timeout(step, dt)
                except Exception:
                    log.exception("watchdog handler failed")

    def stop(self) -> None:
        self._stop.set()
