"""Lock-step driver for multi-rank serving (one process per GPU).

The reference drives every rank from one process with one worker thread per GPU and a host barrier
after each forward (src/distributed/tp_runtime.cpp:92-150, 378-420). Here each GPU has its own
process and its own copy of the deterministic scheduler; before each step rank 0 broadcasts, over a
CPU (gloo) group, the requests added, aborted or finished on the host since the previous step: a
two-word header (payload bytes, stop) and, only when something changed, the pickled commands. A
steady decode step therefore costs one 16-byte broadcast (51 us on two local gloo ranks, against
161 us for broadcast_object_list, which always sends a size and a payload).
Every rank then applies the same commands in the same order and runs the same step, so the
schedules, the collectives and the sampled tokens stay identical without any per-step device sync.
Followers wait with a bounded timeout; rank 0 sends a heartbeat while idle.

Failure detection (parallel/health.py): every rank publishes a heartbeat into the process group's
store; before each control collective a rank checks its peers' heartbeats and raises RankFailure
instead of entering a collective that a dead peer will never join. A peer that is alive but stuck
is caught by the control group's timeout, and the error names the stalled rank. VMC_FAULT injects
host-side faults at step boundaries for testing.
"""
from __future__ import annotations

import pickle
import time
from dataclasses import asdict
from datetime import timedelta

import torch
import torch.distributed as dist

from ..core.sampling_params import FinishReason, SamplingParams
from .health import FaultPlan, Heartbeats, RankFailure


class StepDriver:
    def __init__(self, engine, heartbeat_s: float = 0.05, timeout_s: float = 300.0, peer_timeout_s: float = 10.0,
                 faults: FaultPlan | None = None):
        self.engine = engine
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        self.timeout_s = timeout_s
        self.group = dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))
        self.heartbeat_s = heartbeat_s
        self._finish: list[tuple[str, int]] = []
        self.stopped = False
        self.faults = faults if faults is not None else FaultPlan.from_env()
        self.health = None
        self._hdr = torch.zeros(2, dtype=torch.int64)  # control header: payload bytes, stop
        if self.world > 1:
            store = dist.distributed_c10d._get_default_store()
            # progress = control collectives entered: a peer behind us never joined the current one
            self.health = Heartbeats(store, self.rank, self.world, interval_s=min(0.2, peer_timeout_s / 10),
                                     timeout_s=peer_timeout_s, progress=lambda: self.ncoll)
    ncoll = 0

    # every rank, before each control collective ------------------------------------------------
    def _pre_collective(self) -> None:
        if self.faults is not None:
            step = self.engine.step_id
            if self.faults.due(self.rank, step) is not None:
                # an injected departure happens between steps: no kernel of this rank in flight
                self.engine.quiesce()
            self.faults.fire(self.rank, step)
        if self.health is not None:
            self.health.check()

    def _broadcast(self, cmds: dict | None) -> dict:
        """One control exchange: rank 0 passes its commands, followers pass None; every rank returns
        rank 0's commands."""
        self._pre_collective()
        self.ncoll += 1
        try:
            return self._exchange(cmds)
        except RuntimeError as e:  # the control group's timeout, or a peer's connection went away
            self._diagnose(e)
            raise

    def _exchange(self, cmds: dict | None) -> dict:
        hdr = self._hdr
        if self.rank == 0:
            busy = cmds["add"] or cmds["abort"] or cmds["finish"]
            payload = pickle.dumps(cmds, protocol=pickle.HIGHEST_PROTOCOL) if busy else b""
            hdr[0], hdr[1] = len(payload), int(cmds["stop"])
        dist.broadcast(hdr, src=0, group=self.group)
        n, stop = int(hdr[0]), bool(hdr[1])
        if n == 0:
            return cmds if self.rank == 0 else {"add": [], "abort": [], "finish": [], "stop": stop}
        buf = (torch.frombuffer(bytearray(payload), dtype=torch.uint8) if self.rank == 0
               else torch.empty(n, dtype=torch.uint8))
        dist.broadcast(buf, src=0, group=self.group)
        return cmds if self.rank == 0 else pickle.loads(buf.numpy().tobytes())

    def _diagnose(self, e: BaseException) -> None:
        """After a failed control collective: name the peer that died (its heartbeat goes stale
        within the peer timeout) or that is alive but never joined this collective."""
        if self.health is None:
            return
        deadline = time.time() + self.health.timeout_s + 1.0
        while True:
            try:
                self.health.check()
            except RankFailure as f:
                raise f from e
            behind = [r for r in range(self.world)
                      if r != self.rank and (hb := self.health.read(r)) is not None and hb[1] < self.ncoll]
            if time.time() >= deadline:
                if behind:
                    raise RankFailure(behind[0], f"is alive but stopped taking steps ({e})") from e
                return
            time.sleep(0.05)

    # rank 0 ----------------------------------------------------------------------------------
    def finish(self, request_id: str, reason: FinishReason) -> None:
        self._finish.append((request_id, int(reason)))

    def _collect(self) -> dict:
        eng = self.engine
        with eng._lock:
            pend = list(eng._pending)
            aborts = list(eng._aborts)
        adds = [(r.request_id, r.prompt_token_ids, asdict(r.params)) for r in pend]
        fin, self._finish = self._finish, []
        return {"add": adds, "abort": aborts, "finish": fin, "stop": self.stopped}

    def step(self) -> None:
        """Rank 0: broadcast this step's commands, then step (or idle-wait) like the followers."""
        eng = self.engine
        if not eng.has_unfinished() and not self._finish and not self.stopped:
            time.sleep(self.heartbeat_s)
        cmds = self._broadcast(self._collect())
        self._apply_finish(cmds)
        if eng.has_unfinished():
            eng.step()

    def shutdown(self) -> None:
        self.stopped = True
        self._exchange({"add": [], "abort": [], "finish": [], "stop": True})
        self.close()

    def close(self) -> None:
        if self.health is not None:
            self.health.stop()

    # followers ---------------------------------------------------------------------------------
    def follow(self) -> None:
        eng = self.engine
        while True:
            cmds = self._broadcast(None)
            if cmds["stop"]:
                self.close()
                break
            for rid, prompt, params in cmds["add"]:
                eng.add_request(prompt, SamplingParams(**params), request_id=rid)
            for rid in cmds["abort"]:
                eng.abort_request(rid)
            self._apply_finish(cmds)
            if eng.has_unfinished():
                eng.step()

    def _apply_finish(self, cmds) -> None:
        for rid, reason in cmds["finish"]:
            self.engine.finish_request(rid, FinishReason(reason))
