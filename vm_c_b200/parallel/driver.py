"""Lock-step driver for multi-rank serving (one process per GPU).

The reference drives every rank from one process with one worker thread per GPU and a host barrier
after each forward (src/distributed/tp_runtime.cpp:92-150, 378-420). Here each GPU has its own
process and its own copy of the deterministic scheduler; before each step rank 0 broadcasts, over a
CPU (gloo) group, the requests added, aborted or finished on the host since the previous step.
Every rank then applies the same commands in the same order and runs the same step, so the
schedules, the collectives and the sampled tokens stay identical without any per-step device sync.
Followers wait with a bounded timeout; rank 0 sends a heartbeat while idle.
"""
from __future__ import annotations

import time
from dataclasses import asdict
from datetime import timedelta

import torch.distributed as dist

from ..core.sampling_params import FinishReason, SamplingParams


class StepDriver:
    def __init__(self, engine, heartbeat_s: float = 0.05, timeout_s: float = 300.0):
        self.engine = engine
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        self.group = dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))
        self.heartbeat_s = heartbeat_s
        self._finish: list[tuple[str, int]] = []
        self.stopped = False

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
        cmds = self._collect()
        obj = [cmds]
        dist.broadcast_object_list(obj, src=0, group=self.group)
        self._apply_finish(cmds)
        if eng.has_unfinished():
            eng.step()

    def shutdown(self) -> None:
        self.stopped = True
        obj = [{"add": [], "abort": [], "finish": [], "stop": True}]
        dist.broadcast_object_list(obj, src=0, group=self.group)

    # followers ---------------------------------------------------------------------------------
    def follow(self) -> None:
        eng = self.engine
        while True:
            obj = [None]
            dist.broadcast_object_list(obj, src=0, group=self.group)
            cmds = obj[0]
            if cmds["stop"]:
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
