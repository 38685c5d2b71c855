"""Failure detection on the host (no GPU): fault plans, heartbeats, the step watchdog, and two gloo
ranks where one rank exits, raises or hangs between steps while the other must stop with an error
that names it instead of waiting."""
import json
import os
import socket
import subprocess
import sys
import threading
import time

import pytest
import torch.distributed as dist

from vm_c_b200.core.sampling_params import FinishReason
from vm_c_b200.parallel.health import FaultPlan, Heartbeats, InjectedFault, RankFailure, StepWatchdog

HERE = os.path.dirname(os.path.abspath(__file__))


def test_fault_plan_parse_and_fire():
    p = FaultPlan.parse("raise:1:3, exit:0:7,hang:2:1")
    assert [(f.kind, f.rank, f.step) for f in p.faults] == [("raise", 1, 3), ("exit", 0, 7), ("hang", 2, 1)]
    assert p.due(1, 3).kind == "raise" and p.due(1, 4) is None
    with pytest.raises(InjectedFault):
        p.fire(1, 3)
    p.fire(0, 3)  # nothing due
    t0 = time.time()
    p.fire(2, 1, hang_s=0.2)
    assert time.time() - t0 >= 0.2
    with pytest.raises(ValueError):
        FaultPlan.parse("explode:0:1")


def test_heartbeats_detect_dead_and_stalled_peers():
    store = dist.HashStore()
    step = {"v": 0}
    a = Heartbeats(store, 0, 2, interval_s=0.05, timeout_s=0.5)
    b = Heartbeats(store, 1, 2, interval_s=0.05, timeout_s=0.5, progress=lambda: step["v"])
    time.sleep(0.15)
    a.check()
    assert a.stalled(10.0) == []
    time.sleep(0.3)
    assert a.stalled(0.2) == [1]  # alive, but its step did not move
    step["v"] = 5
    time.sleep(0.15)
    assert a.stalled(0.2) == []
    b.stop()  # the peer dies
    time.sleep(0.8)
    with pytest.raises(RankFailure) as e:
        a.check()
    assert e.value.rank == 1
    a.stop()


def test_step_watchdog_fires_once_per_step():
    hits = []
    w = StepWatchdog(0.2, lambda s, dt: hits.append(s), poll_s=0.02)
    w.begin(1)
    time.sleep(0.05)
    w.end()
    w.begin(2)
    time.sleep(0.4)
    w.end()
    time.sleep(0.1)
    w.stop()
    assert hits == [2]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_pair(tmp_path, fault, ctrl_timeout=4, workload=""):
    out = str(tmp_path / "res")
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(r), WORLD_SIZE="2",
                   LOCAL_RANK=str(r), VMC_FAULT=fault, CTRL_TIMEOUT=str(ctrl_timeout), WORKLOAD=workload)
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "health_worker.py"), out], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    try:
        procs[0].wait(timeout=60)  # rank 0 must end on its own; a hung rank 1 is killed below
        try:
            procs[1].wait(timeout=5)
        except subprocess.TimeoutExpired:
            pass
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    res = {}
    for r in range(2):
        path = out + f".{r}"
        if os.path.exists(path):
            res[r] = json.load(open(path))
    return res, [p.returncode for p in procs]


def test_no_fault_runs_to_completion(tmp_path):
    res, codes = _run_pair(tmp_path, "")
    assert res[0]["error"] is None and res[1]["error"] is None
    assert res[0]["steps"] == res[1]["steps"] >= 40


def test_ranks_stay_in_lock_step(tmp_path):
    """Requests added over several steps, a client abort and a host-side finish reach the follower
    through the control header + payload exchange; both engines emit the same tokens and finishes."""
    res, codes = _run_pair(tmp_path, "", workload="mixed")
    assert res[0]["error"] is None and res[1]["error"] is None
    assert res[0]["steps"] == res[1]["steps"]
    outs = res[0]["outs"]
    assert set(outs) == {"a", "b", "c", "d", "e"}
    assert outs == res[1]["outs"]
    assert all(o[1] for o in outs.values())
    assert outs["c"][2] == int(FinishReason.LENGTH) and len(outs["c"][0]) == 12
    assert outs["a"][2] == int(FinishReason.STOP) and len(outs["a"][0]) < 30
    assert outs["d"][2] == int(FinishReason.ABORTED)


@pytest.mark.parametrize("kind", ["exit", "raise"])
def test_dead_peer_is_named(tmp_path, kind):
    res, codes = _run_pair(tmp_path, f"{kind}:1:5")
    assert res[0]["error"] == "RankFailure" and res[0]["failed_rank"] == 1
    assert res[0]["t"] < 15
    if kind == "exit":
        assert codes[1] == 3 and 1 not in res
    else:
        assert res[1]["error"] == "InjectedFault"


def test_hung_peer_is_named(tmp_path):
    res, codes = _run_pair(tmp_path, "hang:1:5", ctrl_timeout=3)
    assert res[0]["error"] == "RankFailure" and res[0]["failed_rank"] == 1
    assert res[0]["t"] < 20
