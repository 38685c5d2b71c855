"""Concurrency stress on the host (no GPU): eight producer threads add requests and abort a third of
them while the server's engine thread steps. The engine owns the scheduler alone; producers only
append to its locked command queues. Checked: one final callback per request, exact tokens for
completed requests, a correct prefix for aborted ones, and every KV block released at the end."""
import threading
import time

import numpy as np

from vm_c_b200.core.sampling_params import FinishReason, SamplingParams
from vm_c_b200.server.http import EngineLoop

from test_engine_cpu import make


def test_producers_and_aborts_against_the_engine_thread():
    eng = make(budget=48, seqs=6, blocks=64)
    loop = EngineLoop(eng, poll_s=0.001, step_timeout_s=0)
    loop.start()
    lock = threading.Lock()
    got: dict[str, list[int]] = {}
    finals: dict[str, list] = {}
    expect: dict[str, list[int]] = {}
    aborted: set[str] = set()

    def cb(req, toks, fin):
        with lock:
            got.setdefault(req.request_id, []).extend(toks)
            if fin:
                finals.setdefault(req.request_id, []).append(req.finish_reason)

    def producer(p: int):
        rng = np.random.default_rng(p)
        for i in range(25):
            rid = f"p{p}-{i}"
            prompt = rng.integers(0, 90, int(rng.integers(1, 40))).tolist()
            n = int(rng.integers(1, 12))
            with lock:
                expect[rid] = [(prompt[-1] + 1 + j) % 100 for j in range(n)]
            eng.add_request(prompt, SamplingParams.greedy_params(max_tokens=n, ignore_eos=True), request_id=rid,
                            stream_callback=cb)
            loop.wake()
            if rng.random() < 0.33:
                if rng.random() < 0.5:  # the other half is aborted at once, so that some aborts land early
                    time.sleep(float(rng.random()) * 0.003)
                with lock:
                    aborted.add(rid)
                eng.abort_request(rid)
            time.sleep(float(rng.random()) * 0.001)

    threads = [threading.Thread(target=producer, args=(p,)) for p in range(8)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    deadline = time.time() + 60
    while time.time() < deadline:
        with lock:
            if len(finals) == len(expect):
                break
        time.sleep(0.01)
    loop.shutdown()
    loop.join(timeout=10)
    assert loop.error is None
    assert len(finals) == len(expect) == 200
    assert all(len(v) == 1 for v in finals.values())  # exactly one final callback per request
    for rid, want in expect.items():
        toks = got.get(rid, [])
        if finals[rid][0] == FinishReason.ABORTED:
            assert rid in aborted and toks == want[:len(toks)], rid
        else:
            assert finals[rid][0] == FinishReason.LENGTH and toks == want, rid
    n_ab = sum(v[0] == FinishReason.ABORTED for v in finals.values())
    assert n_ab > 0, "no abort landed before its request finished"
    assert not eng.has_unfinished() and eng.sched.num_running == 0
    assert eng.bm.num_free_blocks == 63
