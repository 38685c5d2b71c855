"""The tensor-parallel reduce-scatter / all-gather flag protocol of the fused TP path (comm.cu
rs_norm_ag_kernel with the GEMM scatter epilogue), run on the CPU with ranks and CTAs as threads and
the PTX release / acquire operations as C++ atomics (csrc/host/tp_protocol_sim.cpp), built with
ThreadSanitizer. Counters, targets and buffers are reused across many calls, as on the GPU; the
result must equal a serial computation and ThreadSanitizer must see a happens-before edge for every
reuse. Three deliberate weakenings of the protocol must each be caught."""
import json
import subprocess

import pytest

from vm_c_b200._build import build_protocol_sim


@pytest.fixture(scope="module")
def exe():
    return str(build_protocol_sim())


@pytest.mark.parametrize("ranks,ctas,layers,seed", [(2, 1, 20, 1), (2, 3, 20, 2), (4, 2, 20, 3), (8, 4, 12, 4),
                                                    (8, 1, 12, 5), (3, 8, 10, 6), (8, 8, 6, 7)])
def test_protocol_exact_and_race_free(exe, ranks, ctas, layers, seed):
    r = subprocess.run([exe, str(ranks), str(ctas), str(layers), str(seed)], capture_output=True, text=True,
                       timeout=300, env={"TSAN_OPTIONS": "halt_on_error=0 exitcode=66"})
    assert "ThreadSanitizer" not in r.stderr, r.stderr[-3000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert r.returncode == 0 and out["ok"] and out["mismatches"] == 0, (r.stdout, r.stderr[-2000:])


@pytest.mark.parametrize("mutation", ["relaxed-signal", "no-ag-wait", "early-advance"])
def test_weakened_protocol_is_caught(exe, mutation):
    r = subprocess.run([exe, "4", "2", "10", "1", mutation], capture_output=True, text=True, timeout=300,
                       env={"TSAN_OPTIONS": "halt_on_error=0 exitcode=66"})
    assert r.returncode != 0 and ("ThreadSanitizer" in r.stderr or '"ok": false' in r.stdout), (r.stdout, r.stderr)
