"""The fused reduce-scatter / all-gather of the row-parallel sites (scatter-epilogue GEMM +
rs_norm_ag) on 2, 4 and 8 GPUs: exact sums over bursts of back-to-back calls, normalised rows
gathered on every rank, and agreement with NCCL's all-reduce on the same partials; plus vocabulary-parallel
sampling against the single-GPU sampler on the whole rows (tests/comm_worker.py)."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("n", [2, 4, 8])
def test_reduce_scatter_all_gather_exact(tmp_path, n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    out = tmp_path / "comm.json"
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29633",
           os.path.join(HERE, "comm_worker.py"), str(out), "60", "25"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert r.returncode == 0, r.stderr[-3000:]
    s = json.load(open(out))
    assert s["err"] == 0
    assert s["calls"] == 60 * 25
    assert s["max_resid_err"] == 0.0          # integer partials: exact
    assert s["max_vs_nccl"] == 0.0
    assert s["max_h_rel_err"] < 1e-2          # bf16 output rounding
    assert s["sampler_mismatch"] == 0         # vocabulary-parallel sampling = whole-row sampling
    assert s["sampler_lp_err"] < 1e-3
