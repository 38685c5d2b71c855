"""A rank leaving a two-GPU tensor-parallel job between steps (tests/failure_tp_worker.py): the
departing rank drains its device work and exits on the host; the survivor detects the departure
through the control group / heartbeats before its next step, raises RankFailure naming the rank,
launches no further kernel (none of which could then touch the departed rank's IPC memory), and its
device error words stay clear with a working CUDA context. Peer access is plain CUDA IPC (no NVLink
multicast objects) and NCCL runs with NVLS off."""
import json
import os
import subprocess
import sys

import pytest
import torch

from vm_c_b200.gguf.random_init import preset, write_random_gguf

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_rank_leaves_between_steps(tmp_path):
    model = str(tmp_path / "tiny.gguf")
    write_random_gguf(model, preset("tiny-llama"), "Q8_0", seed=0)
    out = str(tmp_path / "res")
    # The two ranks are plain child processes with the rendezvous variables set here: under
    # torch.distributed.run the departing rank's exit would make the launcher stop the survivor too.
    procs = []
    for r in range(2):
        env = dict(os.environ, NCCL_NVLS_ENABLE="0", VMC_FAULT="exit:1:6", RANK=str(r), LOCAL_RANK=str(r),
                   WORLD_SIZE="2", LOCAL_WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT="29651")
        procs.append(subprocess.Popen(["timeout", "-k", "10", "180", sys.executable,
                                       os.path.join(HERE, "failure_tp_worker.py"), model, out], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    logs = [p.communicate()[0] for p in procs]
    assert procs[1].returncode == 3, logs[1][-2000:]   # the injected departure's exit status
    assert os.path.exists(out + ".0"), logs[0][-3000:]
    r0 = json.load(open(out + ".0"))
    assert not os.path.exists(out + ".1")   # the departed rank wrote nothing
    assert r0["error"] == "RankFailure" and r0["failed_rank"] == 1, r0
    assert 5 <= r0["steps"] <= 7             # the survivor stopped at the departure
    assert r0["launches_after"] == 0
    assert r0["device_error"] == 0 and r0["gemm_error"] == 0
    assert r0["context_ok"]
