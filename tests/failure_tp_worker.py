"""Worker of the tensor-parallel departure test (two GPUs, launched by torch.distributed.run): both
ranks serve through the lock-step driver with the fused peer-memory backend (CUDA IPC peer loads and
stores; no multicast objects, NCCL with NVLS off); VMC_FAULT makes one rank leave between two steps
(after draining its device work). The surviving rank must stop with RankFailure naming the departed
rank before it launches the next step, with no device wait timed out and a usable CUDA context."""
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from vm_c_b200 import ops  # noqa: E402
from vm_c_b200.core.sampling_params import SamplingParams  # noqa: E402
from vm_c_b200.llm import LLM  # noqa: E402
from vm_c_b200.parallel.comm import init_distributed  # noqa: E402
from vm_c_b200.parallel.driver import StepDriver  # noqa: E402
from vm_c_b200.parallel.fused import FusedComm  # noqa: E402
from vm_c_b200.parallel.health import RankFailure  # noqa: E402


def main():
    model, out = sys.argv[1], sys.argv[2]
    rank, world, local = init_distributed(timeout_s=30)
    torch.cuda.set_device(local)
    comm = FusedComm()
    llm = LLM(model, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256, num_gpu_blocks=256,
              tp_rank=rank, tp_size=world, comm=comm, device=f"cuda:{local}")
    eng = llm.engine
    drv = StepDriver(eng, heartbeat_s=0.01, timeout_s=10.0, peer_timeout_s=3.0)
    res = {"rank": rank, "error": None, "failed_rank": None, "steps": 0, "launches_after": 0}
    t0 = time.time()
    try:
        if rank == 0:
            for n in (5, 40, 17):
                eng.add_request(list(range(1, n + 1)), SamplingParams.greedy_params(max_tokens=40, ignore_eos=True))
            while eng.has_unfinished():
                drv.step()
            drv.shutdown()
        else:
            drv.follow()
    except RankFailure as e:
        res["error"], res["failed_rank"] = "RankFailure", e.rank
        launches = llm.runner.launch_count
        eng.quiesce()   # only this rank's own completed work: nothing new is launched
        res["launches_after"] = llm.runner.launch_count - launches
    except Exception as e:  # noqa: BLE001
        res["error"] = f"{type(e).__name__}: {e}"
    torch.cuda.synchronize()
    res["steps"] = eng.step_id
    res["device_error"] = comm.device_error()
    res["gemm_error"] = ops.device_error(f"cuda:{local}")
    x = torch.ones(1024, device=f"cuda:{local}")
    res["context_ok"] = float((x * 2).sum().item()) == 2048.0
    res["t"] = time.time() - t0
    with open(out + f".{rank}", "w") as f:
        json.dump(res, f)
    os._exit(0)   # no NCCL teardown with a departed peer


if __name__ == "__main__":
    main()
