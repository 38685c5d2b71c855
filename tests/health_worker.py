"""Worker for the host-side failure-detection tests: two gloo ranks on the CPU run the lock-step
driver over an engine with a fake model runner; VMC_FAULT injects the failure on one rank."""
import json
import os
import sys
import time
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import numpy as np  # noqa: E402
import torch.distributed as dist  # noqa: E402

from vm_c_b200.config import VmCConfig  # noqa: E402
from vm_c_b200.core.engine import LLMEngine, ModelRunner  # noqa: E402
from vm_c_b200.core.sampling_params import SamplingParams  # noqa: E402
from vm_c_b200.parallel.driver import StepDriver  # noqa: E402
from vm_c_b200.parallel.health import RankFailure  # noqa: E402


class FakeRunner(ModelRunner):
    def __init__(self):
        self.num_kv_blocks = 256
        self.max_model_len = 512

    def bind_layout(self, layout):
        self.layout = layout

    def execute(self, meta, counts, params, penalties=None):
        time.sleep(0.02)
        L = self.layout
        ids = meta[L.off_input_ids:L.off_input_ids + counts.T]
        lidx = meta[L.off_logits_idx:L.off_logits_idx + counts.S]
        return ((ids[lidx] + 1) % 100).astype(np.int32), np.zeros(counts.S, np.float32)


def main():
    out = sys.argv[1]
    dist.init_process_group("gloo", timeout=timedelta(seconds=20))
    rank = dist.get_rank()
    cfg = VmCConfig()
    cfg.model.vocab = 100
    cfg.model.max_model_len = 512
    cfg.model.eos_token_ids = [99]
    cfg.finalize()
    eng = LLMEngine(cfg, FakeRunner())
    drv = StepDriver(eng, heartbeat_s=0.01, timeout_s=float(os.environ.get("CTRL_TIMEOUT", "4")), peer_timeout_s=1.5)
    res = {"rank": rank, "error": None, "failed_rank": None, "steps": 0, "t": 0.0}
    t0 = time.time()
    try:
        if rank == 0:
            eng.add_request([1, 2, 3], SamplingParams.greedy_params(max_tokens=40, ignore_eos=True))
            while eng.has_unfinished():
                drv.step()
            drv.shutdown()
        else:
            drv.follow()
    except RankFailure as e:
        res["error"], res["failed_rank"] = "RankFailure", e.rank
    except Exception as e:  # noqa: BLE001
        res["error"] = type(e).__name__
    res["steps"] = eng.step_id
    res["t"] = time.time() - t0
    with open(out + f".{rank}", "w") as f:
        json.dump(res, f)
    os._exit(0)


if __name__ == "__main__":
    main()
