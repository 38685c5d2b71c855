"""Worker for the host-side failure-detection and lock-step tests: two gloo ranks on the CPU run the
lock-step driver over an engine with a fake model runner; VMC_FAULT injects the failure on one rank.
WORKLOAD=mixed makes rank 0 add requests over several steps, abort one and finish one on the host,
and every rank records what its engine emitted, so the test can check the ranks stayed identical."""
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
from vm_c_b200.core.sampling_params import FinishReason, SamplingParams  # noqa: E402
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
    outs = {}
    finish = eng._finish

    def recording_finish(req, reason, last_tokens=None):  # every way a request ends passes here
        finish(req, reason, last_tokens)
        outs[req.request_id] = [list(req.to_output().output_token_ids), True, int(reason)]
    eng._finish = recording_finish
    try:
        if rank == 0 and os.environ.get("WORKLOAD") == "mixed":
            greedy = lambda n: SamplingParams.greedy_params(max_tokens=n, ignore_eos=True)  # noqa: E731
            eng.add_request([1, 2, 3], greedy(30), request_id="a")
            eng.add_request([5] * 40, SamplingParams(temperature=0.9, top_k=20, max_tokens=25, ignore_eos=True),
                            request_id="b")
            for k in range(60):
                if k == 2:
                    eng.add_request([7, 8], greedy(12), request_id="c")
                    eng.add_request(list(range(10, 60)), greedy(40), request_id="d")
                if k == 5:
                    eng.abort_request("d")
                if k == 7:
                    drv.finish("a", FinishReason.STOP)
                if k == 9:
                    eng.add_request([9] * 3, greedy(8), request_id="e")
                if k > 9 and not eng.has_unfinished():
                    break
                drv.step()
            drv.shutdown()
        elif rank == 0:
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
    res["outs"] = outs
    res["t"] = time.time() - t0
    with open(out + f".{rank}", "w") as f:
        json.dump(res, f)
    os._exit(0)


if __name__ == "__main__":
    main()
