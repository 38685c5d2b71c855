"""Penalty metadata of the engine on the CPU: rows of requests with repetition / frequency / presence
penalties reach the runner as CSR triples (row, token, count of that token in the output so far;
prompt tokens appear with count 0), rows without penalties are left out, and once no running request
uses penalties the runner gets None (the graph-replay path)."""
import numpy as np

from vm_c_b200.config import VmCConfig
from vm_c_b200.core.engine import LLMEngine, ModelRunner
from vm_c_b200.core.sampling_params import SamplingParams

V = 50


class RecordingRunner(ModelRunner):
    """Next token = (last + 1) % V; records the sample ids order and the penalty triples of each step."""

    def __init__(self):
        self.num_kv_blocks = 64
        self.max_model_len = 256
        self.seen = []

    def bind_layout(self, layout):
        self.layout = layout

    def execute(self, meta, counts, params, penalties=None):
        L = self.layout
        lidx = meta[L.off_logits_idx:L.off_logits_idx + counts.S]
        ids = meta[L.off_input_ids + lidx]
        self.seen.append(None if penalties is None else tuple(np.asarray(a).copy() for a in penalties))
        return ((ids + 1) % V).astype(np.int32), np.zeros(counts.S, np.float32)


def test_penalty_rows_and_counts():
    cfg = VmCConfig()
    cfg.model.vocab = V
    cfg.model.max_model_len = 256
    cfg.model.eos_token_ids = [V - 1]
    cfg.finalize()
    r = RecordingRunner()
    eng = LLMEngine(cfg, r)
    plain = eng.add_request([3, 4], SamplingParams.greedy_params(max_tokens=12, ignore_eos=True))
    pen = eng.add_request([10, 10, 11], SamplingParams(temperature=0.0, top_k=1, repetition_penalty=1.3,
                                                       max_tokens=4, ignore_eos=True))
    steps = []
    while eng.has_unfinished():
        before = {plain.request_id: list(plain.output_token_ids), pen.request_id: list(pen.output_token_ids)}
        n = len(r.seen)
        eng.step()
        if len(r.seen) > n:
            steps.append((before, r.seen[-1]))
    with_pen = [(b, p) for b, p in steps if p is not None]
    assert len(with_pen) == 4  # one sampled token per step while the penalised request runs
    for before, (rows, toks, cnts) in with_pen:
        assert len(set(rows.tolist())) == 1  # only the penalised request's row
        out = before[pen.request_id]
        want = {t: 0 for t in pen.prompt_token_ids}
        for t in out:
            want[t] = want.get(t, 0) + 1
        assert dict(zip(toks.tolist(), cnts.tolist())) == want
    # after it finished, the remaining steps carry no penalties
    last_pen = max(i for i, (_, p) in enumerate(steps) if p is not None)
    assert all(p is None for _, p in steps[last_pen + 1:])
    assert len(steps) > last_pen + 1
    assert len(plain.output_token_ids) == 12 and len(pen.output_token_ids) == 4
