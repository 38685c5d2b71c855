"""Engine logic on the CPU with a deterministic fake model runner (next token = (last + 1) % V)."""
import numpy as np
import pytest

from vm_c_b200.config import VmCConfig
from vm_c_b200.core.engine import LLMEngine, ModelRunner
from vm_c_b200.core.sampling_params import FinishReason, SamplingParams


class FakeRunner(ModelRunner):
    def __init__(self, blocks=256, V=100):
        self.num_kv_blocks = blocks
        self.max_model_len = 512
        self.V = V
        self.steps = []

    def execute(self, meta, counts, params, penalties=None):
        self.steps.append(counts)
        L = self.layout
        ids = meta[L.off_input_ids:L.off_input_ids + counts.T]
        lidx = meta[L.off_logits_idx:L.off_logits_idx + counts.S]
        toks = ((ids[lidx] + 1) % self.V).astype(np.int32)
        return toks, np.zeros(counts.S, np.float32)

    def bind_layout(self, layout):
        self.layout = layout


def make(budget=64, seqs=8, blocks=256):
    cfg = VmCConfig()
    cfg.model.vocab = 100
    cfg.model.max_model_len = 512
    cfg.model.eos_token_ids = [99]
    cfg.scheduler.max_num_seqs = seqs
    cfg.scheduler.max_num_batched_tokens = budget
    cfg.finalize()
    return LLMEngine(cfg, FakeRunner(blocks))


def test_generate_counts_and_values():
    eng = make()
    outs = eng.generate([[1, 2, 3], [50]], SamplingParams.greedy_params(max_tokens=5))
    assert outs[0].output_token_ids == [4, 5, 6, 7, 8]
    assert outs[1].output_token_ids == [51, 52, 53, 54, 55]
    assert all(o.finished and o.finish_reason == FinishReason.LENGTH for o in outs)


def test_eos_and_ignore_eos():
    eng = make()
    out = eng.generate([[96]], SamplingParams.greedy_params(max_tokens=10))[0]
    assert out.output_token_ids == [97, 98, 99] and out.finish_reason == FinishReason.STOP
    out = eng.generate([[96]], SamplingParams.greedy_params(max_tokens=5, ignore_eos=True))[0]
    assert out.output_token_ids == [97, 98, 99, 0, 1]


def test_many_requests_chunked_prefill_continuous_batching():
    eng = make(budget=32, seqs=4, blocks=64)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 90, int(n)).tolist() for n in rng.integers(1, 60, 12)]
    outs = eng.generate(prompts, SamplingParams.greedy_params(max_tokens=7, ignore_eos=True))
    for p, o in zip(prompts, outs):
        exp = [(p[-1] + 1 + i) % 100 for i in range(7)]
        assert o.output_token_ids == exp
    assert max(c.T for c in eng.runner.steps) <= 32
    assert eng.sched.num_running == 0 and eng.bm.num_free_blocks == 63


def test_abort_and_stream_callback():
    eng = make()
    seen = []

    def cb(req, toks, fin):
        seen.append((list(toks), fin))

    eng.add_request([1, 2], SamplingParams.greedy_params(max_tokens=50, ignore_eos=True), request_id="a",
                    stream_callback=cb)
    for _ in range(3):
        eng.step()
    eng.abort_request("a")
    eng.step()
    assert seen[-1][1] is True and not eng.has_unfinished()
    assert [t for s in seen for t in s[0]][:2] == [3, 4]


def test_rejects_out_of_vocab():
    eng = make()
    with pytest.raises(ValueError):
        eng.add_request([100])
