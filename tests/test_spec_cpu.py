"""Speculative-decoding bookkeeping on the CPU: engine routing, multi-token scheduler updates,
look-ahead reservation and stop handling, with a fake target (next token = (last + 1) % V) and a
fake draft that is wrong at chosen positions. Output must equal plain greedy decoding."""
import numpy as np

from vm_c_b200.config import VmCConfig
from vm_c_b200.core.engine import LLMEngine, ModelRunner
from vm_c_b200.core.sampling_params import FinishReason, SamplingParams

V = 100


class FakeSpec:
    """Proposes k tokens; the proposal at absolute position p is wrong when bad(p)."""

    def __init__(self, runner, k, bad):
        self.r, self.k, self.bad = runner, k, bad
        self.steps = self.shadows = 0
        self.positions = []
        self.forgotten = []

    def step(self, ids, counts):
        L, h = self.r.layout, self.r.meta
        qs = h[L.off_q_start:L.off_q_start + counts.R + 1]
        x0 = h[L.off_input_ids + qs[:-1]]
        p0 = h[L.off_positions + qs[:-1]]
        self.steps += 1
        out = []
        for i in range(counts.R):
            self.positions.append((int(ids[i]), int(p0[i]), int(x0[i])))
            tgt, drafts, t = [], [], int(x0[i])
            for j in range(self.k + 1):
                t = (t + 1) % V
                tgt.append(t)
            for j in range(self.k):
                drafts.append(tgt[j] if not self.bad(int(p0[i]) + 1 + j) else (tgt[j] + 7) % V)
            a = 0
            while a < self.k and drafts[a] == tgt[a]:
                a += 1
            out.append(drafts[:a] + [tgt[a]])
        return out

    def set_batch(self, ids):
        pass

    def shadow(self, counts):
        self.shadows += 1

    def forget(self, rid):
        self.forgotten.append(rid)


class FakeRunner(ModelRunner):
    def __init__(self, k, bad, blocks=256):
        self.num_kv_blocks = blocks
        self.max_model_len = 512
        self.num_lookahead_tokens = k
        self.spec = FakeSpec(self, k, bad)
        self.plain = 0

    def alloc_meta(self, total):
        self.meta = np.zeros(total, dtype=np.int32)
        return self.meta

    def bind_layout(self, layout):
        self.layout = layout

    def execute(self, meta, counts, params, penalties=None):
        self.plain += 1
        L = self.layout
        ids = meta[L.off_input_ids:L.off_input_ids + counts.T]
        lidx = meta[L.off_logits_idx:L.off_logits_idx + counts.S]
        return ((ids[lidx] + 1) % V).astype(np.int32), np.zeros(counts.S, np.float32)


def make(k=4, bad=lambda p: p % 5 == 0, blocks=256, seqs=8, budget=64):
    cfg = VmCConfig()
    cfg.model.vocab = V
    cfg.model.max_model_len = 512
    cfg.model.eos_token_ids = [99]
    cfg.scheduler.max_num_seqs = seqs
    cfg.scheduler.max_num_batched_tokens = budget
    cfg.finalize()
    return LLMEngine(cfg, FakeRunner(k, bad, blocks))


def test_outputs_equal_plain_greedy_and_positions_advance():
    eng = make()
    prompts = [[1, 2, 3], [10] * 17, [40, 41]]
    outs = eng.generate(prompts, SamplingParams.greedy_params(max_tokens=23, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert o.output_token_ids == [(p[-1] + 1 + i) % V for i in range(23)]
        assert o.finish_reason == FinishReason.LENGTH
    s = eng.runner.spec
    assert s.steps > 0 and eng.runner.plain >= 1
    assert s.steps < 3 * 22  # several tokens per speculative step
    # Every speculative step starts at the position of the request's last known token:
    # (x0 - p0) mod V identifies the prompt (1, 94 and 40 for the three prompts).
    by_req = {}
    for rid, p, x in s.positions:
        by_req.setdefault(rid, []).append((p, (x - p) % V))
    assert len(by_req) == 3
    for ps in by_req.values():
        pos = [p for p, _ in ps]
        assert pos == sorted(pos) and len(set(pos)) == len(pos)
        assert len({d for _, d in ps}) == 1 and ps[0][1] in (1, 94, 40)
    assert eng.sched.num_running == 0 and eng.bm.num_free_blocks == 255
    assert sorted(set(s.forgotten)) == sorted(by_req)


def test_all_accepted_and_none_accepted():
    for bad in (lambda p: False, lambda p: True):
        eng = make(k=3, bad=bad)
        out = eng.generate([[5, 6]], SamplingParams.greedy_params(max_tokens=17, ignore_eos=True))[0]
        assert out.output_token_ids == [(7 + i) % V for i in range(17)]


def test_stop_inside_accepted_run():
    eng = make(k=5, bad=lambda p: False)
    out = eng.generate([[90]], SamplingParams.greedy_params(max_tokens=40))[0]
    assert out.output_token_ids == list(range(91, 100)) and out.finish_reason == FinishReason.STOP
    out = eng.generate([[10]], SamplingParams.greedy_params(max_tokens=8, ignore_eos=True))[0]
    assert out.output_token_ids == list(range(11, 19)) and out.finish_reason == FinishReason.LENGTH
    assert eng.bm.num_free_blocks == 255


def test_sampled_requests_take_the_plain_path():
    eng = make(k=4, bad=lambda p: False)
    eng.generate([[1, 2]], SamplingParams(temperature=0.8, max_tokens=6, ignore_eos=True, seed=1))
    assert eng.runner.spec.steps == 0 and eng.runner.spec.shadows >= 6


def test_token_tree_layout():
    from vm_c_b200.speculative.tree import TokenTree
    t = TokenTree([2, 2, 1])
    assert t.N == 11 and t.D == 3
    assert t.parent.tolist() == [-1, 0, 0, 1, 1, 2, 2, 3, 4, 5, 6]
    assert t.depth.tolist() == [0, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3]
    assert [list(t.level(d)) for d in range(4)] == [[0], [1, 2], [3, 4, 5, 6], [7, 8, 9, 10]]
    m = [int(x) & ((1 << 64) - 1) for x in t.masks]
    assert m[0] == 1 and m[3] == 0b1011 and m[10] == (1 | 1 << 2 | 1 << 6 | 1 << 10)
    import pytest
    with pytest.raises(ValueError):
        TokenTree([8, 8])  # 73 nodes


def test_filtered_probs_matches_sampler_rules():
    import torch
    from vm_c_b200.speculative.draft import filtered_probs
    logits = torch.tensor([[2.0, 1.0, 0.5, 0.0, -1.0, -3.0]] * 5)
    temp = torch.tensor([1.0, 0.5, 1.0, 1.0, 0.0])
    top_k = torch.tensor([0, 0, 3, 0, 0])
    top_p = torch.tensor([1.0, 1.0, 1.0, 0.7, 1.0])
    min_p = torch.tensor([0.0, 0.0, 0.0, 0.0, 0.0])
    p = filtered_probs(logits, temp, top_k, top_p, min_p)
    assert torch.allclose(p[0], torch.softmax(logits[0], -1))
    assert torch.allclose(p[1], torch.softmax(logits[1] / 0.5, -1))
    want = torch.softmax(logits[2, :3], -1)
    assert torch.allclose(p[2, :3], want) and p[2, 3:].sum() == 0
    full = torch.softmax(logits[3], -1)  # 0.61, 0.22, ...: the top two reach 0.7
    assert torch.allclose(p[3, :2], full[:2] / full[:2].sum()) and p[3, 2:].sum() == 0
    assert p[4].tolist() == [1.0, 0, 0, 0, 0, 0]
    mp = filtered_probs(logits[:1], torch.tensor([1.0]), torch.tensor([0]), torch.tensor([1.0]), torch.tensor([0.3]))
    assert (mp[0] > 0).sum() == 2  # p_i >= 0.3 * p_max keeps the two largest
