"""Serving the hybrid Qwen3.5-MoE family (models/qwen35.py) on one GPU: a tiny random checkpoint of
every tensor of the family, four requests whose prompts span several chunked-prefill steps (so the
gated delta-net layers resume from their slot state) and then decode, teacher-forced against the fp32
oracle of tests/ref_qwen35.py along the engine's own greedy tokens. (Measured: 1-2% relative logit
error on compared rows; chunked, unchunked and one-request-at-a-time serving give the same rows.)"""
import numpy as np
import pytest
import torch

import ref_qwen35 as R
from vm_c_b200.core.sampling_params import SamplingParams
from vm_c_b200.gguf.random_init import preset, write_random_gguf

pytestmark = pytest.mark.gpu

LOGIT_BOUND = 0.05   # bf16 activations through three recurrent layers and one attention layer
# A router gap below this (relative to the largest router logit) may pick the other expert in bf16.
# In this family the recurrent state carries such a flip into every later token of the request, so a
# request is compared only up to its first output row with a near-tie at any layer.
ROUTER_TIE = 0.03


def test_tiny_qwen35moe_serves_and_matches_oracle(tmp_path):
    from vm_c_b200.gguf.reader import GgufSource
    from vm_c_b200.llm import LLM
    p = str(tmp_path / "tiny-qwen35moe.gguf")
    write_random_gguf(p, preset("tiny-qwen35moe"), "Q8_0", seed=0)
    llm = LLM(p, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=64, num_gpu_blocks=128)
    rows = []
    llm.engine.logits_hook = lambda ids, lg: rows.append((ids, lg))
    rng = np.random.default_rng(2)
    cfg = llm.cfg.model
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (5, 40, 17, 100)]
    outs = llm.generate(prompts, SamplingParams.greedy_params(max_tokens=8, ignore_eos=True))
    llm.shutdown()
    assert all(len(o.output_token_ids) == 8 for o in outs)
    got = {}
    for ids, lg in rows:
        for k, i in enumerate(ids):
            got.setdefault(i, []).append(lg[k])
    src = GgufSource(p)
    W = R.load(src)
    worst, flips, tied, compared = 0.0, 0, 0, 0
    for idx, (pr, o) in enumerate(zip(prompts, outs)):
        margins = []
        ref = R.forward(W, cfg, pr + o.output_token_ids[:-1], R.new_state(cfg), margins)[len(pr) - 1:]
        keep = torch.cumprod((torch.stack(margins).min(0).values[len(pr) - 1:] >= ROUTER_TIE).int(), 0).bool()
        tied += int((~keep).sum())
        mine = torch.stack(got[sorted(got)[idx]])[keep]
        ref = ref[keep]
        if ref.shape[0] == 0:
            continue
        compared += ref.shape[0]
        scale = ref.abs().max(-1).values
        worst = max(worst, float(((mine - ref).abs().max(-1).values / scale).max()))
        top2 = torch.topk(ref, 2, -1).values
        decided = (top2[:, 0] - top2[:, 1]) > 0.05 * scale
        flips += int(((mine.argmax(-1) != ref.argmax(-1)) & decided).sum())
    assert compared >= 8, (compared, tied)
    assert worst < LOGIT_BOUND and flips == 0, (worst, flips, tied)
