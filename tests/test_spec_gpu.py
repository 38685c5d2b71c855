"""Draft-model speculative decoding on the sm_100a kernels (tiny llama, Q8_0): greedy output equals
plain greedy decoding of the target, with a perfect draft (the target itself) and with an unrelated
draft (acceptance near zero)."""
import numpy as np
import pytest

from vm_c_b200.core.sampling_params import SamplingParams
from vm_c_b200.gguf.random_init import preset, write_random_gguf
from vm_c_b200.gguf.reader import GgufSource

from ref_llama import forward_logits, load_dense

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("spec")
    tgt, other = str(d / "target.gguf"), str(d / "other.gguf")
    write_random_gguf(tgt, preset("tiny-llama"), "Q8_0", seed=0)
    write_random_gguf(other, preset("tiny-llama"), "Q8_0", seed=7)
    return tgt, other


def _gen(path, prompts, n, draft="", k=4):
    from vm_c_b200.llm import LLM
    llm = LLM(path, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256, num_gpu_blocks=256,
              enable_prefix_caching=False, draft_model=draft, num_speculative_tokens=k)
    outs = llm.generate(prompts, SamplingParams.greedy_params(max_tokens=n, ignore_eos=True))
    stats = llm.runner.spec.stats.as_dict() if llm.runner.spec is not None else None
    llm.shutdown()
    return [o.output_token_ids for o in outs], stats


def _same_up_to_ties(W, cfg, prompts, a, b):
    # The verification pass runs the prefill kernels and plain decoding the decode kernels, whose
    # fp32 sums round differently: trajectories agree until a step whose two candidates are within
    # that noise in the fp32 oracle.
    for p, x, y in zip(prompts, a, b):
        assert len(x) == len(y)
        i = next((j for j in range(len(x)) if x[j] != y[j]), None)
        if i is None:
            continue
        row = forward_logits(W, cfg, p + x[:i])[-1]
        gap = abs(float(row[x[i]] - row[y[i]]))
        assert gap < 0.05 * float(row.abs().max()), (i, x[i], y[i], gap)


@pytest.mark.parametrize("which", ["self", "other"])
def test_spec_equals_plain_greedy(models, which):
    tgt, other = models
    src = GgufSource(tgt)
    cfg = src.model_config()
    W = load_dense(src, cfg)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (7, 33, 16, 70, 3)]
    n = 24
    plain, _ = _gen(tgt, prompts, n)
    spec, st = _gen(tgt, prompts, n, draft=tgt if which == "self" else other, k=4)
    _same_up_to_ties(W, cfg, prompts, spec, plain)
    assert st["steps"] > 0
    if which == "self":
        assert st["acceptance_rate"] > 0.8, st
        assert st["tokens_per_step"] > 3.5, st
    else:
        assert st["acceptance_rate"] < 0.2, st


def _gen_tree(path, prompts, n, draft, tree):
    from vm_c_b200.llm import LLM
    llm = LLM(path, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256, num_gpu_blocks=256,
              enable_prefix_caching=False, draft_model=draft, spec_tree=tree)
    outs = llm.generate(prompts, SamplingParams.greedy_params(max_tokens=n, ignore_eos=True))
    stats = llm.runner.spec.stats.as_dict()
    llm.shutdown()
    return [o.output_token_ids for o in outs], stats


@pytest.mark.parametrize("which,tree", [("self", "2,2,1"), ("other", "3,2"), ("other", "1,1,1,1")])
def test_tree_spec_equals_plain_greedy(models, which, tree):
    tgt, other = models
    src = GgufSource(tgt)
    cfg = src.model_config()
    W = load_dense(src, cfg)
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (7, 33, 16, 70)]
    n = 20
    plain, _ = _gen(tgt, prompts, n)
    spec, st = _gen_tree(tgt, prompts, n, tgt if which == "self" else other, tree)
    _same_up_to_ties(W, cfg, prompts, spec, plain)
    assert st["steps"] > 0
    if which == "self":
        assert st["tokens_per_step"] > 3.0, st


def _gen_sampled(path, prompts, n, draft, sp, k=4):
    from vm_c_b200.llm import LLM
    llm = LLM(path, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256, num_gpu_blocks=256,
              enable_prefix_caching=False, draft_model=draft, num_speculative_tokens=k)
    outs = llm.generate(prompts, sp)
    stats = llm.runner.spec.stats.as_dict() if llm.runner.spec is not None else None
    llm.shutdown()
    return [o.output_token_ids for o in outs], stats


def test_speculative_sampling_self_draft_accepts_nearly_all(models):
    # p and q come from the same weights (decode vs prefill kernels): min(1, p/q) is ~1 everywhere.
    tgt, _ = models
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 32000, n).tolist() for n in (9, 40, 20)]
    sp = SamplingParams(temperature=1.0, top_k=40, top_p=0.95, max_tokens=16, ignore_eos=True, seed=3)
    toks, st = _gen_sampled(tgt, prompts, 16, tgt, sp)
    assert all(len(t) == 16 for t in toks)
    assert st["steps"] > 0 and st["acceptance_rate"] > 0.9, st


def test_speculative_sampling_cold_temperature_is_greedy(models):
    # At a temperature this low both distributions are one-hot at the argmax: rejection sampling
    # with an unrelated draft must reproduce plain greedy decoding (up to near-ties).
    tgt, other = models
    src = GgufSource(tgt)
    cfg = src.model_config()
    W = load_dense(src, cfg)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (7, 33, 16)]
    plain, _ = _gen(tgt, prompts, 12)
    sp = SamplingParams(temperature=1e-4, top_k=0, top_p=1.0, max_tokens=12, ignore_eos=True, seed=5)
    spec, st = _gen_sampled(tgt, prompts, 12, other, sp)
    assert st["steps"] > 0
    _same_up_to_ties(W, cfg, prompts, spec, plain)
