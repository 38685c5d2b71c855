"""The native step forward (csrc/kernels/forward.cpp) against the Python step path of
models/llama.py: the same kernels in the same order, so greedy tokens and every sampled row's logits
must be bit-identical, for prefill, mixed and decode (CUDA-graph) steps, with K-split GEMMs (a
model whose decode GEMMs split K) and with a TurboQuant KV cache."""
import os

import numpy as np
import pytest
import torch

from vm_c_b200.core.sampling_params import SamplingParams
from vm_c_b200.gguf.random_init import preset, write_random_gguf

pytestmark = pytest.mark.gpu


def _small_cfg():
    c = preset("tiny-llama")
    c.name, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.n_layers = "small", 1024, 8, 4, 128, 2816, 2
    return c


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    d = tmp_path_factory.mktemp("nat")
    tiny, small = str(d / "tiny.gguf"), str(d / "small.gguf")
    write_random_gguf(tiny, preset("tiny-llama"), "Q8_0", seed=0)
    write_random_gguf(small, _small_cfg(), "Q4_K_M", seed=1)
    return {"tiny": tiny, "small": small}


def _run(path, native: bool, kv="auto"):
    from vm_c_b200 import ops
    from vm_c_b200.llm import LLM
    os.environ["VMC_NATIVE"] = "1" if native else "0"
    try:
        llm = LLM(path, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=128, num_gpu_blocks=256,
                  kv_cache_dtype=kv)
    finally:
        os.environ.pop("VMC_NATIVE", None)
    rows = []
    llm.engine.logits_hook = lambda ids, lg: rows.append((ids, lg))
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, llm.cfg.model.vocab, n).tolist() for n in (5, 70, 17, 150)]
    n0 = ops.LAUNCHES[0]
    outs = llm.generate(prompts, SamplingParams.greedy_params(max_tokens=10, ignore_eos=True))
    launches = ops.LAUNCHES[0] - n0
    llm.shutdown()
    return [o.output_token_ids for o in outs], rows, launches


@pytest.mark.parametrize("name,kv", [("tiny", "auto"), ("small", "auto"), ("small", "turboquant_4bit_nc")])
def test_native_matches_python_path(models, name, kv):
    t_py, r_py, _ = _run(models[name], False, kv)
    t_nat, r_nat, _ = _run(models[name], True, kv)
    assert t_nat == t_py
    assert len(r_nat) == len(r_py)
    for (ia, la), (ib, lb) in zip(r_py, r_nat):
        assert ia == ib
        assert torch.equal(la, lb)


def test_native_splits_policy_matches_python(cuda_ext):
    from vm_c_b200 import ops
    for wf, N, K in [(1, 6144, 4096), (1, 28672, 4096), (2, 4096, 14336), (3, 768, 4096), (0, 512, 512)]:
        for M in (1, 4, 16, 64, 100, 256, 300, 2048):
            w = ops.TiledWeight(wf, torch.empty(ops.tiled_bytes(wf, N, K), dtype=torch.uint8), N, K)
            assert cuda_ext.gemm_pick_splits(wf, N, K, M, ops.NUM_SMS) == ops.pick_splits(w, M), (wf, N, K, M)
