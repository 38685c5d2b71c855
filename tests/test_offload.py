"""CPU weight offload: the reference's name-segment rule and the byte budget (CPU), and offloaded
layers giving the same tokens as resident ones (GPU)."""
import types

import numpy as np
import pytest
import torch

from vm_c_b200.models.offload import apply_offload, matches


def test_segment_rule():
    assert matches("blk.3.attn_q.weight", ["attn_q"])
    assert matches("blk.3.attn_q.weight", ["weight"])
    assert not matches("blk.3.attn_q.weight", ["attn"])
    assert not matches("blk.3.ffn_down.weight", ["ffn_gate", "attn_q"])
    assert matches("anything", [])


def _fake_weights(n_layers=3, nbytes=1000):
    def tw():
        return types.SimpleNamespace(data=torch.arange(nbytes, dtype=torch.int64).to(torch.uint8), nbytes=nbytes)
    layers = [types.SimpleNamespace(index=i, wqkv=[tw()], wo=tw(), w_gate_up=tw(), w_down=tw(), offload=[])
              for i in range(n_layers)]
    return types.SimpleNamespace(layers=layers)


@pytest.mark.gpu
def test_budget_and_selection_gpu():
    w = _fake_weights()
    plan = apply_offload(w, 3500 / (1 << 30), ["ffn_down", "attn_output"], "cuda")
    # 3 ffn_down + ... within 3500 bytes: wo(0), w_down(0), wo(1) fit (3000), the 4th does not
    assert plan.tensors == 3 and plan.bytes_offloaded == 3000
    assert [len(lw.offload) for lw in w.layers] == [2, 1, 0]
    host, view = w.layers[0].offload[0]
    assert host.is_pinned() and view.is_cuda and view.numel() == 1000


@pytest.mark.gpu
def test_offloaded_model_same_tokens(tmp_path):
    from vm_c_b200.core.sampling_params import SamplingParams
    from vm_c_b200.gguf.random_init import preset, write_random_gguf
    from vm_c_b200.llm import LLM
    p = str(tmp_path / "t.gguf")
    write_random_gguf(p, preset("tiny-llama"), "Q8_0", seed=0)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 32000, n).tolist() for n in (9, 30)]
    sp = SamplingParams.greedy_params(max_tokens=8, ignore_eos=True)
    outs = []
    for gb, segs in ((0.0, ()), (0.002, ()), (1.0, ("ffn_down",))):
        llm = LLM(p, max_model_len=256, max_num_seqs=4, max_num_batched_tokens=256, num_gpu_blocks=128,
                  cpu_offload_gb=gb, cpu_offload_params=segs)
        if gb:
            assert llm.runner.offload.tensors > 0
        outs.append([o.output_token_ids for o in llm.generate(prompts, sp)])
        llm.shutdown()
    assert outs[0] == outs[1] == outs[2]
