"""The PyTorch-free runtime (csrc/runtime/vmc_run.cpp): the native scheduler, native step forward
and decode CUDA graphs driven from C++ must produce the Python engine's greedy tokens on the same
checkpoint, prompts and scheduler settings, and the executable must not map libtorch or libpython.

Token equality is required up to the first position where the Python engine's own logits put the
two best tokens within rounding of each other (random-weight models have such near-ties): there the
runtime may pick the other of the two, and that request is not compared further."""
import json
import os
import struct
import subprocess

import numpy as np
import pytest

from vm_c_b200.core.sampling_params import SamplingParams
from vm_c_b200.gguf.random_init import preset, write_random_gguf

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "vm_c_b200", "_ext", "runtime", "vmc_run")


@pytest.fixture(scope="module")
def exe():
    if not os.path.exists(EXE):
        from vm_c_b200._build import build_runtime
        build_runtime()
    return EXE


def test_runtime_links_no_torch(exe):
    out = subprocess.run(["ldd", exe], capture_output=True, text=True).stdout
    assert "torch" not in out and "python" not in out, out


@pytest.mark.parametrize("model,mix", [("tiny-llama", "Q8_0"), ("tiny-llama", "Q4_K_M"), ("tiny-mixtral", "Q8_0")])
def test_runtime_matches_python_engine(exe, tmp_path, model, mix):
    # tiny-mixtral: the runtime serves Mixtral-architecture checkpoints with every expert on the GPU
    # (router, routing, grouped expert GEMMs and combine of the native forward).
    cfg = preset(model)
    if mix == "Q4_K_M":
        cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.n_layers = 1024, 8, 4, 128, 2816, 2
    path = str(tmp_path / "m.gguf")
    write_random_gguf(path, cfg, mix, seed=3)
    rng = np.random.default_rng(9)
    prompts = rng.integers(0, cfg.vocab, (6, 40)).astype(np.int32)
    pf = tmp_path / "p.bin"
    pf.write_bytes(struct.pack("<ii", *prompts.shape) + prompts.tobytes())
    dump = tmp_path / "t.json"
    r = subprocess.run([exe, path, "--prompts", str(pf), "--gen", "12", "--max-num-seqs", "8",
                        "--max-num-batched-tokens", "128", "--max-model-len", "256", "--num-blocks", "256",
                        "--dump-tokens", str(dump)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["device_error"] == 0
    native = json.load(open(dump))
    from vm_c_b200.llm import LLM
    llm = LLM(path, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=128, num_gpu_blocks=256)
    rows = []
    llm.engine.logits_hook = lambda ids, lg: rows.append((ids, lg))
    outs = llm.generate(prompts.tolist(), SamplingParams.greedy_params(max_tokens=12, ignore_eos=True))
    llm.shutdown()
    per_req = {}
    for ids, lg in rows:
        for k, i in enumerate(ids):
            per_req.setdefault(i, []).append(lg[k].float())
    py_logits = [per_req[i] for i in sorted(per_req)]
    ties, equal = 0, 0
    for n, p, lg in zip(native, [o.output_token_ids for o in outs], py_logits):
        assert len(n) == len(p) == 12
        for j, (a, b) in enumerate(zip(n, p)):
            if a == b:
                equal += 1
                continue
            row = lg[j]
            gap = float(row[b] - row[a])
            assert 0 <= gap < 2e-3 * float(row.abs().max()), (j, a, b, gap, float(row.abs().max()))
            ties += 1
            break
    assert ties <= 1 and equal >= 6 * 12 - 12, (ties, equal, native, [o.output_token_ids for o in outs])
