"""BASELINE config 1 against the reference's own CPU output.

tests/data/config1_reference_cpu.json holds the 32 greedy tokens that the reference's CPU stack (its
vendored libllama + ggml-cpu, driven by baseline/ref_bench.cpp) produced for the config-1 tiny Llama
(Q8_0 GGUF written by this repository's seeded random-init writer) and a 16-token prompt. This test
rebuilds the same GGUF, checks that it is byte-identical to the file the reference read, and compares
the model definition with the reference:
  * teacher-forced on the reference's tokens, this repository's fp32 oracle picks the same argmax at
    all but at most one of the 32 positions, and only where its top-1 / top-2 logit margin is below
    0.01 (ggml-cpu quantises activations to Q8_0 in its Q8_0 dot products, so near-ties may flip);
  * free-running greedy decoding agrees on every token before the first disagreement (28 tokens).
If baseline/_ref/vmc_ref_cpu has been built, the reference binary is also re-run on the file.
"""
import hashlib
import json
import os
import struct
import subprocess
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(__file__))
from ref_llama import forward_logits, greedy, load_dense  # noqa: E402

from vm_c_b200.gguf.random_init import preset, write_random_gguf  # noqa: E402
from vm_c_b200.llm import make_source  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "data", "config1_reference_cpu.json")))
MARGIN = 0.01


def _gguf(tmp_path):
    path = str(tmp_path / "tiny.gguf")
    write_random_gguf(path, preset("tiny-llama"), "Q8_0", seed=0)
    return path


def test_prompt_rule():
    assert np.random.default_rng(1).integers(0, 32000, 16).tolist() == GOLD["prompt"]


def test_config1_matches_reference_cpu(tmp_path):
    path = _gguf(tmp_path)
    assert hashlib.sha256(open(path, "rb").read()).hexdigest() == GOLD["gguf_sha256"]
    src, cfg = make_source(path, "cpu")
    W = load_dense(src, cfg)
    prompt, ref = GOLD["prompt"], GOLD["tokens"]
    lg = forward_logits(W, cfg, prompt + ref[:-1])[len(prompt) - 1:]
    top2 = torch.topk(lg, 2, -1).values
    margin = (top2[:, 0] - top2[:, 1]).tolist()
    am = lg.argmax(-1).tolist()
    differ = [i for i in range(len(ref)) if am[i] != ref[i]]
    assert len(differ) <= 1, differ
    assert all(margin[i] <= MARGIN for i in differ), [(i, margin[i]) for i in differ]
    first = differ[0] if differ else len(ref)
    assert first >= 28
    assert greedy(W, cfg, prompt, first) == ref[:first]


def test_reference_binary_if_built(tmp_path):
    exe = os.path.join(HERE, "..", "baseline", "_ref", "vmc_ref_cpu")
    if not os.path.exists(exe):
        import pytest
        pytest.skip("reference CPU stack not built (baseline/build_ref.sh)")
    path = _gguf(tmp_path)
    pf = tmp_path / "p.bin"
    pf.write_bytes(struct.pack("<ii", 1, 16) + np.asarray(GOLD["prompt"], np.int32).tobytes())
    out = tmp_path / "t.json"
    subprocess.run([exe, "bench", "--model", path, "--prompts", str(pf), "--gen", "32", "--batch", "512", "--runs",
                    "1", "--warmup", "0", "--cpu", "--dump-tokens", str(out)], check=True, capture_output=True,
                   timeout=300)
    assert json.load(open(out))[0] == GOLD["tokens"]
