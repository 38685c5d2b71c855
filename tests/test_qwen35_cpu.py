"""Hybrid Qwen3.5-MoE (gated delta-net) on CPU: GGUF hyper-parameters parse, the layer schedule follows
full_attention_interval, the fp32 oracle gives the same logits for a prompt run in one pass, in pieces
and token by token (conv, delta-rule and K/V state carried between calls), and loading for serving
is refused with a clear message."""
import numpy as np
import pytest
import torch

from vm_c_b200.gguf.random_init import preset, write_random_gguf
from vm_c_b200.gguf.reader import GgufSource

import ref_qwen35 as R


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("q35") / "tiny-qwen35moe.gguf")
    write_random_gguf(p, preset("tiny-qwen35moe"), "Q8_0", seed=0)
    src = GgufSource(p)
    return src, src.model_config()


def test_config(model):
    _, cfg = model
    want = preset("tiny-qwen35moe")
    for f in ("arch", "n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "ffn_shexp", "ssm_conv",
              "ssm_state", "ssm_k_heads", "ssm_v_heads", "full_attn_interval", "rope_dims", "n_experts",
              "n_experts_used", "nextn_layers", "vocab"):
        assert getattr(cfg, f) == getattr(want, f), f
    assert cfg.is_hybrid and cfg.rope_neox
    assert [cfg.is_recurrent(i) for i in range(cfg.n_layers)] == [True, True, True, False]


def test_oracle_state_carry(model):
    src, cfg = model
    W = R.load(src)
    toks = np.random.default_rng(0).integers(0, cfg.vocab, 9).tolist()
    full = R.forward(W, cfg, toks, R.new_state(cfg))
    st = R.new_state(cfg)
    pieces = torch.cat([R.forward(W, cfg, toks[:4], st), R.forward(W, cfg, toks[4:7], st),
                        R.forward(W, cfg, toks[7:], st)])
    st1 = R.new_state(cfg)
    single = torch.cat([R.forward(W, cfg, [t], st1) for t in toks])
    tol = 1e-4 * float(full.abs().max())
    assert torch.allclose(full, pieces, atol=tol, rtol=0)
    assert torch.allclose(full, single, atol=tol, rtol=0)
    assert torch.isfinite(full).all() and float(full.std()) > 0


def test_tensor_parallel_refused_with_message(model):
    # The family is served on one GPU; a tensor-parallel load is refused after the tensor check,
    # before anything is moved to a device.
    src, cfg = model
    from vm_c_b200.models.llama import load_weights
    with pytest.raises(ValueError, match="qwen35moe"):
        load_weights(src, cfg, "cpu", 0, 2)


@pytest.mark.parametrize("chunk", [1, 16, 64])
def test_chunked_delta_rule_equals_recurrence(chunk):
    # The chunked (matrix-product) form of the gated delta rule, the planned prefill algorithm,
    # equals the token-serial recurrence, including a partial last chunk and a non-zero entering state.
    torch.manual_seed(1)
    T, Hk, Hv, D, eps = 100, 2, 4, 32, 1e-6
    y = torch.randn(T, (2 * Hk + Hv) * D)
    alpha, beta, z = torch.randn(T, Hv), torch.randn(T, Hv), torch.randn(T, Hv * D)
    a_neg, dt_bias, norm_w = -torch.exp(torch.randn(Hv) * 0.5), torch.randn(Hv) * 0.1, 1 + 0.1 * torch.randn(D)
    S0 = torch.randn(Hv, D, D) * 0.1
    o1, s1 = R.ref_gdn(y, alpha, beta, z, a_neg, dt_bias, norm_w, S0, Hk, eps)
    o2, s2 = R.ref_gdn_chunked(y, alpha, beta, z, a_neg, dt_bias, norm_w, S0, Hk, eps, chunk)
    torch.testing.assert_close(o2, o1, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(s2, s1, rtol=1e-4, atol=1e-5)


def test_tensor_plan_matches_checkpoint(model):
    from vm_c_b200.models.hybrid import check_hybrid_tensors, hybrid_tensor_plan
    src, cfg = model
    plan = hybrid_tensor_plan(cfg)
    assert set(plan) == set(src.tensors)
    check_hybrid_tensors(src, cfg)

    class Missing:
        def has(self, n):
            return n != "blk.1.ssm_a" and src.has(n)

        def info(self, n):
            return src.info(n)
    with pytest.raises(ValueError, match="blk.1.ssm_a"):
        check_hybrid_tensors(Missing(), cfg)
