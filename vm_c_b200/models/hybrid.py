"""Tensor plan of hybrid Qwen3.5-MoE checkpoints (gated delta-net + full attention, MoE with a shared
expert), the first step of serving them: every tensor a layer needs with its GGUF shape (ne order:
row length first), as the reference creates them (src/official/llama/models/qwen35moe.cpp:60-112,
load_arch_tensors), and a check of a checkpoint against it."""
from __future__ import annotations

from ..config import ModelConfig


def hybrid_tensor_plan(cfg: ModelConfig) -> dict[str, list[int]]:
    H, D, V = cfg.hidden, cfg.head_dim, cfg.vocab
    Ds, Hk, Hv, E, F, Fs = cfg.ssm_state, cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.n_experts, cfg.ffn, cfg.ffn_shexp
    conv_dim = 2 * Hk * Ds + Hv * Ds
    plan = {"token_embd.weight": [H, V], "output_norm.weight": [H]}
    if not cfg.tie_embeddings:
        plan["output.weight"] = [H, V]
    for i in range(cfg.n_layers - cfg.nextn_layers):
        b = f"blk.{i}."
        plan[b + "attn_norm.weight"] = [H]
        plan[b + "post_attention_norm.weight"] = [H]
        if cfg.is_recurrent(i):
            plan.update({b + "attn_qkv.weight": [H, conv_dim], b + "attn_gate.weight": [H, Hv * Ds],
                         b + "ssm_conv1d.weight": [cfg.ssm_conv, conv_dim], b + "ssm_dt.bias": [Hv],
                         b + "ssm_a": [Hv], b + "ssm_beta.weight": [H, Hv], b + "ssm_alpha.weight": [H, Hv],
                         b + "ssm_norm.weight": [Ds], b + "ssm_out.weight": [Hv * Ds, H]})
        else:
            plan.update({b + "attn_q.weight": [H, 2 * cfg.n_heads * D], b + "attn_k.weight": [H, cfg.kv_size],
                         b + "attn_v.weight": [H, cfg.kv_size], b + "attn_output.weight": [cfg.q_size, H],
                         b + "attn_q_norm.weight": [D], b + "attn_k_norm.weight": [D]})
        plan.update({b + "ffn_gate_inp.weight": [H, E], b + "ffn_gate_exps.weight": [H, F, E],
                     b + "ffn_up_exps.weight": [H, F, E], b + "ffn_down_exps.weight": [F, H, E]})
        if Fs:
            plan.update({b + "ffn_gate_inp_shexp.weight": [H], b + "ffn_gate_shexp.weight": [H, Fs],
                         b + "ffn_up_shexp.weight": [H, Fs], b + "ffn_down_shexp.weight": [Fs, H]})
    return plan


def check_hybrid_tensors(src, cfg: ModelConfig) -> None:
    """Raise ValueError naming the first missing or mis-shaped tensor of a hybrid checkpoint."""
    for name, ne in hybrid_tensor_plan(cfg).items():
        if not src.has(name):
            raise ValueError(f"hybrid checkpoint is missing tensor {name}")
        got = list(src.info(name).ne)
        if got != ne:
            raise ValueError(f"tensor {name} has shape {got}, expected {ne}")
