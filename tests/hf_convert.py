"""Test helper: write a GGUF checkpoint out as a HuggingFace directory (config.json + two safetensors
shards + index). Q/K rows go back from the GGUF adjacent-pair order to HF's rotate-half order, so
the HF model with half-rotation RoPE computes the same function as the GGUF one."""
import json
import os

import numpy as np
import torch

from vm_c_b200 import _native
from vm_c_b200.gguf.constants import GType
from vm_c_b200.hf import save_file


def _dense(src, name):
    spec = src.info(name)
    raw = src.rows(name).cpu().numpy()
    K = spec.ne[0]
    if spec.gtype == GType.F32:
        return torch.from_numpy(raw.reshape(-1, K).astype(np.float32))
    return torch.from_numpy(_native.host().dequantize(int(spec.gtype), raw, spec.rows, K))


def unpermute_qk(w: torch.Tensor, n_heads: int) -> torch.Tensor:
    """GGUF row 2i + j of a head -> HF row j * D/2 + i."""
    R, H = w.shape
    D = R // n_heads
    return w.reshape(n_heads, D // 2, 2, H).transpose(1, 2).reshape(R, H)


def gguf_to_hf(src, cfg, out_dir: str, dtype=torch.bfloat16) -> None:
    os.makedirs(out_dir, exist_ok=True)
    t = {}
    t["model.embed_tokens.weight"] = _dense(src, "token_embd.weight").to(dtype)
    t["model.norm.weight"] = _dense(src, "output_norm.weight").view(-1)
    if src.has("output.weight"):
        t["lm_head.weight"] = _dense(src, "output.weight").to(dtype)
    for i in range(cfg.n_layers):
        p, b = f"model.layers.{i}.", f"blk.{i}."
        t[p + "input_layernorm.weight"] = _dense(src, b + "attn_norm.weight").view(-1)
        t[p + "post_attention_layernorm.weight"] = _dense(src, b + "ffn_norm.weight").view(-1).to(dtype)
        t[p + "self_attn.q_proj.weight"] = unpermute_qk(_dense(src, b + "attn_q.weight"), cfg.n_heads).to(dtype)
        t[p + "self_attn.k_proj.weight"] = unpermute_qk(_dense(src, b + "attn_k.weight"), cfg.n_kv_heads).to(dtype)
        t[p + "self_attn.v_proj.weight"] = _dense(src, b + "attn_v.weight").to(dtype)
        t[p + "self_attn.o_proj.weight"] = _dense(src, b + "attn_output.weight").to(dtype)
        if cfg.is_moe:
            E, F, H = cfg.n_experts, cfg.ffn, cfg.hidden
            t[p + "block_sparse_moe.gate.weight"] = _dense(src, b + "ffn_gate_inp.weight").to(dtype)
            g = _dense(src, b + "ffn_gate_exps.weight").reshape(E, F, H)
            u = _dense(src, b + "ffn_up_exps.weight").reshape(E, F, H)
            d = _dense(src, b + "ffn_down_exps.weight").reshape(E, H, F)
            for e in range(E):
                q = p + f"block_sparse_moe.experts.{e}."
                t[q + "w1.weight"], t[q + "w3.weight"], t[q + "w2.weight"] = (g[e].to(dtype), u[e].to(dtype),
                                                                              d[e].to(dtype))
        else:
            t[p + "mlp.gate_proj.weight"] = _dense(src, b + "ffn_gate.weight").to(dtype)
            t[p + "mlp.up_proj.weight"] = _dense(src, b + "ffn_up.weight").to(dtype)
            t[p + "mlp.down_proj.weight"] = _dense(src, b + "ffn_down.weight").to(dtype)
    names = sorted(t)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    wmap = {}
    for fn, ns in shards.items():
        save_file({n: t[n] for n in ns}, os.path.join(out_dir, fn), metadata={"format": "pt"})
        wmap.update({n: fn for n in ns})
    json.dump({"metadata": {}, "weight_map": wmap}, open(os.path.join(out_dir, "model.safetensors.index.json"), "w"))
    hc = {"model_type": "mixtral" if cfg.is_moe else "llama", "num_hidden_layers": cfg.n_layers,
          "hidden_size": cfg.hidden, "num_attention_heads": cfg.n_heads, "num_key_value_heads": cfg.n_kv_heads,
          "head_dim": cfg.head_dim, "intermediate_size": cfg.ffn, "vocab_size": cfg.vocab,
          "rms_norm_eps": cfg.rms_eps, "rope_theta": cfg.rope_theta, "max_position_embeddings": cfg.context_length,
          "bos_token_id": cfg.bos_token_id, "eos_token_id": cfg.eos_token_ids[0],
          "tie_word_embeddings": not src.has("output.weight")}
    if cfg.is_moe:
        hc.update(num_local_experts=cfg.n_experts, num_experts_per_tok=cfg.n_experts_used)
    json.dump(hc, open(os.path.join(out_dir, "config.json"), "w"))
