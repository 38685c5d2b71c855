"""Test oracle: an fp32 PyTorch Llama forward over whole sequences (no KV cache), from the same
dequantised GGUF weights the engine loads. Used only by tests."""
from __future__ import annotations

import numpy as np
import torch

from vm_c_b200 import _native
from vm_c_b200.config import rope_inv_freq
from vm_c_b200.gguf.constants import GType, blk


def load_dense(src, cfg):
    h = _native.host()

    def get(name):
        spec = src.info(name)
        raw = src.rows(name).cpu().numpy()
        K = spec.ne[0]
        if spec.gtype == GType.F32:
            return torch.from_numpy(raw.reshape(-1, K).astype(np.float32))
        return torch.from_numpy(h.dequantize(int(spec.gtype), raw, spec.rows, K))

    W = {"embd": get("token_embd.weight"), "norm": get("output_norm.weight").view(-1),
         "out": get("output.weight") if src.has("output.weight") else get("token_embd.weight"), "layers": []}
    ffn = ["ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"] if cfg.is_moe else \
        ["ffn_gate", "ffn_up", "ffn_down"]
    for i in range(cfg.n_layers):
        L = {k: get(blk(i, k)) for k in ["attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm"] + ffn}
        if cfg.is_moe:
            E, F, H = cfg.n_experts, cfg.ffn, cfg.hidden
            L["ffn_gate_exps"] = L["ffn_gate_exps"].reshape(E, F, H)
            L["ffn_up_exps"] = L["ffn_up_exps"].reshape(E, F, H)
            L["ffn_down_exps"] = L["ffn_down_exps"].reshape(E, H, F)
        W["layers"].append(L)
    return W


def moe_ffn(L, cfg, h, margins=None):
    """Mixtral FFN: softmax router, top-k, renormalised weights, weighted sum of SwiGLU experts.
    With `margins` (a list), appends per token the gap between the k-th and (k+1)-th router logit
    relative to the largest router logit magnitude: how close the expert choice is to a tie."""
    logits = h @ L["ffn_gate_inp"].T
    if margins is not None:
        top = torch.topk(logits, min(cfg.n_experts_used + 1, cfg.n_experts), -1).values
        gap = top[:, cfg.n_experts_used - 1] - top[:, -1] if cfg.n_experts > cfg.n_experts_used else \
            torch.full_like(top[:, 0], float("inf"))
        margins.append(gap / logits.abs().max(-1).values.clamp_min(1e-30))
    probs = torch.softmax(logits, -1)
    w, idx = torch.topk(probs, cfg.n_experts_used, -1)
    w = w / w.sum(-1, keepdim=True)
    out = torch.zeros_like(h)
    for t in range(h.shape[0]):
        for j in range(cfg.n_experts_used):
            e = int(idx[t, j])
            g = torch.nn.functional.silu(h[t] @ L["ffn_gate_exps"][e].T) * (h[t] @ L["ffn_up_exps"][e].T)
            out[t] += w[t, j] * (g @ L["ffn_down_exps"][e].T)
    return out


def rope(x, pos, inv, neox):
    # x: [T, H, D]
    ang = pos[:, None].double() * torch.tensor(inv, dtype=torch.float64)[None, :]
    c, s = torch.cos(ang).float()[:, None, :], torch.sin(ang).float()[:, None, :]
    if neox:
        d = x.shape[-1] // 2
        x0, x1 = x[..., :d], x[..., d:]
        return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], -1)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def forward_logits(W, cfg, tokens: list[int], margins=None) -> torch.Tensor:
    """Logits for every position of `tokens` (fp32). `margins`: see moe_ffn (one entry per layer)."""
    T = len(tokens)
    D, Hq, Hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    x = W["embd"][torch.tensor(tokens)]
    pos = torch.arange(T)
    inv = rope_inv_freq(cfg)

    def rms(v, w):
        return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * w.view(-1)

    mask = torch.full((T, T), float("-inf")).triu(1)
    for L in W["layers"]:
        h = rms(x, L["attn_norm"])
        q = (h @ L["attn_q"].T).view(T, Hq, D)
        k = (h @ L["attn_k"].T).view(T, Hkv, D)
        v = (h @ L["attn_v"].T).view(T, Hkv, D)
        q, k = rope(q, pos, inv, cfg.rope_neox), rope(k, pos, inv, cfg.rope_neox)
        G = Hq // Hkv
        k = k.repeat_interleave(G, 1)
        v = v.repeat_interleave(G, 1)
        s = torch.einsum("thd,shd->hts", q, k) / D ** 0.5 + mask
        a = torch.einsum("hts,shd->thd", torch.softmax(s, -1), v).reshape(T, Hq * D)
        x = x + a @ L["attn_output"].T
        h = rms(x, L["ffn_norm"])
        if cfg.is_moe:
            x = x + moe_ffn(L, cfg, h, margins)
        else:
            x = x + (torch.nn.functional.silu(h @ L["ffn_gate"].T) * (h @ L["ffn_up"].T)) @ L["ffn_down"].T
    return rms(x, W["norm"]) @ W["out"].T


def greedy(W, cfg, prompt: list[int], n: int) -> list[int]:
    toks = list(prompt)
    out = []
    for _ in range(n):
        nxt = int(forward_logits(W, cfg, toks)[-1].argmax())
        out.append(nxt)
        toks.append(nxt)
    return out
