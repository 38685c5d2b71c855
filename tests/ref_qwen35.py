"""fp32 CPU oracle of the hybrid Qwen3.5-MoE forward (gated delta-net + gated full attention, MoE with a
sigmoid-gated shared expert), restated from the reference graph
(src/official/llama/models/qwen35moe.cpp:164-590, delta-net-base.cpp:289-363), with explicit
per-layer state so a prompt can be run in pieces: conv history + delta-rule state for GDN layers,
K/V rows for attention layers."""
import numpy as np
import torch
import torch.nn.functional as Fn

from vm_c_b200 import _native
from vm_c_b200.gguf.constants import GType


def ref_conv(x, w, hist):
    """silu(causal depthwise conv) of x [T, C] with kernel w [C, K] after the K-1 rows of hist."""
    K = w.shape[1]
    xin = torch.cat([hist, x], 0)
    y = torch.stack([(w * xin[t:t + K].T).sum(1) for t in range(x.shape[0])])
    return Fn.silu(y), xin[-(K - 1):]


def ref_gdn(y, alpha, beta, z, a_neg, dt_bias, norm_w, S, Hk, eps):
    """Gated delta rule over the tokens of y (q | k | v heads) + gated RMSNorm; returns (out, S)."""
    T = y.shape[0]
    Hv, D = S.shape[0], S.shape[1]
    out = torch.empty(T, Hv * D)
    S = S.clone()
    for t in range(T):
        for h in range(Hv):
            kh = h % Hk
            q = y[t, kh * D:(kh + 1) * D]
            k = y[t, (Hk + kh) * D:(Hk + kh + 1) * D]
            v = y[t, 2 * Hk * D + h * D:2 * Hk * D + (h + 1) * D]
            q = q / torch.clamp(q.norm(), min=eps) / D ** 0.5
            k = k / torch.clamp(k.norm(), min=eps)
            g = torch.exp(a_neg[h] * Fn.softplus(alpha[t, h] + dt_bias[h]))
            b = torch.sigmoid(beta[t, h])
            S[h] = g * S[h]
            d = b * (v - S[h].T @ k)
            S[h] = S[h] + torch.outer(k, d)
            o = S[h].T @ q
            zz = z[t, h * D:(h + 1) * D]
            out[t, h * D:(h + 1) * D] = o * torch.rsqrt(o.pow(2).mean() + eps) * norm_w * Fn.silu(zz)
    return out, S


def ref_gdn_chunked(y, alpha, beta, z, a_neg, dt_bias, norm_w, S, Hk, eps, chunk):
    """The same recurrence in chunks of `chunk` tokens, written as matrix products (the form a
    tensor-core prefill kernel computes). Per chunk, with gamma the cumulative log decay, S0 the
    entering state, A[t, s] = beta_t e^(gamma_t - gamma_s) k_t.k_s (s < t) and
    M[t, s] = e^(gamma_t - gamma_s) (s <= t):
        D   = (I + A)^-1 (beta * (V - e^gamma * K S0))      (the delta rows d_t)
        O   = e^gamma * Q S0 + (M * Q K^T) D
        S_C = e^gamma_C S0 + K^T (e^(gamma_C - gamma) * D)
    """
    T = y.shape[0]
    Hv, D = S.shape[0], S.shape[1]
    out = torch.empty(T, Hv * D)
    S = S.clone().double()
    for h in range(Hv):
        kh = h % Hk
        Q = y[:, kh * D:(kh + 1) * D].double()
        K = y[:, (Hk + kh) * D:(Hk + kh + 1) * D].double()
        V = y[:, 2 * Hk * D + h * D:2 * Hk * D + (h + 1) * D].double()
        Q = Q / torch.clamp(Q.norm(dim=1, keepdim=True), min=eps) / D ** 0.5
        K = K / torch.clamp(K.norm(dim=1, keepdim=True), min=eps)
        lg = (a_neg[h] * Fn.softplus(alpha[:, h] + dt_bias[h])).double()
        b = torch.sigmoid(beta[:, h]).double()
        O = torch.empty(T, D, dtype=torch.float64)
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            q, k, v, bb = Q[c0:c1], K[c0:c1], V[c0:c1], b[c0:c1]
            gam = torch.cumsum(lg[c0:c1], 0)
            n = c1 - c0
            diff = gam[:, None] - gam[None, :]
            tril = torch.tril(torch.ones(n, n, dtype=torch.bool))
            Mx = torch.where(tril, torch.exp(torch.where(tril, diff, torch.zeros_like(diff))), torch.zeros_like(diff))
            A = (bb[:, None] * Mx * (k @ k.T)).tril(-1)
            rhs = bb[:, None] * (v - torch.exp(gam)[:, None] * (k @ S[h]))
            Dm = torch.linalg.solve_triangular(torch.eye(n, dtype=torch.float64) + A, rhs, upper=False,
                                               unitriangular=True)
            O[c0:c1] = torch.exp(gam)[:, None] * (q @ S[h]) + (Mx * (q @ k.T)) @ Dm
            S[h] = torch.exp(gam[-1]) * S[h] + k.T @ (torch.exp(gam[-1] - gam)[:, None] * Dm)
        O = O.float()
        zz = z[:, h * D:(h + 1) * D]
        out[:, h * D:(h + 1) * D] = O * torch.rsqrt(O.pow(2).mean(1, keepdim=True) + eps) * norm_w * Fn.silu(zz)
    return out, S.float()


def load(src):
    """Every tensor of the GGUF as a dense fp32 matrix [rows, ne0] (1-D tensors as vectors)."""
    h = _native.host()
    W = {}
    for name in src.tensors:
        spec = src.info(name)
        raw = src.rows(name).cpu().numpy()
        K = spec.ne[0]
        if spec.gtype == GType.F32:
            m = torch.from_numpy(raw.reshape(-1, K).astype(np.float32))
        else:
            m = torch.from_numpy(h.dequantize(int(spec.gtype), raw, spec.rows, K))
        W[name] = m.view(-1) if len(spec.ne) == 1 else m
    return W


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _rope_partial(x, pos, n_rot, theta):
    """Half-rotation RoPE on the first n_rot dims of every head of x [T, H, D]."""
    half = n_rot // 2
    inv = 1.0 / theta ** (torch.arange(half, dtype=torch.float64) * 2 / n_rot)
    ang = (pos[:, None].double() * inv[None, :]).float()
    c, s = ang.cos()[:, None, :], ang.sin()[:, None, :]
    x = x.clone()
    a, b = x[..., :half].clone(), x[..., half:n_rot].clone()
    x[..., :half] = a * c - b * s
    x[..., half:n_rot] = a * s + b * c
    return x


def new_state(cfg):
    st = []
    C = 2 * cfg.ssm_k_heads * cfg.ssm_state + cfg.ssm_v_heads * cfg.ssm_state
    for i in range(cfg.n_layers - cfg.nextn_layers):
        if cfg.is_recurrent(i):
            st.append({"conv": torch.zeros(cfg.ssm_conv - 1, C),
                       "S": torch.zeros(cfg.ssm_v_heads, cfg.ssm_state, cfg.ssm_state)})
        else:
            st.append({"k": torch.zeros(0, cfg.n_kv_heads, cfg.head_dim),
                       "v": torch.zeros(0, cfg.n_kv_heads, cfg.head_dim)})
    return {"pos": 0, "layers": st}


def forward(W, cfg, tokens, state, margins=None):
    """Logits [T, V] of `tokens` continuing from `state` (updated in place). With `margins` (a list),
    appends per layer and token the gap between the k-th and (k+1)-th router logit relative to the
    largest router logit magnitude (how close the expert choice is to a tie)."""
    T, eps, D = len(tokens), cfg.rms_eps, cfg.head_dim
    pos = torch.arange(state["pos"], state["pos"] + T)
    h = W["token_embd.weight"][torch.tensor(tokens)]
    for i, ls in enumerate(state["layers"]):
        b = f"blk.{i}."
        x = _rms(h, W[b + "attn_norm.weight"], eps)
        if cfg.is_recurrent(i):
            mixed = x @ W[b + "attn_qkv.weight"].T
            z = x @ W[b + "attn_gate.weight"].T
            beta = x @ W[b + "ssm_beta.weight"].T
            alpha = x @ W[b + "ssm_alpha.weight"].T
            y, ls["conv"] = ref_conv(mixed, W[b + "ssm_conv1d.weight"], ls["conv"])
            o, ls["S"] = ref_gdn(y, alpha, beta, z, W[b + "ssm_a"], W[b + "ssm_dt.bias"], W[b + "ssm_norm.weight"],
                                 ls["S"], cfg.ssm_k_heads, eps)
            a = o @ W[b + "ssm_out.weight"].T
        else:
            Hq, Hkv = cfg.n_heads, cfg.n_kv_heads
            qg = (x @ W[b + "attn_q.weight"].T).view(T, Hq, 2 * D)
            q, gate = qg[..., :D], qg[..., D:]
            q = _rms(q, W[b + "attn_q_norm.weight"], eps)
            k = _rms((x @ W[b + "attn_k.weight"].T).view(T, Hkv, D), W[b + "attn_k_norm.weight"], eps)
            v = (x @ W[b + "attn_v.weight"].T).view(T, Hkv, D)
            n_rot = cfg.rope_dims or D
            q, k = _rope_partial(q, pos, n_rot, cfg.rope_theta), _rope_partial(k, pos, n_rot, cfg.rope_theta)
            ls["k"], ls["v"] = torch.cat([ls["k"], k]), torch.cat([ls["v"], v])
            K_, V_ = ls["k"], ls["v"]
            N = K_.shape[0]
            rep = Hq // Hkv
            o = torch.empty(T, Hq, D)
            for hh in range(Hq):
                kv = hh // rep
                s = (q[:, hh] @ K_[:, kv].T) / D ** 0.5
                mask = torch.arange(N)[None, :] > (N - T + torch.arange(T))[:, None]
                s = s.masked_fill(mask, float("-inf"))
                o[:, hh] = torch.softmax(s, -1) @ V_[:, kv]
            o = o * torch.sigmoid(gate)
            a = o.reshape(T, Hq * D) @ W[b + "attn_output.weight"].T
        h = h + a
        x2 = _rms(h, W[b + "post_attention_norm.weight"], eps)
        rl = x2 @ W[b + "ffn_gate_inp.weight"].T
        if margins is not None:
            top = torch.topk(rl, cfg.n_experts_used + 1, -1).values
            margins.append((top[:, -2] - top[:, -1]) / rl.abs().max(-1).values.clamp_min(1e-30))
        probs = torch.softmax(rl, -1)
        wts, idx = torch.topk(probs, cfg.n_experts_used, -1)
        wts = wts / wts.sum(-1, keepdim=True)
        E, F, H = cfg.n_experts, cfg.ffn, cfg.hidden
        Wg = W[b + "ffn_gate_exps.weight"].view(E, F, H)
        Wu = W[b + "ffn_up_exps.weight"].view(E, F, H)
        Wd = W[b + "ffn_down_exps.weight"].view(E, H, F)
        moe = torch.zeros_like(h)
        for t in range(T):
            for j in range(cfg.n_experts_used):
                e = int(idx[t, j])
                moe[t] += wts[t, j] * ((Fn.silu(x2[t] @ Wg[e].T) * (x2[t] @ Wu[e].T)) @ Wd[e].T)
        sh = (Fn.silu(x2 @ W[b + "ffn_gate_shexp.weight"].T) * (x2 @ W[b + "ffn_up_shexp.weight"].T)) \
            @ W[b + "ffn_down_shexp.weight"].T
        sg = torch.sigmoid(x2 @ W[b + "ffn_gate_inp_shexp.weight"])[:, None]
        h = h + moe + sg * sh
    state["pos"] += T
    out = W["output.weight"] if "output.weight" in W else W["token_embd.weight"]
    return _rms(h, W["output_norm.weight"], eps) @ out.T
