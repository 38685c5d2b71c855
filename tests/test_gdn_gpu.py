"""Gated delta-net kernels (causal conv + SiLU, gated delta-rule recurrence + gated RMSNorm) against a
plain fp32 PyTorch restatement of the same ops, for a varlen batch mixing new sequences and
sequences that continue from a stored state."""
import pytest
import torch

from vm_c_b200 import ops

pytestmark = pytest.mark.gpu


def ref_conv(x, w, hist):
    K = w.shape[1]
    xin = torch.cat([hist, x], 0)
    y = torch.stack([(w * xin[t:t + K].T).sum(1) for t in range(x.shape[0])])
    return torch.nn.functional.silu(y), xin[-(K - 1):]


def ref_gdn(y, alpha, beta, z, a_neg, dt_bias, norm_w, S, Hk, eps):
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
            g = torch.exp(a_neg[h] * torch.nn.functional.softplus(alpha[t, h] + dt_bias[h]))
            b = torch.sigmoid(beta[t, h])
            S[h] = g * S[h]
            d = b * (v - S[h].T @ k)
            S[h] = S[h] + torch.outer(k, d)
            o = S[h].T @ q
            zz = z[t, h * D:(h + 1) * D]
            out[t, h * D:(h + 1) * D] = o * torch.rsqrt(o.pow(2).mean() + eps) * norm_w * torch.nn.functional.silu(zz)
    return out, S


@pytest.mark.parametrize("D,Hk,Hv", [(128, 2, 4), (64, 1, 2)])
def test_gdn_conv_and_recurrence(cuda_ext, D, Hk, Hv):
    torch.manual_seed(0)
    dev = "cuda"
    lens, has = [1, 7, 33, 1], [1, 0, 0, 1]
    nseq, T = len(lens), sum(lens)
    C, K, eps = (2 * Hk + Hv) * D, 4, 1e-6
    slots = [3, 0, 2, 1]
    nslots = 4
    x = torch.randn(T, C)
    w = torch.randn(C, K) * 0.5
    alpha, beta = torch.randn(T, Hv), torch.randn(T, Hv)
    z = torch.randn(T, Hv * D)
    a_neg = -torch.exp(torch.randn(Hv) * 0.5)
    dt_bias = torch.randn(Hv) * 0.1
    norm_w = 1 + 0.1 * torch.randn(D)
    conv_state = torch.randn(nslots, K - 1, C)
    state = torch.randn(nslots, Hv, D, D) * 0.1
    qs = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)

    # fp32 oracle
    y_ref = torch.empty(T, C)
    out_ref = torch.empty(T, Hv * D)
    cs_ref, st_ref = conv_state.clone(), state.clone()
    for s in range(nseq):
        a, b = int(qs[s]), int(qs[s + 1])
        hist = conv_state[slots[s]] if has[s] else torch.zeros(K - 1, C)
        y_ref[a:b], cs_ref[slots[s]] = ref_conv(x[a:b], w, hist)
        S0 = state[slots[s]] if has[s] else torch.zeros(Hv, D, D)
        out_ref[a:b], st_ref[slots[s]] = ref_gdn(y_ref[a:b], alpha[a:b], beta[a:b], z[a:b], a_neg, dt_bias,
                                                 norm_w, S0, Hk, eps)

    g = lambda t: t.to(dev).contiguous()  # noqa: E731
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731
    cs_d, st_d = g(conv_state), g(state)
    y_d = torch.empty(T, C, device=dev)
    ops.gdn_conv(g(x), g(w), g(qs), i32(slots), i32(has), nseq, cs_d, y_d)
    out_d = torch.empty(T, Hv * D, dtype=torch.bfloat16, device=dev)
    ops.gdn_recurrent(y_d, g(alpha), g(beta), g(z), g(a_neg), g(dt_bias), g(norm_w), st_d, i32(slots), i32(has),
                      g(qs), nseq, Hk, eps, out_d)
    torch.cuda.synchronize()
    torch.testing.assert_close(y_d.cpu(), y_ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(cs_d.cpu(), cs_ref, rtol=0, atol=0)
    torch.testing.assert_close(st_d.cpu(), st_ref, rtol=1e-3, atol=1e-4)
    torch.testing.assert_close(out_d.float().cpu(), out_ref, rtol=2e-2, atol=2e-2)
