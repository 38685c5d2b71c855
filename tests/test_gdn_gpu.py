"""Gated delta-net kernels (causal conv + SiLU, gated delta-rule recurrence + gated RMSNorm) against a
plain fp32 PyTorch restatement of the same ops, for a varlen batch mixing new sequences and
sequences that continue from a stored state."""
import pytest
import torch

from vm_c_b200 import ops

from ref_qwen35 import ref_conv, ref_gdn

pytestmark = pytest.mark.gpu


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
