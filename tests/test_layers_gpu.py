"""Residual add + RMSNorm and RoPE + paged-KV store kernels vs fp32 PyTorch restatements."""
import pytest
import torch

from vm_c_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,T", [(4096, 64), (256, 5), (100, 3), (8192, 2)])
@pytest.mark.parametrize("nd,f32", [(0, True), (1, True), (4, True), (9, True), (1, False)])
def test_add_rmsnorm(cuda_ext, H, T, nd, f32):
    torch.manual_seed(H + nd)
    resid = torch.randn(T, H, device="cuda")
    w = torch.randn(H, device="cuda")
    dt = torch.float32 if f32 else torch.bfloat16
    delta = torch.randn(max(nd, 1), T, H, device="cuda").to(dt)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    want = resid.clone()
    for j in range(nd):
        want += delta[j].float()
    ref = (want * torch.rsqrt(want.pow(2).mean(-1, keepdim=True) + 1e-5) * w)
    r = resid.clone()
    ops.add_rmsnorm(r, w, T, H, 1e-5, out=out, delta=delta if nd else None, ndelta=max(nd, 1),
                    delta_stride=T * H)
    torch.cuda.synchronize()
    assert torch.allclose(r, want, atol=1e-4, rtol=1e-5)
    assert (out.float() - ref).abs().max().item() <= 0.01 * ref.abs().max().item()


def _rope_ref(x, pos, D, neox, theta=10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = pos.double().cpu()[:, None] * inv[None, :]
    c, s = ang.cos().float().cuda(), ang.sin().float().cuda()
    c, s = c[:, None, :], s[:, None, :]
    if neox:
        a, b = x[..., :D // 2], x[..., D // 2:]
        return torch.cat([a * c - b * s, a * s + b * c], -1)
    a, b = x[..., 0::2], x[..., 1::2]
    y = torch.empty_like(x)
    y[..., 0::2] = a * c - b * s
    y[..., 1::2] = a * s + b * c
    return y


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("neox", [False, True])
@pytest.mark.parametrize("nsplit,f32", [(1, True), (3, True), (1, False)])
def test_rope_store(cuda_ext, D, neox, nsplit, f32):
    torch.manual_seed(D + nsplit)
    T, Hq, Hkv = 37, 8, 2
    W = (Hq + 2 * Hkv) * D
    parts = torch.randn(nsplit, T, W, device="cuda")
    qkv = parts.sum(0)
    src = parts if f32 else qkv.bfloat16()
    if not f32:
        qkv = src.float()
    pos = torch.randint(0, 500, (T,), dtype=torch.int32, device="cuda")
    slots = torch.randperm(8 * 16, device="cuda")[:T].int()
    slots[3] = -1
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = torch.arange(512, dtype=torch.float64)[:, None] * inv[None, :]
    cos_sin = torch.stack([ang.cos(), ang.sin()], -1).float().cuda().contiguous()
    q_out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(8, 2, Hkv, 16, D, dtype=torch.bfloat16, device="cuda")
    ops.rope_store(src[0] if f32 else src, T, Hq, Hkv, D, pos, slots, cos_sin, neox, q_out, kv, nsplit=nsplit,
                   split_stride=T * W)
    torch.cuda.synchronize()
    x = qkv.view(T, Hq + 2 * Hkv, D)
    q_ref = _rope_ref(x[:, :Hq], pos, D, neox)
    k_ref = _rope_ref(x[:, Hq:Hq + Hkv], pos, D, neox)
    v_ref = x[:, Hq + Hkv:]
    tol = 0.02 * x.abs().max().item()
    assert (q_out.float() - q_ref).abs().max().item() <= tol
    for t in range(T):
        sl = int(slots[t])
        if sl < 0:
            continue
        blk, off = sl // 16, sl % 16
        assert (kv[blk, 0, :, off].float() - k_ref[t]).abs().max().item() <= tol
        assert (kv[blk, 1, :, off].float() - v_ref[t]).abs().max().item() <= tol
