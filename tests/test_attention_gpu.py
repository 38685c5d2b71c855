"""Paged attention (decode, split-KV decode, prefill chunks) vs an fp32 PyTorch reference."""
import math

import pytest
import torch

from vm_c_b200 import ops

pytestmark = pytest.mark.gpu


def _setup(ctx_lens, q_lens, Hq, Hkv, D, nblocks=512, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kv = (torch.randn(nblocks, 2, Hkv, 16, D, generator=g, device="cuda") * 0.5).bfloat16()
    R = len(ctx_lens)
    max_blocks = max((c + 15) // 16 for c in ctx_lens) + 1
    perm = torch.randperm(nblocks - 1, generator=torch.Generator().manual_seed(seed)) + 1
    bt = torch.zeros(R, max_blocks, dtype=torch.int32)
    o = 0
    for r, c in enumerate(ctx_lens):
        nb = (c + 15) // 16
        bt[r, :nb] = perm[o:o + nb].int()
        o += nb
    T = sum(q_lens)
    q = (torch.randn(T, Hq, D, generator=g, device="cuda")).bfloat16()
    qs = torch.tensor([0] + list(torch.cumsum(torch.tensor(q_lens), 0)), dtype=torch.int32)
    return kv, bt.cuda(), q, qs.cuda(), torch.tensor(ctx_lens, dtype=torch.int32).cuda(), T


def _ref(kv, bt, q, qs, ctx, Hq, Hkv, D):
    G = Hq // Hkv
    out = torch.zeros_like(q, dtype=torch.float32)
    for r in range(ctx.numel()):
        c = int(ctx[r]); a, b = int(qs[r]), int(qs[r + 1]); ql = b - a
        nb = (c + 15) // 16
        blocks = bt[r, :nb].long()
        K = kv[blocks, 0].permute(1, 0, 2, 3).reshape(Hkv, nb * 16, D)[:, :c].float()
        V = kv[blocks, 1].permute(1, 0, 2, 3).reshape(Hkv, nb * 16, D)[:, :c].float()
        for h in range(Hq):
            kvh = h // G
            s = q[a:b, h].float() @ K[kvh].T / math.sqrt(D)
            qpos = torch.arange(c - ql, c, device=q.device)[:, None]
            kpos = torch.arange(c, device=q.device)[None, :]
            s = s.masked_fill(kpos > qpos, float("-inf"))
            out[a:b, h] = torch.softmax(s, -1) @ V[kvh]
    return out


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 32, 8), (64, 32, 8), (32, 8, 4), (128, 8, 1)])
def test_decode(cuda_ext, D, Hq, Hkv):
    ctx = [1, 17, 100, 515, 1024, 33]
    kv, bt, q, qs, cl, T = _setup(ctx, [1] * len(ctx), Hq, Hkv, D)
    out = torch.empty_like(q)
    ops.paged_attention(q, kv, qs, cl, bt, len(ctx), 0, 1, T, Hq, Hkv, D, 1 / math.sqrt(D), True, out)
    torch.cuda.synchronize()
    ref = _ref(kv, bt, q, qs, cl, Hq, Hkv, D)
    assert (out.float() - ref).abs().max().item() < 2e-2


def test_decode_split_kv(cuda_ext):
    D, Hq, Hkv = 128, 32, 8
    ctx = [700, 1500, 3]
    kv, bt, q, qs, cl, T = _setup(ctx, [1] * 3, Hq, Hkv, D, nblocks=300)
    out = torch.empty_like(q)
    S = 5
    po = torch.empty(S, T, Hq, D, device="cuda")
    pl = torch.empty(S, T, Hq, device="cuda")
    ops.paged_attention(q, kv, qs, cl, bt, 3, 0, 1, T, Hq, Hkv, D, 1 / math.sqrt(D), True, out, S, po, pl)
    torch.cuda.synchronize()
    ref = _ref(kv, bt, q, qs, cl, Hq, Hkv, D)
    assert (out.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 32, 8), (32, 8, 4), (64, 16, 2)])
def test_prefill_chunks(cuda_ext, D, Hq, Hkv):
    # (context after step, q_len): fresh prompt, chunk continuing a cached prefix, tiny extends
    ctx = [100, 300, 64, 5, 1024]
    ql = [100, 77, 64, 2, 512]
    kv, bt, q, qs, cl, T = _setup(ctx, ql, Hq, Hkv, D)
    out = torch.empty_like(q)
    ops.paged_attention(q, kv, qs, cl, bt, len(ctx), 0, max(ql), T, Hq, Hkv, D, 1 / math.sqrt(D), False, out)
    torch.cuda.synchronize()
    ref = _ref(kv, bt, q, qs, cl, Hq, Hkv, D)
    assert (out.float() - ref).abs().max().item() < 2e-2


def test_mixed_offsets(cuda_ext):
    # decodes first (req_offset 0), then prefill requests launched with req_offset = num_decode
    D, Hq, Hkv = 128, 32, 8
    ctx = [50, 60, 200, 129]
    ql = [1, 1, 120, 129]
    kv, bt, q, qs, cl, T = _setup(ctx, ql, Hq, Hkv, D)
    out = torch.empty_like(q)
    ops.paged_attention(q, kv, qs, cl, bt, 2, 0, 1, 2, Hq, Hkv, D, 1 / math.sqrt(D), True, out)
    ops.paged_attention(q, kv, qs, cl, bt, 2, 2, 129, T, Hq, Hkv, D, 1 / math.sqrt(D), False, out)
    torch.cuda.synchronize()
    ref = _ref(kv, bt, q, qs, cl, Hq, Hkv, D)
    assert (out.float() - ref).abs().max().item() < 2e-2
