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


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (64, 8), (8, 8), (4, 1)])
@pytest.mark.parametrize("tc", [True, False])
def test_prefill_head128_paths(cuda_ext, Hq, Hkv, tc):
    # Head dim 128, bf16 pages: the tcgen05 kernel (tc=True, 128 packed rows x 128-key tiles) and the
    # mma.sync kernel, on fresh prompts, chunks continuing a cached prefix (context > q_len), ragged
    # row and key counts, and a 2048-token context.
    D = 128
    ctx = [1024, 2048, 300, 129, 17, 640]
    ql = [1024, 700, 77, 129, 17, 1]
    kv, bt, q, qs, cl, T = _setup(ctx, ql, Hq, Hkv, D, nblocks=400)
    out = torch.full_like(q, float("nan"))
    ops.C().attention_tc(tc)
    try:
        ops.paged_attention(q, kv, qs, cl, bt, len(ctx), 0, max(ql), T, Hq, Hkv, D, 1 / math.sqrt(D), False, out)
        torch.cuda.synchronize()
    finally:
        ops.C().attention_tc(True)
    assert ops.device_error() == 0
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


@pytest.mark.parametrize("span_extra", [0, 3])
def test_prefill_tree_mask(cuda_ext, span_extra):
    # Queries are the last q_len positions; the tree spans the last q_len + span_extra positions
    # (span_extra > 0: earlier tree levels that are keys only, as in the draft's per-depth passes).
    from vm_c_b200.speculative.tree import TokenTree
    tree = TokenTree([2, 2, 1])
    Hq, Hkv, D = 32, 8, 128
    span = tree.N
    ql = span - span_extra
    ctx = [40 + span, 300 + span]
    kv, bt, q, qs, cl, T = _setup(ctx, [ql, ql], Hq, Hkv, D, seed=4)
    masks = torch.tensor(list(tree.masks[span_extra:span]) * 2, dtype=torch.int64, device="cuda")
    out = torch.empty_like(q)
    ops.paged_attention(q, kv, qs, cl, bt, 2, 0, ql, T, Hq, Hkv, D, 1 / math.sqrt(D), False, out,
                        tree_mask=masks, tree_span=span)
    torch.cuda.synchronize()
    G = Hq // Hkv
    ref = torch.zeros_like(q, dtype=torch.float32)
    for r in range(2):
        c = ctx[r]; a = int(qs[r])
        nb = (c + 15) // 16
        blocks = bt[r, :nb].long()
        K = kv[blocks, 0].permute(1, 0, 2, 3).reshape(Hkv, nb * 16, D)[:, :c].float()
        V = kv[blocks, 1].permute(1, 0, 2, 3).reshape(Hkv, nb * 16, D)[:, :c].float()
        allow = torch.ones(ql, c, dtype=torch.bool, device="cuda")
        base = c - span
        for t in range(ql):
            m = int(tree.masks[span_extra + t]) & ((1 << 64) - 1)
            for i in range(span):
                allow[t, base + i] = bool((m >> i) & 1)
        for h in range(Hq):
            s = q[a:a + ql, h].float() @ K[h // G].T / math.sqrt(D)
            s = s.masked_fill(~allow, float("-inf"))
            ref[a:a + ql, h] = torch.softmax(s, -1) @ V[h // G]
    assert (out.float() - ref).abs().max().item() < 2e-2


def test_kv_move_reads_before_writes(cuda_ext):
    L, nb, Hkv, D = 3, 8, 2, 64
    cache = torch.randn(L, nb, 2, Hkv, 16, D, device="cuda").bfloat16()
    before = cache.clone()
    # request 0: 20 -> 17, 23 -> 18 (18's old content is not a source); request 1: 34 -> 33, 36 -> 34
    src = torch.tensor([[20, 23] + [0] * 14, [34, 36] + [0] * 14], dtype=torch.int32, device="cuda")
    dst = torch.tensor([[17, 18] + [0] * 14, [33, 34] + [0] * 14], dtype=torch.int32, device="cuda")
    cnt = torch.tensor([2, 2], dtype=torch.int32, device="cuda")
    ops.kv_move(cache, Hkv, D, src, dst, cnt, 2, 16)
    torch.cuda.synchronize()

    def row(c, s):
        return c[:, s // 16, :, :, s % 16]

    for s_, d_ in ((20, 17), (23, 18), (34, 33), (36, 34)):
        assert torch.equal(row(cache, d_), row(before, s_))
    for s_ in (20, 23, 36, 0, 5):
        assert torch.equal(row(cache, s_), row(before, s_))
