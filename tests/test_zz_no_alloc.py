"""The allocation-free C entry point of split-KV decode attention (attention_noalloc.cu).

Calls the exported symbol through ctypes, twice in a row, and compares both results with the
regular entry point (ops.paged_attention with PyTorch-allocated partial buffers) and with an fp32
PyTorch reference. The file name sorts last so that it also runs after every other GPU test.
"""
import ctypes
import math

import pytest
import torch

from vm_c_b200 import ops

pytestmark = pytest.mark.gpu


def _lib():
    from vm_c_b200 import _native
    lib = ctypes.CDLL(_native.cuda().__file__)
    fn = lib.vmc_paged_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = ([ctypes.c_void_p] * 5 + [ctypes.c_int] * 6 +
                   [ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int])
    return fn


def _setup(ctx_lens, Hq, Hkv, D, q_len=1, nblocks=400, seed=3):
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
    q = torch.randn(R * q_len, Hq, D, generator=g, device="cuda").bfloat16()
    qs = torch.arange(0, R * q_len + 1, q_len, dtype=torch.int32, device="cuda")
    return kv, bt.cuda(), q, qs, torch.tensor(ctx_lens, dtype=torch.int32, device="cuda")


def _ref(kv, bt, q, ctx, Hq, Hkv, D, q_len=1):
    """fp32 causal attention: token j (of q_len) of request r sees the first ctx - q_len + 1 + j keys."""
    G = Hq // Hkv
    out = torch.zeros_like(q, dtype=torch.float32)
    for r in range(ctx.numel()):
        c = int(ctx[r])
        nb = (c + 15) // 16
        blocks = bt[r, :nb].long()
        K = kv[blocks, 0].permute(1, 0, 2, 3).reshape(Hkv, nb * 16, D)[:, :c].float()
        V = kv[blocks, 1].permute(1, 0, 2, 3).reshape(Hkv, nb * 16, D)[:, :c].float()
        for j in range(q_len):
            row = r * q_len + j
            n = c - q_len + 1 + j
            for h in range(Hq):
                s = q[row, h].float() @ K[h // G, :n].T / math.sqrt(D)
                out[row, h] = torch.softmax(s, -1) @ V[h // G, :n]
    return out


def _call(fn, kv, bt, q, qs, cl, Hq, Hkv, D, splits, out, q_len=1):
    err = ctypes.create_string_buffer(256)
    rc = fn(q.data_ptr(), kv.data_ptr(), qs.data_ptr(), cl.data_ptr(), bt.data_ptr(), bt.shape[1],
            q.shape[0] // q_len, q_len, Hq, Hkv, D, 1.0 / math.sqrt(D), splits, out.data_ptr(),
            torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode()


@pytest.fixture(scope="module")
def fn(cuda_ext):
    return _lib()


@pytest.mark.parametrize("q_len,D,splits", [(1, 128, 4), (1, 64, 1), (2, 128, 8), (2, 64, 8), (1, 128, 8)])
def test_noalloc_matches_regular_entry_point(fn, q_len, D, splits):
    # GQA 4 (q_len 1 or 2 rows per KV group fit the 16-row decode tile); one context of 3 tokens,
    # shorter than `splits` pages, leaves most of its split ranges empty (the -inf LSE path).
    Hq, Hkv = 32, 8
    ctx = [700, 1500, 3, 64, 257]
    kv, bt, q, qs, cl = _setup(ctx, Hq, Hkv, D, q_len=q_len)
    R = len(ctx)
    T = R * q_len
    want = torch.empty_like(q)
    po = torch.empty(splits, T, Hq, D, device="cuda")
    pl = torch.empty(splits, T, Hq, device="cuda")
    ops.paged_attention(q, kv, qs, cl, bt, R, 0, q_len, T, Hq, Hkv, D, 1 / math.sqrt(D), True, want, splits,
                        po if splits > 1 else None, pl if splits > 1 else None)
    ref = _ref(kv, bt, q, cl, Hq, Hkv, D, q_len)
    for _ in range(2):  # two calls in a row reuse the same static scratch
        got = torch.full_like(q, float("nan"))
        rc, msg = _call(fn, kv, bt, q, qs, cl, Hq, Hkv, D, splits, got, q_len)
        assert rc == 0, msg
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert (got.float() - want.float()).abs().max().item() < 1e-2
        assert (got.float() - ref).abs().max().item() < 2e-2


def test_noalloc_rejects_oversized_request(fn):
    Hq, Hkv, D = 32, 8, 128
    kv, bt, q, qs, cl = _setup([40] * 64, Hq, Hkv, D)
    out = torch.empty_like(q)
    rc, msg = _call(fn, kv, bt, q, qs, cl, Hq, Hkv, D, 16, out)  # 16 * 64 * 32 * 129 floats > 4 MiB
    assert rc == -2 and "scratch" in msg
