"""TurboQuant KV cache on the GPU: the fused RoPE + rotate + quantise store against a PyTorch
restatement of the slot format, and decode / prefill attention over the compressed cache against
fp32 attention over the same dequantised values."""
import math

import numpy as np
import pytest
import torch
from scipy.linalg import hadamard

from vm_c_b200 import ops

pytestmark = pytest.mark.gpu

METHODS = ["turboquant_4bit_nc", "turboquant_k8v4", "turboquant_k3v4_nc", "turboquant_3bit_nc"]


def _sign(seed, layer, kvh, d):
    if seed == 0:
        return 1.0
    m = 0xFFFFFFFF
    x = (seed ^ ((layer * 0x9E3779B1) & m) ^ ((kvh * 0x85EBCA77) & m) ^ ((d * 0xC2B2AE3D) & m)) & m
    x ^= x >> 16
    x = (x * 0x7FEB352D) & m
    x ^= x >> 15
    x = (x * 0x846CA68B) & m
    x ^= x >> 16
    return -1.0 if x & 1 else 1.0


def _rope(x, pos, D, theta=10000.0):
    inv = 1.0 / (theta ** (np.arange(0, D, 2) / D))
    ang = pos[:, None].double() * torch.tensor(inv)[None, :]
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def _bf16(x):
    return torch.tensor(x, dtype=torch.float32).bfloat16().float().item()


def _bits(byts, nbits, n):
    """Unpack n little-endian nbits-wide fields from a uint8 array."""
    v = 0
    for i, b in enumerate(byts):
        v |= int(b) << (8 * i)
    return [(v >> (nbits * i)) & ((1 << nbits) - 1) for i in range(n)]


def _setup(method, D, Hq=8, Hkv=2, ctx=(37, 70, 16), seed=11, rot_seed=0):
    torch.manual_seed(seed)
    dev = "cuda"
    tab = ops.TqTables(method, D, dev, rot_seed=rot_seed)
    T = sum(ctx)
    qkv = (torch.randn(T, (Hq + 2 * Hkv) * D, device=dev) * 0.7).bfloat16()
    pos = torch.cat([torch.arange(c) for c in ctx]).int().to(dev)
    nblocks = sum((c + 15) // 16 for c in ctx) + 1
    bt = torch.zeros(len(ctx), max((c + 15) // 16 for c in ctx), dtype=torch.int32)
    slots = []
    o = 1
    for r, c in enumerate(ctx):
        nb = (c + 15) // 16
        bt[r, :nb] = torch.arange(o, o + nb)
        slots += [int(bt[r, i // 16]) * 16 + i % 16 for i in range(c)]
        o += nb
    slots = torch.tensor(slots, dtype=torch.int32, device=dev)
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = torch.arange(4096, dtype=torch.float64)[:, None] * inv[None, :]
    cos_sin = torch.stack([ang.cos(), ang.sin()], -1).float().to(dev).contiguous()
    cache = torch.zeros(nblocks, 16, Hkv, tab.slot_bytes, dtype=torch.uint8, device=dev)
    q_out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
    ops.rope_store_tq(qkv, T, Hq, Hkv, D, pos, slots, cos_sin, False, q_out, cache, tab, layer=3)
    torch.cuda.synchronize()
    return dict(tab=tab, qkv=qkv, pos=pos, slots=slots, bt=bt.to(dev), cache=cache, q_out=q_out, ctx=ctx, T=T, Hq=Hq,
                Hkv=Hkv, D=D, cos_sin=cos_sin)


def _dequant(S):
    """fp32 K [T, Hkv, D] (rotated space) and V from the cache bytes (restated decoder)."""
    L, tab, D, Hkv = S["tab"].layout, S["tab"], S["D"], S["Hkv"]
    cache = S["cache"].cpu().numpy()
    cent = tab.centroids.cpu().numpy()
    K = torch.zeros(S["T"], Hkv, D)
    V = torch.zeros(S["T"], Hkv, D)
    for t, sl in enumerate(S["slots"].tolist()):
        for h in range(Hkv):
            sp = cache[sl // 16, sl % 16, h]
            if L["key_fp8"]:
                k = torch.from_numpy(sp[:D].copy()).view(torch.float8_e4m3fn).float()
            else:
                idx = _bits(sp[:L["mse_bytes"]], L["key_bits"], D)
                c = torch.tensor(cent[idx], dtype=torch.float64)
                norm = torch.from_numpy(sp[L["mse_bytes"]:L["mse_bytes"] + 2].copy()).view(torch.bfloat16).float()
                k = c * (norm / torch.sqrt((c * c).sum() + 1e-16) if L["norm_correction"] else norm)
            vb = sp[L["key_packed"]:]
            q = torch.tensor(_bits(vb[:L["val_bytes"]], L["value_bits"], D), dtype=torch.float64)
            sc = torch.from_numpy(vb[L["val_bytes"]:L["val_bytes"] + 2].copy()).view(torch.bfloat16).float()
            mn = torch.from_numpy(vb[L["val_bytes"] + 2:L["val_bytes"] + 4].copy()).view(torch.bfloat16).float()
            K[t, h] = k.float()
            V[t, h] = (q * sc + mn).float()
    return K, V


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("rot_seed", [0, 12345])
def test_store_matches_restatement(cuda_ext, method, D, rot_seed):
    S = _setup(method, D, rot_seed=rot_seed)
    L, tab, Hq, Hkv = S["tab"].layout, S["tab"], S["Hq"], S["Hkv"]
    x = S["qkv"].float().cpu().view(S["T"], Hq + 2 * Hkv, D).double()
    pos = S["pos"].cpu()
    q = _rope(x[:, :Hq], pos, D)
    k = _rope(x[:, Hq:Hq + Hkv], pos, D)
    v = x[:, Hq + Hkv:]
    Hm = torch.tensor(hadamard(D), dtype=torch.float64) / math.sqrt(D)
    mids = tab.midpoints.cpu().double().numpy()
    cache = S["cache"].cpu().numpy()
    qo = S["q_out"].float().cpu()
    G = Hq // Hkv
    idx_bad = idx_tot = v_bad = 0
    for t, sl in enumerate(S["slots"].tolist()):
        for h in range(Hq):
            ref = q[t, h]
            if not L["key_fp8"]:
                s = torch.tensor([_sign(rot_seed, 3, h // G, d) for d in range(D)], dtype=torch.float64)
                ref = Hm @ (s * ref)
            assert torch.allclose(qo[t, h].double(), ref, atol=2e-2 * ref.abs().max().item() + 1e-3)
        for h in range(Hkv):
            sp = cache[sl // 16, sl % 16, h]
            if L["key_fp8"]:
                got = torch.from_numpy(sp[:D].copy()).view(torch.float8_e4m3fn).float()
                want = k[t, h].float().to(torch.float8_e4m3fn).float()
                idx_bad += int((got != want).sum())
                idx_tot += D
            else:
                s = torch.tensor([_sign(rot_seed, 3, h, d) for d in range(D)], dtype=torch.float64)
                norm = k[t, h].norm()
                y = (Hm @ (s * k[t, h] / norm)).numpy()
                want = np.searchsorted(mids, y, side="right")
                got = np.array(_bits(sp[:L["mse_bytes"]], L["key_bits"], D))
                idx_bad += int((got != want).sum())
                idx_tot += D
                gn = torch.from_numpy(sp[L["mse_bytes"]:L["mse_bytes"] + 2].copy()).view(torch.bfloat16).float()
                assert abs(gn.item() - _bf16(norm.item())) <= 1e-2 * norm.item()
            vb = sp[L["key_packed"]:]
            qmax = (1 << L["value_bits"]) - 1
            mn, mx = v[t, h].min().item(), v[t, h].max().item()
            scale = max((mx - mn) / qmax, 1e-8)
            want_q = np.clip(np.floor((v[t, h].numpy() - mn) / scale + 0.5), 0, qmax)
            got_q = np.array(_bits(vb[:L["val_bytes"]], L["value_bits"], D))
            v_bad += int((got_q != want_q).sum())
            sc = torch.from_numpy(vb[L["val_bytes"]:L["val_bytes"] + 2].copy()).view(torch.bfloat16).float().item()
            m0 = torch.from_numpy(vb[L["val_bytes"] + 2:L["val_bytes"] + 4].copy()).view(torch.bfloat16).float().item()
            assert abs(sc - _bf16(scale)) <= 1e-2 * scale and abs(m0 - _bf16(mn)) <= 1e-2 * abs(mn) + 1e-6
    # fp32 rounding order may move a value across a quantisation boundary now and then
    assert idx_bad <= 0.01 * idx_tot, (idx_bad, idx_tot)
    assert v_bad <= 0.01 * S["T"] * Hkv * D, v_bad


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("decode", [True, False])
def test_attention_over_compressed_cache(cuda_ext, method, D, decode):
    S = _setup(method, D)
    K, V = _dequant(S)
    Hq, Hkv, ctx = S["Hq"], S["Hkv"], S["ctx"]
    G = Hq // Hkv
    qall = S["q_out"]
    starts = np.cumsum([0] + list(ctx))
    if decode:
        rows = [int(starts[r + 1] - 1) for r in range(len(ctx))]
        q = qall[rows].contiguous()
        qs = torch.arange(len(ctx) + 1, dtype=torch.int32, device="cuda")
        qlens = [1] * len(ctx)
    else:
        q = qall
        qs = torch.tensor(starts, dtype=torch.int32, device="cuda")
        qlens = list(ctx)
    cl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    ops.paged_attention(q, S["cache"], qs, cl, S["bt"], len(ctx), 0, max(qlens), q.shape[0], Hq, Hkv, D,
                        1 / math.sqrt(D), decode, out, tq=(S["cache"], S["tab"]))
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    qf = q.float().cpu()
    o = 0
    for r, c in enumerate(ctx):
        kr, vr = K[starts[r]:starts[r] + c], V[starts[r]:starts[r] + c]
        ql = qlens[r]
        for i in range(ql):
            qpos = c - ql + i
            for h in range(Hq):
                s = (kr[:qpos + 1, h // G] @ qf[o + i, h]) / math.sqrt(D)
                ref = torch.softmax(s, 0) @ vr[:qpos + 1, h // G]
                got = out[o + i, h].float().cpu()
                assert (got - ref).abs().max().item() < 3e-2 * max(1.0, ref.abs().max().item()), (r, i, h)
        o += ql


def test_tiny_llama_turboquant_runs(tmp_path):
    from vm_c_b200.core.sampling_params import SamplingParams
    from vm_c_b200.gguf.random_init import preset, write_random_gguf
    from vm_c_b200.llm import LLM
    p = tmp_path / "tiny.gguf"
    write_random_gguf(str(p), preset("tiny-llama"), "Q8_0", seed=0)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 32000, n).tolist() for n in (5, 40, 100)]
    sp = SamplingParams.greedy_params(max_tokens=8, ignore_eos=True)
    ref = LLM(str(p), max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256, num_gpu_blocks=256)
    want = [o.output_token_ids for o in ref.generate(prompts, sp)]
    ref_bytes = ref.runner.kv_bytes_per_token
    ref.shutdown()
    # no prefix caching: a second run must recompute the same prompts the same way
    llm = LLM(str(p), max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256, num_gpu_blocks=256,
              kv_cache_dtype="turboquant_4bit_nc", tq_rotation_seed=7, enable_prefix_caching=False)
    assert llm.runner.kv.dtype == torch.uint8
    assert llm.runner.kv_bytes_per_token < ref_bytes / 3
    got = [o.output_token_ids for o in llm.generate(prompts, sp)]
    assert got == [o.output_token_ids for o in llm.generate(prompts, sp)]  # deterministic
    # 4-bit keys / values change the logits a little: most greedy tokens still agree
    agree = sum(a == b for g, w in zip(got, want) for a, b in zip(g, w))
    assert agree >= 0.6 * sum(len(w) for w in want), (got, want)
    llm.shutdown()
