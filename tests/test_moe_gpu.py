"""Mixture of experts: routing kernel, grouped tcgen05 GEMM, expert placements and the end-to-end
tiny Mixtral model, each against an fp32 PyTorch restatement."""
import types

import numpy as np
import pytest
import torch

from vm_c_b200 import _native, ops
from vm_c_b200.core.sampling_params import SamplingParams
from vm_c_b200.gguf.constants import GType
from vm_c_b200.gguf.random_init import preset, write_random_gguf
from vm_c_b200.gguf.reader import GgufSource

from ref_llama import forward_logits, load_dense

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_moe(tmp_path_factory):
    p = tmp_path_factory.mktemp("moe") / "tiny-mixtral-q8.gguf"
    write_random_gguf(str(p), preset("tiny-mixtral"), "Q8_0", seed=0)
    return str(p)


def _route(logits, k, e0, el):
    T, E = logits.shape
    dev = logits.device
    i32 = dict(dtype=torch.int32, device=dev)
    out = dict(topk_id=torch.zeros(T * k, **i32), topk_w=torch.zeros(T * k, device=dev),
               counts=torch.zeros(el, **i32), offsets=torch.zeros(el, **i32), sorted_src=torch.zeros(T * k, **i32),
               slot_row=torch.zeros(T * k, **i32), total=torch.zeros(1, **i32))
    ops.moe_route(logits, T, E, k, True, e0, el, out["topk_id"], out["topk_w"], out["counts"], out["offsets"],
                  out["sorted_src"], out["slot_row"], out["total"])
    torch.cuda.synchronize()
    return {n: v.cpu() for n, v in out.items()}


@pytest.mark.parametrize("e0,el", [(0, 8), (4, 4), (2, 1)])
def test_route_matches_torch(cuda_ext, e0, el):
    torch.manual_seed(0)
    T, E, k = 37, 8, 2
    logits = torch.randn(T, E, device="cuda")
    r = _route(logits, k, e0, el)
    p = torch.softmax(logits.cpu(), -1)
    w, idx = torch.topk(p, k, -1)
    w = w / w.sum(-1, keepdim=True)
    assert torch.equal(r["topk_id"].view(T, k), idx.int())
    assert torch.allclose(r["topk_w"].view(T, k), w, atol=1e-5)
    pos = 0
    for j, e in enumerate(range(e0, e0 + el)):
        toks = [t for t in range(T) for s in range(k) if int(idx[t, s]) == e]
        assert int(r["counts"][j]) == len(toks) and int(r["offsets"][j]) == pos
        assert r["sorted_src"][pos:pos + len(toks)].tolist() == toks  # stable: token order
        pos += len(toks)
    assert int(r["total"][0]) == pos
    for t in range(T):
        for s in range(k):
            row = int(r["slot_row"][t * k + s])
            if e0 <= int(idx[t, s]) < e0 + el:
                assert int(r["sorted_src"][row]) == t
            else:
                assert row == -1


@pytest.mark.parametrize("counts", [[5, 0, 70], [130, 0, 300], [1, 1, 1]])
@pytest.mark.parametrize("gt,mode", [(GType.Q4_K, ops.OUT_F32), (GType.Q8_0, ops.OUT_SWIGLU)])
def test_grouped_gemm(cuda_ext, counts, gt, mode):
    torch.manual_seed(1)
    G, N, K = len(counts), 512, 512
    h = _native.host()
    tiles, dense = [], []
    for g in range(G):
        x = torch.randn(N, K, device="cuda") * 0.02
        raw = ops.quantize_blocks(int(gt), x)
        dense.append(torch.from_numpy(h.dequantize(int(gt), raw.cpu().numpy(), N, K)))
        tiles.append(ops.tile_weight(raw, int(gt), N, K))
    w = ops.TiledWeight(tiles[0].wf, torch.cat([t.data for t in tiles]), N, K, interleaved_swiglu=mode == ops.OUT_SWIGLU)
    R = sum(counts)
    xs = torch.randn(R + 3, K, device="cuda").bfloat16()
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    off = torch.tensor(np.cumsum([0] + counts[:-1]), dtype=torch.int32, device="cuda")
    ncol = N // 2 if mode == ops.OUT_SWIGLU else N
    out = torch.full((R + 3, ncol), float("nan"), device="cuda",
                     dtype=torch.bfloat16 if mode == ops.OUT_SWIGLU else torch.float32)
    bn = ops.pick_bn(max(1, R // G))
    ops.gemm_grouped(xs, w, G, tiles[0].nbytes, R, cnt, off, max(counts), out, mode, bn=bn)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    o = 0
    for g, c in enumerate(counts):
        if c:
            ref = xs[o:o + c].float().cpu() @ dense[g].T
            if mode == ops.OUT_SWIGLU:
                ref = torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2]
            got = out[o:o + c].float().cpu()
            err = (got - ref).abs().max().item()
            assert err < 2e-2 * max(1.0, ref.abs().max().item()), (g, err)
        o += c
    assert torch.isnan(out[R:].float()).all()  # rows past the groups untouched


def _moe_out(src, cfg, layer, h, tp_rank, tp_size, ep_size):
    from vm_c_b200.models.moe import MoERunner, load_moe_layer
    moe = load_moe_layer(src, cfg, layer, torch.device("cuda"), tp_rank, tp_size, ep_size)
    shim = types.SimpleNamespace(cfg=cfg, dev=h.device, w=types.SimpleNamespace(layers=[types.SimpleNamespace(moe=moe)]))
    run = MoERunner(shim, h.shape[0])
    out, _ = run.forward(moe, h, h.shape[0])
    torch.cuda.synchronize()
    return out.clone()


@pytest.fixture(scope="module")
def tiny_moe8(tmp_path_factory):
    p = tmp_path_factory.mktemp("moe8") / "tiny-mixtral8-q8.gguf"
    write_random_gguf(str(p), preset("tiny-mixtral8"), "Q8_0", seed=0)
    return str(p)


@pytest.mark.parametrize("model,tp,ep,T", [("tiny_moe", 2, 1, 23), ("tiny_moe", 2, 2, 23), ("tiny_moe", 4, 4, 23),
                                           ("tiny_moe8", 2, 2, 23), ("tiny_moe8", 2, 2, 162),
                                           ("tiny_moe8", 4, 4, 8), ("tiny_moe8", 8, 8, 162)])
def test_expert_placements_sum_to_full(cuda_ext, request, model, tp, ep, T):
    # Every placement's per-rank partial outputs sum to the single-rank output (the all-reduce of
    # the expert-parallel NCCL path), for 4 and 8 experts and decode- and prefill-sized batches.
    src = GgufSource(request.getfixturevalue(model))
    cfg = src.model_config()
    torch.manual_seed(2)
    h = (torch.randn(T, cfg.hidden, device="cuda")).bfloat16()
    full = _moe_out(src, cfg, 1, h, 0, 1, 1)
    parts = sum(_moe_out(src, cfg, 1, h, r, tp, ep) for r in range(tp))
    assert (parts - full).abs().max().item() < 2e-2 * full.abs().max().item()
    # and the full output against the fp32 restatement
    W = load_dense(src, cfg)
    from ref_llama import moe_ffn
    ref = moe_ffn(W["layers"][1], cfg, h.float().cpu())
    assert (full.cpu() - ref).abs().max().item() < 3e-2 * ref.abs().max().item()


def test_tiny_mixtral_matches_oracle(tiny_moe):
    from vm_c_b200.llm import LLM
    llm = LLM(tiny_moe, max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256, num_gpu_blocks=256)
    src = GgufSource(tiny_moe)
    cfg = src.model_config()
    W = load_dense(src, cfg)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, cfg.vocab, 16).tolist()
    toks = llm.generate([prompt], SamplingParams.greedy_params(max_tokens=8, ignore_eos=True))[0].output_token_ids
    logits = forward_logits(W, cfg, prompt + toks[:-1])
    agree = 0
    for i, t in enumerate(toks):
        row = logits[len(prompt) - 1 + i]
        if int(row.argmax()) == t:
            agree += 1
        else:
            assert float(row.max() - row[t]) < 0.05 * float(row.abs().max()), (i, t, int(row.argmax()))
    assert agree >= len(toks) - 1
    llm.shutdown()
