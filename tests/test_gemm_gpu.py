"""tcgen05 fused-dequant GEMM vs an fp32 PyTorch reference of the same op."""
import numpy as np
import pytest
import torch

from vm_c_b200 import ops
from vm_c_b200.gguf.constants import GType

pytestmark = pytest.mark.gpu


def _ref(x, host, gtype, raw_np, N, K):
    if gtype in (GType.F32, GType.F16, GType.BF16):
        w = raw_np.astype(np.float32)
    else:
        w = host.dequantize(int(gtype), raw_np, N, K)
    w = torch.from_numpy(np.asarray(w, dtype=np.float32)).cuda()
    # dequantised weights are rounded to bf16 by the kernel before the MMA
    w = w.to(torch.bfloat16).float()
    return x.float() @ w.T


def _make(host, gtype, N, K, seed=0):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    if gtype == GType.F32:
        raw = w
        t = torch.from_numpy(w).cuda()
    elif gtype == GType.BF16:
        t = torch.from_numpy(w).cuda().bfloat16()
        raw = t.float().cpu().numpy()
    else:
        q = host.quantize(int(gtype), w)
        raw = q
        t = torch.from_numpy(q).cuda()
    tw = ops.tile_weight(t, int(gtype), N, K)
    return tw, raw


@pytest.mark.parametrize("gtype", [GType.Q4_K, GType.Q6_K, GType.Q8_0, GType.BF16, GType.F32])
@pytest.mark.parametrize("M", [1, 5, 64, 130, 300])
def test_gemm_matches_reference(host, cuda_ext, gtype, M):
    N, K = 384, 512
    tw, raw = _make(host, gtype, N, K, seed=M)
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, tw, out, M, ops.OUT_BF16, 1)
    torch.cuda.synchronize()
    ref = _ref(x, host, gtype, raw, N, K)
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert ops.device_error() == 0
    assert err <= 0.02 * scale + 1e-3, (err, scale)


@pytest.mark.parametrize("gtype", [GType.Q4_K, GType.Q6_K, GType.BF16])
def test_gemm_split_k_f32_accumulate(host, cuda_ext, gtype):
    N, K, M = 256, 2048, 48
    tw, raw = _make(host, gtype, N, K, seed=3)
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    ops.gemm(x, tw, out, M, ops.OUT_F32_ADD, 4)
    torch.cuda.synchronize()
    ref = _ref(x, host, gtype, raw, N, K)
    assert (out - ref).abs().max().item() <= 0.01 * ref.abs().max().item() + 1e-3


def test_gemm_odd_k_bf16(host, cuda_ext):
    # K not a multiple of 64 (tiny-llama FFN 688): zero-filled tails on both operands.
    N, K, M = 256, 688, 17
    tw, raw = _make(host, GType.F32, N, K, seed=5)
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, tw, out, M, ops.OUT_BF16, 1)
    torch.cuda.synchronize()
    ref = _ref(x, host, GType.F32, raw, N, K)
    assert (out.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item() + 1e-3


@pytest.mark.parametrize("M", [3, 64, 257])
def test_gemm_fused_swiglu(host, cuda_ext, M):
    F, K = 256, 512
    rng = np.random.default_rng(11)
    g = (rng.standard_normal((F, K)) * 0.05).astype(np.float32)
    u = (rng.standard_normal((F, K)) * 0.05).astype(np.float32)
    inter = np.stack([g, u], 1).reshape(2 * F, K)
    q = host.quantize(int(GType.Q4_K), inter)
    tw = ops.tile_weight(torch.from_numpy(q).cuda(), int(GType.Q4_K), 2 * F, K)
    x = (torch.randn(M, K, device="cuda")).bfloat16()
    out = torch.empty(M, F, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, tw, out, M, ops.OUT_SWIGLU, 1)
    torch.cuda.synchronize()
    w = torch.from_numpy(host.dequantize(int(GType.Q4_K), q, 2 * F, K)).cuda().bfloat16().float()
    y = x.float() @ w.T
    gg, uu = y[:, 0::2], y[:, 1::2]
    ref = torch.nn.functional.silu(gg) * uu
    assert (out.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item() + 1e-3


def test_gpu_quantizers_match_host(host, cuda_ext):
    x = torch.randn(64, 1024) * 0.02
    for gt in (GType.Q8_0, GType.Q4_K, GType.Q6_K):
        dev = ops.quantize_blocks(int(gt), x.cuda()).cpu().numpy()
        ref = host.quantize(int(gt), x.numpy())
        diff = (dev != ref).mean()
        assert diff < 1e-3, (gt, diff)


@pytest.mark.parametrize("gtype", [GType.Q4_K, GType.Q8_0, GType.BF16])
@pytest.mark.parametrize("M", [1, 64])
def test_gemm_split_partials(host, cuda_ext, gtype, M):
    # per-split fp32 partials (no atomics): their sum equals the full product
    N, K, S = 640, 2048, 3
    tw, raw = _make(host, gtype, N, K, seed=7)
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    out = torch.full((S, M, N), float("nan"), dtype=torch.float32, device="cuda")
    ops.gemm(x, tw, out[0], M, ops.OUT_F32_SPLIT, S, split_stride=M * N)
    torch.cuda.synchronize()
    ref = _ref(x, host, gtype, raw, N, K)
    assert (out.sum(0) - ref).abs().max().item() <= 0.01 * ref.abs().max().item() + 1e-3


def test_gemm_many_units_persistent(host, cuda_ext):
    # more work units than SMs: every CTA walks several units with the double-buffered accumulator
    N, K, M = 128 * 200, 512, 300
    tw, raw = _make(host, GType.Q4_K, N, K, seed=9)
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, tw, out, M, ops.OUT_BF16, 1)
    torch.cuda.synchronize()
    ref = _ref(x, host, GType.Q4_K, raw, N, K)
    assert (out.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item() + 1e-3


@pytest.mark.parametrize("gtype,N,K,M", [(GType.Q4_K, 1024, 14336, 64), (GType.Q6_K, 512, 4096, 7),
                                         (GType.Q8_0, 4096, 512, 33), (GType.Q4_K, 6144, 4096, 1)])
def test_gemm_stream_k_decode_shapes(host, cuda_ext, gtype, N, K, M):
    # Decode-width quantized GEMMs run the stream-K schedule: tiles are cut across CTAs (heads,
    # middles and tails), the finisher adds the later CTAs' partials. Repeated launches check that the
    # per-tile arrival counters are reset by their finishers.
    tw, raw = _make(host, gtype, N, K, seed=N + M)
    ref = None
    for rep in range(3):
        x = (torch.randn(M, K, device="cuda", generator=torch.Generator(device="cuda").manual_seed(rep)) * 0.5
             ).bfloat16()
        out = torch.empty(M, N, dtype=torch.float32, device="cuda")
        ops.gemm(x, tw, out, M, ops.OUT_F32, 1)
        torch.cuda.synchronize()
        ref = _ref(x, host, gtype, raw, N, K)
        err = (out - ref).abs().max().item()
        assert ops.device_error() == 0
        assert err <= 0.01 * ref.abs().max().item() + 1e-3, (rep, err)


def test_gemm_stream_k_swiglu(host, cuda_ext):
    N, K, M = 2 * 2816, 4096, 24   # interleaved gate / up rows
    tw, raw = _make(host, GType.Q4_K, N, K, seed=5)
    tw.interleaved_swiglu = True
    x = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    out = torch.empty(M, N // 2, dtype=torch.bfloat16, device="cuda")
    ops.gemm(x, tw, out, M, ops.OUT_SWIGLU, 1)
    torch.cuda.synchronize()
    y = _ref(x, host, GType.Q4_K, raw, N, K)
    g, u = y[:, 0::2], y[:, 1::2]
    ref = torch.nn.functional.silu(g) * u
    assert ops.device_error() == 0
    assert (out.float() - ref).abs().max().item() <= 0.02 * ref.abs().max().item() + 1e-3
