"""Kernel microbenchmarks at the shapes of the Llama-3-8B serving config (one GPU).

    python -m vm_c_b200.ops.bench [case ...] [--reps N]

Cases: gemm:<name> (decode / prefill projections of the 8B model, see GEMM_CASES), attn:decode,
attn:prefill (one 2048-token prompt), attn:prefill2 (two 1024-token prompts), norm, rope, swiglu,
sample, gdn:decode / gdn:prefill2 (gated delta-net conv + recurrence, 64 x 1 and 2 x 1024 tokens), and
step:decode (a whole engine decode step; not part of "all"). Each case is captured in a CUDA graph after warm-up and timed with CUDA events around the
graph replay (no host launch overhead, as in the engine's decode graphs), with a 256 MB buffer
written between repetitions so that every repetition reads its inputs from HBM; the median is reported with the achieved bandwidth / FLOP rate. These are the
cases the committed ncu summaries were captured on.
"""
from __future__ import annotations

import argparse
import math

import torch

from . import (OUT_BF16, OUT_F32_SPLIT, OUT_SWIGLU, add_rmsnorm, decode_slots, decode_splits, device_error,
               effective_splits, gemm, paged_attention, pick_splits, quantize_blocks, rope_store, sample, swiglu,
               tile_weight)
from ..gguf.constants import GType

# name: (weight type, N, K, tokens M, output mode)
GEMM_CASES = {
    "dec_qkv": (GType.Q4_K, 6144, 4096, 64, OUT_F32_SPLIT),
    "dec_o": (GType.Q4_K, 4096, 4096, 64, OUT_F32_SPLIT),
    "dec_gu": (GType.Q4_K, 28672, 4096, 64, OUT_SWIGLU),
    "dec_down": (GType.Q4_K, 4096, 14336, 64, OUT_F32_SPLIT),
    "dec_down6": (GType.Q6_K, 4096, 14336, 64, OUT_F32_SPLIT),
    "dec_lm": (GType.Q6_K, 128256, 4096, 64, OUT_F32_SPLIT),
    "dec1_gu": (GType.Q4_K, 28672, 4096, 1, OUT_SWIGLU),
    "pre_qkv": (GType.Q4_K, 6144, 4096, 2048, OUT_BF16),
    "pre_gu": (GType.Q4_K, 28672, 4096, 2048, OUT_SWIGLU),
    "pre_o": (GType.Q4_K, 4096, 4096, 2048, OUT_F32_SPLIT),
    "pre_down": (GType.Q4_K, 4096, 14336, 2048, OUT_F32_SPLIT),
    "pre_down6": (GType.Q6_K, 4096, 14336, 2048, OUT_F32_SPLIT),
    "pre_bf16": (GType.BF16, 8192, 4096, 2048, OUT_BF16),
    # per-rank shapes of the 8B model at tensor parallel 8 (decode, 64 tokens)
    "tp8_qkv": (GType.Q4_K, 768, 4096, 64, OUT_F32_SPLIT),
    "tp8_o": (GType.Q4_K, 4096, 512, 64, OUT_F32_SPLIT),
    "tp8_gu": (GType.Q4_K, 3584, 4096, 64, OUT_F32_SPLIT),
    "tp8_down": (GType.Q4_K, 4096, 1792, 64, OUT_F32_SPLIT),
}


def _time(fn, reps: int, flush: torch.Tensor) -> float:
    """Median device time of `fn` in microseconds. `fn` is captured once in a CUDA graph and the
    graph is replayed between two events, so host launch overhead (argument marshalling, tensor-map
    encoding) is not in the number, as in the engine's decode graphs."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    del g
    return sorted(ts)[len(ts) // 2]


def bench_gemm(name: str, reps: int, flush: torch.Tensor, splits: int = 0) -> str:
    gt, N, K, M, mode = GEMM_CASES[name]
    g = torch.Generator(device="cuda").manual_seed(0)
    x32 = torch.randn(N, K, device="cuda", generator=g) * 0.02
    raw = x32.bfloat16() if gt == GType.BF16 else quantize_blocks(int(gt), x32)
    del x32
    w = tile_weight(raw, int(gt), N, K)
    del raw
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    s = effective_splits(w, splits or pick_splits(w, M)) if mode == OUT_F32_SPLIT else 1
    if mode == OUT_SWIGLU:
        out = torch.empty(M, N // 2, dtype=torch.bfloat16, device="cuda")
    elif mode == OUT_BF16:
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    else:
        out = torch.empty(s * M, N, dtype=torch.float32, device="cuda")
    t = _time(lambda: gemm(x, w, out[:M] if mode == OUT_F32_SPLIT else out, M, mode, s, split_stride=M * N),
              reps, flush)
    return (f"gemm:{name:9s} M={M:5d} N={N:6d} K={K:6d} splits={s} {t:8.1f} us  weight bytes {w.nbytes / t / 1e6:5.2f} TB/s"
            f"  {2 * M * N * K / t / 1e6:7.1f} TFLOP/s")


def _paged_setup(ctx, qlen, Hq=32, Hkv=8, D=128, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nblocks = sum((c + 15) // 16 for c in ctx) + 1
    kv = (torch.randn(nblocks, 2, Hkv, 16, D, device="cuda", generator=g) * 0.5).bfloat16()
    maxb = max((c + 15) // 16 for c in ctx)
    bt = torch.zeros(len(ctx), maxb, dtype=torch.int32)
    o = 1
    for r, c in enumerate(ctx):
        nb = (c + 15) // 16
        bt[r, :nb] = torch.arange(o, o + nb, dtype=torch.int32)
        o += nb
    T = sum(qlen)
    q = torch.randn(T, Hq, D, device="cuda", generator=g).bfloat16()
    qs = torch.tensor([0] + list(torch.cumsum(torch.tensor(qlen), 0)), dtype=torch.int32, device="cuda")
    return kv, bt.cuda(), q, qs, torch.tensor(ctx, dtype=torch.int32, device="cuda"), T


def bench_attn(kind: str, reps: int, flush: torch.Tensor, splits: int = 0) -> str:
    Hq, Hkv, D = 32, 8, 128
    if kind == "decode":
        ctx, ql = [1280] * 64, [1] * 64
    elif kind == "decode_tp8":  # one rank of tensor parallel 8: 4 query heads, 1 KV head
        Hq, Hkv = 4, 1
        ctx, ql = [1040] * 64, [1] * 64
    elif kind == "prefill2":  # two 1024-token prompts: the 2048-token chunked-prefill step of serving
        ctx, ql = [1024, 1024], [1024, 1024]
    else:
        ctx, ql = [2048], [2048]
    kv, bt, q, qs, cl, T = _paged_setup(ctx, ql, Hq, Hkv, D)
    out = torch.empty_like(q)
    dec = kind.startswith("decode")
    s = (splits or decode_splits(len(ctx) * Hkv, decode_slots(D))) if dec else 1
    po = torch.empty(s, T, Hq, D, device="cuda") if s > 1 else None
    pl = torch.empty(s, T, Hq, device="cuda") if s > 1 else None
    t = _time(lambda: paged_attention(q, kv, qs, cl, bt, len(ctx), 0, max(ql), T, Hq, Hkv, D, 1 / math.sqrt(D), dec,
                                      out, s, po, pl), reps, flush)
    kv_bytes = sum(ctx) * Hkv * D * 2 * 2
    flops = sum(4 * q_ * c * Hq * D for q_, c in zip(ql, ctx)) / (1 if dec else 2)
    return (f"attn:{kind:7s} reqs={len(ctx)} ctx={ctx[0]} qlen={ql[0]} splits={s} {t:8.1f} us  KV {kv_bytes / t / 1e6:5.2f} TB/s"
            f"  {flops / t / 1e6:7.1f} TFLOP/s")


def bench_small(kind: str, reps: int, flush: torch.Tensor) -> str:
    T, H, F = 2048, 4096, 14336
    dev = "cuda"
    if kind == "norm":
        resid = torch.randn(T, H, device=dev)
        delta = torch.randn(T, H, device=dev)
        w = torch.randn(H, device=dev)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        t = _time(lambda: add_rmsnorm(resid, w, T, H, 1e-5, out=out, delta=delta), reps, flush)
        nbytes = T * H * (4 + 4 + 4 + 2)
    elif kind == "swiglu":
        gu = torch.randn(T, 2 * F, device=dev).bfloat16()
        out = torch.empty(T, F, dtype=torch.bfloat16, device=dev)
        t = _time(lambda: swiglu(gu, T, F, out, interleaved=True), reps, flush)
        nbytes = T * F * 2 * 3
    elif kind == "rope":
        Hq, Hkv, D = 32, 8, 128
        qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev).bfloat16()
        pos = torch.arange(T, dtype=torch.int32, device=dev)
        slots = torch.arange(T, dtype=torch.int32, device=dev)
        inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
        ang = torch.arange(4096, dtype=torch.float64)[:, None] * inv[None, :]
        cos_sin = torch.stack([ang.cos(), ang.sin()], -1).float().to(dev).contiguous()
        q_out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=dev)
        kv = torch.zeros(T // 16 + 1, 2, Hkv, 16, D, dtype=torch.bfloat16, device=dev)
        t = _time(lambda: rope_store(qkv, T, Hq, Hkv, D, pos, slots, cos_sin, False, q_out, kv), reps, flush)
        nbytes = T * (Hq + 2 * Hkv) * D * 2 * 2
    else:  # sample: greedy over a 128K vocabulary for 64 rows
        from . import SAMPLE_PARAMS_DTYPE
        import numpy as np
        S, V = 64, 128256
        logits = torch.randn(S, V, device=dev)
        p = np.zeros(S, dtype=SAMPLE_PARAMS_DTYPE)
        params = torch.from_numpy(p.view(np.uint8)).to(dev)
        tok = torch.empty(S, dtype=torch.int32, device=dev)
        t = _time(lambda: sample(logits, S, V, params, tok), reps, flush)
        nbytes = S * V * 4
    return f"{kind:12s} {t:8.1f} us  {nbytes / t / 1e6:5.2f} TB/s"


def bench_step(kind: str, reps: int) -> str:
    """Whole engine steps of the 8B serving config (random-init Q4_K_M weights, 64 requests with
    1024-token prompts): run until every request decodes, time `reps` decode steps (wall clock
    around a synchronised step; the step replays a CUDA graph), then run one more step between
    cudaProfilerStart / Stop so that `ncu --profile-from-start off` captures exactly one step."""
    import time

    import numpy as np

    from ..core.sampling_params import SamplingParams
    from ..llm import LLM
    R, P = 64, 1024
    llm = LLM("random:llama3-8b:Q4_K_M:0", max_model_len=2048, max_num_seqs=R, max_num_batched_tokens=2048,
              num_gpu_blocks=R * ((P + 300) // 16) + 64)
    eng = llm.engine
    rng = np.random.default_rng(0)
    sp = SamplingParams.greedy_params(max_tokens=64, ignore_eos=True)
    reqs = [eng.add_request(rng.integers(0, llm.cfg.model.vocab, P).tolist(), sp) for _ in range(R)]
    while any(len(r.output_token_ids) < 2 for r in reqs):   # requests join the scheduler at a step
        eng.step()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        eng.step()
        torch.cuda.synchronize()
        ts.append((time.perf_counter() - t0) * 1e3)
    torch.cuda.profiler.start()
    eng.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    llm.shutdown()
    return f"step:decode  64 requests, context ~{P + 8}  median {sorted(ts)[len(ts) // 2]:.3f} ms  ({len(ts)} steps)"


def bench_gdn(kind: str, reps: int, flush: torch.Tensor) -> str:
    """Gated delta-net layer core (conv + recurrence + gated norm) at 16 key / 32 value heads of dim
    128, conv kernel 4: `decode` = 64 sequences x 1 token, `prefill2` = two 1024-token prompts."""
    from . import gdn_conv, gdn_recurrent
    Hk, Hv, D, K = 16, 32, 128, 4
    C = (2 * Hk + Hv) * D
    lens = [1] * 64 if kind == "decode" else [1024, 1024]
    nseq, T = len(lens), sum(lens)
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(T, C, device=dev, generator=g)
    w = torch.randn(C, K, device=dev, generator=g) * 0.5
    ab = torch.randn(T, 2 * Hv, device=dev, generator=g)
    z = torch.randn(T, Hv * D, device=dev, generator=g)
    a_neg, dt_bias, norm_w = -torch.ones(Hv, device=dev), torch.zeros(Hv, device=dev), torch.ones(D, device=dev)
    conv_state = torch.zeros(nseq, K - 1, C, device=dev)
    state = torch.randn(nseq, Hv, D, D, device=dev, generator=g) * 0.01
    qs = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=dev)
    slot = torch.arange(nseq, dtype=torch.int32, device=dev)
    has = torch.ones(nseq, dtype=torch.int32, device=dev)
    y = torch.empty(T, C, device=dev)
    out = torch.empty(T, Hv * D, dtype=torch.bfloat16, device=dev)

    def run():
        gdn_conv(x, w, qs, slot, has, nseq, conv_state, y)
        gdn_recurrent(y, ab[:, :Hv], ab[:, Hv:], z, a_neg, dt_bias, norm_w, state, slot, has, qs, nseq, Hk, 1e-6, out)
    t = _time(run, reps, flush)
    nbytes = state.numel() * 4 * 2 + conv_state.numel() * 4 * 2 + T * (C * 4 * 2 + 2 * Hv * 4 + Hv * D * (4 + 2))
    return f"gdn:{kind:8s} {t:8.1f} us  {nbytes / t / 1e6:5.2f} TB/s  ({nseq} seqs, {T} tokens)"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("cases", nargs="*", default=["all"])
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--splits", type=int, default=0,
                    help="force the split count: K splits of gemm cases with split-K output, KV splits of decode attention")
    a = ap.parse_args(argv)
    cases = a.cases
    if cases == ["all"]:
        cases = [f"gemm:{k}" for k in GEMM_CASES if not k.startswith("tp8_")] + ["attn:decode", "attn:prefill", "attn:prefill2", "norm", "rope",
                                                      "swiglu", "sample", "gdn:decode", "gdn:prefill2"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for c in cases:
        if c.startswith("gemm:"):
            line = bench_gemm(c[5:], a.reps, flush, a.splits)
        elif c.startswith("step:"):
            line = bench_step(c[5:], min(a.reps, 10))
        elif c.startswith("attn:"):
            line = bench_attn(c[5:], a.reps, flush, a.splits)
        elif c.startswith("gdn:"):
            line = bench_gdn(c[4:], a.reps, flush)
        else:
            line = bench_small(c, a.reps, flush)
        print(line, flush=True)
    print("device error word:", device_error())


if __name__ == "__main__":
    main()
