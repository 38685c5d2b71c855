"""Micro-benchmark of a tensor-parallel row-parallel site (the down projection of the Llama-3-8B layer,
W [4096, 14336 / N] Q4_K on each rank) as the engine runs it:

  * fused: the GEMM with the reduce-scatter in its epilogue (bf16 rows stored into their owner's
    buffer over NVLink) followed by rs_norm_ag (sum, residual, RMSNorm, all-gather by push);
  * nccl:  the GEMM into an fp32 buffer, NCCL all-reduce, then the residual + RMSNorm kernel;
  * gemm:  the GEMM alone (bf16 output, local) - the compute part of the site.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m vm_c_b200.parallel.bench_comm

Each case captures 20 calls in a CUDA graph, replays it once untimed and once between CUDA events;
the time per call is the maximum over ranks. Roofline of the fused site: the slowest of the GEMM's
FLOPs at the measured bf16 peak, its Q4_K weight bytes (4.5 bits per weight) at the measured HBM
bandwidth, and the bytes that must leave each GPU over NVLink (the reduce-scatter and the all-gather
each send (N - 1) / N x T x 4096 x 2 bytes) at the measured 770 GB/s per direction.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

from .. import ops
from ..gguf.constants import GType
from .comm import init_distributed
from .fused import FusedComm

H, F = 4096, 14336
NVLINK_GBS = 770.0


def _peaks() -> tuple[float, float]:
    """(bf16 TFLOP/s, HBM GB/s) measured on this pool (MEASURED_PEAKS.json at the repository root),
    else the pool's earlier measurement."""
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0


def _time(fn, n: int = 20) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=st):
        for _ in range(n):
            fn()
    torch.cuda.synchronize()
    dist.barrier()
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    t = torch.tensor([e0.elapsed_time(e1) / n * 1e3], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    rank, world, local = init_distributed(timeout_s=120)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = FusedComm()
    T_MAX = 2048
    comm.setup(T_MAX, H, 256)
    K = F // world
    gen = torch.Generator(device=dev).manual_seed(rank)
    w = ops.tile_weight(ops.quantize_blocks(int(GType.Q4_K), torch.randn(H, K, device=dev, generator=gen) * 0.02),
                        int(GType.Q4_K), H, K)
    x = (torch.randn(T_MAX, K, device=dev, generator=gen) * 0.5).bfloat16()
    resid = torch.randn(T_MAX, H, device=dev)
    norm_w = torch.ones(H, device=dev)
    out16 = torch.empty(T_MAX, H, dtype=torch.bfloat16, device=dev)
    o32 = torch.zeros(T_MAX, H, device=dev)
    peak, hbm = _peaks()
    lines = []
    for T in (64, 256, 2048):
        s = ops.pick_splits(w, T)

        def fused():
            comm.row_parallel_rs(1, x, w, T, resid, norm_w, 1e-5, s)

        def nccl():
            ops.gemm(x, w, o32, T, ops.OUT_F32, 1)
            comm.all_reduce(o32[:T])
            ops.add_rmsnorm(resid, norm_w, T, H, 1e-5, out=out16, delta=o32[:T])

        def gemm():
            ops.gemm(x, w, out16, T, ops.OUT_BF16, 1)

        tf, tn, tg = _time(fused), _time(nccl), _time(gemm)
        flop = 2.0 * T * H * K
        t_compute = flop / (peak * 1e12) * 1e6
        t_hbm = H * K * 4.5 / 8 / (hbm * 1e9) * 1e6
        t_link = 2 * (world - 1) / world * T * H * 2 / (NVLINK_GBS * 1e9) * 1e6
        target = max(t_compute, t_hbm, t_link)
        lines.append(f"T={T:5d} ranks={world} K_local={K:5d} splits={s}  fused {tf:8.2f} us  nccl+norm {tn:8.2f} us  "
                     f"gemm alone (1 split) {tg:8.2f} us  roofline {target:7.2f} us (compute {t_compute:.2f}, HBM "
                     f"{t_hbm:.2f}, NVLink {t_link:.2f})  fused/roofline {target / tf:.2f}")
    err = comm.device_error()
    if rank == 0:
        for ln in lines:
            print(ln, flush=True)
        print("device error word:", err, flush=True)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
