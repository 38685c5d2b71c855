"""Micro-benchmark of the tensor-parallel reduction sites: the fused peer-memory all-reduce +
residual + RMSNorm kernel against NCCL all-reduce followed by the separate residual + RMSNorm
kernel, at decode and small-prefill sizes (hidden 4096, fp32 partials).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m vm_c_b200.parallel.bench_comm

Each case captures 50 calls in a CUDA graph and times one replay with CUDA events; the reported
time per call is the maximum over ranks.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .comm import init_distributed
from .fused import FusedComm

CASES = ((64, 4), (64, 1), (256, 2))  # (tokens, split-K partials per rank)


def main() -> None:
    rank, world, local = init_distributed(timeout_s=60)
    torch.cuda.set_device(local)
    H = 4096
    comm = FusedComm()
    comm.setup(2048, H)
    res = {}
    for T, S in CASES:
        resid = torch.randn(T, H, device="cuda")
        w = torch.ones(H, device="cuda")
        out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
        comm.partial(0).view(-1)[:S * T * H].normal_()
        o = torch.randn(T, H, device="cuda")

        def fused():
            comm.allreduce_add_rmsnorm(0, T, resid, w, 1e-5, out, nsplit=S, split_stride=T * H)

        def nccl():
            comm.all_reduce(o)
            ops.add_rmsnorm(resid, w, T, H, 1e-5, out=out, delta=o)

        for name, fn in (("fused", fused), ("nccl+norm", nccl)):
            for _ in range(20):
                fn()
            torch.cuda.synchronize()
            dist.barrier()
            n = 50
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
            res[(name, T, S)] = t.item()
    if rank == 0:
        for (name, T, S), v in res.items():
            print(f"{name:10s} tokens={T:4d} partials={S} ranks={world}  {v:7.2f} us per call", flush=True)
    err = comm.device_error()
    if rank == 0:
        print("device error word:", err)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
