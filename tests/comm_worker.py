"""Worker of the fused reduce-scatter / all-gather GPU test (launched by torch.distributed.run, one rank
per GPU). Each rank multiplies its own integer-valued activations by its own integer-valued weight
shard through the scatter-epilogue GEMM and rs_norm_ag (FusedComm.row_parallel_rs); every partial sum
is an integer that bf16 holds exactly, so the residual rows each rank owns must equal the exact sum
of all ranks' products. Calls run in bursts of back-to-back launches (no host synchronisation inside
a burst) with random token counts, K splits and sites; the gathered activations h are checked against
an fp32 RMSNorm, and the sums against NCCL's all-reduce of the same partials."""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from vm_c_b200 import ops  # noqa: E402
from vm_c_b200.gguf.constants import GType  # noqa: E402
from vm_c_b200.parallel.comm import init_distributed  # noqa: E402


def gen(seed):
    return torch.Generator().manual_seed(seed)


def sampler_check(comm, rank, world, dev):
    """Vocabulary-parallel sampling (tp_sample) against the single-GPU sampler on the whole row: the
    same tokens for greedy, unrestricted and top-k / top-p / min-p rows, and the same log-probs."""
    from types import SimpleNamespace
    from vm_c_b200.core.engine import SAMPLE_DTYPE
    V, S = 128256, 48
    V_local = V // world
    g = gen(11)
    full = (torch.randn(S, V, generator=g) * 3).to(dev)
    rec = np.zeros(S, dtype=SAMPLE_DTYPE)
    for r in range(S):
        kind = r % 4
        rec[r]["temperature"] = 0.0 if kind == 0 else 0.7 + 0.1 * (r % 3)
        rec[r]["top_k"] = [0, 0, 40, 0][kind]
        rec[r]["top_p"] = [1.0, 1.0, 0.95, 0.9][kind]
        rec[r]["min_p"] = [0.0, 0.0, 0.0, 0.05][kind]
        rec[r]["repetition_penalty"] = 1.0
        rec[r]["step"] = r
        rec[r]["seed"] = 1234 + 17 * r
    params = torch.from_numpy(rec.view(np.uint8).copy()).to(dev)
    tok_ref = torch.zeros(S, dtype=torch.int32, device=dev)
    lp_ref = torch.zeros(S, dtype=torch.float32, device=dev)
    ops.sample(full, S, V, params, tok_ref, lp_ref)
    model = SimpleNamespace(ws=SimpleNamespace(logits=full[:, rank * V_local:(rank + 1) * V_local].contiguous()),
                            v_local=V_local)
    mism = 0
    lp_err = 0.0
    for _ in range(3):   # repeated calls advance the exchange counters
        tok = torch.zeros(S, dtype=torch.int32, device=dev)
        lp = torch.zeros(S, dtype=torch.float32, device=dev)
        comm.sample_vocab_parallel(model, S, params, tok, lp)
        torch.cuda.synchronize(dev)
        mism += int((tok != tok_ref).sum())
        lp_err = max(lp_err, float((lp - lp_ref).abs().max()))
    return {"sampler_mismatch": mism, "sampler_lp_err": lp_err}


def main():
    out, bursts, per_burst = sys.argv[1], int(sys.argv[2]), int(sys.argv[3])
    rank, world, local = init_distributed(timeout_s=120)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from vm_c_b200.parallel.fused import FusedComm
    comm = FusedComm()
    H, K, T_MAX, eps = 1024, 256, 2048, 1e-5
    comm.setup(T_MAX, H, 64)
    W = [torch.randint(-1, 2, (H, K), generator=gen(7 + r)).float() for r in range(world)]
    Wd = [w.to(dev) for w in W]
    tw = ops.tile_weight(Wd[rank], int(GType.F32), H, K)
    norm_w = (torch.rand(H, generator=gen(3)) + 0.5).to(dev)
    xbuf = torch.zeros(T_MAX, K, dtype=torch.bfloat16, device=dev)
    resid = torch.zeros(T_MAX, H, dtype=torch.float32, device=dev)
    rng = np.random.default_rng(123)   # the same call schedule on every rank
    stats = {"calls": 0, "max_resid_err": 0.0, "max_h_rel_err": 0.0, "max_vs_nccl": 0.0, "bursts": bursts}
    for b in range(bursts):
        M = int(rng.choice([1, 3, 8, 17, 64, 100, 256, 511, 1024, 2048]))
        r0 = torch.randint(-4, 5, (M, H), generator=gen(100000 + b)).float().to(dev)
        resid[:M] = r0
        total = torch.zeros(M, H, device=dev)
        mine = torch.zeros(M, H, device=dev)
        for c in range(per_burst):
            site = int(rng.integers(0, 2))
            splits = int(rng.choice([1, 2, 4])) if M <= 256 else 1
            xs = [torch.randint(-1, 2, (M, K), generator=gen(1000 * (b * per_burst + c) + r)).float().to(dev)
                  for r in range(world)]
            xbuf[:M] = xs[rank].bfloat16()
            comm.row_parallel_rs(site, xbuf, tw, M, resid, norm_w, eps, splits)
            for r in range(world):
                p = xs[r] @ Wd[r].T
                total += p
                if r == rank:
                    mine += p
            stats["calls"] += 1
        torch.cuda.synchronize(dev)
        expect = r0 + total
        rpr = (M + world - 1) // world
        lo, hi = rank * rpr, min(M, (rank + 1) * rpr)
        if hi > lo:
            stats["max_resid_err"] = max(stats["max_resid_err"], float((resid[lo:hi] - expect[lo:hi]).abs().max()))
        # the last call's normalised rows, gathered from every owner into this rank's h
        hx = expect * torch.rsqrt(expect.pow(2).mean(-1, keepdim=True) + eps) * norm_w
        herr = float((comm.h[:M].float() - hx).abs().max() / hx.abs().max())
        stats["max_h_rel_err"] = max(stats["max_h_rel_err"], herr)
        # NCCL all-reduce of this rank's partials over the burst
        dist.all_reduce(mine)
        if hi > lo:
            stats["max_vs_nccl"] = max(stats["max_vs_nccl"], float((resid[lo:hi] - (r0 + mine)[lo:hi]).abs().max()))
    stats.update(sampler_check(comm, rank, world, dev))
    stats["err"] = comm.device_error()
    stats["world"] = world
    if rank == 0:
        json.dump(stats, open(out, "w"))
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
