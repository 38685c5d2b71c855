"""Speculative sampling under tensor parallelism, host side (two gloo ranks on the CPU): the
vocab-parallel logit shards gather into the full distribution on every rank, and rank 0's draws are
what every rank keeps."""
import json
import os
import socket
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vm_c_b200.speculative.draft import filtered_probs, from_rank0, gather_vocab


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        R, V = 3, 64
        full = torch.randn(R, V)
        per = V // world
        model = SimpleNamespace(tp=world, ws=SimpleNamespace(logits=full[:, rank * per:(rank + 1) * per].clone()))
        got = gather_vocab(model, R)
        p = filtered_probs(got, torch.ones(R), torch.zeros(R, dtype=torch.int32), torch.ones(R), torch.zeros(R))
        gen = torch.Generator().manual_seed(100 + rank)  # different streams: rank 0's draw must win
        draw = from_rank0(torch.multinomial(p, 1, generator=gen).squeeze(1), world)
        json.dump({"gather_ok": bool(torch.equal(got, full)), "draw": draw.tolist()},
                  open(os.path.join(out_dir, f"r{rank}.json"), "w"))
    finally:
        dist.destroy_process_group()


def test_gather_and_rank0_draws(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    res = [json.load(open(tmp_path / f"r{r}.json")) for r in range(world)]
    assert all(r["gather_ok"] for r in res)
    assert res[0]["draw"] == res[1]["draw"]
