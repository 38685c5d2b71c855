"""Tensor-parallel communication for one process per GPU.

``NcclComm`` is the baseline backend: torch.distributed (NCCL) all-reduce at the reference's two
sites (after Wo and after the FFN down projection; reference NcclComm::allreduce,
src/distributed/nccl_comm.cu:259-327, which calls ncclAllReduce in place on the ggml stream) and an
all-gather of vocab-parallel logits before sampling. The fused peer-memory backend lives in
parallel/fused.py and replaces the all-reduce with kernels that read and write peer GPUs' memory.
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist

from .. import ops
from ..utils.nvtx import nvtx_range


def init_distributed(timeout_s: float = 120.0) -> tuple[int, int, int]:
    """Initialise the default process group from torchrun's environment. Returns (rank, world, local)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local


class NcclComm:
    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._gather_buf = None

    def all_reduce(self, t: torch.Tensor) -> None:
        with nvtx_range("allreduce"):
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def barrier(self) -> None:
        dist.barrier(group=self.group)

    def gather_logits(self, model, S: int) -> torch.Tensor:
        """Full-vocabulary logits of the last step's S rows (after sample_vocab_parallel)."""
        return self._full[:S]

    def sample_vocab_parallel(self, model, S: int, params: torch.Tensor, out_tok: torch.Tensor, out_lp) -> None:
        """Gather the vocab-parallel logits of the S sampled rows, then sample identically on every rank."""
        ws = model.ws
        vl = model.v_local
        if self._gather_buf is None or self._gather_buf.shape[1] < S:
            self._gather_buf = torch.empty(self.world, model.max_samples, vl, dtype=torch.float32, device=ws.logits.device)
            self._full = torch.empty(model.max_samples, self.world * vl, dtype=torch.float32, device=ws.logits.device)
        buf = self._gather_buf
        # Gather the whole (static-shape) logits buffer so the collective is CUDA-graph capturable.
        dist.all_gather_into_tensor(buf.view(-1), ws.logits.view(-1), group=self.group)
        full = self._full[:S].view(S, self.world, vl)
        full.copy_(buf[:, :S].permute(1, 0, 2))
        V = model.cfg.vocab
        ops.sample(self._full[:S], S, V, params, out_tok, out_lp)
