"""Fused peer-memory tensor-parallel communication (the product path; NCCL is the baseline).

Every rank allocates one symmetric region (cudaMalloc + CUDA IPC handle, exchanged through the
process group) holding two fp32 partial buffers [max_tokens, hidden] (the two all-reduce sites of
a layer alternate between them) and a flag array. The row-parallel O / down GEMMs write their
partial sums straight into this rank's buffer; ``ar_add_rmsnorm`` then reads every rank's partial
over NVLink, adds the residual and applies the next RMSNorm in one kernel (csrc/kernels/comm.cu).
No NCCL call sits on the per-layer path; NCCL is used only to exchange the IPC handles at start-up
and to gather the vocab-parallel logits before sampling.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .comm import NcclComm

_FLAG_SLOTS = 256
_MAX_RANKS = 8


class FusedComm(NcclComm):
    """`max_fused_tokens`: steps with more tokens (prefill chunks) take the NCCL all-reduce and a
    separate residual + RMSNorm kernel instead: a one-shot all-reduce reads every peer's whole
    partial, (world - 1) times the data, where NCCL's bandwidth-optimal algorithms move about twice
    the data whatever the world size; decode-sized steps are latency-bound and take the fused
    kernel."""

    def __init__(self, group=None, max_ctas: int = 148, max_fused_tokens: int = 512):
        super().__init__(group)
        self.max_fused_tokens = max_fused_tokens
        if self.world > _MAX_RANKS:
            raise ValueError("fused communication supports up to 8 ranks")
        self.max_ctas = min(max_ctas, _FLAG_SLOTS)
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self._ready = False

    def setup(self, max_tokens: int, hidden: int) -> None:
        """Allocate and map the symmetric region (collective: every rank must call it)."""
        if self._ready:
            return
        C = ops.C()
        self.max_tokens, self.hidden = max_tokens, hidden
        self.buf_elems = max_tokens * hidden
        flag_bytes = _FLAG_SLOTS * _MAX_RANKS * 4
        data_bytes = 2 * self.buf_elems * 4
        total = data_bytes + flag_bytes
        self.local_ptr, handle = C.sym_alloc(total)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        self.peer_ptrs = []
        self._opened = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.peer_ptrs.append(self.local_ptr)
            else:
                p = C.sym_open(h)
                self._opened.append(p)
                self.peer_ptrs.append(p)
        self.flag_ptrs = [p + data_bytes for p in self.peer_ptrs]
        dev = self.dev.index
        f32 = 6  # c10::ScalarType::Float
        self.partials = [C.wrap_ptr(self.local_ptr + s * self.buf_elems * 4, [max_tokens, hidden], f32, dev)
                         for s in range(2)]
        self.epochs = torch.zeros(_FLAG_SLOTS, dtype=torch.int32, device=self.dev)
        self.err = torch.zeros(4, dtype=torch.int32, device=self.dev)
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        self._ready = True

    def partial(self, site: int) -> torch.Tensor:
        """This rank's fp32 partial buffer for all-reduce site `site` (0 or 1)."""
        return self.partials[site & 1]

    def allreduce_add_rmsnorm(self, site: int, T: int, resid: torch.Tensor, w: torch.Tensor, eps: float,
                              out: torch.Tensor, nsplit: int = 1, split_stride: int = 0) -> None:
        off = (site & 1) * self.buf_elems * 4
        ops.C().ar_add_rmsnorm([p + off for p in self.peer_ptrs], self.flag_ptrs, self.epochs, self.rank, T,
                               self.hidden, nsplit, split_stride, resid, w, eps, out, self.err, self.max_ctas)
        ops._count()

    def device_error(self) -> int:
        return int(self.err.max().item())

    def close(self) -> None:
        if not self._ready:
            return
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        C = ops.C()
        for p in self._opened:
            C.sym_close(p)
        C.sym_free(self.local_ptr)
        self._ready = False
