"""Fused peer-memory tensor-parallel communication (the product path; NCCL is the baseline).

Every rank allocates one symmetric region (cudaMalloc + CUDA IPC handle, exchanged through the
process group) and maps every peer's. It holds:

* for the reduce-scatter / all-gather design used by the native step forward (csrc/kernels/forward.cpp):
  two bf16 receive buffers (one per row-parallel site) into which the row-parallel O / down GEMMs of
  all ranks store the partial rows that this rank owns (the GEMM epilogue writes over NVLink), the
  bf16 activations ``h`` that every owner fills with its normalised rows (all-gather by push) and that
  the next column-parallel GEMM reads locally, and four monotonic arrival counters;
* for the one-shot all-reduce of the Python step path: two fp32 partial buffers and a flag array
  (``ar_add_rmsnorm`` reads every rank's partial over NVLink, adds the residual and applies RMSNorm).

No NCCL call sits on the per-layer path; NCCL is used only to exchange the IPC handles at start-up
and, for now, to gather the vocab-parallel logits before sampling.
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

    def setup(self, max_tokens: int, hidden: int, max_samples: int = 0) -> None:
        """Allocate and map the symmetric region (collective: every rank must call it)."""
        if self._ready:
            return
        C = ops.C()
        self.max_tokens, self.hidden = max_tokens, hidden
        self.max_samples = max_samples or max_tokens
        nr = self.world
        self.buf_elems = max_tokens * hidden
        # Receive rows: K-split partials only occur for steps of at most 256 tokens (one token tile),
        # with at most 8 splits; unsplit steps need one slot of ceil(T / nr) rows per source.
        rpr256 = (256 + nr - 1) // nr
        self.recv_rows = max(8 * nr * rpr256, nr * ((max_tokens + nr - 1) // nr))
        a = 256
        rnd = lambda x: (x + a - 1) // a * a  # noqa: E731
        off = 0
        self.off_partial = [off, off + rnd(self.buf_elems * 4)]
        off += 2 * rnd(self.buf_elems * 4)
        self.off_recv = [off, off + rnd(self.recv_rows * hidden * 2)]
        off += 2 * rnd(self.recv_rows * hidden * 2)
        self.off_h = off
        off += rnd(max_tokens * hidden * 2)
        # uint32 counters, 64 bytes apart: rs0, rs1, ag0, ag1, sampler, ag2 (MoE combine), MoE dispatch,
        # MoE combine arrivals
        self.off_count = off
        off += 512
        off = rnd(off)
        self.off_xbuf = off           # vocabulary-parallel sampler exchange [nr][max_samples][row bytes]
        off += rnd(nr * self.max_samples * C.tp_sample_row_bytes())
        self.off_flags = off
        off += rnd(_FLAG_SLOTS * _MAX_RANKS * 4)
        total = off
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
        self.flag_ptrs = [p + self.off_flags for p in self.peer_ptrs]
        dev = self.dev.index
        f32, bf16 = 6, 15  # c10::ScalarType::Float, BFloat16
        self.partials = [C.wrap_ptr(self.local_ptr + self.off_partial[s], [max_tokens, hidden], f32, dev)
                         for s in range(2)]
        self.h = C.wrap_ptr(self.local_ptr + self.off_h, [max_tokens, hidden], bf16, dev)
        self.epochs = torch.zeros(_FLAG_SLOTS, dtype=torch.int32, device=self.dev)
        self.err = torch.zeros(4, dtype=torch.int32, device=self.dev)
        self.state = torch.zeros(12, dtype=torch.int32, device=self.dev)   # 3 sites x 4 words
        self.xstate = torch.zeros(2, dtype=torch.int32, device=self.dev)
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        self._ready = True

    def tp_desc(self) -> dict:
        """Peer addresses of the reduce-scatter / all-gather buffers (TpComm, csrc/kernels/comm.h)."""
        P = self.peer_ptrs
        cnt = [[p + self.off_count + 64 * k for p in P] for k in range(4)]
        return {"nranks": self.world, "rank": self.rank, "recv_rows": self.recv_rows, "max_ctas": self.max_ctas,
                "recv0": [p + self.off_recv[0] for p in P], "recv1": [p + self.off_recv[1] for p in P],
                "h": [p + self.off_h for p in P], "rs0": cnt[0], "rs1": cnt[1], "ag0": cnt[2], "ag1": cnt[3],
                "ag2": [p + self.off_count + 320 for p in P],
                "state": self.state.data_ptr(), "err": self.err.data_ptr(),
                "xbuf": [p + self.off_xbuf for p in P], "xcount": [p + self.off_count + 256 for p in P],
                "xstate": self.xstate.data_ptr(), "max_rows": self.max_samples}

    def setup_moe(self, E: int, k: int, e_local: int, f_local: int, hidden: int) -> None:
        """Expert-parallel buffers (collective): a second symmetric region with every rank's expert
        input rows, their return words, the per-expert row counters (two layer parities) and the rows
        that come back to their token's owner; plus this rank's routing and expert activations."""
        if getattr(self, "_moe_ready", False):
            return
        C = ops.C()
        nr, T = self.world, self.max_tokens
        cap = T                       # a token selects an expert at most once
        rpr = (T + nr - 1) // nr
        rnd = lambda x: (x + 255) // 256 * 256  # noqa: E731
        off = 0
        o_x = off
        off += rnd(e_local * cap * hidden * 2)
        o_ret = off
        off += rnd(e_local * cap * 4)
        o_cnt = [off, off + rnd(e_local * 4)]
        off += 2 * rnd(e_local * 4)
        o_comb = off
        off += rnd(rpr * k * hidden * 2)
        total = off
        self.moe_local, handle = C.sym_alloc(total)
        handles = [None] * nr
        dist.all_gather_object(handles, handle, group=self.group)
        peers = []
        for r, h in enumerate(handles):
            if r == self.rank:
                peers.append(self.moe_local)
            else:
                p = C.sym_open(h)
                self._opened.append(p)
                peers.append(p)
        dev = self.dev
        self.moe_peers = peers
        self._moe_off = dict(x=o_x, ret=o_ret, cnt=o_cnt, comb=o_comb)
        self.moe_dims = dict(E=E, k=k, e_local=e_local, f_local=f_local, cap=cap, rpr=rpr)
        self.disp_state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.ep_logits = torch.zeros(rpr, E, dtype=torch.float32, device=dev)
        self.ep_topk_w = torch.zeros(rpr, k, dtype=torch.float32, device=dev)
        self.ep_act = torch.zeros(e_local * cap, f_local, dtype=torch.bfloat16, device=dev)
        self.ep_offsets = torch.arange(0, e_local * cap, cap, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)
        self._moe_ready = True

    def moe_desc(self) -> dict:
        """MoeBuffers (csrc/kernels/forward.h) of the expert-parallel path."""
        P, o, md = self.moe_peers, self._moe_off, self.moe_dims
        cnt = [p + self.off_count for p in self.peer_ptrs]
        return {"E": md["E"], "k": md["k"], "norm_topk": 1, "ep": True, "cap": md["cap"],
                "recv_x": [p + o["x"] for p in P], "recv_ret": [p + o["ret"] for p in P],
                "cnt0": [p + o["cnt"][0] for p in P], "cnt1": [p + o["cnt"][1] for p in P],
                "comb": [p + o["comb"] for p in P], "disp_arrive": [c + 384 for c in cnt],
                "comb_arrive": [c + 448 for c in cnt], "disp_state": self.disp_state.data_ptr(),
                "ep_logits": self.ep_logits.data_ptr(), "ep_topk_w": self.ep_topk_w.data_ptr(),
                "ep_act": self.ep_act.data_ptr(), "ep_offsets": self.ep_offsets.data_ptr()}

    def sample_vocab_parallel(self, model, S: int, params: torch.Tensor, out_tok: torch.Tensor, out_lp) -> None:
        """Sample the S rows from this rank's vocabulary shard of the logits: a local reduction and a
        candidate exchange through peer memory (no logits all-gather)."""
        ops.C().tp_sample(self.tp_desc(), model.ws.logits, S, model.v_local, params, out_tok, out_lp)
        ops._count(2)

    def gather_logits(self, model, S: int) -> torch.Tensor:
        """Full-vocabulary logits of the last step's S rows (diagnostics and tests; NCCL, not captured)."""
        shard = model.ws.logits[:S].contiguous()
        parts = [torch.empty_like(shard) for _ in range(self.world)]
        dist.all_gather(parts, shard, group=self.group)
        return torch.cat(parts, dim=1)

    def partial(self, site: int) -> torch.Tensor:
        """This rank's fp32 partial buffer for all-reduce site `site` (0 or 1)."""
        return self.partials[site & 1]

    def allreduce_add_rmsnorm(self, site: int, T: int, resid: torch.Tensor, w: torch.Tensor, eps: float,
                              out: torch.Tensor, nsplit: int = 1, split_stride: int = 0) -> None:
        off = self.off_partial[site & 1]
        ops.C().ar_add_rmsnorm([p + off for p in self.peer_ptrs], self.flag_ptrs, self.epochs, self.rank, T,
                               self.hidden, nsplit, split_stride, resid, w, eps, out, self.err, self.max_ctas)
        ops._count()

    def row_parallel_rs(self, site: int, x: torch.Tensor, w, M: int, resid: torch.Tensor, norm_w: torch.Tensor,
                        eps: float, splits: int = 1) -> int:
        """One row-parallel site through the reduce-scatter design: x[:M] @ w^T with the partial rows
        scattered to their owners in the GEMM epilogue, then residual + RMSNorm on the owned rows and
        the all-gather into every rank's ``self.h``. Returns the K splits used."""
        used = ops.C().tp_row_parallel(self.tp_desc(), site & 1, w.wf, w.data, w.N, w.K, x, M, splits, resid, norm_w,
                                      eps, self.err)
        ops._count(2)
        return used

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
