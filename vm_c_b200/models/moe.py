"""Mixture-of-experts FFN (Mixtral) on the sm_100a kernels.

Reference behaviour (llama.cpp build_moe_ffn as vendored by vm_c, src/llama-graph.cpp): router
logits = x @ W_gate_inp, softmax over the E experts, top-k (Mixtral: k = 2), weights renormalised
to sum 1, out = sum_j w_j * down_j(silu(gate_j(x)) * up_j(x)). vm_c runs it with every expert
sliced across the tensor-parallel ranks and an all-reduce after the FFN
(src/official/llama/models/llama.cpp:196).

Two placements here:
  * expert-sliced (``ep_size == 1``): every rank holds the FFN columns [r F/tp, (r+1) F/tp) of all
    E experts (the reference's layout);
  * expert-parallel (``ep_size == tp_size``): rank r holds experts [r E/ep, (r+1) E/ep) whole.
Attention stays tensor-parallel, so after its all-reduce every rank holds the hidden states of
all tokens: routing is computed redundantly on every rank (bit-identical: a stable sort in a
single CTA), each rank runs its own experts on the rows routed to them, and the cross-rank sum of
the weighted expert outputs is the layer's usual all-reduce -- on the peer-memory path fused with
the residual add and the next RMSNorm. Dispatch therefore moves no data.

Per layer: router GEMM (tcgen05, N = E) -> moe_route (softmax/top-k + stable counting sort by
expert, one CTA) -> gather of the token rows in expert order -> grouped gate/up GEMM with fused
SwiGLU -> grouped down GEMM (one launch each for all local experts; counts stay on the device, so
the step remains CUDA-graph capturable) -> moe_combine (weighted sum per token).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..config import ModelConfig
from ..gguf.constants import GType


@dataclass
class MoEWeights:
    router: ops.TiledWeight        # [E, H] (bf16 tiles)
    gate_up: ops.TiledWeight       # descriptor of ONE expert: [2 F_local, H], rows gate/up interleaved
    gate_up_stride: int            # bytes between consecutive experts in gate_up.data
    down: ops.TiledWeight          # descriptor of ONE expert: [H, F_local]
    down_stride: int
    e0: int                        # first local expert
    e_local: int                   # number of local experts
    f_local: int                   # FFN columns per expert on this rank


def moe_placement(cfg: ModelConfig, tp_rank: int, tp_size: int, ep_size: int) -> tuple[int, int, int, int]:
    """(e0, e_local, f0, f_local) of this rank."""
    E, F = cfg.n_experts, cfg.ffn
    if ep_size > 1:
        if ep_size != tp_size:
            raise ValueError(f"expert parallelism needs ep_size == tp_size (attention is tensor-parallel): "
                             f"ep {ep_size}, tp {tp_size}")
        if E % ep_size:
            raise ValueError(f"{E} experts are not divisible by ep_size {ep_size}")
        per = E // ep_size
        return tp_rank * per, per, 0, F
    if F % tp_size:
        raise ValueError(f"expert FFN {F} not divisible by tp {tp_size}")
    fl = F // tp_size
    return 0, E, tp_rank * fl, fl


def _interleave_tile(g: torch.Tensor, u: torch.Tensor, tg: int, tu: int, F: int, H: int, dev) -> ops.TiledWeight:
    if tg == tu:
        inter = torch.stack([g, u], 1).reshape(2 * F, -1)
        return ops.tile_weight(inter, tg, 2 * F, H)
    from .. import _native
    h = _native.host()
    gf = torch.from_numpy(h.dequantize(int(tg), g.cpu().numpy(), F, H))
    uf = torch.from_numpy(h.dequantize(int(tu), u.cpu().numpy(), F, H))
    inter = torch.stack([gf, uf], 1).reshape(2 * F, H).to(dev)
    return ops.tile_weight(inter, int(GType.F32), 2 * F, H)


def load_moe_layer(src, cfg: ModelConfig, i: int, dev, tp_rank: int, tp_size: int, ep_size: int = 1) -> MoEWeights:
    from .llama import _col_slice, _tile_raw, _to_dev
    H, F, E = cfg.hidden, cfg.ffn, cfg.n_experts
    e0, el, f0, fl = moe_placement(cfg, tp_rank, tp_size, ep_size)
    from ..gguf.constants import blk
    rn = blk(i, "ffn_gate_inp")
    rspec = src.info(rn)
    rraw = _to_dev(src.rows(rn), dev)
    if rspec.gtype != GType.F32:
        from .. import _native
        rraw = torch.from_numpy(_native.host().dequantize(int(rspec.gtype), rraw.cpu().numpy(), E, H)).to(dev)
    router = ops.tile_weight(rraw.float().reshape(E, H), int(GType.F32), E, H)

    gn, un, dn = blk(i, "ffn_gate_exps"), blk(i, "ffn_up_exps"), blk(i, "ffn_down_exps")
    tg, tu, td = src.info(gn).gtype, src.info(un).gtype, src.info(dn).gtype
    gus, downs = [], []
    for e in range(e0, e0 + el):
        g = _to_dev(src.rows(gn, e * F + f0, e * F + f0 + fl), dev)
        u = _to_dev(src.rows(un, e * F + f0, e * F + f0 + fl), dev)
        gus.append(_interleave_tile(g, u, tg, tu, fl, H, dev))
        d = _to_dev(src.rows(dn, e * H, (e + 1) * H), dev)
        d = _col_slice(d, td, F, f0, f0 + fl).contiguous()
        downs.append(_tile_raw(d, td, H, fl))
        del g, u, d
    gu_stride, dn_stride = gus[0].nbytes, downs[0].nbytes
    if any(w.wf != gus[0].wf or w.nbytes != gu_stride for w in gus) or \
            any(w.wf != downs[0].wf or w.nbytes != dn_stride for w in downs):
        raise ValueError(f"layer {i}: experts must share one weight type per projection")
    gate_up = ops.TiledWeight(gus[0].wf, torch.cat([w.data for w in gus]), 2 * fl, H, interleaved_swiglu=True)
    down = ops.TiledWeight(downs[0].wf, torch.cat([w.data for w in downs]), H, fl)
    return MoEWeights(router=router, gate_up=gate_up, gate_up_stride=gu_stride, down=down, down_stride=dn_stride,
                      e0=e0, e_local=el, f_local=fl)


class MoERunner:
    """Device workspace and launch sequence of the MoE FFN for up to ``max_tokens`` tokens."""

    def __init__(self, model, max_tokens: int):
        cfg = model.cfg
        dev = model.dev
        self.E, self.k, self.H = cfg.n_experts, cfg.n_experts_used, cfg.hidden
        self.norm_topk = True  # Mixtral renormalises the selected weights
        moe0 = next(lw.moe for lw in model.w.layers if lw.moe is not None)
        el, fl = moe0.e_local, moe0.f_local
        R = max_tokens * self.k
        i32, f32 = dict(dtype=torch.int32, device=dev), dict(dtype=torch.float32, device=dev)
        self.logits = torch.zeros(max_tokens, self.E, **f32)
        self.topk_id = torch.zeros(R, **i32)
        self.topk_w = torch.zeros(R, **f32)
        self.counts = torch.zeros(el, **i32)
        self.offsets = torch.zeros(el, **i32)
        self.sorted_src = torch.zeros(R, **i32)
        self.slot_row = torch.zeros(R, **i32)
        self.total = torch.zeros(1, **i32)
        self.xs = torch.zeros(R, self.H, dtype=torch.bfloat16, device=dev)
        self.act = torch.zeros(R, fl, dtype=torch.bfloat16, device=dev)
        self.y = torch.zeros(R, self.H, **f32)
        self.out = torch.zeros(max_tokens, self.H, **f32)

    def native_desc(self) -> dict:
        """MoeBuffers (csrc/kernels/forward.h) of the expert-sliced path of the native forward."""
        t = lambda x: x.data_ptr()  # noqa: E731
        return {"E": self.E, "k": self.k, "norm_topk": int(self.norm_topk), "ep": False,
                "logits": t(self.logits), "topk_id": t(self.topk_id), "topk_w": t(self.topk_w),
                "counts": t(self.counts), "offsets": t(self.offsets), "sorted_src": t(self.sorted_src),
                "slot_row": t(self.slot_row), "total": t(self.total), "xs": t(self.xs), "act": t(self.act),
                "y": t(self.y), "out": t(self.out)}

    def forward(self, moe: MoEWeights, h: torch.Tensor, T: int, out: torch.Tensor | None = None):
        """Weighted sum of this rank's expert outputs for tokens h[:T] into out[:T] (fp32)."""
        if out is None:
            out = self.out
        k, H = self.k, self.H
        R = T * k
        ops.gemm(h, moe.router, self.logits[:T], T, ops.OUT_F32, 1)
        ops.moe_route(self.logits, T, self.E, k, self.norm_topk, moe.e0, moe.e_local, self.topk_id, self.topk_w,
                      self.counts, self.offsets, self.sorted_src, self.slot_row, self.total)
        ops.gather_rows(h, self.sorted_src, R, H, self.xs)
        bn = ops.pick_bn(max(1, -(-R // moe.e_local)))
        ops.gemm_grouped(self.xs, moe.gate_up, moe.e_local, moe.gate_up_stride, R, self.counts, self.offsets, T,
                         self.act, ops.OUT_SWIGLU, bn=bn)
        ops.gemm_grouped(self.act, moe.down, moe.e_local, moe.down_stride, R, self.counts, self.offsets, T,
                         self.y, ops.OUT_F32, bn=bn)
        ops.moe_combine(self.y, self.slot_row, self.topk_w, T, k, H, out)
        return out, (self.topk_id, self.topk_w)
