"""Llama / Mixtral-architecture model on the sm_100a kernels, with Megatron tensor parallelism.

Forward of one engine step over a flat token batch (decodes first, then prefill chunks), reading
the step metadata written by the native scheduler (csrc/host/scheduler.cpp build_batch):

  embed (GGUF row dequant) -> [per layer] RMSNorm -> QKV GEMM -> RoPE + paged KV store ->
  paged attention -> O GEMM -> (TP reduce) -> residual + RMSNorm -> gate/up GEMM with fused SwiGLU
  (or MoE) -> down GEMM -> (TP reduce) -> residual + RMSNorm -> ... -> final norm on the sampled
  rows -> vocab-parallel lm_head -> sampler.

This is the graph the reference builds with libllama (src/official/llama/models/llama.cpp:98-253)
including vm_c's two all-reduce sites after Wo and after the FFN / MoE down projection (:171,196,221).
Weight sharding follows the reference's layout plan (src/model/weight_layout_plan.cpp:38-81,114-131):
Q/K/V and gate/up column-parallel (KV heads replicated when n_kv_heads < tp), O and down
row-parallel, embedding replicated; the lm_head is vocab-parallel here (the reference replicates it).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field

import torch

from .. import ops
from ..utils.nvtx import LayerRanges
from ..config import ModelConfig, rope_inv_freq
from ..gguf.constants import GType, blk, row_bytes


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    wqkv: list                     # TiledWeight(s): one fused QKV weight, or [QK, V] when types differ
    qkv_split: list                # output column offsets of each part
    wo: ops.TiledWeight
    w_gate_up: ops.TiledWeight | None = None   # rows interleave gate/up (fused SwiGLU)
    w_down: ops.TiledWeight | None = None
    moe: object | None = None      # MoE weights (models/moe.py)
    index: int = 0                 # layer number
    offload: list = field(default_factory=list)  # (pinned host tensor, device view) copied before the layer


@dataclass
class ModelWeights:
    cfg: ModelConfig
    layers: list[LayerWeights]
    embd: torch.Tensor             # raw GGUF rows [V, row_bytes] (replicated)
    embd_type: int
    embd_row_bytes: int
    output_norm: torch.Tensor
    lm_head: ops.TiledWeight       # rows [vocab_begin, vocab_end) of the output projection
    vocab_begin: int = 0
    vocab_end: int = 0
    tp_rank: int = 0
    tp_size: int = 1
    bytes_total: int = 0


# ------------------------------------------------------------------------------------------------
# Sharding helpers


def _kv_heads_local(cfg: ModelConfig, rank: int, tp: int) -> tuple[int, int]:
    """(first kv head, number of kv heads) held by `rank`."""
    if cfg.n_kv_heads >= tp:
        n = cfg.n_kv_heads // tp
        return rank * n, n
    return (rank * cfg.n_kv_heads) // tp, 1


def check_tp(cfg: ModelConfig, tp: int) -> None:
    if cfg.n_heads % tp:
        raise ValueError(f"n_heads {cfg.n_heads} not divisible by tp {tp}")
    if cfg.n_kv_heads >= tp and cfg.n_kv_heads % tp:
        raise ValueError(f"n_kv_heads {cfg.n_kv_heads} not divisible by tp {tp}")
    if cfg.n_kv_heads < tp and tp % cfg.n_kv_heads:
        raise ValueError(f"tp {tp} not a multiple of n_kv_heads {cfg.n_kv_heads}")
    if cfg.ffn % tp:
        raise ValueError(f"ffn {cfg.ffn} not divisible by tp {tp}")
    if tp > 1 and (cfg.ffn // tp) % 8:
        # the down projection reads bf16 activation rows of ffn / tp columns through TMA
        raise ValueError(f"ffn {cfg.ffn} / tp {tp} = {cfg.ffn // tp} columns per rank: not a multiple of 8 "
                         f"(16-byte activation rows)")


def _to_dev(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device, non_blocking=False).contiguous()


def _col_slice(raw: torch.Tensor, gtype: int, K: int, c0: int, c1: int) -> torch.Tensor:
    """Columns [c0, c1) (elements) of GGUF rows: a byte slice of every row (block aligned)."""
    if c0 == 0 and c1 == K:
        return raw
    if gtype == GType.F32:
        return raw[:, c0:c1]
    b0, b1 = row_bytes(gtype, c0) if c0 else 0, row_bytes(gtype, c1)
    return raw[:, b0:b1]


def _tile(src, name: str, device, r0=0, r1=None, c0=0, c1=None, rows_override=None) -> ops.TiledWeight:
    spec = src.info(name)
    K = spec.ne[0]
    r1 = spec.rows if r1 is None else r1
    c1 = K if c1 is None else c1
    raw = _to_dev(src.rows(name, r0, r1), device)
    raw = _col_slice(raw, spec.gtype, K, c0, c1).contiguous()
    return _tile_raw(raw, spec.gtype, r1 - r0, c1 - c0)


def _tile_raw(raw: torch.Tensor, gtype: int, N: int, K: int) -> ops.TiledWeight:
    if ops.wf_for_gtype(gtype) is None:
        # No native GPU format (Q2_K, Q3_K, Q5_K, IQ4, ...): dequantise on the host, tile as bf16.
        from .. import _native
        f = _native.host().dequantize(int(gtype), raw.cpu().numpy(), N, K)
        return ops.tile_weight(torch.from_numpy(f).to(raw.device), int(GType.F32), N, K)
    return ops.tile_weight(raw, gtype, N, K)


def load_weights(src, cfg: ModelConfig, device, tp_rank: int = 0, tp_size: int = 1, ep_size: int = 1) -> ModelWeights:
    """Load (and shard) the weights of a llama-architecture model from a tensor source."""
    if cfg.is_hybrid:
        from .qwen35 import load_hybrid_weights
        return load_hybrid_weights(src, cfg, device, tp_rank, tp_size)
    check_tp(cfg, tp_size)
    dev = torch.device(device)
    D = cfg.head_dim
    hq_local = cfg.n_heads // tp_size
    kv0, nkv = _kv_heads_local(cfg, tp_rank, tp_size)
    f_local = cfg.ffn // tp_size
    layers = []
    total = 0
    for i in range(cfg.n_layers):
        qn, kn, vn = blk(i, "attn_q"), blk(i, "attn_k"), blk(i, "attn_v")
        q_rows = (tp_rank * hq_local * D, (tp_rank + 1) * hq_local * D)
        kv_rows = (kv0 * D, (kv0 + nkv) * D)
        tq, tk, tv = src.info(qn).gtype, src.info(kn).gtype, src.info(vn).gtype
        raw_q = _to_dev(src.rows(qn, *q_rows), dev)
        raw_k = _to_dev(src.rows(kn, *kv_rows), dev)
        raw_v = _to_dev(src.rows(vn, *kv_rows), dev)
        H = cfg.hidden
        if tq == tk == tv:
            wqkv = [_tile_raw(torch.cat([raw_q, raw_k, raw_v], 0), tq, (hq_local + 2 * nkv) * D, H)]
            split = [0]
        elif tq == tk:
            wqkv = [_tile_raw(torch.cat([raw_q, raw_k], 0), tq, (hq_local + nkv) * D, H),
                    _tile_raw(raw_v, tv, nkv * D, H)]
            split = [0, (hq_local + nkv) * D]
        else:
            wqkv = [_tile_raw(raw_q, tq, hq_local * D, H), _tile_raw(raw_k, tk, nkv * D, H),
                    _tile_raw(raw_v, tv, nkv * D, H)]
            split = [0, hq_local * D, (hq_local + nkv) * D]
        del raw_q, raw_k, raw_v
        on = blk(i, "attn_output")
        wo = _tile(src, on, dev, c0=tp_rank * hq_local * D, c1=(tp_rank + 1) * hq_local * D)
        lw = LayerWeights(attn_norm=_to_dev(src.rows(blk(i, "attn_norm")), dev).view(-1).float(),
                          ffn_norm=_to_dev(src.rows(blk(i, "ffn_norm")), dev).view(-1).float(),
                          wqkv=wqkv, qkv_split=split, wo=wo, index=i)
        if cfg.is_moe:
            from .moe import load_moe_layer
            lw.moe = load_moe_layer(src, cfg, i, dev, tp_rank, tp_size, ep_size)
        else:
            gn, un, dn = blk(i, "ffn_gate"), blk(i, "ffn_up"), blk(i, "ffn_down")
            fr = (tp_rank * f_local, (tp_rank + 1) * f_local)
            tg, tu = src.info(gn).gtype, src.info(un).gtype
            raw_g = _to_dev(src.rows(gn, *fr), dev)
            raw_u = _to_dev(src.rows(un, *fr), dev)
            if tg == tu:
                inter = torch.stack([raw_g, raw_u], 1).reshape(2 * f_local, -1)
                lw.w_gate_up = _tile_raw(inter, tg, 2 * f_local, H)
            else:
                # Mixed types: dequantise both to F32 rows, interleave, tile as bf16.
                from .. import _native
                h = _native.host()
                g = torch.from_numpy(h.dequantize(int(tg), raw_g.cpu().numpy(), f_local, H))
                u = torch.from_numpy(h.dequantize(int(tu), raw_u.cpu().numpy(), f_local, H))
                inter = torch.stack([g, u], 1).reshape(2 * f_local, H).to(dev)
                lw.w_gate_up = ops.tile_weight(inter, int(GType.F32), 2 * f_local, H)
            lw.w_gate_up.interleaved_swiglu = True
            del raw_g, raw_u
            lw.w_down = _tile(src, dn, dev, c0=fr[0], c1=fr[1])
        layers.append(lw)
        for w in lw.wqkv + [lw.wo, lw.w_gate_up, lw.w_down]:
            if w is not None:
                total += w.nbytes
        if lw.moe is not None:
            total += lw.moe.router.nbytes + lw.moe.gate_up.nbytes + lw.moe.down.nbytes
    # Embedding (replicated raw rows) and output projection (vocab-parallel).
    es = src.info("token_embd.weight")
    embd = _to_dev(src.rows("token_embd.weight"), dev)
    if es.gtype == GType.F32:
        embd = embd.view(torch.uint8).reshape(es.ne[1], -1)
    V = cfg.vocab
    if V % tp_size:
        raise ValueError(f"vocab {V} not divisible by tp {tp_size} (vocab-parallel lm_head)")
    per = V // tp_size
    v0, v1 = tp_rank * per, min(V, (tp_rank + 1) * per)
    out_name = "output.weight" if src.has("output.weight") else "token_embd.weight"
    lm_head = _tile(src, out_name, dev, r0=v0, r1=v1)
    total += lm_head.nbytes + embd.numel()
    torch.cuda.synchronize(dev)
    return ModelWeights(cfg=cfg, layers=layers, embd=embd, embd_type=es.gtype,
                        embd_row_bytes=row_bytes(es.gtype, cfg.hidden),
                        output_norm=_to_dev(src.rows("output_norm.weight"), dev).view(-1).float(),
                        lm_head=lm_head, vocab_begin=v0, vocab_end=v1, tp_rank=tp_rank, tp_size=tp_size,
                        bytes_total=total)


def rope_table(cfg: ModelConfig, max_pos: int, device) -> torch.Tensor:
    inv = torch.tensor(rope_inv_freq(cfg), dtype=torch.float64)
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = pos[:, None] * inv[None, :]
    cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).to(torch.float32)
    return cs.contiguous().to(device)   # [max_pos, D/2, 2]


# ------------------------------------------------------------------------------------------------
# Forward


@dataclass
class StepMeta:
    """Device views of one step's metadata (see BatchLayout in csrc/host/scheduler.hpp)."""
    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    q_start: torch.Tensor
    ctx_len: torch.Tensor
    block_tables: torch.Tensor
    logits_idx: torch.Tensor
    T: int            # tokens (including padding rows)
    R: int            # requests (including padding rows)
    S: int            # sampled rows
    num_decode: int   # leading decode requests (one token each)
    max_qlen: int     # max q_len over the prefill requests
    decode_qlen: int = 1
    tree_mask: torch.Tensor | None = None  # int64 [T]: token-tree masks (prefill path)
    tree_span: int = 0                     # bit 0 of a mask = key at position ctx - tree_span
    seq_slot: torch.Tensor | None = None   # int32 [R]: the scheduler's sequence slot of each request


@dataclass
class Workspace:
    resid: torch.Tensor
    h: torch.Tensor
    qkv: torch.Tensor      # fp32 (split-K accumulate) or bf16 view on the same storage
    q: torch.Tensor
    attn: torch.Tensor
    o: torch.Tensor        # fp32
    act: torch.Tensor      # bf16 [T, F_local]
    down: torch.Tensor     # fp32
    gu32: torch.Tensor     # fp32 [T, 2F_local] (split-K gate/up)
    hs: torch.Tensor       # bf16 [S, H]
    logits: torch.Tensor   # fp32 [S, V_local]
    part_o: torch.Tensor | None = None
    part_lse: torch.Tensor | None = None


class LlamaModel:
    def __init__(self, w: ModelWeights, max_tokens: int, max_samples: int, max_model_len: int, comm=None,
                 attn_splits: int = 0):
        self.w = w
        self.cfg = cfg = w.cfg
        self.dev = w.output_norm.device
        self.tp = w.tp_size
        self.comm = comm
        self.hq = cfg.n_heads // self.tp
        _, self.hkv = _kv_heads_local(cfg, w.tp_rank, self.tp)
        self.D = cfg.head_dim
        self.H = cfg.hidden
        self.f_local = cfg.ffn // self.tp
        self.v_local = w.vocab_end - w.vocab_begin
        self.max_tokens = max_tokens
        self.max_samples = max_samples
        self.cos_sin = rope_table(cfg, max_model_len + 1, self.dev)
        self.scale = 1.0 / math.sqrt(self.D)
        self.attn_splits = attn_splits
        T, S = max_tokens, max_samples
        qkv_n = (self.hq + 2 * self.hkv) * self.D
        dev = self.dev
        qkv32 = torch.empty(T, qkv_n, dtype=torch.float32, device=dev)
        self.ws = Workspace(
            resid=torch.empty(T, self.H, dtype=torch.float32, device=dev),
            h=torch.empty(T, self.H, dtype=torch.bfloat16, device=dev),
            qkv=qkv32,
            q=torch.empty(T, self.hq * self.D, dtype=torch.bfloat16, device=dev),
            attn=torch.empty(T, self.hq * self.D, dtype=torch.bfloat16, device=dev),
            o=torch.empty(T, self.H, dtype=torch.float32, device=dev),
            act=torch.empty(T, max(self.f_local, 1), dtype=torch.bfloat16, device=dev),
            down=torch.empty(T, self.H, dtype=torch.float32, device=dev),
            gu32=torch.empty(T, 2 * max(self.f_local, 1), dtype=torch.float32, device=dev),
            hs=torch.empty(S, self.H, dtype=torch.bfloat16, device=dev),
            logits=torch.empty(S, self.v_local, dtype=torch.float32, device=dev),
        )
        self.qkv_bf16 = torch.empty(T, qkv_n, dtype=torch.bfloat16, device=dev)
        self.o16 = torch.empty(T, self.H, dtype=torch.bfloat16, device=dev)
        # Split-K partials: [splits][M][N] fp32, summed by the consumer kernel (no atomics, no memset).
        self.qkv_n = qkv_n
        self.split_ws = torch.empty(T * max(qkv_n, 2 * max(self.f_local, 1), self.H), dtype=torch.float32, device=dev)
        if attn_splits > 1:
            self.ws.part_o = torch.empty(attn_splits, max_samples, self.hq, self.D, dtype=torch.float32, device=dev)
            self.ws.part_lse = torch.empty(attn_splits, max_samples, self.hq, dtype=torch.float32, device=dev)
        ops.C().gemm_prepare()  # per-device GEMM workspace, before any CUDA-graph capture
        self.fused = self.tp > 1 and comm is not None and hasattr(comm, "allreduce_add_rmsnorm")
        if self.fused:
            comm.setup(max_tokens, self.H, max_samples)
            # The gathered activations live in the symmetric region: owners push their rows there.
            self.ws.h = comm.h
        # Native step forward (csrc/kernels/forward.cpp): the whole kernel program of a step issued
        # from C++. VMC_NATIVE=0 keeps every step on the Python path below.
        self.use_native = os.environ.get("VMC_NATIVE", "1") != "0"
        self._nat = None
        self._nat_key = None
        self.moe_runner = None
        self.ep = 1
        self.tq = None  # TurboQuant tables when the KV cache is compressed (set by the runner)
        self.tracer = None  # utils.trace.HiddenTracer when VMC_LOG_HIDDEN / VMC_LOG_LOGITS is set
        if cfg.is_moe:
            from .moe import MoERunner
            self.moe_runner = MoERunner(self, max_tokens)
            moe0 = next(lw.moe for lw in w.layers if lw.moe is not None)
            self.ep = cfg.n_experts // moe0.e_local if moe0.e_local < cfg.n_experts else 1
            if self.ep > 1 and self.fused and self.use_native:
                comm.setup_moe(cfg.n_experts, cfg.n_experts_used, moe0.e_local, moe0.f_local, self.H)

    # -- split-K policy ----------------------------------------------------------------------------
    def _splits(self, w: ops.TiledWeight, M: int) -> int:
        s = ops.pick_splits(w, M)
        while s > 1 and s * M > self.max_tokens:
            s -= 1
        return ops.effective_splits(w, s)

    def _split_view(self, M: int, N: int) -> torch.Tensor:
        return self.split_ws[:M * N].view(M, N)

    def _qkv(self, lw: LayerWeights, x: torch.Tensor, M: int, m: StepMeta, kv_layer: torch.Tensor) -> None:
        """QKV GEMM(s) + RoPE + paged KV store."""
        s = self._splits(lw.wqkv[0], M)
        if s > 1:
            out = self._split_view(M, self.qkv_n)
            for w, c0 in zip(lw.wqkv, lw.qkv_split):
                ops.gemm(x, w, out[:, c0:c0 + w.N], M, ops.OUT_F32_SPLIT, s, split_stride=M * self.qkv_n)
            self._rope_store(out, M, m, kv_layer, lw.index, nsplit=s, split_stride=M * self.qkv_n)
            return
        for w, c0 in zip(lw.wqkv, lw.qkv_split):
            ops.gemm(x, w, self.qkv_bf16[:M, c0:c0 + w.N], M, ops.OUT_BF16, 1)
        self._rope_store(self.qkv_bf16[:M], M, m, kv_layer, lw.index)

    def _rope_store(self, qkv, M: int, m: StepMeta, kv_layer: torch.Tensor, layer: int, nsplit=1,
                    split_stride=0) -> None:
        if self.tq is None:
            ops.rope_store(qkv, M, self.hq, self.hkv, self.D, m.positions, m.slot_mapping, self.cos_sin,
                           self.cfg.rope_neox, self.ws.q, kv_layer, nsplit=nsplit, split_stride=split_stride)
        else:
            ops.rope_store_tq(qkv, M, self.hq, self.hkv, self.D, m.positions, m.slot_mapping, self.cos_sin,
                              self.cfg.rope_neox, self.ws.q, kv_layer, self.tq, layer, nsplit=nsplit,
                              split_stride=split_stride)

    def _row_parallel_norm(self, x: torch.Tensor, w: ops.TiledWeight, M: int, norm_w: torch.Tensor) -> None:
        """Row-parallel GEMM, (TP reduce), residual add + RMSNorm into ws.h."""
        ws, eps = self.ws, self.cfg.rms_eps
        if self.tp > 1:
            # NCCL baseline: one fp32 partial, all-reduced in place.
            s = self._splits(w, M)
            o = ws.o[:M]
            if s > 1:
                o.zero_()
            ops.gemm(x, w, o, M, ops.OUT_F32_ADD if s > 1 else ops.OUT_F32, s)
            self.comm.all_reduce(o)
            ops.add_rmsnorm(ws.resid, norm_w, M, self.H, eps, out=ws.h, delta=o)
            return
        s = self._splits(w, M)
        if s > 1:
            out = self._split_view(M, self.H)
            ops.gemm(x, w, out, M, ops.OUT_F32_SPLIT, s, split_stride=M * self.H)
            ops.add_rmsnorm(ws.resid, norm_w, M, self.H, eps, out=ws.h, delta=out, ndelta=s, delta_stride=M * self.H)
        else:
            ops.gemm(x, w, self.o16[:M], M, ops.OUT_BF16, 1)
            ops.add_rmsnorm(ws.resid, norm_w, M, self.H, eps, out=ws.h, delta=self.o16[:M])

    def _row_parallel_fused(self, site: int, x: torch.Tensor, w: ops.TiledWeight, M: int,
                            norm_w: torch.Tensor) -> None:
        """Row-parallel GEMM into this rank's symmetric partial buffer, then one kernel that
        all-reduces over NVLink, adds the residual and applies the next RMSNorm."""
        s = self._splits(w, M)
        part = self.comm.partial(site).view(-1)[:s * M * self.H].view(s * M, self.H)
        ops.gemm(x, w, part[:M], M, ops.OUT_F32_SPLIT if s > 1 else ops.OUT_F32, s, split_stride=M * self.H)
        self.comm.allreduce_add_rmsnorm(site, M, self.ws.resid, norm_w, self.cfg.rms_eps, self.ws.h, nsplit=s,
                                        split_stride=M * self.H)

    def _gate_up(self, lw: LayerWeights, M: int) -> None:
        ws = self.ws
        w = lw.w_gate_up
        s = self._splits(w, M)
        if s > 1:
            out = self._split_view(M, w.N)
            ops.gemm(ws.h, w, out, M, ops.OUT_F32_SPLIT, s, split_stride=M * w.N)
            ops.swiglu(out, M, w.N // 2, ws.act, interleaved=True, nsplit=s, split_stride=M * w.N)
        else:
            ops.gemm(ws.h, w, ws.act[:M], M, ops.OUT_SWIGLU, 1)

    # -- native step forward ----------------------------------------------------------------------
    def native_ok(self, m: StepMeta) -> bool:
        """Steps the C++ forward handles: dense layers, no tracing, no CPU-offloaded weights, no
        token-tree masks; one rank, or tensor parallel over the fused peer-memory backend."""
        if not (self.use_native and self.tracer is None and m.tree_mask is None
                and not any(lw.offload for lw in self.w.layers) and (self.tp == 1 or self.fused)):
            return False
        # MoE layers: one rank (expert-sliced), or expert parallelism over the fused backend
        return self.moe_runner is None or self.tp == 1 or self.ep > 1

    @staticmethod
    def _lin(w: ops.TiledWeight) -> list[int]:
        return [w.wf, w.data.data_ptr(), w.N, w.K]

    def _native(self, kv_cache: torch.Tensor, m: StepMeta, params: torch.Tensor, out_tok: torch.Tensor,
                out_lp: torch.Tensor | None):
        key = (kv_cache.data_ptr(), m.input_ids.data_ptr(), m.block_tables.data_ptr(), params.data_ptr(),
               out_tok.data_ptr(), 0 if out_lp is None else out_lp.data_ptr())
        if self._nat is not None and self._nat_key == key:
            return self._nat
        w, ws, cfg = self.w, self.ws, self.cfg
        zero = [0, 0, 0, 0]
        layers = []
        for lw in w.layers:
            q = [self._lin(x) for x in lw.wqkv] + [zero] * (3 - len(lw.wqkv))
            cols = list(lw.qkv_split) + [0] * (3 - len(lw.qkv_split))
            ffn = (self._lin(lw.w_gate_up) + self._lin(lw.w_down)) if lw.moe is None else zero + zero
            d = [lw.attn_norm.data_ptr(), lw.ffn_norm.data_ptr(), len(lw.wqkv)] + q[0] + q[1] + q[2] + cols \
                + self._lin(lw.wo) + ffn
            if lw.moe is not None:
                mo = lw.moe
                d += [1] + self._lin(mo.router) + self._lin(mo.gate_up) + [mo.gate_up_stride] + self._lin(mo.down) \
                    + [mo.down_stride, mo.e0, mo.e_local, mo.f_local]
            layers.append(d)
        c = dict(L=len(w.layers), H=self.H, Hq=self.hq, Hkv=self.hkv, D=self.D, F=max(self.f_local, 1),
                 V_local=self.v_local, max_tokens=self.max_tokens, max_samples=self.max_samples,
                 max_blocks=int(m.block_tables.shape[-1]), eps=float(cfg.rms_eps), scale=float(self.scale),
                 neox=bool(cfg.rope_neox), embd=w.embd.data_ptr(), embd_type=int(w.embd_type),
                 embd_row_bytes=int(w.embd_row_bytes), out_norm=w.output_norm.data_ptr(), lm_head=self._lin(w.lm_head),
                 cos_sin=self.cos_sin.data_ptr(), num_sms=ops.NUM_SMS)
        b = dict(resid=ws.resid.data_ptr(), h=ws.h.data_ptr(), qkv_bf16=self.qkv_bf16.data_ptr(),
                 split_ws=self.split_ws.data_ptr(), split_ws_elems=self.split_ws.numel(), q=ws.q.data_ptr(),
                 attn=ws.attn.data_ptr(), o16=self.o16.data_ptr(), act=ws.act.data_ptr(), hs=ws.hs.data_ptr(),
                 logits=ws.logits.data_ptr(), attn_max_splits=1, ids=m.input_ids.data_ptr(),
                 pos=m.positions.data_ptr(), slots=m.slot_mapping.data_ptr(), q_start=m.q_start.data_ptr(),
                 ctx_len=m.ctx_len.data_ptr(), block_tables=m.block_tables.data_ptr(),
                 logits_idx=m.logits_idx.data_ptr(), params=params.data_ptr(), out_tok=out_tok.data_ptr(),
                 kv=kv_cache.data_ptr(), kv_layer_bytes=kv_cache.stride(0) * kv_cache.element_size(),
                 err=ops._err_word(self.dev).data_ptr())
        if out_lp is not None:
            b["out_lp"] = out_lp.data_ptr()
        if ws.part_o is not None:
            b.update(part_o=ws.part_o.data_ptr(), part_lse=ws.part_lse.data_ptr(), attn_max_splits=ws.part_o.shape[0])
        if self.tq is not None:
            b.update(tq_meta=self.tq.meta(), tq_centroids=self.tq.centroids.data_ptr(),
                     tq_midpoints=self.tq.midpoints.data_ptr())
        nat = ops.C().make_forward(c, layers, b)
        if self.fused:
            nat.set_comm(self.comm.tp_desc())
        if self.moe_runner is not None:
            if self.ep > 1:
                nat.set_moe(self.comm.moe_desc())
            else:
                nat.set_moe(self.moe_runner.native_desc())
        self._nat, self._nat_key = nat, key
        return nat

    def forward(self, kv_cache: torch.Tensor, m: StepMeta, params: torch.Tensor, out_tok: torch.Tensor,
                out_lp: torch.Tensor | None = None, pre_sample=None) -> None:
        """One step: writes sampled token ids for the m.S sample rows into out_tok."""
        if self.native_ok(m):
            nat = self._native(kv_cache, m, params, out_tok, out_lp)
            local_sample = pre_sample is None and (self.tp == 1 or self.fused)
            ops._count(nat.run(m.T, m.R, m.S, m.num_decode, m.max_qlen, m.decode_qlen, self.attn_splits, local_sample))
            if not local_sample and m.S > 0:
                if pre_sample is not None:
                    pre_sample(self)
                self._sample(m.S, params, out_tok, out_lp)
            return
        cfg, ws = self.cfg, self.ws
        T = m.T
        tr = self.tracer
        ops.embed(m.input_ids, T, self.w.embd, self.w.embd_type, self.w.embd_row_bytes, self.H, resid=ws.resid)
        if tr:
            tr.probe("inp_embd", ws.resid[:T])
        layers = self.w.layers
        ops.add_rmsnorm(ws.resid, layers[0].attn_norm, T, self.H, cfg.rms_eps, out=ws.h)
        rng = LayerRanges()
        for li, lw in enumerate(layers):
            rng.next(li)
            for host, dev in lw.offload:  # CPU-offloaded weights of this layer into the staging buffer
                dev.copy_(host, non_blocking=True)
            if tr:
                tr.probe(f"attn_norm-{li}", ws.h[:T])
            self._qkv(lw, ws.h, T, m, kv_cache[li])
            self._attention(kv_cache[li], m)
            if tr:
                tr.probe(f"kqv_out-{li}", ws.attn[:T])
            nxt = layers[li + 1].attn_norm if li + 1 < len(layers) else self.w.output_norm
            if self.fused and T <= self.comm.max_fused_tokens:
                self._row_parallel_fused(0, ws.attn, lw.wo, T, lw.ffn_norm)
                if tr:
                    tr.probe(f"ffn_inp-{li}", ws.resid[:T])
                if lw.moe is not None:
                    part = self.comm.partial(1).view(-1)[:T * self.H].view(T, self.H)
                    self.moe_runner.forward(lw.moe, ws.h, T, out=part)
                    self.comm.allreduce_add_rmsnorm(1, T, ws.resid, nxt, cfg.rms_eps, ws.h)
                    if tr:
                        tr.probe(f"l_out-{li}", ws.resid[:T])
                    continue
                self._gate_up(lw, T)
                if tr:
                    tr.probe(f"ffn_swiglu-{li}", ws.act[:T])
                self._row_parallel_fused(1, ws.act, lw.w_down, T, nxt)
                if tr:
                    tr.probe(f"l_out-{li}", ws.resid[:T])
                continue
            self._row_parallel_norm(ws.attn, lw.wo, T, lw.ffn_norm)
            if tr:
                tr.probe(f"ffn_inp-{li}", ws.resid[:T])
            if lw.moe is not None:
                d, _ = self.moe_runner.forward(lw.moe, ws.h, T)
                if self.tp > 1:
                    self.comm.all_reduce(d[:T])
                ops.add_rmsnorm(ws.resid, nxt, T, self.H, cfg.rms_eps, out=ws.h, delta=d[:T])
                if tr:
                    tr.probe(f"l_out-{li}", ws.resid[:T])
                continue
            self._gate_up(lw, T)
            if tr:
                tr.probe(f"ffn_swiglu-{li}", ws.act[:T])
            self._row_parallel_norm(ws.act, lw.w_down, T, nxt)
            if tr:
                tr.probe(f"l_out-{li}", ws.resid[:T])
        rng.close()
        ops.gather_rows(ws.h, m.logits_idx, m.S, self.H, ws.hs)
        if tr:
            tr.probe("result_norm", ws.hs[:m.S])
        ops.gemm(ws.hs, self.w.lm_head, ws.logits[:m.S], m.S, ops.OUT_F32, 1)
        if pre_sample is not None:
            pre_sample(self)
        if tr:
            tr.probe("result_output", ws.logits[:m.S])
            if self.tp == 1:
                tr.probe_logits(ws.logits, m.S)
        self._sample(m.S, params, out_tok, out_lp)

    def _attention(self, kv_layer: torch.Tensor, m: StepMeta) -> None:
        ws = self.ws
        tq = None if self.tq is None else (kv_layer, self.tq)
        nd = m.num_decode
        G = self.hq // self.hkv
        if nd > 0:
            dec_ok = m.decode_qlen * G <= 16
            splits = self.attn_splits if (self.attn_splits > 1 and dec_ok and nd <= self.max_samples) else 1
            ops.paged_attention(ws.q, kv_layer, m.q_start, m.ctx_len, m.block_tables, nd, 0, m.decode_qlen,
                                nd * m.decode_qlen, self.hq, self.hkv, self.D, self.scale, dec_ok, ws.attn,
                                splits, ws.part_o if splits > 1 else None, ws.part_lse if splits > 1 else None,
                                tq=tq)
        if m.R > nd:
            ops.paged_attention(ws.q, kv_layer, m.q_start, m.ctx_len, m.block_tables, m.R - nd, nd, m.max_qlen,
                                m.T, self.hq, self.hkv, self.D, self.scale, False, ws.attn, tq=tq,
                                tree_mask=m.tree_mask, tree_span=m.tree_span)

    def _sample(self, S: int, params: torch.Tensor, out_tok: torch.Tensor, out_lp) -> None:
        if self.tp > 1:
            self.comm.sample_vocab_parallel(self, S, params, out_tok, out_lp)
        else:
            ops.sample(self.ws.logits, S, self.v_local, params, out_tok, out_lp)
