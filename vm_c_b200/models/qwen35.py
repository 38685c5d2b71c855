"""Serving forward of the hybrid Qwen3.5-MoE family (gated delta-net + gated full attention, MoE with a
sigmoid-gated shared expert), one GPU.

Reference graph: src/official/llama/models/qwen35moe.cpp:164-590 (build_layer_attn_linear /
build_layer_attn / build_moe_ffn with the shared expert) and delta-net-base.cpp:289-363. Per layer:

  x  = rmsnorm(h) * attn_norm
  GDN layer:   one GEMM gives mixed q|k|v, the output gate z, beta and alpha; gdn_conv (causal conv +
               SiLU, conv history in a slot pool); gdn_recurrent (gated delta rule with the fp32 state
               in a slot pool, fused q/k l2 norms, gates and gated RMSNorm); ssm_out GEMM
  attention:   q (with a per-head output gate) / k / v GEMMs; Q and K RMSNorm per head; RoPE on the
               first rope_dims dims of each head (half rotation); paged KV store; paged attention
               (tcgen05 prefill kernel for head dim 128, mma.sync otherwise); o * sigmoid(gate); o GEMM
  h += that;  x2 = rmsnorm(h) * post_attention_norm
  h += routed experts (router GEMM, moe_route, grouped GEMMs, combine) + sigmoid(x2 . w_shexp_gate) *
       shared expert (gate/up GEMM with fused SwiGLU, down GEMM)

Recurrent state lives in per-request slots: the scheduler's sequence slot (held from admission to
finish or preemption) indexes the conv-history and delta-state pools, and a request whose context
before the step is empty (new, or recomputed after preemption) starts from zero, so slots are never
cleared. Prefix caching is off for this family (cached KV blocks cannot restore a recurrent state)
and steps run eagerly (no CUDA graphs). Q/K RMSNorm, the partial RoPE with the KV store, and the
two sigmoid gates are small element-wise steps done with torch ops on the device; everything else
runs on this library's kernels. Tensor parallelism, speculative decoding, TurboQuant KV and CPU
offload are refused for this family.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .. import ops
from ..config import ModelConfig
from ..gguf.constants import GType, blk, row_bytes
from .llama import ModelWeights, _tile, _tile_raw, _to_dev


@dataclass
class GdnWeights:
    w_in: ops.TiledWeight      # rows: mixed q|k|v [C], z [Hv*Ds], beta [Hv], alpha [Hv]
    conv_w: torch.Tensor       # fp32 [C, ssm_conv]
    a_neg: torch.Tensor        # fp32 [Hv]
    dt_bias: torch.Tensor      # fp32 [Hv]
    norm_w: torch.Tensor       # fp32 [Ds]
    w_out: ops.TiledWeight     # [H, Hv*Ds]


@dataclass
class GatedAttnWeights:
    wq: ops.TiledWeight        # [2 Hq D, H]: per head D query rows then D gate rows
    wk: ops.TiledWeight
    wv: ops.TiledWeight
    q_norm: torch.Tensor       # fp32 [D]
    k_norm: torch.Tensor
    wo: ops.TiledWeight        # [H, Hq D]


@dataclass
class HybridLayer:
    index: int
    attn_norm: torch.Tensor
    post_norm: torch.Tensor
    gdn: GdnWeights | None
    attn: GatedAttnWeights | None
    moe: object                # models/moe.py MoEWeights
    sh_gate_up: ops.TiledWeight  # shared expert, gate/up rows interleaved (fused SwiGLU)
    sh_down: ops.TiledWeight
    sh_gate: torch.Tensor      # fp32 [H]: the shared expert's sigmoid gate
    offload: tuple = ()


def _dense(src, name: str, dev) -> torch.Tensor:
    """A tensor as dense fp32 rows [rows, ne0] on the device (1-D tensors as vectors)."""
    spec = src.info(name)
    raw = src.rows(name)
    K = spec.ne[0]
    if spec.gtype == GType.F32:
        m = raw.float().reshape(-1, K)
    else:
        from .. import _native
        m = torch.from_numpy(_native.host().dequantize(int(spec.gtype), raw.cpu().numpy(), spec.rows, K))
    m = m.to(dev).contiguous()
    return m.view(-1) if len(spec.ne) == 1 else m


def _tile_rows(src, names: list[str], dev) -> ops.TiledWeight:
    """The rows of several [*, H] tensors stacked into one GEMM weight (raw blocks when they share a
    type, else dequantised rows tiled as bf16)."""
    specs = [src.info(n) for n in names]
    K = specs[0].ne[0]
    N = sum(s.rows for s in specs)
    if all(s.gtype == specs[0].gtype for s in specs):
        raw = torch.cat([_to_dev(src.rows(n), dev).view(torch.uint8).reshape(s.rows, -1) for n, s in zip(names, specs)])
        return _tile_raw(raw, specs[0].gtype, N, K)
    rows = torch.cat([_dense(src, n, dev) for n in names])
    return ops.tile_weight(rows, int(GType.F32), N, K)


def _interleaved_gate_up(src, gate: str, up: str, dev) -> ops.TiledWeight:
    sg, su = src.info(gate), src.info(up)
    F, H = sg.rows, sg.ne[0]
    if sg.gtype == su.gtype:
        g = _to_dev(src.rows(gate), dev).view(torch.uint8).reshape(F, -1)
        u = _to_dev(src.rows(up), dev).view(torch.uint8).reshape(F, -1)
        w = _tile_raw(torch.stack([g, u], 1).reshape(2 * F, -1), sg.gtype, 2 * F, H)
    else:
        w = ops.tile_weight(torch.stack([_dense(src, gate, dev), _dense(src, up, dev)], 1).reshape(2 * F, H),
                            int(GType.F32), 2 * F, H)
    w.interleaved_swiglu = True
    return w


def load_hybrid_weights(src, cfg: ModelConfig, dev, tp_rank: int = 0, tp_size: int = 1) -> ModelWeights:
    """Every tensor of a Qwen3.5-MoE checkpoint (main layers; MTP blocks are not loaded) on one GPU."""
    from .hybrid import check_hybrid_tensors
    from .moe import load_moe_layer
    check_hybrid_tensors(src, cfg)
    if tp_size != 1:
        raise ValueError("GGUF architecture 'qwen35moe' is served on one GPU (tensor parallelism is not "
                         "implemented for the gated delta-net layers)")
    if cfg.n_heads % max(1, cfg.n_kv_heads):
        raise ValueError("n_heads must be a multiple of n_kv_heads")
    layers, total = [], 0
    for i in range(cfg.n_layers - cfg.nextn_layers):
        b = lambda n: blk(i, n)  # noqa: E731
        gdn = attn = None
        if cfg.is_recurrent(i):
            gdn = GdnWeights(
                w_in=_tile_rows(src, [b("attn_qkv"), b("attn_gate"), b("ssm_beta"), b("ssm_alpha")], dev),
                conv_w=_dense(src, b("ssm_conv1d"), dev), a_neg=_dense(src, f"blk.{i}.ssm_a", dev),
                dt_bias=_dense(src, f"blk.{i}.ssm_dt.bias", dev),
                norm_w=_dense(src, b("ssm_norm"), dev), w_out=_tile(src, b("ssm_out"), dev))
            total += gdn.w_in.nbytes + gdn.w_out.nbytes
        else:
            attn = GatedAttnWeights(wq=_tile(src, b("attn_q"), dev), wk=_tile(src, b("attn_k"), dev),
                                    wv=_tile(src, b("attn_v"), dev), q_norm=_dense(src, b("attn_q_norm"), dev),
                                    k_norm=_dense(src, b("attn_k_norm"), dev), wo=_tile(src, b("attn_output"), dev))
            total += attn.wq.nbytes + attn.wk.nbytes + attn.wv.nbytes + attn.wo.nbytes
        moe = load_moe_layer(src, cfg, i, dev, 0, 1, 1)
        lw = HybridLayer(index=i, attn_norm=_dense(src, b("attn_norm"), dev),
                         post_norm=_dense(src, b("post_attention_norm"), dev), gdn=gdn, attn=attn, moe=moe,
                         sh_gate_up=_interleaved_gate_up(src, b("ffn_gate_shexp"), b("ffn_up_shexp"), dev),
                         sh_down=_tile(src, b("ffn_down_shexp"), dev), sh_gate=_dense(src, b("ffn_gate_inp_shexp"), dev))
        total += moe.router.nbytes + moe.gate_up.nbytes + moe.down.nbytes + lw.sh_gate_up.nbytes + lw.sh_down.nbytes
        layers.append(lw)
    es = src.info("token_embd.weight")
    embd = _to_dev(src.rows("token_embd.weight"), dev)
    if es.gtype == GType.F32:
        embd = embd.view(torch.uint8).reshape(es.ne[1], -1)
    out_name = "output.weight" if src.has("output.weight") else "token_embd.weight"
    lm_head = _tile(src, out_name, dev)
    total += lm_head.nbytes + embd.numel()
    torch.cuda.synchronize(dev)
    return ModelWeights(cfg=cfg, layers=layers, embd=embd, embd_type=es.gtype, embd_row_bytes=row_bytes(es.gtype, cfg.hidden),
                        output_norm=_dense(src, "output_norm.weight", dev), lm_head=lm_head, vocab_begin=0,
                        vocab_end=cfg.vocab, tp_rank=0, tp_size=1, bytes_total=total)


class HybridModel:
    """Workspaces, recurrent-state pools and the step forward of one Qwen3.5-MoE model (one GPU)."""

    def __init__(self, w: ModelWeights, max_tokens: int, max_samples: int, max_model_len: int, num_slots: int):
        from .moe import MoERunner
        self.w = w
        self.cfg = cfg = w.cfg
        self.dev = dev = w.output_norm.device
        self.tp = 1
        self.comm = None
        self.fused = False
        self.hq, self.hkv, self.D, self.H = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden
        self.v_local = cfg.vocab
        self.max_tokens, self.max_samples = max_tokens, max_samples
        self.scale = 1.0 / math.sqrt(self.D)
        self.attn_splits = 1
        self.tq = None
        self.tracer = None
        self.Hk, self.Hv, self.Ds = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_state
        self.C = 2 * self.Hk * self.Ds + self.Hv * self.Ds
        self.Cw = self.C + self.Hv * self.Ds + 2 * self.Hv
        T, S, f32, bf16 = max_tokens, max_samples, torch.float32, torch.bfloat16
        e = lambda *shape, dt=f32: torch.empty(*shape, dtype=dt, device=dev)  # noqa: E731
        self.resid, self.h, self.a = e(T, self.H), e(T, self.H, dt=bf16), e(T, self.H)
        self.proj, self.y, self.gout = e(T, self.Cw), e(T, self.C), e(T, self.Hv * self.Ds, dt=bf16)
        self.qg, self.kf, self.vf = e(T, 2 * self.hq * self.D), e(T, self.hkv * self.D), e(T, self.hkv * self.D)
        self.q16, self.attn_out, self.o16 = (e(T, self.hq * self.D, dt=bf16) for _ in range(3))
        self.act, self.sh = e(T, max(cfg.ffn_shexp, 1), dt=bf16), e(T, self.H)

        class _Ws:  # what the runner and the sampler read: the logits of the sampled rows
            pass
        self.ws = _Ws()
        self.ws.h = self.h
        self.ws.hs = e(S, self.H, dt=bf16)
        self.ws.logits = e(S, cfg.vocab)
        # attention layers own the KV cache layers in order; GDN layers own state-pool layers
        self.kv_index, self.gdn_index = {}, {}
        for lw in w.layers:
            if lw.attn is not None:
                self.kv_index[lw.index] = len(self.kv_index)
            else:
                self.gdn_index[lw.index] = len(self.gdn_index)
        self.n_kv_layers = max(1, len(self.kv_index))
        n_gdn = len(self.gdn_index)
        self.conv = torch.zeros(max(n_gdn, 1), num_slots, cfg.ssm_conv - 1, self.C, dtype=f32, device=dev)
        self.state = torch.zeros(max(n_gdn, 1), num_slots, self.Hv, self.Ds, self.Ds, dtype=f32, device=dev)
        # partial RoPE: half rotation over the first n_rot dims of each head
        self.n_rot = cfg.rope_dims or self.D
        half = self.n_rot // 2
        inv = 1.0 / cfg.rope_theta ** (torch.arange(half, dtype=torch.float64) * 2 / self.n_rot)
        ang = torch.arange(max_model_len + 1, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos, self.sin = ang.cos().float().to(dev), ang.sin().float().to(dev)
        self.moe_runner = MoERunner(self, max_tokens)
        ops.C().gemm_prepare()

    # -- per-layer parts --------------------------------------------------------------------------------
    def _gdn(self, g: GdnWeights, gi: int, T: int, R: int, q_start, slot, has) -> None:
        C, HD, Hv = self.C, self.Hv * self.Ds, self.Hv
        ops.gemm(self.h, g.w_in, self.proj[:T], T, ops.OUT_F32, 1)
        mixed, z = self.proj[:T, :C], self.proj[:T, C:C + HD]
        beta, alpha = self.proj[:T, C + HD:C + HD + Hv], self.proj[:T, C + HD + Hv:C + HD + 2 * Hv]
        ops.gdn_conv(mixed, g.conv_w, q_start, slot, has, R, self.conv[gi], self.y[:T])
        ops.gdn_recurrent(self.y[:T], alpha, beta, z, g.a_neg, g.dt_bias, g.norm_w, self.state[gi], slot, has,
                          q_start, R, self.Hk, self.cfg.rms_eps, self.gout[:T])
        ops.gemm(self.gout, g.w_out, self.a[:T], T, ops.OUT_F32, 1)

    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        half = self.n_rot // 2
        c, s = self.cos[pos][:, None, :], self.sin[pos][:, None, :]
        a, b = x[..., :half], x[..., half:self.n_rot]
        return torch.cat([a * c - b * s, a * s + b * c, x[..., self.n_rot:]], -1)

    def _attention(self, at: GatedAttnWeights, kv_layer: torch.Tensor, m, T: int) -> None:
        Hq, Hkv, D, eps = self.hq, self.hkv, self.D, self.cfg.rms_eps
        ops.gemm(self.h, at.wq, self.qg[:T], T, ops.OUT_F32, 1)
        ops.gemm(self.h, at.wk, self.kf[:T], T, ops.OUT_F32, 1)
        ops.gemm(self.h, at.wv, self.vf[:T], T, ops.OUT_F32, 1)
        qg = self.qg[:T].view(T, Hq, 2 * D)
        q, gate = qg[..., :D], qg[..., D:]
        k = self.kf[:T].view(T, Hkv, D)
        rms = lambda x, w: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w  # noqa: E731
        pos = m.positions[:T].long()
        q = self._rope(rms(q, at.q_norm), pos)
        k = self._rope(rms(k, at.k_norm), pos)
        self.q16[:T].view(T, Hq, D).copy_(q)
        slots = m.slot_mapping[:T].long()
        ok = slots >= 0
        bs = kv_layer.shape[3]
        sl = slots[ok]
        kv_layer[sl // bs, 0, :, sl % bs, :] = k[ok].to(torch.bfloat16)
        kv_layer[sl // bs, 1, :, sl % bs, :] = self.vf[:T].view(T, Hkv, D)[ok].to(torch.bfloat16)
        nd, R = m.num_decode, m.R
        if nd > 0:
            dec_ok = m.decode_qlen * (Hq // Hkv) <= 16
            ops.paged_attention(self.q16, kv_layer, m.q_start, m.ctx_len, m.block_tables, nd, 0, m.decode_qlen,
                                nd * m.decode_qlen, Hq, Hkv, D, self.scale, dec_ok, self.attn_out)
        if R > nd:
            ops.paged_attention(self.q16, kv_layer, m.q_start, m.ctx_len, m.block_tables, R - nd, nd, m.max_qlen, T,
                                Hq, Hkv, D, self.scale, False, self.attn_out)
        o = self.attn_out[:T].view(T, Hq, D).float() * torch.sigmoid(gate)
        self.o16[:T].copy_(o.reshape(T, Hq * D))
        ops.gemm(self.o16, at.wo, self.a[:T], T, ops.OUT_F32, 1)

    # -- step ---------------------------------------------------------------------------------------------
    def forward(self, kv_cache: torch.Tensor, m, params: torch.Tensor, out_tok: torch.Tensor,
                out_lp: torch.Tensor | None = None, pre_sample=None) -> None:
        """One step: writes sampled token ids for the m.S sample rows into out_tok."""
        cfg, w, T, R, H, eps = self.cfg, self.w, m.T, m.R, self.H, self.cfg.rms_eps
        if m.seq_slot is None:
            raise ValueError("hybrid models need the sequence slots of the step metadata")
        ops.embed(m.input_ids, T, w.embd, w.embd_type, w.embd_row_bytes, H, resid=self.resid)
        ops.add_rmsnorm(self.resid, w.layers[0].attn_norm, T, H, eps, out=self.h)
        # recurrent-state slots: the scheduler's sequence slots; no context before this step = zero state
        q_start = m.q_start[:R + 1]
        slot = m.seq_slot[:R].contiguous()
        has = ((m.ctx_len[:R] - (q_start[1:] - q_start[:-1])) > 0).to(torch.int32)
        for li, lw in enumerate(w.layers):
            if lw.gdn is not None:
                self._gdn(lw.gdn, self.gdn_index[lw.index], T, R, q_start, slot, has)
            else:
                self._attention(lw.attn, kv_cache[self.kv_index[lw.index]], m, T)
            ops.add_rmsnorm(self.resid, lw.post_norm, T, H, eps, out=self.h, delta=self.a[:T])
            d, _ = self.moe_runner.forward(lw.moe, self.h, T)
            ops.gemm(self.h, lw.sh_gate_up, self.act[:T], T, ops.OUT_SWIGLU, 1)
            ops.gemm(self.act, lw.sh_down, self.sh[:T], T, ops.OUT_F32, 1)
            sg = torch.sigmoid(self.h[:T].float() @ lw.sh_gate)
            d[:T].add_(sg[:, None] * self.sh[:T])
            nxt = w.layers[li + 1].attn_norm if li + 1 < len(w.layers) else w.output_norm
            ops.add_rmsnorm(self.resid, nxt, T, H, eps, out=self.h, delta=d[:T])
        ops.gather_rows(self.h, m.logits_idx, m.S, H, self.ws.hs)
        ops.gemm(self.ws.hs, w.lm_head, self.ws.logits[:m.S], m.S, ops.OUT_F32, 1)
        if pre_sample is not None:
            pre_sample(self)
        ops.sample(self.ws.logits, m.S, self.v_local, params, out_tok, out_lp)
