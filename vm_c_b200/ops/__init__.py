"""Python entry points of the sm_100a kernels (thin wrappers over the ``_cuda`` extension).

Every function launches on the current CUDA stream and writes into caller-provided tensors, so a
sequence of them can be captured into a CUDA graph. There is no PyTorch fallback: if the CUDA
extension is missing the first call raises ImportError.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from .. import _native
from ..gguf.constants import GType

# Tiled weight formats (csrc/kernels/weight_formats.cuh).
WF_BF16, WF_Q4K, WF_Q6K, WF_Q8_0 = 0, 1, 2, 3
OUT_BF16, OUT_F32, OUT_F32_ADD, OUT_SWIGLU, OUT_F32_SPLIT = 0, 1, 2, 3, 4
NUM_SMS = 148
# Decode-width quantized GEMMs that the split policy leaves unsplit run a stream-K schedule
# (csrc/kernels/gemm_tcgen05.cu); VMC_STREAMK=0 turns it off (read by the C++ side).
STREAMK = os.environ.get("VMC_STREAMK", "1") != "0"

_WF_FOR_GTYPE = {GType.Q4_K: WF_Q4K, GType.Q6_K: WF_Q6K, GType.Q8_0: WF_Q8_0,
                 GType.F32: WF_BF16, GType.F16: WF_BF16, GType.BF16: WF_BF16}
_CHUNK = {WF_BF16: 64, WF_Q4K: 256, WF_Q6K: 256, WF_Q8_0: 256}
_ROWB = {WF_BF16: 128, WF_Q4K: 160, WF_Q6K: 224, WF_Q8_0: 272}


def C():
    return _native.cuda()


# Number of kernel launches issued through these wrappers (for the bench's launch count).
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def wf_for_gtype(t: int) -> int | None:
    return _WF_FOR_GTYPE.get(GType(t))


def tiled_bytes(wf: int, N: int, K: int) -> int:
    return ((N + 127) // 128) * ((K + _CHUNK[wf] - 1) // _CHUNK[wf]) * 128 * _ROWB[wf]


@dataclass
class TiledWeight:
    """A linear weight [N, K] in a tiled on-device format (see weight_formats.cuh)."""
    wf: int
    data: torch.Tensor   # uint8, tiled bytes
    N: int
    K: int
    interleaved_swiglu: bool = False   # rows alternate gate/up (fused SwiGLU epilogue)

    @property
    def chunks(self) -> int:
        return (self.K + _CHUNK[self.wf] - 1) // _CHUNK[self.wf]

    @property
    def nbytes(self) -> int:
        return self.data.numel()


def tile_weight(raw: torch.Tensor, gtype: int, N: int, K: int, wf: int | None = None) -> TiledWeight:
    """Repack GGUF rows (uint8 bytes, or an F32/F16/BF16 tensor) already on the GPU into tiles."""
    if wf is None:
        wf = wf_for_gtype(gtype)
        if wf is None:
            raise ValueError(f"no tiled GPU format for GGUF type {GType(gtype).name}; dequantise first")
    out = torch.empty(tiled_bytes(wf, N, K), dtype=torch.uint8, device=raw.device)
    C().repack_weight(wf, int(gtype), raw.contiguous(), N, K, out)
    return TiledWeight(wf, out, N, K)


def pick_bn(M: int) -> int:
    for b in (16, 32, 64, 128):
        if M <= b:
            return b
    return 256


def pick_splits(w: TiledWeight, M: int, bn: int = 0, sms: int = NUM_SMS, max_splits: int = 8) -> int:
    """K splits for the persistent GEMM: minimise (weight bytes + partial-sum traffic) divided by the
    SM-balance efficiency of the resulting work units. Multi-token-tile problems are not split."""
    bn = bn or pick_bn(M)
    m_tiles = (M + bn - 1) // bn
    if m_tiles > 1 or w.chunks < 2:
        return 1
    base = (w.N + 127) // 128
    wbytes = w.nbytes

    def cost(s: int) -> float:
        units = base * s
        eff = units / (math.ceil(units / sms) * sms)
        partial = (s * M * w.N * 8) if s > 1 else M * w.N * 2
        return (wbytes + partial) / eff

    best = min(range(1, min(max_splits, w.chunks) + 1), key=lambda s: (cost(s), s))
    return effective_splits(w, best)


def effective_splits(w: TiledWeight, s: int) -> int:
    """The split count the kernel actually runs for `s` requested splits (each split covers
    ceil(chunks / s) chunks, so trailing splits can vanish). Consumers must sum exactly this many."""
    s = max(1, min(s, w.chunks))
    per = (w.chunks + s - 1) // s
    return (w.chunks + per - 1) // per


def gemm(x: torch.Tensor, w: TiledWeight, out: torch.Tensor, M: int, mode: int = OUT_BF16, splits: int = 1,
         bn: int = 0, err: torch.Tensor | None = None, split_stride: int = 0) -> torch.Tensor:
    """out[:M] (=|+=) x[:M] @ W^T. OUT_F32_ADD requires a zeroed fp32 output; OUT_F32_SPLIT writes
    one fp32 partial per K split, `split_stride` elements apart (consumers sum them)."""
    if err is None:
        err = _err_word(x.device)
    C().gemm(w.wf, w.data, w.N, w.K, x, M, out, mode, splits, bn, err, split_stride)
    _count()
    return out


def gemm_grouped(x: torch.Tensor, w: TiledWeight, groups: int, group_stride: int, rows_total: int,
                 counts: torch.Tensor, offsets: torch.Tensor, max_rows: int, out: torch.Tensor,
                 mode: int = OUT_BF16, bn: int = 0, err: torch.Tensor | None = None) -> torch.Tensor:
    """Per-group GEMM in one launch (MoE experts): rows [offsets[g], offsets[g] + counts[g]) of x
    times expert g's weight (``group_stride`` bytes after expert g-1 in ``w.data``; ``w`` describes
    one expert). Counts and offsets stay on the device."""
    if err is None:
        err = _err_word(x.device)
    C().gemm_grouped(w.wf, w.data, group_stride, w.N, w.K, x, rows_total, out, mode, groups, counts, offsets,
                     max_rows, bn, err)
    _count()
    return out


def moe_route(logits, T, E, k, norm_topk, e0, e_local, topk_id, topk_w, counts, offsets, sorted_src, slot_row,
              total_rows):
    C().moe_route(logits, T, E, k, norm_topk, e0, e_local, topk_id, topk_w, counts, offsets, sorted_src, slot_row,
                  total_rows)
    _count()


def moe_combine(y, slot_row, topk_w, T, k, H, out):
    C().moe_combine(y, slot_row, topk_w, T, k, H, out)
    _count()


_ERR: dict = {}


def _err_word(device) -> torch.Tensor:
    key = str(device)
    if key not in _ERR:
        _ERR[key] = torch.zeros(4, dtype=torch.int32, device=device)
    return _ERR[key]


def device_error(device="cuda") -> int:
    """Error code recorded by a kernel whose bounded wait expired (0 = none)."""
    return int(_err_word(torch.device(device)).max().item())


def quantize_blocks(gtype: int, x: torch.Tensor) -> torch.Tensor:
    """fp32 tensor [..., K] -> GGUF block bytes (uint8) on the device."""
    x = x.contiguous().float()
    K = x.shape[-1]
    rows = x.numel() // K
    from ..gguf.constants import row_bytes
    out = torch.empty(rows * row_bytes(gtype, K), dtype=torch.uint8, device=x.device)
    C().quantize_blocks(int(gtype), x, out)
    return out.view(rows, -1)


def untile_bf16(w: TiledWeight) -> torch.Tensor:
    out = torch.empty(w.N, w.K, dtype=torch.bfloat16, device=w.data.device)
    C().untile_bf16(w.data, w.N, w.K, out)
    return out


def embed(ids, T, table, gtype, row_bytes, H, resid=None, out_bf16=None):
    C().embed(ids, T, table, int(gtype), row_bytes, H, resid, out_bf16)
    _count()


def add_rmsnorm(resid, w, T, H, eps, out=None, delta=None, ndelta=1, delta_stride=0):
    C().add_rmsnorm(resid, delta, ndelta, delta_stride, w, T, H, eps, out)
    _count()


def rope_store(qkv, T, Hq, Hkv, D, pos, slots, cos_sin, neox, q_out, kv, nsplit=1, split_stride=0):
    C().rope_store(qkv, nsplit, split_stride, T, Hq, Hkv, D, pos, slots, cos_sin, neox, q_out, kv)
    _count()


def gdn_conv(x, w, q_start, slot, has_state, nseq, conv_state, y):
    """Causal depthwise conv + SiLU of the gated delta-net mixed q|k|v channels (gdn.cu)."""
    C().gdn_conv(x, w, q_start, slot, has_state, nseq, conv_state, y)
    _count()


def gdn_recurrent(qkv, alpha, beta, z, a_neg, dt_bias, norm_w, state, slot, has_state, q_start, nseq, Hk, eps, out):
    """Gated delta-rule recurrence over each sequence's tokens + gated RMSNorm (gdn.cu)."""
    C().gdn_recurrent(qkv, alpha, beta, z, a_neg, dt_bias, norm_w, state, slot, has_state, q_start, nseq, Hk, eps, out)
    _count()


class TqTables:
    """TurboQuant layout of one model (csrc/host/turboquant.hpp) and its Lloyd-Max tables on the
    device. ``layer`` selects the random rotation of a layer (set per call through ``for_layer``)."""

    def __init__(self, method: str, head_dim: int, device, rot_seed: int = 0):
        from .. import _native
        h = _native.host()
        self.method = method
        self.layout = dict(h.tq_layout(method, head_dim))
        self.head_dim = head_dim
        self.rot_seed = int(rot_seed) & 0xFFFFFFFF
        L = self.layout
        if L["key_fp8"]:
            cent = [0.0]
        else:
            cent = list(h.lloyd_max_gaussian(L["key_bits"], 1.0 / math.sqrt(head_dim)))
        mids = [(a + b) / 2 for a, b in zip(cent[:-1], cent[1:])] or [0.0]
        self.centroids = torch.tensor(cent, dtype=torch.float32, device=device)
        self.midpoints = torch.tensor(mids, dtype=torch.float32, device=device)
        self.layer = 0

    @property
    def slot_bytes(self) -> int:
        return self.layout["slot_aligned"]

    def meta(self) -> list[int]:
        L = self.layout
        return [L["slot_aligned"], L["mse_bytes"], L["key_packed"], L["val_bytes"], L["key_bits"], L["value_bits"],
                int(L["norm_correction"]), int(L["key_fp8"]), self.rot_seed, self.layer]


def rope_store_tq(qkv, T, Hq, Hkv, D, pos, slots, cos_sin, neox, q_out, cache, tab: TqTables, layer: int,
                  nsplit=1, split_stride=0):
    """RoPE + rotation of Q (written to q_out) and TurboQuant quantisation of K / V into ``cache``
    (one layer: uint8 [num_blocks, 16, Hkv, slot])."""
    tab.layer = layer
    C().rope_store_tq(qkv, nsplit, split_stride, T, Hq, Hkv, D, pos, slots, cos_sin, neox, q_out, cache, tab.meta(),
                      tab.centroids, tab.midpoints)
    _count()


def swiglu(gu, T, F, out, interleaved=False, nsplit=1, split_stride=0):
    C().swiglu(gu, nsplit, split_stride, T, F, interleaved, out)
    _count()


def gather_rows(src, idx, n, H, dst):
    C().gather_rows(src, idx, n, H, dst)
    _count()


def paged_attention(q, kv, q_start, ctx_len, block_tables, num_reqs, req_offset, max_qlen, total_tokens, Hq, Hkv,
                    D, scale, decode, out, splits=1, part_o=None, part_lse=None, tq=None, tree_mask=None,
                    tree_span=0):
    """Paged attention over bf16 pages ``kv``, or over a TurboQuant cache layer when ``tq`` is a
    (cache layer, TqTables) pair (``kv`` is then ignored). ``tree_mask`` (int64 [T], prefill path):
    bit i of a token's mask lets it attend to the key at position ctx - tree_span + i of its
    request (token trees; keys before that are context, visible to all); null = causal."""
    if tq is None:
        C().paged_attention(q, kv, q_start, ctx_len, block_tables, num_reqs, req_offset, max_qlen, total_tokens, Hq,
                            Hkv, D, scale, decode, splits, part_o, part_lse, out, tree_mask=tree_mask,
                            tree_span=tree_span, err=_err_word(q.device))
    else:
        cache, tab = tq
        C().paged_attention(q, cache, q_start, ctx_len, block_tables, num_reqs, req_offset, max_qlen, total_tokens,
                            Hq, Hkv, D, scale, decode, splits, part_o, part_lse, out, cache, tab.meta(),
                            tab.centroids, tab.midpoints, tree_mask, tree_span, _err_word(q.device))
    _count(2 if (decode and splits > 1) else 1)


def kv_move(cache, Hkv, D, src, dst, cnt, num_reqs, max_moves):
    """Move KV rows (all layers, K and V) of a bf16 paged cache [L, blocks, 2, Hkv, 16, D]: request r
    moves cnt[r] slots src[r, i] -> dst[r, i]; all reads happen before the writes."""
    C().kv_move(cache, Hkv, D, src, dst, cnt, num_reqs, max_moves)
    _count()


# Sampling parameters: one 40-byte record per row (csrc/kernels/sampling.h SampleParams).
SAMPLE_PARAMS_DTYPE = [("temperature", "<f4"), ("top_k", "<i4"), ("top_p", "<f4"), ("min_p", "<f4"),
                       ("repetition_penalty", "<f4"), ("frequency_penalty", "<f4"), ("presence_penalty", "<f4"),
                       ("step", "<i4"), ("seed", "<u8")]


def decode_splits(ctas: int, slots: int, max_splits: int = 16) -> int:
    """Split-KV factor for decode attention with `ctas` (request, KV head) pairs on a GPU with
    `slots` resident CTA slots. Splitting only pays when the pairs alone leave SMs idle: measured on
    the 8B shapes, filling the last wave of a >1-wave grid with splits gains nothing, and at one
    rank of tensor parallel 8 (64 requests x 1 KV head, ~1040 tokens of context) one CTA per SM was
    fastest: 2 splits 20.5 us, 5 splits 26.6 us, 16 splits 32.8 us."""
    sms = slots // max(1, slots // 148) if slots >= 148 else slots
    ctas = max(1, ctas)
    if ctas >= sms:
        return 1
    return max(1, min(max_splits, sms // ctas))


def decode_slots(D: int) -> int:
    """Resident decode-attention CTAs on the whole GPU for head dim D."""
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return sms * max(1, C().attn_decode_ctas_per_sm(D))


def sample(logits, S, V, params, out_tok, out_lp=None):
    C().sample(logits, S, V, params, out_tok, out_lp)
    _count()


def apply_penalties(logits, row_of, tok, out_count, params, n):
    C().apply_penalties(logits, row_of, tok, out_count, params, n)
    _count()
