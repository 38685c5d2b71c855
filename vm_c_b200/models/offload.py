"""CPU weight offload (``--cpu-offload-gb``, ``--cpu-offload-params``).

Counterpart of the reference's UVA offload (src/model/model_loader.cpp:706-760: tensors whose
dotted name contains a ``--cpu-offload-params`` segment move to pinned host memory while the
``--cpu-offload-gb`` budget lasts; src/model/weight_layout_plan.cpp:268-281 for the matching).
Selection is the same rule over GGUF tensor names (``blk.3.attn_q.weight`` matches ``attn_q``,
``blk`` or ``weight``; no segments = every layer weight, in layer order), and a tensor that does
not fit the remaining budget stays on the GPU.

The GEMMs stream their weight tiles into shared memory with bulk copies from device memory, so an
offloaded layer's tiles are copied from pinned host memory into one device staging buffer right
before the layer runs (a stream-ordered copy, captured in the decode CUDA graphs like any kernel).
The staging buffer is as large as the largest offloaded layer; every other offloaded byte stays
on the host. Offload trades speed (host-link bandwidth per step) for device memory.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..gguf.constants import blk
from ..utils.logging import get_logger

log = get_logger("offload")

_ALIGN = 256
# layer attribute -> GGUF tensor names (per layer) that it is built from
_PARTS = (("wqkv", ("attn_q", "attn_k", "attn_v")), ("wo", ("attn_output",)),
          ("w_gate_up", ("ffn_gate", "ffn_up")), ("w_down", ("ffn_down",)))


def matches(name: str, segments: list[str]) -> bool:
    """The reference's rule: '.' + segment + '.' occurs in '.' + name + '.'."""
    if not segments:
        return True
    full = f".{name}."
    return any(f".{s}." in full for s in segments)


@dataclass
class OffloadPlan:
    staging: torch.Tensor | None
    bytes_offloaded: int
    tensors: int


def apply_offload(weights, budget_gb: float, segments: list[str], device) -> OffloadPlan:
    """Move the selected layer weights to pinned host memory and point them at a device staging
    buffer; layers get an ``offload`` list of (host tensor, device view) copies to run first."""
    budget = int(budget_gb * (1 << 30))
    if budget <= 0:
        return OffloadPlan(None, 0, 0)
    used = 0
    chosen = []  # (layer, [TiledWeight])
    for lw in weights.layers:
        tws = []
        for attr, parts in _PARTS:
            obj = getattr(lw, attr, None)
            if obj is None:
                continue
            names = [blk(lw.index, p) for p in parts]
            if not any(matches(n, segments) for n in names):
                continue
            for tw in (obj if isinstance(obj, list) else [obj]):
                if used + tw.nbytes > budget:
                    continue
                used += tw.nbytes
                tws.append(tw)
        if tws:
            chosen.append((lw, tws))
    if not chosen:
        return OffloadPlan(None, 0, 0)
    per_layer = [sum((tw.nbytes + _ALIGN - 1) // _ALIGN * _ALIGN for tw in tws) for _, tws in chosen]
    staging = torch.empty(max(per_layer), dtype=torch.uint8, device=device)
    n = 0
    for lw, tws in chosen:
        off = 0
        for tw in tws:
            host = tw.data.cpu().pin_memory()
            view = staging[off:off + tw.nbytes]
            tw.data = view
            lw.offload.append((host, view))
            off += (tw.nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
            n += 1
    torch.cuda.empty_cache()
    log.info("CPU offload: %d weight tensors, %.3f GB on the host, %.3f GB device staging buffer", n, used / 1e9,
             staging.numel() / 1e9)
    return OffloadPlan(staging, used, n)
