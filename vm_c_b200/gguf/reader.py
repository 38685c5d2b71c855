"""GGUF checkpoint access on top of the native memory-mapped reader (csrc/host/gguf.cpp)."""
from __future__ import annotations

import numpy as np

from .. import _native
from ..config import ModelConfig, model_config_from_gguf
from .constants import GType, row_bytes
from .random_init import TensorSpec


class GgufSource:
    """Tensor source backed by a GGUF file: rows come out as zero-copy CPU views of the mapping."""

    def __init__(self, path: str):
        self.path = path
        self.f = _native.host().GgufFile.open(path)
        self.tensors = {t["name"]: t for t in self.f.tensors()}

    def model_config(self) -> ModelConfig:
        return model_config_from_gguf(self.f)

    def metadata(self, key: str, default=None):
        if not self.f.has(key):
            return default
        v = self.f.get(key)
        return v.decode("utf-8", "replace") if isinstance(v, bytes) else v

    def has(self, name: str) -> bool:
        return name in self.tensors

    def info(self, name: str) -> TensorSpec:
        t = self.tensors[name]
        return TensorSpec(name, list(t["ne"]), int(t["type"]))

    def rows(self, name: str, r0: int = 0, r1: int | None = None):
        import torch
        t = self.tensors[name]
        K = t["ne"][0]
        nrows = 1
        for d in t["ne"][1:]:
            nrows *= d
        r1 = nrows if r1 is None else r1
        rb = row_bytes(t["type"], K)
        buf = self.f.tensor_bytes(name)  # read-only numpy view over the mapping
        arr = np.asarray(buf)[r0 * rb:r1 * rb].reshape(r1 - r0, rb)
        # torch cannot wrap read-only memory; copy the slice (one pass over the needed bytes).
        tt = torch.from_numpy(arr.copy())
        if t["type"] == GType.F32:
            return tt.view(torch.float32)
        return tt
