"""Reader and writer of the safetensors container (HuggingFace checkpoints).

Counterpart of the reference's ``SafeTensorsLoader`` (src/model/model_loader.cpp:78-296). The
format is fixed by its public specification: an 8-byte little-endian header length N, N bytes of
JSON (``{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}``; the
offsets are relative to the first byte after the header), then the tensor bytes, row-major. The
reader is the native host library's (csrc/host/safetensors.cpp: memory map, header parse, byte
range checks); tensors come out as zero-copy read-only views of the mapping, so a row slice costs
one copy of the bytes it covers. The writer (tests, conversions) is plain Python.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass

import numpy as np

# safetensors dtype -> (numpy dtype used to view the bytes, bytes per element)
DTYPES = {"F64": (np.float64, 8), "F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2),
          "I64": (np.int64, 8), "I32": (np.int32, 4), "I16": (np.int16, 2), "I8": (np.int8, 1),
          "U8": (np.uint8, 1), "BOOL": (np.bool_, 1), "F8_E4M3": (np.uint8, 1), "F8_E5M2": (np.uint8, 1)}


@dataclass
class StEntry:
    name: str
    dtype: str
    shape: list[int]
    begin: int   # absolute file offset of the first byte
    end: int

    @property
    def itemsize(self) -> int:
        return DTYPES[self.dtype][1]


class SafetensorsFile:
    def __init__(self, path: str):
        from .. import _native
        try:
            self.f = _native.host().SafetensorsFile.open(path)
        except RuntimeError as e:
            raise ValueError(str(e)) from e
        self.path = path
        self.metadata = dict(self.f.metadata())
        self.entries: dict[str, StEntry] = {}
        for t in self.f.tensors():
            if t["dtype"] not in DTYPES:
                raise ValueError(f"{path}: tensor {t['name']} has unsupported dtype {t['dtype']}")
            self.entries[t["name"]] = StEntry(t["name"], t["dtype"], list(t["shape"]), int(t["begin"]), int(t["end"]))

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the mapping."""
        return self.f.tensor_bytes(name)

    def rows_bytes(self, name: str, r0: int, r1: int) -> np.ndarray:
        """Rows [r0, r1) of the tensor viewed as [prod(shape[:-1]), shape[-1]] (bytes, a view)."""
        e = self.entries[name]
        rb = (e.shape[-1] if e.shape else 1) * e.itemsize
        return self.raw(name)[r0 * rb:r1 * rb].reshape(r1 - r0, rb)


def save_file(tensors: dict, path: str, metadata: dict | None = None) -> None:
    """Write torch tensors (any of the dtypes above) as one safetensors file."""
    import torch
    names = sorted(tensors)
    rev = {torch.float64: "F64", torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16",
           torch.int64: "I64", torch.int32: "I32", torch.int16: "I16", torch.int8: "I8", torch.uint8: "U8",
           torch.bool: "BOOL"}
    header, blobs, off = {}, [], 0
    for n in names:
        t = tensors[n].detach().contiguous().cpu()
        if t.dtype not in rev:
            raise ValueError(f"save_file: dtype {t.dtype} of {n} is not supported")
        b = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[n] = {"dtype": rev[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * (-len(h) % 8)  # the data section starts 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
