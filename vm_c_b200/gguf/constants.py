"""GGUF format constants (type ids, value types, metadata keys, tensor names).

The numeric ids are fixed by the GGUF file format; see csrc/host/ggml_types.hpp for the block
geometry of each tensor type.
"""
from __future__ import annotations

from enum import IntEnum


class GType(IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    IQ4_NL = 20
    IQ4_XS = 23
    I8 = 24
    I16 = 25
    I32 = 26
    I64 = 27
    F64 = 28
    BF16 = 30


# (elements per block, bytes per block)
BLOCK = {
    GType.F32: (1, 4), GType.F16: (1, 2), GType.BF16: (1, 2), GType.F64: (1, 8),
    GType.I8: (1, 1), GType.I16: (1, 2), GType.I32: (1, 4), GType.I64: (1, 8),
    GType.Q4_0: (32, 18), GType.Q4_1: (32, 20), GType.Q5_0: (32, 22), GType.Q5_1: (32, 24),
    GType.Q8_0: (32, 34), GType.Q8_1: (32, 36), GType.Q2_K: (256, 84), GType.Q3_K: (256, 110),
    GType.Q4_K: (256, 144), GType.Q5_K: (256, 176), GType.Q6_K: (256, 210), GType.Q8_K: (256, 292),
    GType.IQ4_NL: (32, 18), GType.IQ4_XS: (256, 136),
}


def row_bytes(t: int, n: int) -> int:
    be, bb = BLOCK[GType(t)]
    if n % be:
        raise ValueError(f"row of {n} elements is not a multiple of the {GType(t).name} block ({be})")
    return n // be * bb


class VType(IntEnum):
    UINT8 = 0
    INT8 = 1
    UINT16 = 2
    INT16 = 3
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10
    INT64 = 11
    FLOAT64 = 12


# llama.cpp's file-type codes (general.file_type) for the mixes this engine writes.
FILE_TYPE = {"F32": 0, "F16": 1, "Q8_0": 7, "Q4_K_M": 15, "Q4_K_S": 14, "BF16": 32, "Q6_K": 18}

# Per-layer tensor names (llama / mixtral architectures).
T_TOKEN_EMBD = "token_embd.weight"
T_OUTPUT_NORM = "output_norm.weight"
T_OUTPUT = "output.weight"
T_ROPE_FREQS = "rope_freqs.weight"


def blk(i: int, name: str) -> str:
    return f"blk.{i}.{name}.weight"
