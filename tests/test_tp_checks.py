"""Tensor-parallel shape checks done at load time (models/llama.py check_tp), on CPU."""
import pytest

from vm_c_b200.gguf.random_init import preset
from vm_c_b200.models.llama import check_tp


def test_check_tp_accepts_the_8b_shape_at_every_size():
    cfg = preset("llama3-8b")
    for tp in (1, 2, 4, 8):
        check_tp(cfg, tp)


def test_check_tp_rejects_unaligned_ffn_slices():
    cfg = preset("tiny-llama")   # ffn 688: 86 columns per rank at tp 8
    check_tp(cfg, 2)             # 344 columns: 688 bytes, 16-byte aligned
    with pytest.raises(ValueError, match="not a multiple of 8"):
        check_tp(cfg, 8)
    cfg.ffn = 768
    check_tp(cfg, 8)


def test_check_tp_rejects_indivisible_heads():
    cfg = preset("tiny-llama")   # 8 query heads, 4 KV heads
    with pytest.raises(ValueError):
        check_tp(cfg, 3)
