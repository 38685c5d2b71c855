"""GGUF container round trip and metadata -> ModelConfig (native reader / writer)."""
import numpy as np
import pytest

from vm_c_b200.config import model_config_from_gguf
from vm_c_b200.gguf.constants import GType, VType, row_bytes
from vm_c_b200.gguf.random_init import preset, tensor_plan, write_random_gguf
from vm_c_b200.gguf.reader import GgufSource


def test_roundtrip_metadata_and_tensors(host, tmp_path):
    w = host.GgufWriter(32)
    w.set("general.architecture", int(VType.STRING), "llama")
    w.set("a.u32", int(VType.UINT32), 7)
    w.set("a.i64", int(VType.INT64), -5)
    w.set("a.f32", int(VType.FLOAT32), 1.5)
    w.set("a.b", int(VType.BOOL), True)
    w.set("a.arr_s", int(VType.ARRAY), ["x", "yz", ""], int(VType.STRING))
    w.set("a.arr_i", int(VType.ARRAY), [1, -2, 3], int(VType.INT32))
    w.set("a.arr_f", int(VType.ARRAY), [0.25, -1.0], int(VType.FLOAT32))
    t0 = np.arange(64, dtype=np.float32).reshape(2, 32)
    t1 = host.quantize(int(GType.Q8_0), np.random.default_rng(0).standard_normal((3, 64)).astype(np.float32))
    w.add_tensor("t0", [32, 2], int(GType.F32))
    w.add_tensor("t1", [64, 3], int(GType.Q8_0))
    p = tmp_path / "x.gguf"
    w.write(str(p), lambda i: [t0, t1][i])
    f = host.GgufFile.open(str(p))
    assert f.version == 3
    assert f.get("general.architecture") == b"llama"
    assert f.get("a.u32") == 7 and f.get("a.i64") == -5 and f.get("a.f32") == 1.5 and f.get("a.b") is True
    assert f.get("a.arr_s") == [b"x", b"yz", b""]
    assert f.get("a.arr_i") == [1, -2, 3] and f.get("a.arr_f") == [0.25, -1.0]
    ts = {t["name"]: t for t in f.tensors()}
    assert ts["t0"]["ne"] == [32, 2] and ts["t1"]["type"] == int(GType.Q8_0)
    assert ts["t1"]["offset"] % 32 == 0
    assert np.array_equal(np.frombuffer(f.tensor_bytes("t0"), np.float32).reshape(2, 32), t0)
    assert np.array_equal(np.asarray(f.tensor_bytes("t1")).reshape(3, -1), t1)


def test_truncated_file_rejected(host, tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUF\x03\x00\x00\x00" + b"\x01" * 5)
    with pytest.raises(RuntimeError):
        host.GgufFile.open(str(p))


def test_random_tiny_checkpoint(tmp_path):
    cfg = preset("tiny-llama")
    p = tmp_path / "tiny.gguf"
    write_random_gguf(str(p), cfg, "Q8_0", seed=0)
    src = GgufSource(str(p))
    m = src.model_config()
    assert (m.n_layers, m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn, m.vocab) == (4, 256, 8, 4, 32, 688, 32000)
    assert m.rms_eps == pytest.approx(1e-5) and m.rope_theta == pytest.approx(10000.0)
    # ffn_down rows of 688 elements are not Q8_0-aligned -> F16 (llama.cpp convention)
    assert src.info("blk.0.ffn_down.weight").gtype == GType.F16
    assert src.info("blk.0.attn_q.weight").gtype == GType.Q8_0
    assert src.rows("blk.1.attn_norm.weight").numpy().tolist()[0][:3] == [1.0, 1.0, 1.0]
    # deterministic in the seed
    p2 = tmp_path / "tiny2.gguf"
    write_random_gguf(str(p2), cfg, "Q8_0", seed=0)
    assert p.read_bytes() == p2.read_bytes()


def test_q4km_mix_plan():
    cfg = preset("llama3-8b")
    plan = {s.name: s.gtype for s in tensor_plan(cfg, "Q4_K_M")}
    assert plan["output.weight"] == GType.Q6_K
    assert plan["blk.0.attn_v.weight"] == GType.Q6_K and plan["blk.0.ffn_down.weight"] == GType.Q6_K
    assert plan["blk.4.attn_v.weight"] == GType.Q4_K and plan["blk.6.ffn_down.weight"] == GType.Q6_K
    assert plan["blk.10.attn_q.weight"] == GType.Q4_K and plan["token_embd.weight"] == GType.Q4_K
    total = sum(s.nbytes for s in tensor_plan(cfg, "Q4_K_M"))
    assert 4.5e9 < total < 5.2e9   # ~4.9 GB like a llama.cpp Llama-3-8B Q4_K_M


def test_row_bytes():
    assert row_bytes(GType.Q4_K, 4096) == 16 * 144
    assert row_bytes(GType.Q8_0, 64) == 68
    with pytest.raises(ValueError):
        row_bytes(GType.Q4_K, 100)


def _raw_gguf(path, ne, gtype=0, offset=0, data=b"\0" * 64):
    """A GGUF v3 file with one tensor and no metadata, written byte by byte (dimensions and offset
    as given, not as a writer would compute them)."""
    import struct
    name = b"t"
    hdr = b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + struct.pack("<Q", len(name)) + name
    hdr += struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", n) for n in ne)
    hdr += struct.pack("<IQ", gtype, offset)
    hdr += b"\0" * ((32 - len(hdr) % 32) % 32)
    open(path, "wb").write(hdr + data)


def test_reader_rejects_corrupt_tensor_infos(host, tmp_path):
    """Dimensions, sizes and offsets that would wrap 64-bit arithmetic are refused at open, so no
    tensor view can point outside the mapped file."""
    ok = str(tmp_path / "ok.gguf")
    _raw_gguf(ok, [4, 4])
    assert host.GgufFile.open(ok) is not None
    for i, (ne, off) in enumerate([([4, 2 ** 63], 0),            # negative as int64
                                   ([2 ** 33, 2 ** 33], 0),      # 64-bit size overflow
                                   ([4, 4], 2 ** 64 - 16),       # offset wraps the end check
                                   ([4, 5], 0),                  # past the end of the file
                                   ([2 ** 41], 0)]):             # implausible dimension
        p = str(tmp_path / f"bad{i}.gguf")
        _raw_gguf(p, ne, offset=off)
        with pytest.raises(RuntimeError):
            host.GgufFile.open(p)
