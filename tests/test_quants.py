"""CPU quant codecs: independent numpy restatements of the GGUF block formats vs the C++ codecs,
and a bit-exact numpy emulation of the GPU tiled formats + dequant tricks (csrc/kernels)."""
import numpy as np
import pytest

from vm_c_b200.gguf.constants import GType


def f16(b):
    return np.frombuffer(bytes(b), np.float16).astype(np.float32)


def np_deq_q8_0(raw):
    out = []
    for blk in raw.reshape(-1, 34):
        d = f16(blk[:2])[0]
        out.append(d * blk[2:].view(np.int8).astype(np.float32))
    return np.concatenate(out)


def k4(sc, j):
    if j < 4:
        return sc[j] & 63, sc[j + 4] & 63
    return (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4), (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)


def np_deq_q4_k(raw):
    out = []
    for b in raw.reshape(-1, 144):
        d, dmin = f16(b[0:2])[0], f16(b[2:4])[0]
        sc = b[4:16].astype(np.int32)
        qs = b[16:]
        y = np.zeros(256, np.float32)
        for j in range(8):
            s, m = k4(sc, j)
            q = (qs[32 * (j // 2):32 * (j // 2) + 32] >> (4 * (j % 2))) & 15
            y[32 * j:32 * j + 32] = d * s * q - dmin * m
        out.append(y)
    return np.concatenate(out)


def np_deq_q6_k(raw):
    out = []
    for b in raw.reshape(-1, 210):
        ql, qh, sc, d = b[:128].astype(np.int32), b[128:192].astype(np.int32), b[192:208].view(np.int8), f16(b[208:210])[0]
        y = np.zeros(256, np.float32)
        for e in range(256):
            h, r = divmod(e, 128)
            k, l = divmod(r, 32)
            lo = (ql[64 * h + l + 32 * (k & 1)] >> (4 * (k >> 1))) & 15
            hi = (qh[32 * h + l] >> (2 * k)) & 3
            y[e] = d * sc[e // 16] * ((lo | (hi << 4)) - 32)
        out.append(y)
    return np.concatenate(out)


@pytest.mark.parametrize("gt,fn,n", [(GType.Q8_0, np_deq_q8_0, 128), (GType.Q4_K, np_deq_q4_k, 512),
                                     (GType.Q6_K, np_deq_q6_k, 512)])
def test_dequant_matches_numpy_restatement(host, gt, fn, n):
    rng = np.random.default_rng(int(gt))
    x = (rng.standard_normal((1, n)) * 0.05).astype(np.float32)
    q = host.quantize(int(gt), x)
    ref = fn(q.reshape(-1))
    got = host.dequantize(int(gt), q, 1, n).reshape(-1)
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("gt,tol", [(GType.Q8_0, 0.01), (GType.Q4_K, 0.12), (GType.Q6_K, 0.03), (GType.Q4_0, 0.15),
                                    (GType.F16, 1e-3), (GType.BF16, 8e-3)])
def test_quantize_error_bounds(host, gt, tol):
    x = (np.random.default_rng(1).standard_normal((8, 1024)) * 0.02).astype(np.float32)
    y = host.dequantize(int(gt), host.quantize(int(gt), x), 8, 1024)
    rel = np.abs(y - x).max() / np.abs(x).max()
    assert rel < tol, rel


def test_other_formats_dequantize(host):
    # Q2_K/Q3_K/Q5_K/IQ4_XS blocks: decode random blocks without error and with finite values.
    rng = np.random.default_rng(0)
    for gt, bb in [(GType.Q2_K, 84), (GType.Q3_K, 110), (GType.Q5_K, 176), (GType.IQ4_XS, 136), (GType.Q5_0, 22),
                   (GType.Q5_1, 24), (GType.Q4_1, 20)]:
        raw = rng.integers(0, 255, (2, bb * (256 // host.type_traits(int(gt))[1]) if host.type_traits(int(gt))[1] == 32 else bb), dtype=np.uint8)
        # keep the fp16 scales small and finite
        n = 256 if host.type_traits(int(gt))[1] == 256 else 256
        raw = np.zeros((1, host.row_bytes(int(gt), n)), np.uint8) + rng.integers(0, 255, (1, host.row_bytes(int(gt), n)), dtype=np.uint8)
        y = host.dequantize(int(gt), raw, 1, n)
        assert y.shape == (1, n)


# ----------------------------------------------------------------------------------------------
# numpy emulation of the tiled GPU formats (weights.cu repack) and the bf16x2 dequant tricks
# (gemm_tcgen05.cu dq_*). bf16 arithmetic: exact op then round-to-nearest-even to bf16.

def bf16(x):
    x = np.asarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return r.astype(np.uint32).view(np.float32)


def bits_to_bf16(h):  # uint16 array -> float
    return (np.asarray(h, np.uint32) << 16).view(np.float32)


def halves(w):  # uint32 word -> (lo, hi) bf16 floats
    return bits_to_bf16(w & 0xFFFF), bits_to_bf16(w >> 16)


def emu_q4k_row(block144, s, h):
    b = np.asarray(block144, np.uint8)
    d, dmin = f16(b[0:2])[0], f16(b[2:4])[0]
    j = 2 * s + h
    sc, m = k4(b[4:16].astype(np.int32), j)
    ds = bf16(np.float32(d) * np.float32(sc))
    ndm = bf16(-np.float32(dmin) * np.float32(m))
    # repacked nibble bytes: 4-byte groups in order (0,2,1,3)
    qs = b[16:].copy()
    rep = qs.reshape(-1, 4)[:, [0, 2, 1, 3]].reshape(-1)
    words = rep[32 * s:32 * s + 32].view("<u4")
    out = []
    sh0, sh1 = (4, 12) if h else (0, 8)
    for w in words:
        for sh in (sh0, sh1):
            x = ((int(w) >> sh) & 0x000F000F) | 0x43004300
            lo, hi = halves(np.uint32(x))
            q = bf16(np.array([lo, hi]) - 128.0)
            out += list(bf16(q * ds + ndm))  # fma: one rounding
    return np.array(out, np.float32)


def test_q4k_gpu_dequant_emulation(host):
    x = (np.random.default_rng(5).standard_normal((1, 256)) * 0.05).astype(np.float32)
    q = host.quantize(int(GType.Q4_K), x)[0]
    ref = host.dequantize(int(GType.Q4_K), q[None], 1, 256)[0]
    got = np.concatenate([emu_q4k_row(q, s, h) for s in range(4) for h in range(2)])
    # bf16x2 arithmetic with bf16-rounded scale/min: error bounded relative to the block's range
    assert np.max(np.abs(got - ref)) < 2 ** -7 * np.abs(ref).max()


def test_q8_0_sign_trick():
    # (128 + low7) - {128, 256} reproduces every int8 value exactly in bf16
    for v in range(-128, 128):
        byte = v & 0xFF
        y = bits_to_bf16(0x4300 | (byte & 0x7F))
        z = bits_to_bf16(0x4300 | (byte & 0x80))
        assert float(bf16(y - z)) == v


def test_q6_offset_constant():
    assert float(bits_to_bf16(0x4320)) == 160.0 and float(bits_to_bf16(0x4300)) == 128.0
    assert float(bits_to_bf16(0x4380)) == 256.0
