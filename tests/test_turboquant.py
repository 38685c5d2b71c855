"""TurboQuant host side: slot layouts of the four variants and the Lloyd-Max quantiser tables."""
import math

import numpy as np
import pytest
from scipy import integrate, stats


@pytest.mark.parametrize("method,D,expect", [
    ("turboquant_4bit_nc", 128, dict(mse_bytes=64, key_packed=66, val_bytes=64, value_packed=68, slot=134, slot_aligned=134)),
    ("turboquant_k8v4", 128, dict(mse_bytes=128, key_packed=128, val_bytes=64, value_packed=68, slot=196, slot_aligned=196)),
    ("turboquant_k3v4_nc", 128, dict(mse_bytes=48, key_packed=50, val_bytes=64, value_packed=68, slot=118, slot_aligned=118)),
    ("turboquant_3bit_nc", 128, dict(mse_bytes=48, key_packed=50, val_bytes=48, value_packed=52, slot=102, slot_aligned=102)),
    ("turboquant_3bit_nc", 64, dict(mse_bytes=24, key_packed=26, val_bytes=24, value_packed=28, slot=54, slot_aligned=54)),
])
def test_layouts(host, method, D, expect):
    lay = dict(host.tq_layout(method, D))
    for k, v in expect.items():
        assert lay[k] == v, (k, lay[k], v)
    assert lay["slot_aligned"] % 2 == 0


def test_unknown_method_rejected(host):
    with pytest.raises(Exception):
        host.tq_layout("turboquant_9bit", 128)
    assert not host.is_turboquant_method("fp8_e4m3")


def _lloyd_max_scipy(bits, sigma):
    n = 1 << bits
    c = np.linspace(-2.5 * sigma, 2.5 * sigma, n)
    pdf = stats.norm(0, sigma).pdf
    for _ in range(400):
        b = np.concatenate([[-np.inf], (c[:-1] + c[1:]) / 2, [np.inf]])
        c = np.array([integrate.quad(lambda x: x * pdf(x), b[i], b[i + 1])[0] /
                      integrate.quad(pdf, b[i], b[i + 1])[0] for i in range(n)])
    return c


@pytest.mark.parametrize("bits", [3, 4])
def test_lloyd_max_matches_numerical_fixed_point(host, bits):
    D = 128
    sigma = 1 / math.sqrt(D)
    got = np.array(host.lloyd_max_gaussian(bits, sigma))
    ref = _lloyd_max_scipy(bits, sigma)
    assert np.all(np.diff(got) > 0)
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(got, -got[::-1], atol=1e-12)  # symmetric


def test_lloyd_max_known_values(host):
    # Unit-variance 1-bit and 2-bit optimum (Max, 1960): +-0.7979 and +-0.4528, +-1.5104.
    np.testing.assert_allclose(host.lloyd_max_gaussian(1, 1.0), [-0.7978846, 0.7978846], atol=1e-6)
    np.testing.assert_allclose(host.lloyd_max_gaussian(2, 1.0), [-1.5104, -0.4528, 0.4528, 1.5104], atol=1e-4)
