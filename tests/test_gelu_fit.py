"""The GELU the CUDA epilogues evaluate (csrc/common.cuh gelu_erf): its
coefficients, read from the source, evaluated here in emulated fp32 against
the exact x Phi(x), and re-derived from the fit the source describes.
No GPU: the device result is checked against the oracle in test_gemv_gpu."""
import os
import re

import numpy as np
from scipy.special import log_ndtr, ndtr

SRC = os.path.join(os.path.dirname(__file__), "..", "gpt-sovits-native_b200", "csrc", "common.cuh")
L2E = 1.0 / np.log(2.0)


def _source():
    text = open(SRC).read()
    body = text[text.index("float gelu_erf(float x)"):]
    body = body[:body.index("\n}\n")]
    coef = [float(v) for v in re.findall(r"([-+]?\d\.\d+e[-+]\d+)f", body)]
    clamp = float(re.search(r"fminf\(fabsf\(x\), ([\d.]+)f\)", body).group(1))
    scale = float(re.search(r"fmaf\((-0\.\d+)f, x \* x, h\)", body).group(1))
    return coef, clamp, scale


def _fma32(a, b, c):
    return (a.astype(np.float64) * b + c).astype(np.float32)


def gelu_fp32(x):
    """The device expression step by step in fp32 (fma as one rounding)."""
    coef, clamp, scale = _source()
    x = np.asarray(x, np.float32)
    u = np.minimum(np.abs(x), np.float32(clamp))
    h = np.full_like(x, coef[0])
    for c in coef[1:]:
        h = _fma32(h, u, np.float32(c))
    q = np.exp2(_fma32(np.full_like(x, scale), (x * x).astype(np.float32), h).astype(np.float64))
    q = q.astype(np.float32)
    return (x * np.where(x >= 0, (np.float32(1) - q).astype(np.float32), q)).astype(np.float32)


def test_source_constants():
    coef, clamp, scale = _source()
    assert len(coef) == 11 and clamp == 5.5
    assert abs(scale + L2E / 2) < 1e-9
    assert abs(coef[-1] + 1.0) < 1e-6  # h(0) = log2 Phi(0) = -1


def test_gelu_fit_accuracy():
    x = np.linspace(-9, 9, 400_001).astype(np.float32)
    ref = x.astype(np.float64) * ndtr(x.astype(np.float64))
    got = gelu_fp32(x).astype(np.float64)
    err = np.abs(got - ref)
    assert err.max() <= 5e-7
    big = np.abs(ref) > 1e-6
    assert (err[big] / np.abs(ref[big])).max() <= 5e-6
    # tails and specials
    assert gelu_fp32(np.float32(40))[()] == np.float32(40)
    assert gelu_fp32(np.float32(-40))[()] == 0
    assert np.isnan(gelu_fp32(np.float32(np.nan))[()])


def test_coefficients_reproduce_the_stated_fit():
    coef, clamp, _ = _source()
    n = 6000
    k = np.arange(n)
    u = (clamp / 2) * (1 - np.cos(np.pi * (k + 0.5) / n))
    h = log_ndtr(-u) * L2E + u * u * L2E / 2
    fit = np.polynomial.polynomial.polyfit(u, h, 10)[::-1]
    np.testing.assert_allclose(np.float32(fit), np.float32(coef), rtol=1e-6, atol=1e-12)
