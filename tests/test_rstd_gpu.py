"""The LayerNorm reciprocal square root of every T2S decode kernel.

kern.cpp:55 forms rstd = (float)(1.0 / std::sqrt((double)var + eps)): a
correctly rounded double sqrt, a correctly rounded double divide, then a
rounding to float.  numpy's float64 sqrt and divide are IEEE correctly
rounded, so `np.float32(1.0 / np.sqrt(v))` is that value exactly.  The device
routine takes a float candidate and proves it with exact midpoint tests,
falling back to the sqrt-then-divide path near a midpoint; it must agree bit
for bit everywhere, including on inputs built to sit next to a midpoint.
"""
import numpy as np
import pytest


def _device_rstd(dev, v):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(v, dtype=np.float64)).cuda()
    out = torch.empty(t.numel(), dtype=torch.float32, device="cuda")
    dev.check(dev.lib().gsvk_test_rstd(t.data_ptr(), out.data_ptr(), t.numel(),
                                       torch.cuda.current_stream().cuda_stream))
    return out.cpu().numpy()


def _reference(v):
    return (1.0 / np.sqrt(v)).astype(np.float32)


@pytest.mark.gpu
def test_rstd_random_variances(dev):
    rng = np.random.default_rng(0)
    # LayerNorm variances over many decades, plus eps-dominated ones
    var = np.concatenate([
        10.0 ** rng.uniform(-12, 12, 1 << 20),
        rng.uniform(0, 4, 1 << 20),
        np.zeros(16),
    ]).astype(np.float32).astype(np.float64)
    v = var + 1e-5
    got = _device_rstd(dev, v)
    ref = _reference(v)
    bad = np.flatnonzero(got.view(np.uint32) != ref.view(np.uint32))
    assert bad.size == 0, f"{bad.size} mismatches, first v={v[bad[0]]!r}: {got[bad[0]]} vs {ref[bad[0]]}"


@pytest.mark.gpu
def test_rstd_next_to_rounding_midpoints(dev):
    # v = 1 / m^2 for m the midpoint between adjacent floats: 1/sqrt(v) lies
    # within a few double ulps of m, where only the exact path can decide
    rng = np.random.default_rng(1)
    r = (10.0 ** rng.uniform(-6, 3, 1 << 18)).astype(np.float32)
    up = np.nextafter(r, np.float32(np.inf))
    m = 0.5 * (r.astype(np.float64) + up.astype(np.float64))
    v = 1.0 / (m * m)
    v = np.concatenate([v, np.nextafter(v, 0), np.nextafter(v, np.inf)])
    got = _device_rstd(dev, v)
    ref = _reference(v)
    bad = np.flatnonzero(got.view(np.uint32) != ref.view(np.uint32))
    assert bad.size == 0, f"{bad.size} mismatches, first v={v[bad[0]]!r}: {got[bad[0]]} vs {ref[bad[0]]}"
