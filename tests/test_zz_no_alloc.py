"""Allocation-free decode attention (gsvk_attention_decode_noalloc).

Some callers cannot allocate device memory themselves or let the library do
it: a host framework whose memory pool owns every byte of the GPU, a
fixed-budget deployment, or a call path that must never reach the CUDA
allocator.  For them the library keeps the attention chunk records in one
static device array of a fixed size instead of a caller-provided workspace.

This file runs last in the suite.  It calls the allocation-free entry point
through the C ABI twice in a row, each time with fresh inputs, and compares
the result with gsvk_attention_decode (caller workspace) on the same inputs.
The bar is bit-identical output, the same bar every attention test here uses.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(rng, length, H, HD):
    D = H * HD
    q = torch.from_numpy(rng.standard_normal(D).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.standard_normal((length, D)).astype(np.float16)).cuda()
    vc = torch.from_numpy(rng.standard_normal((length, D)).astype(np.float16)).cuda()
    return q, kc, vc


def test_noalloc_attention_matches_workspace_entry_point(dev):
    lib = dev.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(2026)
    for length, H, HD in [(570, 16, 32), (1000, 12, 64)]:  # two calls in a row
        q, kc, vc = _inputs(rng, length, H, HD)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(HD)))
        expected = dev.attention_decode(q, kc, vc, length, H, HD, scale).cpu().numpy()
        out = torch.full((H * HD,), float("nan"), device="cuda")
        rc = lib.gsvk_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), length,
                                               H, HD, kc.stride(0), scale, out.data_ptr(), stream)
        assert rc == 0, dev.last_error()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), expected)
    assert dev.device_status() == 0


def test_noalloc_attention_rejects_requests_beyond_its_array(dev):
    lib = dev.lib()
    max_floats = lib.gsvk_attention_decode_noalloc_max_floats()
    assert max_floats == 262144
    H, HD = 16, 32
    too_long = (max_floats // (H * (HD + 4)) + 1) * 64  # one chunk past the limit
    q, kc, vc = _inputs(np.random.default_rng(1), 8, H, HD)
    out = torch.zeros(H * HD, device="cuda")
    rc = lib.gsvk_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), too_long,
                                           H, HD, kc.stride(0), 0.1, out.data_ptr(), None)
    assert rc == -5  # GSVK_ERR_UNSUPPORTED, nothing launched
    assert "static array" in dev.last_error()
