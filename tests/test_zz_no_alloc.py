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
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_FLOATS = 262144
H32 = 16
CHUNKS_THAT_FIT = MAX_FLOATS // (H32 * (32 + 4))  # 455 chunks of 64 keys at 16 heads x 32


def _inputs(rng, length, H, HD):
    D = H * HD
    q = torch.from_numpy(rng.standard_normal(D).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.standard_normal((length, D)).astype(np.float16)).cuda()
    vc = torch.from_numpy(rng.standard_normal((length, D)).astype(np.float16)).cuda()
    return q, kc, vc


def _noalloc(dev, q, kc, vc, length, H, HD, scale):
    lib = dev.lib()
    stream = torch.cuda.current_stream().cuda_stream
    out = torch.full((H * HD,), float("nan"), device="cuda")
    rc = lib.gsvk_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), length,
                                           H, HD, kc.stride(0), scale, out.data_ptr(), stream)
    assert rc == 0, dev.last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_noalloc_attention_matches_workspace_entry_point(dev):
    rng = np.random.default_rng(2026)
    for length, H, HD in [(570, 16, 32), (1000, 12, 64)]:  # two calls in a row
        q, kc, vc = _inputs(rng, length, H, HD)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(HD)))
        expected = dev.attention_decode(q, kc, vc, length, H, HD, scale).cpu().numpy()
        np.testing.assert_array_equal(_noalloc(dev, q, kc, vc, length, H, HD, scale), expected)
    assert dev.device_status() == 0


def test_noalloc_attention_fills_its_array_exactly(dev):
    """The largest accepted request: 455 chunks x 16 heads x 36 floats =
    262,080 of the 262,144 floats, so the last chunk records sit at the end
    of the array."""
    length = CHUNKS_THAT_FIT * 64
    assert dev.lib().gsvk_attention_workspace_floats(length, H32, 32) <= MAX_FLOATS
    q, kc, vc = _inputs(np.random.default_rng(7), length, H32, 32)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(32)))
    expected = dev.attention_decode(q, kc, vc, length, H32, 32, scale).cpu().numpy()
    np.testing.assert_array_equal(_noalloc(dev, q, kc, vc, length, H32, 32, scale), expected)
    assert dev.device_status() == 0


def test_noalloc_attention_rejects_requests_beyond_its_array(dev):
    lib = dev.lib()
    assert lib.gsvk_attention_decode_noalloc_max_floats() == MAX_FLOATS
    too_long = (CHUNKS_THAT_FIT + 1) * 64  # one chunk past the limit
    # K/V really hold too_long rows, so a broken size check would compute on
    # valid memory and fail the return-code assert instead of reading past them
    q, kc, vc = _inputs(np.random.default_rng(1), too_long, H32, 32)
    out = torch.zeros(H32 * 32, device="cuda")
    rc = lib.gsvk_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), too_long,
                                           H32, 32, kc.stride(0), 0.1, out.data_ptr(), None)
    assert rc == -5  # GSVK_ERR_UNSUPPORTED, nothing launched
    assert "static array" in dev.last_error()
    # absurd head counts are refused by the size check, not wrapped past it
    rc = lib.gsvk_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), 64,
                                           2**62, 32, kc.stride(0), 0.1, out.data_ptr(), None)
    assert rc == -5
