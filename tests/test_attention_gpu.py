"""GPU parity of the decode attention op (a17 support op) through the C-ABI.

The op evaluates the canonical chunked softmax (64-slot chunks, dot_f16kv
scores, deterministic exp), so the bar is bit-exactness against the oracle.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def case(rng, length, H, HD, stride_pad=0):
    D = H * HD + stride_pad
    q = rng.standard_normal(H * HD).astype(np.float32)
    kc = rng.standard_normal((length, D)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((length, D)).astype(np.float16).view(np.uint16)
    return q, kc, vc


@pytest.mark.parametrize("length,H,HD,pad", [(1, 16, 32, 0), (63, 16, 32, 0), (64, 16, 32, 0),
                                            (65, 4, 32, 0), (570, 16, 32, 0), (1000, 12, 64, 0),
                                            (333, 3, 64, 64), (4097, 2, 32, 8)])
def test_attention_decode_bit_exact(dev, ora, length, H, HD, pad):
    rng = np.random.default_rng(length * 31 + H + HD)
    q, kc, vc = case(rng, length, H, HD, pad)
    scale = np.float32(1.0) / np.sqrt(np.float32(HD))
    ref = ora.attention_decode(q, kc, vc, length, H, HD, float(scale))
    got = dev.attention_decode(torch.from_numpy(q).cuda(),
                               torch.from_numpy(kc.view(np.float16)).cuda(),
                               torch.from_numpy(vc.view(np.float16)).cuda(), length, H, HD,
                               float(scale))
    np.testing.assert_array_equal(got.cpu().numpy(), ref)
    # against a float64 softmax: the canonical order is a reassociation only
    kf = kc.view(np.float16).astype(np.float64)
    vf = vc.view(np.float16).astype(np.float64)
    for h in range(H):
        s = kf[:, h * HD:(h + 1) * HD] @ q[h * HD:(h + 1) * HD].astype(np.float64) * float(scale)
        p = np.exp(s - s.max())
        p /= p.sum()
        np.testing.assert_allclose(ref[h * HD:(h + 1) * HD], p @ vf[:, h * HD:(h + 1) * HD],
                                   atol=1e-5, rtol=1e-4)


def test_attention_decode_rejects_bad_args(dev):
    q = torch.zeros(16 * 32, device="cuda")
    kc = torch.zeros(10, 512, dtype=torch.float16, device="cuda")
    ws = torch.zeros(1024, device="cuda")
    L = dev.lib()
    assert L.gsvk_attention_decode(q.data_ptr(), kc.data_ptr(), kc.data_ptr(), 10, 16, 48, 512,
                                   1.0, q.data_ptr(), ws.data_ptr(), None) == -5
    assert L.gsvk_attention_decode(q.data_ptr(), kc.data_ptr(), kc.data_ptr(), 0, 16, 32, 512,
                                   1.0, q.data_ptr(), ws.data_ptr(), None) == -1
    assert L.gsvk_attention_decode(q.data_ptr(), kc.data_ptr(), kc.data_ptr(), 10, 16, 32, 500,
                                   1.0, q.data_ptr(), ws.data_ptr(), None) == -1
