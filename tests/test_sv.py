"""The SV speaker encoder (ERes2NetV2 w24 s4 e4, sv.cpp:130-885): the
conv2d_f16 restatement against an independent numpy im2col, then the whole
device forward against the oracle.

The device runs each conv as an fp16 im2col and one tensor-core GEMM with
fp32 accumulation (the reference's conv2d_f16 arithmetic, in another
summation order) and BatchNorm in the same fp64 chain; the bar is max
|error| <= 1e-2 of the peak and cos >= 0.9999 on the embedding."""
import numpy as np
import pytest


def _rel_cos(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    return (float(np.abs(got - ref).max() / np.abs(ref).max()),
            float(got @ ref / np.sqrt((got @ got) * (ref @ ref))))


@pytest.fixture(scope="module")
def model(gsv):
    return gsv.workloads.sv_model(seed=3)


@pytest.mark.parametrize("c_in,h,w,c_out,k,stride,pad", [
    (1, 9, 11, 8, 3, 1, 1), (5, 7, 6, 4, 1, 2, 0), (8, 10, 9, 6, 3, 2, 1), (3, 4, 5, 7, 1, 1, 0)])
def test_oracle_conv2d_f16_matches_numpy(ora, c_in, h, w, c_out, k, stride, pad):
    rng = np.random.default_rng(c_in * 100 + h)
    x = rng.standard_normal((c_in, h, w), dtype=np.float32)
    w16 = (rng.standard_normal((c_out, c_in, k, k), dtype=np.float32) * 0.3).astype(np.float16)
    got = ora.sv_conv2d_f16(x, w16.view(np.uint16), stride, pad)
    xp = np.pad(x.astype(np.float16).astype(np.float64), ((0, 0), (pad, pad), (pad, pad)))
    oh, ow = (h + 2 * pad - k) // stride + 1, (w + 2 * pad - k) // stride + 1
    ref = np.zeros((c_out, oh, ow))
    for oy in range(oh):
        for ox in range(ow):
            patch = xp[:, oy * stride:oy * stride + k, ox * stride:ox * stride + k]
            ref[:, oy, ox] = np.tensordot(w16.astype(np.float64), patch, axes=3)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


def test_oracle_forward_shape(gsv, ora, model):
    fb = gsv.workloads.sv_fbank(16, seed=1)
    e = ora.sv_forward(model, fb)
    assert e.shape == (2048 * 10,) and np.isfinite(e).all()
    m2 = dict(model)
    m2["tensors"] = {k: v for k, v in model["tensors"].items() if k != "layer2.1.bn3.running_var"}
    with pytest.raises(ValueError):
        ora.sv_forward(m2, fb)


@pytest.mark.gpu
@pytest.mark.parametrize("frames", [32, 45])
def test_sv_matches_oracle(dev, ora, model, frames):
    import torch

    fb = dev.workloads.sv_fbank(frames, seed=frames)
    ref = ora.sv_forward(model, fb)
    enc = dev.SvEncoder(model, max_frames=64)
    assert enc.embedding_size() == ref.size
    got = enc.forward(torch.from_numpy(fb).cuda()).cpu().numpy()
    enc.close()
    d, c = _rel_cos(got, ref)
    assert d <= 1e-2 and c >= 0.9999, f"max rel {d:.3e} cos {c:.8f}"
    assert dev.device_status() == 0


@pytest.mark.gpu
def test_sv_from_gsv_and_rejections(dev, model, tmp_path):
    import os
    import sys

    import torch

    sys.path.insert(0, os.path.dirname(__file__))
    import gsv_writer

    tensors = [(k, a.view(np.float16).astype(np.float32), a) if a.dtype == np.uint16 else (k, a, None)
               for k, a in model["tensors"].items()]
    path = str(tmp_path / "sv.gsv")
    gsv_writer.write(path, "sv", {"meta": {"source": "synthetic"}}, tensors, slim=True)
    f = dev.GsvFile(path)
    fb = torch.from_numpy(dev.workloads.sv_fbank(24, seed=2)).cuda()
    a = dev.SvEncoder(model, max_frames=24)
    b = dev.SvEncoder(None, max_frames=24, gsv=f)
    np.testing.assert_array_equal(a.forward(fb).cpu().numpy(), b.forward(fb).cpu().numpy())
    with pytest.raises(dev.GsvkError):
        a.forward(torch.zeros(25, 80, device="cuda"))
    a.close()
    b.close()
    f.close()
    m2 = dict(model)
    m2["tensors"] = {k: v for k, v in model["tensors"].items() if k != "fuse34.local_att.3.bias"}
    with pytest.raises(dev.GsvkError):
        dev.SvEncoder(m2, max_frames=8)
    assert dev.device_status() == 0
