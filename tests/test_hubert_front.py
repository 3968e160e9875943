"""The HuBERT feature front-end (hubert.cpp:439-580): strided CNN with
GroupNorm and GELU, feature projection, grouped positional conv, encoder
LayerNorm.  The device rounds activations to fp16 for every convolution and
GEMM as the reference's im2col + FMLAL path does and accumulates in fp32 on
the tensor cores, so the bar is the GEMM tolerance on the output: max
relative error 1e-2 of the peak, cos >= 0.9999."""
import numpy as np
import pytest
import torch


def _rel_cos(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    return (float(np.abs(got - ref).max() / np.abs(ref).max()),
            float(got @ ref / np.sqrt((got @ got) * (ref @ ref))))


def test_oracle_frame_count_and_shape(gsv, ora):
    m = gsv.workloads.hubert_front_model(seed=1)
    wav = gsv.workloads.hubert_waveform(4000, seed=1)
    out = ora.hubert_front(m, wav)
    assert out.shape == (12, 768)  # 4000 samples -> 799, 399, 199, 99, 49, 24, 12 frames
    assert np.isfinite(out).all()


@pytest.mark.gpu
@pytest.mark.parametrize("n", [16000, 12345])
def test_hubert_front_matches_oracle(dev, ora, n):
    m = dev.workloads.hubert_front_model(seed=3)
    wav = dev.workloads.hubert_waveform(n, seed=n)
    ref = ora.hubert_front(m, wav)
    fe = dev.HubertFront(m, max_samples=16000)
    assert fe.frames(n) == ref.shape[0]
    got = fe.forward(torch.from_numpy(wav).cuda()).cpu().numpy()
    fe.close()
    d, c = _rel_cos(got, ref)
    assert d <= 1e-2 and c >= 0.9999, f"max rel {d:.3e} cos {c:.8f}"
    assert dev.device_status() == 0


@pytest.mark.gpu
def test_hubert_front_rejects_long_input(dev):
    m = dev.workloads.hubert_front_model(seed=3)
    fe = dev.HubertFront(m, max_samples=8000)
    with pytest.raises(dev.GsvkError):
        fe.forward(torch.zeros(9000, device="cuda"))
    fe.close()
