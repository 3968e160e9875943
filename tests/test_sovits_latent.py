"""The SoVITS latent path (sovits_engine.hpp:48-93 steps 1-5): RVQ decode,
nearest x2, TextEncoder with relative-position attention and MRTE, the z_p
draw and the reverse WaveNet flow, against the oracle restatement.

The device runs every Conv1d with fp16 activations on the tensor cores and
the attention in fp32, the oracle rounds the conv inputs to fp16 the same
way; the remaining differences are summation order and library exp/tanh.
The bar is the SoVITS generator's: max |error| <= 1e-2 of the peak, cos >=
0.9999, on m_p, logs_p and z."""
import numpy as np
import pytest


def _rel_cos(got, ref):
    got = np.asarray(got, np.float64).ravel()
    ref = np.asarray(ref, np.float64).ravel()
    return (float(np.abs(got - ref).max() / np.abs(ref).max()),
            float(got @ ref / np.sqrt((got @ got) * (ref @ ref))))


@pytest.fixture(scope="module")
def model(gsv):
    return gsv.workloads.sovits_latent_model(seed=2)


def test_oracle_shapes_and_errors(gsv, ora, model):
    W = gsv.workloads
    codes, phones, ge, ge_text, nz = W.sovits_latent_inputs(6, 5, seed=3)
    mp, lp, z = ora.sovits_latent(model, codes, phones, ge, ge_text, nz)
    assert mp.shape == lp.shape == z.shape == (192, 12)
    assert np.isfinite(z).all()
    # deterministic
    z2 = ora.sovits_latent(model, codes, phones, ge, ge_text, nz)[2]
    np.testing.assert_array_equal(z, z2)
    # no noise: z_p = m_p enters the flow
    z0 = ora.sovits_latent(model, codes, phones, ge, ge_text, None)[2]
    assert not np.array_equal(z0, z)
    bad = codes.copy()
    bad[2] = 1024
    with pytest.raises(ValueError, match="-2"):
        ora.sovits_latent(model, bad, phones, ge, ge_text, nz)
    m2 = dict(model)
    m2["tensors"] = {k: v for k, v in model["tensors"].items() if "flow.flows.4.post" not in k}
    with pytest.raises(ValueError, match="-1"):
        ora.sovits_latent(m2, codes, phones, ge, ge_text, nz)


def _run(dev, ora, model, n_codes, n_phones, seed, noise=True, max_codes=256, max_phones=256):
    import torch

    W = dev.workloads
    codes, phones, ge, ge_text, nz = W.sovits_latent_inputs(n_codes, n_phones, cfg=model,
                                                            seed=seed, noise=noise)
    ref = ora.sovits_latent(model, codes, phones, ge, ge_text, nz)
    eng = dev.SovitsLatent(model, max_codes, max_phones)
    Tq = 2 * n_codes
    mp = torch.empty(model["hidden"], Tq, device="cuda")
    lp = torch.empty_like(mp)
    z = eng.forward(codes, phones, torch.from_numpy(ge).cuda(), torch.from_numpy(ge_text).cuda(),
                    None if nz is None else torch.from_numpy(nz).cuda(), m_p=mp, logs_p=lp)
    got = [t.cpu().numpy() for t in (mp, lp, z)]
    eng.close()
    return got, ref


@pytest.mark.gpu
@pytest.mark.parametrize("n_codes,n_phones,noise", [(20, 15, True), (1, 1, False), (3, 40, True),
                                                    (150, 120, True)])
def test_latent_matches_oracle(dev, ora, model, n_codes, n_phones, noise):
    got, ref = _run(dev, ora, model, n_codes, n_phones, seed=n_codes, noise=noise)
    for name, g, r in zip(("m_p", "logs_p", "z"), got, ref):
        d, c = _rel_cos(g, r)
        assert d <= 1e-2 and c >= 0.9999, f"{name}: max rel {d:.3e} cos {c:.8f}"
    assert dev.device_status() == 0


@pytest.mark.gpu
def test_latent_odd_flow_count(dev, ora, gsv):
    """Three coupling layers leave the flips' orientation reversed at the end."""
    cfg = dict(gsv.workloads.SOVITS_LATENT, flows=3, layers_ssl=1, layers_text=1, layers_2=1)
    m = gsv.workloads.sovits_latent_model(seed=4, cfg=cfg)
    got, ref = _run(dev, ora, m, 12, 9, seed=5)
    d, c = _rel_cos(got[2], ref[2])
    assert d <= 1e-2 and c >= 0.9999, f"z: max rel {d:.3e} cos {c:.8f}"


@pytest.mark.gpu
def test_latent_from_gsv_file(dev, model, tmp_path):
    """A .gsv container with the same tensors (slim: fp16 copies only for the
    conv weights) gives the identical output."""
    import sys
    import os
    import torch

    sys.path.insert(0, os.path.dirname(__file__))
    import gsv_writer

    tensors = []
    for k, a in model["tensors"].items():
        if a.dtype == np.uint16:
            tensors.append((k, a.view(np.float16).astype(np.float32), a))
        else:
            tensors.append((k, a, None))
    path = str(tmp_path / "latent.gsv")
    gsv_writer.write(path, "sovits", {"meta": {"source": "synthetic"}}, tensors, slim=True)
    f = dev.GsvFile(path)
    W = dev.workloads
    codes, phones, ge, ge_text, nz = W.sovits_latent_inputs(10, 7, seed=6)
    args = (codes, phones, torch.from_numpy(ge).cuda(), torch.from_numpy(ge_text).cuda(),
            torch.from_numpy(nz).cuda())
    a = dev.SovitsLatent(model, 16, 16)
    b = dev.SovitsLatent(model, 16, 16, gsv=f)
    za, zb = a.forward(*args).cpu().numpy(), b.forward(*args).cpu().numpy()
    a.close()
    b.close()
    f.close()
    np.testing.assert_array_equal(za, zb)


@pytest.mark.gpu
def test_latent_rejections(dev, model):
    import torch

    W = dev.workloads
    codes, phones, ge, ge_text, nz = W.sovits_latent_inputs(8, 6, seed=7)
    g, gt = torch.from_numpy(ge).cuda(), torch.from_numpy(ge_text).cuda()
    eng = dev.SovitsLatent(model, 8, 6)
    bad = codes.copy()
    bad[3] = -1
    with pytest.raises(dev.GsvkError):
        eng.forward(bad, phones, g, gt)
    badp = phones.copy()
    badp[0] = 732
    with pytest.raises(dev.GsvkError):
        eng.forward(codes, badp, g, gt)
    with pytest.raises(dev.GsvkError):
        eng.forward(np.zeros(9, np.int64), phones, g, gt)
    eng.forward(codes, phones, g, gt)  # still usable
    eng.close()
    m2 = dict(model)
    m2["tensors"] = {k: v for k, v in model["tensors"].items() if k != "enc_p.proj.weight"}
    with pytest.raises(dev.GsvkError):
        dev.SovitsLatent(m2, 8, 6)
    assert dev.device_status() == 0
