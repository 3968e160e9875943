"""The .gsv weight container (GsvFile, src/runtime/gsv_loader.hpp:50-114;
format per tools/convert.py:3-28) read through the C-ABI: round trip of a
synthetic T2S file, the reference loader's validation rules on corrupted
files, and (GPU) a T2S engine built from the file that decodes exactly like
one built from the same arrays."""
import numpy as np
import pytest

import gsv_writer


@pytest.fixture(scope="module")
def small(gsv):
    return gsv.workloads.t2s_model(n_layers=2, seed=7)


def _write(tmp_path, model, **kw):
    tensors, config = gsv_writer.t2s_tensors(model)
    path = str(tmp_path / "ar_test.gsv")
    gsv_writer.write(path, "ar_test", config, tensors, **kw)
    return path, tensors, config


@pytest.mark.parametrize("slim", [False, True])
def test_round_trip(gsv, tmp_path, small, slim):
    path, tensors, config = _write(tmp_path, small, slim=slim)
    f = gsv.GsvFile(path)
    assert f.model_name == "ar_test" and len(f) == len(tensors)
    assert '"model_config"' in f.config
    got = {t[0]: t for t in f.tensors()}
    for name, f32, f16 in tensors:
        gname, shape, dtype, g32, g16 = got[name]
        assert shape == f32.shape and dtype == (2 if f16 is not None else 1)
        if f16 is not None:
            np.testing.assert_array_equal(g16, f16)
            assert (g32 is None) == slim
        if g32 is not None:
            np.testing.assert_array_equal(g32, f32)
    _, shape, _, _, w16 = f.tensor("h.layers.1.linear2.weight")
    assert shape == (512, 2048)
    np.testing.assert_array_equal(w16, small["w2"][1])
    with pytest.raises(gsv.GsvkError):
        f.tensor("no.such.tensor")
    f.close()


def _corrupt(name, fn):
    return pytest.param(fn, id=name)


CASES = [
    ("wrong rank", lambda es: es[0].update(dims=[1] * 9)),
    ("unknown dtype", lambda es: es[0].update(dtype=3)),
    ("fp32 size", lambda es: es[1].update(f32_n=es[1]["f32_n"] - 4)),
    ("fp16 size", lambda es: es[0].update(f16_n=es[0]["f16_n"] + 2)),
    ("unaligned", lambda es: es[0].update(f32_off=es[0]["f32_off"] + 4)),
    ("out of file", lambda es: es[2].update(f16_off=es[2]["f16_off"] + (1 << 40))),
    ("flag bit", lambda es: es[0].update(flags=0)),
]


@pytest.mark.parametrize("what,patch", CASES, ids=[c[0] for c in CASES])
def test_rejects_corrupt_directories(gsv, tmp_path, small, what, patch):
    path, _, _ = _write(tmp_path, small, patch=patch)
    with pytest.raises(gsv.GsvkError) as ei:
        gsv.GsvFile(path)
    assert ei.value.code == -1  # GSVK_ERR_INVALID


def test_rejects_bad_headers(gsv, tmp_path, small):
    path, _, _ = _write(tmp_path, small)
    raw = open(path, "rb").read()
    for name, data in [("magic", b"GSV2" + raw[4:]), ("version", raw[:4] + b"\x02" + raw[5:]),
                       ("truncated", raw[:20]), ("empty directory cut", raw[:200])]:
        p = tmp_path / f"bad_{name}.gsv"
        p.write_bytes(data)
        with pytest.raises(gsv.GsvkError):
            gsv.GsvFile(str(p))


@pytest.mark.gpu
def test_t2s_from_gsv_decodes_like_the_arrays(dev, tmp_path, small):
    path, _, _ = _write(tmp_path, small, slim=True)
    f = dev.GsvFile(path)
    prefix, P, steps = 40, 12, 50
    cap = prefix + P + steps
    k0, v0 = dev.workloads.t2s_kv_prefix(small, cap, prefix, seed=3)
    prompt = dev.workloads.t2s_prompt(P, small["vocab"], seed=5)
    a = dev.T2S.from_gsv(f, cap)
    f.close()  # the engine holds device copies
    b = dev.T2S(small, cap)
    out = []
    for eng in (a, b):
        eng.load_kv(k0, v0, prefix)
        out.append(eng.generate(prefix, prompt, steps, False))
        eng.close()
    np.testing.assert_array_equal(out[0][0], out[1][0])
    np.testing.assert_array_equal(out[0][1], out[1][1])
