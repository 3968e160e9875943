"""GPU parity of the T2S path (a16-a19) through the C-ABI against the oracle.

The T2S path evaluates the canonical association of every sum (oracle.h,
"T2S numerics"), so the bar is bit-exactness:
  * prefill rows and the KV slots they write: identical bits;
  * greedy decode: identical token stream (north star), identical per-step
    margins and identical final logits.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


@pytest.fixture(scope="module")
def small(dev):
    m = dev.workloads.t2s_model(n_layers=3, seed=5)
    return m


def test_prefill_matches_oracle(dev, ora, small):
    m = small
    D, cap, prefix, S = m["d_model"], 128, 40, 23
    k0, v0 = dev.workloads.t2s_kv_prefix(m, cap, prefix, seed=3)
    x0 = np.random.default_rng(8).standard_normal((S, D)).astype(np.float32)
    # oracle
    kc, vc, xo = k0.copy(), v0.copy(), x0.copy()
    for layer in range(m["n_layers"]):
        ora.t2s_prefill_layer(m, layer, xo, prefix, 5, kc[layer], vc[layer])
    # device
    eng = dev.T2S(m, cap)
    eng.load_kv(k0, v0, prefix)
    xd = torch.from_numpy(x0).cuda()
    eng.prefill(xd, prefix, 5)
    got = xd.cpu().numpy()
    np.testing.assert_array_equal(got, xo)
    eng.close()


@pytest.mark.parametrize("kernel", [1, 2, 3], ids=["grid", "cluster", "flow"])
@pytest.mark.parametrize("stop_on_eos", [False, True])
def test_generate_small_token_identity(dev, ora, small, stop_on_eos, kernel):
    m = dict(small)
    if stop_on_eos:
        # make EOS competitive so the stop path is exercised after the 11-step mask
        m["wpred"] = m["wpred"].copy()
        row = m["wpred"][m["vocab"] - 1].view(np.float16).astype(np.float32) * 6.0
        m["wpred"][m["vocab"] - 1] = row.astype(np.float16).view(np.uint16)
    prefix, P, steps = 50, 16, 60
    cap = prefix + P + steps
    k0, v0 = dev.workloads.t2s_kv_prefix(m, cap, prefix, seed=1)
    prompt = dev.workloads.t2s_prompt(P, m["vocab"], seed=4)
    toks_ref, marg_ref, logits_ref = ora.t2s_generate(m, k0.copy(), v0.copy(), prefix, prompt,
                                                      steps, stop_on_eos, with_logits=True)
    eng = dev.T2S(m, cap)
    eng.set_decode_kernel(kernel)
    assert eng.decode_kernel() == kernel
    eng.load_kv(k0, v0, prefix)
    toks, marg = eng.generate(prefix, prompt, steps, stop_on_eos)
    logits = eng.read_logits()
    eng.close()
    if stop_on_eos:
        assert len(toks_ref) < steps, "EOS never sampled: the stop path was not exercised"
    first_bad = next((i for i in range(min(len(toks), len(toks_ref))) if toks[i] != toks_ref[i]),
                     None)
    assert first_bad is None and len(toks) == len(toks_ref), (
        f"token streams diverge at step {first_bad} (oracle margin "
        f"{marg_ref[first_bad] if first_bad is not None else 'n/a'})")
    n_steps = len(toks) + (1 if len(toks) < steps else 0)
    np.testing.assert_array_equal(marg[:n_steps], marg_ref[:n_steps])
    np.testing.assert_array_equal(logits, logits_ref)
    assert dev.device_status() == 0


def test_generate_config2_full_model_token_identity(dev, ora):
    """24 layers, d=512, KV prefix 256 (N(0,1)), 64-token prompt,
    500 greedy steps; identical token stream."""
    m, k0, v0, prompt = dev.workloads.t2s_decode_b1()
    cap = k0.shape[1]
    steps = 500
    toks_ref, marg_ref = ora.t2s_generate(m, k0.copy(), v0.copy(), 256, prompt, steps, False)
    eng = dev.T2S(m, cap)
    assert eng.decode_kernel() == eng.DECODE_FLOW  # the default on a B200
    for kernel in (eng.DECODE_FLOW, eng.DECODE_CLUSTER, eng.DECODE_GRID):
        eng.set_decode_kernel(kernel)
        eng.load_kv(k0, v0, 256)
        toks, marg = eng.generate(256, prompt, steps, False)
        assert len(toks) == len(toks_ref) == steps
        bad = np.nonzero(toks != toks_ref)[0]
        assert bad.size == 0, (f"kernel {kernel}: first divergence at step {bad[0]}: oracle "
                               f"margin {marg_ref[bad[0]]:.3e}, device margin {marg[bad[0]]:.3e}")
        np.testing.assert_array_equal(marg, marg_ref)
    eng.close()


def test_decode_kernels_write_identical_kv(dev, small):
    """All decode kernels leave the same KV cache and the same final logits."""
    m = small
    prefix, P, steps = 30, 8, 40
    cap = prefix + P + steps
    k0, v0 = dev.workloads.t2s_kv_prefix(m, cap, prefix, seed=2)
    prompt = dev.workloads.t2s_prompt(P, m["vocab"], seed=6)
    out = {}
    for kernel in (1, 2, 3):
        eng = dev.T2S(m, cap)
        eng.set_decode_kernel(kernel)
        eng.load_kv(k0, v0, prefix)
        toks, marg = eng.generate(prefix, prompt, steps, False)
        kv = eng.read_kv()
        out[kernel] = (toks, marg, eng.read_logits(), kv)
        eng.close()
    for other in (2, 3):
        for a, b in zip(out[1], out[other]):
            if isinstance(a, tuple):
                for x, y in zip(a, b):
                    np.testing.assert_array_equal(x, y)
            else:
                np.testing.assert_array_equal(a, b)
    assert dev.device_status() == 0


def test_generate_rejects_oversized_request(dev, small):
    eng = dev.T2S(small, 64)
    with pytest.raises(dev.GsvkError):
        eng.generate(40, np.zeros(16, np.int32), 20)
    eng.close()


def test_decode_cta_count_does_not_change_results(dev, small):
    """The grid decode kernel on fewer CTAs than SMs: identical tokens and margins."""
    m = small
    prefix, P, steps = 30, 8, 40
    cap = prefix + P + steps
    k0, v0 = dev.workloads.t2s_kv_prefix(m, cap, prefix, seed=7)
    prompt = dev.workloads.t2s_prompt(P, m["vocab"], seed=9)
    out = []
    for ctas in (0, 100, 120):
        eng = dev.T2S(m, cap)
        eng.set_decode_ctas(ctas)
        eng.load_kv(k0, v0, prefix)
        out.append(eng.generate(prefix, prompt, steps, False))
        eng.close()
    for toks, marg in out[1:]:
        np.testing.assert_array_equal(toks, out[0][0])
        np.testing.assert_array_equal(marg, out[0][1])
    # too few CTAs: their weight slices no longer fit shared memory; the plan is kept
    eng = dev.T2S(m, cap)
    with pytest.raises(dev.GsvkError) as ei:
        eng.set_decode_ctas(37)
    assert ei.value.code == -5
    eng.load_kv(k0, v0, prefix)
    toks, marg = eng.generate(prefix, prompt, steps, False)
    np.testing.assert_array_equal(toks, out[0][0])
    eng.close()
    assert dev.device_status() == 0


def test_exchange_wait_timeout_is_reported_and_recovers(dev, ora, small):
    """Failure detection without a fault: with the test spin limit every
    exchange poll of the per-head cluster decode gives up after a few polls,
    so the launch records GSVK_ERR_TIMEOUT, winds down (no wait, every bulk
    copy drained) and the host call reports it; the next healthy generate on
    the same handle and context matches the oracle bit for bit."""
    m = small
    prefix, P, steps = 30, 8, 40
    cap = prefix + P + steps
    k0, v0 = dev.workloads.t2s_kv_prefix(m, cap, prefix, seed=12)
    prompt = dev.workloads.t2s_prompt(P, m["vocab"], seed=13)
    eng = dev.T2S(m, cap)
    if eng.decode_kernel() != eng.DECODE_FLOW:
        pytest.skip("the per-head cluster decode kernel does not fit this GPU")
    lib = dev.lib()
    try:
        assert lib.gsvk_set_spin_limit_for_test(1) == 0
        eng.load_kv(k0, v0, prefix)
        with pytest.raises(dev.GsvkError) as ei:
            eng.generate(prefix, prompt, steps, False)
        assert ei.value.code == -4, ei.value  # GSVK_ERR_TIMEOUT
    finally:
        lib.gsvk_set_spin_limit_for_test(0)
    assert dev.device_status() == 0  # the failing call read and cleared the status
    eng.load_kv(k0, v0, prefix)
    toks, marg = eng.generate(prefix, prompt, steps, False)
    eng.close()
    ref, ref_marg = ora.t2s_generate(m, k0.copy(), v0.copy(), prefix, prompt, steps, False)
    np.testing.assert_array_equal(toks, ref)
    np.testing.assert_array_equal(marg, ref_marg)
