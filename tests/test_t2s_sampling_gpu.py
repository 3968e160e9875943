"""Top-k sampling of the T2S decode (SamplingParams + topk_sample,
t2s_engine.hpp:69-77, t2s_engine.cpp:1640-1737) against the oracle.

Sampling is integer and comparison work on top of the canonical logits, and
the draws come from the same std::mt19937_64 stream, so the bar is the same
as greedy decoding: identical token streams and identical per-step margins.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PARAMS = [
    dict(top_k=15, top_p=1.0, temperature=1.0, rep_penalty=1.35, seed=42),   # the reference default
    dict(top_k=15, top_p=0.8, temperature=0.7, rep_penalty=1.35, seed=7),
    dict(top_k=5, top_p=0.5, temperature=1.3, rep_penalty=1.2, seed=123),
    dict(top_k=40, top_p=1.0, temperature=0.0, rep_penalty=1.1, seed=9),    # temperature 0: top-1
    dict(top_k=1500, top_p=0.95, temperature=1.0, rep_penalty=1.35, seed=2), # k beyond the vocab
]


def _oracle(ora, m, k0, v0, prefix, prompt, steps, p, stop_on_eos):
    sp = ora.Sampling(1, p["top_k"], p["top_p"], p["temperature"], p["rep_penalty"], p["seed"])
    return ora.t2s_generate_sampled(m, k0.copy(), v0.copy(), prefix, prompt, steps, sp,
                                    stop_on_eos)


@pytest.mark.parametrize("p", PARAMS, ids=[f"k{p['top_k']}-p{p['top_p']}-t{p['temperature']}"
                                           for p in PARAMS])
@pytest.mark.parametrize("stop_on_eos", [False, True])
def test_sampled_stream_matches_oracle(dev, ora, p, stop_on_eos):
    W = dev.workloads
    m = W.t2s_model(n_layers=3, seed=5)
    if stop_on_eos:  # make EOS reachable so the stop path is exercised
        m = dict(m)
        m["wpred"] = m["wpred"].copy()
        row = m["wpred"][m["vocab"] - 1].view(np.float16).astype(np.float32) * 4.0
        m["wpred"][m["vocab"] - 1] = row.astype(np.float16).view(np.uint16)
    prefix, P, steps = 50, 16, 80
    cap = prefix + P + steps
    k0, v0 = W.t2s_kv_prefix(m, cap, prefix, seed=1)
    prompt = W.t2s_prompt(P, m["vocab"], seed=4)
    ref, ref_marg = _oracle(ora, m, k0, v0, prefix, prompt, steps, p, stop_on_eos)
    eng = dev.T2S(m, cap)
    if eng.decode_kernel() != eng.DECODE_FLOW:
        pytest.skip("top-k sampling runs on the per-head cluster decode kernel")
    eng.set_sampling(1, **p)
    eng.load_kv(k0, v0, prefix)
    toks, marg = eng.generate(prefix, prompt, steps, stop_on_eos)
    eng.close()
    assert len(toks) == len(ref), (len(toks), len(ref))
    bad = np.nonzero(toks != ref)[0]
    assert bad.size == 0, f"first divergence at step {bad[0]}"
    n = len(toks) + (1 if len(toks) < steps else 0)
    np.testing.assert_array_equal(marg[:n], ref_marg[:n])
    assert dev.device_status() == 0


def test_sampled_config2_full_model(dev, ora):
    """BASELINE config 2's model and cache, 500 sampled steps with the
    reference's default sampling (top-k 15, temperature 1, penalty 1.35)."""
    m, k0, v0, prompt = dev.workloads.t2s_decode_b1()
    steps = 500
    p = dict(top_k=15, top_p=1.0, temperature=1.0, rep_penalty=1.35, seed=20251202)
    ref, ref_marg = _oracle(ora, m, k0, v0, 256, prompt, steps, p, False)
    eng = dev.T2S(m, k0.shape[1])
    eng.set_sampling(1, **p)
    eng.load_kv(k0, v0, 256)
    toks, marg = eng.generate(256, prompt, steps, False)
    eng.close()
    assert len(toks) == steps
    np.testing.assert_array_equal(toks, ref)
    np.testing.assert_array_equal(marg, ref_marg)


def test_sampling_greedy_restore_and_rejections(dev, ora):
    W = dev.workloads
    m = W.t2s_model(n_layers=2, seed=8)
    prefix, P, steps = 20, 8, 20
    cap = prefix + P + steps
    k0, v0 = W.t2s_kv_prefix(m, cap, prefix, seed=2)
    prompt = W.t2s_prompt(P, m["vocab"], seed=3)
    eng = dev.T2S(m, cap)
    with pytest.raises(dev.GsvkError):
        eng.set_sampling(1, top_k=0)
    with pytest.raises(dev.GsvkError):
        eng.set_sampling(1, top_p=0.0)
    with pytest.raises(dev.GsvkError):
        eng.set_sampling(2)
    # sampling, then back to greedy: the greedy stream of the oracle
    eng.set_sampling(1, seed=5)
    eng.load_kv(k0, v0, prefix)
    eng.generate(prefix, prompt, steps, False)
    eng.set_sampling(0)
    eng.load_kv(k0, v0, prefix)
    toks, _ = eng.generate(prefix, prompt, steps, False)
    ref, _ = ora.t2s_generate(m, k0.copy(), v0.copy(), prefix, prompt, steps, False)
    np.testing.assert_array_equal(toks, ref)
    # top-k sampling on the grid kernel is refused at decode time
    eng.set_sampling(1, seed=5)
    eng.set_decode_kernel(eng.DECODE_GRID)
    eng.load_kv(k0, v0, prefix)
    with pytest.raises(dev.GsvkError):
        eng.generate(prefix, prompt, steps, False)
    eng.close()
