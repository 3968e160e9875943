"""CPU checks of the oracle's top-k sampler (t2s_engine.cpp:1640-1737):
mode 0 is the greedy generate, temperature 0 takes the best of the top k,
and a fixed seed reproduces its stream."""
import numpy as np


def _setup(gsv):
    W = gsv.workloads
    m = W.t2s_model(n_layers=2, seed=5)
    k0, v0 = W.t2s_kv_prefix(m, 30 + 8 + 40, 30, seed=1)
    return m, k0, v0, W.t2s_prompt(8, m["vocab"], seed=4)


def test_greedy_mode_equals_greedy_generate(gsv, ora):
    m, k0, v0, pr = _setup(gsv)
    sp = ora.Sampling(0, 15, 1.0, 1.0, 1.35, 0)
    t, _ = ora.t2s_generate_sampled(m, k0.copy(), v0.copy(), 30, pr, 40, sp, False)
    g, _ = ora.t2s_generate(m, k0.copy(), v0.copy(), 30, pr, 40, False)
    np.testing.assert_array_equal(t, g)


def test_zero_temperature_with_reference_penalty_is_greedy(gsv, ora):
    """Temperature 0 returns the best of the top k: with the greedy penalty
    (1.35) that is the greedy token every step."""
    m, k0, v0, pr = _setup(gsv)
    sp = ora.Sampling(1, 15, 1.0, 0.0, 1.35, 3)
    t, _ = ora.t2s_generate_sampled(m, k0.copy(), v0.copy(), 30, pr, 40, sp, False)
    g, _ = ora.t2s_generate(m, k0.copy(), v0.copy(), 30, pr, 40, False)
    np.testing.assert_array_equal(t, g)


def test_seeded_stream_is_reproducible_and_seed_dependent(gsv, ora):
    m, k0, v0, pr = _setup(gsv)
    runs = {}
    for seed in (11, 11, 12):
        sp = ora.Sampling(1, 15, 1.0, 1.0, 1.35, seed)
        runs.setdefault(seed, []).append(
            ora.t2s_generate_sampled(m, k0.copy(), v0.copy(), 30, pr, 40, sp, False)[0])
    np.testing.assert_array_equal(runs[11][0], runs[11][1])
    assert not np.array_equal(runs[11][0], runs[12][0])
