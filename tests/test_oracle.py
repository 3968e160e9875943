"""CPU oracle pinned against the reference's golden vectors and known-answer tests.

Restates the reference's tests/test_kern.cpp and tests/test_accel.cpp cases on
the oracle (the parity checker for every CUDA test), plus torch-CPU cross-checks
for the operators the golden files do not cover (convolutions, GELU).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F


def check_close(got, want, max_rel, min_cos):
    """test_kern.cpp:60-80: peak-normalised max error and cosine similarity."""
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    peak = np.abs(want).max()
    worst = np.abs(got - want).max() / peak
    cos = float(got @ want / np.sqrt((got @ got) * (want @ want)))
    assert worst <= max_rel, f"max_rel={worst:.3e}"
    assert cos >= min_cos, f"cos={cos:.12f}"


def f16(a):
    return np.asarray(a, np.float16).view(np.uint16)


def w16(rng, shape, scale):
    return f16(rng.uniform(-1, 1, size=shape).astype(np.float32) * scale)


# ---------------------------------------------------------------- golden pins
@pytest.mark.parametrize("tag", ["gemv_a", "gemv_b"])
def test_gemv_matches_torch_golden(ora, golden, tag):
    """test_kern.cpp:96-120."""
    w, x, y = golden[f"{tag}_w"], golden[f"{tag}_x"], golden[f"{tag}_y"]
    got = ora.gemv_f16w_f32acc(w, x)
    check_close(got, y, 2e-5, 1.0 - 1e-12)
    got_ref = ora.gemv_f16w_f32acc(w, x, ref=True)
    check_close(got_ref, y, 2e-5, 1.0 - 1e-12)
    peak = max(1.0, np.abs(got_ref).max())
    assert np.all(np.abs(got - got_ref) <= 1e-5 * peak)


def test_layernorm_matches_golden(ora, golden):
    """test_kern.cpp:207-216."""
    got = ora.layernorm(golden["ln_x"], golden["ln_g"], golden["ln_b"], 1e-5)
    check_close(got, golden["ln_y"], 1e-5, 1.0 - 1e-12)


def test_rmsnorm_matches_golden(ora, golden):
    """test_kern.cpp:198-205."""
    got = ora.rmsnorm(golden["rms_x"], golden["rms_g"], 1e-5)
    check_close(got, golden["rms_y"], 1e-6, 1.0 - 1e-12)


def test_softmax_matches_golden_and_sums_to_one(ora, golden):
    """test_kern.cpp:218-229."""
    got = ora.softmax_rows(golden["sm_x"])
    check_close(got, golden["sm_y"], 1e-6, 1.0 - 1e-12)
    np.testing.assert_allclose(got.astype(np.float64).sum(-1), 1.0, atol=1e-6)


def test_activations_match_golden(ora, golden):
    """test_kern.cpp:231-239 (relu bit-exact)."""
    v = golden["act_v"]
    check_close(ora.silu(v), golden["act_silu"], 1e-6, 1.0 - 1e-12)
    assert np.array_equal(ora.relu(v), golden["act_relu"])


def test_f16_special_values_exact(ora):
    """test_accel.cpp:85-100: widening is exact, RNE narrowing round-trips."""
    bits = np.array([0x0000, 0x8000, 0x3C00, 0xC000, 0x7BFF, 0x0400, 0x3555, 0xABCD], np.uint16)
    got = ora.f16_to_f32(bits)
    np.testing.assert_array_equal(got, bits.view(np.float16).astype(np.float32))
    assert got[2] == 1.0 and got[3] == -2.0 and got[4] == 65504.0
    assert np.array_equal(ora.f32_to_f16(got), bits)
    # round-to-nearest-even at a tie: 1 + 2^-11 lies halfway between 1 and 1+2^-10
    tie = np.array([1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11], np.float32)
    assert list(ora.f32_to_f16(tie)) == [0x3C00, 0x3C02]


# ------------------------------------------------------ restated known answers
@pytest.mark.parametrize("out_,in_", [(17, 131), (3, 8), (1, 1), (64, 7), (1536, 512)])
def test_gemv_blocked_vs_scalar_ref(ora, out_, in_):
    """test_kern.cpp:122-139."""
    rng = np.random.default_rng(out_ * 1000 + in_)
    w = w16(rng, (out_, in_), 0.3)
    x = rng.uniform(-1, 1, in_).astype(np.float32)
    a = ora.gemv_f16w_f32acc(w, x)
    b = ora.gemv_f16w_f32acc(w, x, ref=True)
    assert np.all(np.abs(a - b) <= 1e-5 * max(1.0, np.abs(b).max()))


GEMM_SHAPES = [(8, 1024, 1024), (32, 4096, 1024), (14, 768, 768), (96, 200, 9),
               (2048, 50, 1024), (17, 31, 7), (1, 1, 1), (64, 3, 1536)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_f16x_fmlal_matches_fp64(ora, M, N, K):
    """test_kern.cpp:145-196: |acc - got| <= 1e-4 (1 + |acc|) against an fp64 dot."""
    rng = np.random.default_rng(M * 7 + N * 13 + K)
    a = w16(rng, (M, K), 0.5)
    b = w16(rng, (N, K), 0.5)
    got = ora.gemm_f16x_fmlal(a, b)
    acc = a.view(np.float16).astype(np.float64) @ b.view(np.float16).astype(np.float64).T
    assert np.all(np.abs(acc - got) <= 1e-4 * (1.0 + np.abs(acc)))


def test_gemv_fmlal_equals_exact_products(ora):
    """gemv_fmlal.hpp:22-26: fp16 x fp16 products are exact in fp32."""
    rng = np.random.default_rng(5)
    w = w16(rng, (1025, 512), 0.05)
    xh = f16(rng.standard_normal(512))
    got = ora.gemv_f16x_fmlal(w, xh)
    acc = w.view(np.float16).astype(np.float64) @ xh.view(np.float16).astype(np.float64)
    assert np.all(np.abs(acc - got) <= 1e-5 * (1.0 + np.abs(acc)))


def test_sgemm_matches_naive_loop(ora):
    """test_accel.cpp:102-133: NN alpha=1 beta=0 ignores NaN C; TT alpha=2 beta=1."""
    rng = np.random.default_rng(7)
    M, N, K = 5, 7, 3
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    C = np.full((M, N), np.nan, np.float32)
    ora.sgemm("N", "N", M, N, K, 1.0, A, K, B, N, 0.0, C, N)
    np.testing.assert_allclose(C, A.astype(np.float64) @ B, atol=1e-5)
    P = rng.uniform(-1, 1, (K, M)).astype(np.float32)
    Q = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    C = np.full((M, N), 0.5, np.float32)
    ora.sgemm("T", "T", M, N, K, 2.0, P, M, Q, K, 1.0, C, N)
    np.testing.assert_allclose(C, 2.0 * (P.T.astype(np.float64) @ Q.T) + 0.5, atol=1e-5)


def test_dense_rows_match_gemv(ora, golden):
    """test_accel.cpp:135-158: y[T,out] = x W^T row t equals the GEMV of row t."""
    w = golden["gemv_a_w"]
    rng = np.random.default_rng(17)
    x = rng.uniform(-1, 1, (17, w.shape[1])).astype(np.float32)
    wf = ora.f16_to_f32(w)
    y = np.zeros((17, w.shape[0]), np.float32)
    ora.sgemm("N", "T", 17, w.shape[0], w.shape[1], 1.0, x, w.shape[1], wf, w.shape[1], 0.0, y,
              w.shape[0])
    for t in range(17):
        yr = ora.gemv_f16w_f32acc(w, x[t])
        assert np.all(np.abs(y[t] - yr) <= 1e-5 * np.abs(yr).max())


def test_gelu_and_leaky_match_torch(ora):
    v = np.random.default_rng(3).standard_normal(4097).astype(np.float32) * 3
    np.testing.assert_allclose(ora.gelu_erf(v), F.gelu(torch.from_numpy(v)).numpy(), atol=2e-6)
    np.testing.assert_array_equal(ora.leaky_relu(v, 0.1),
                                  F.leaky_relu(torch.from_numpy(v), 0.1).numpy())


# ---------------------------------------------------------------- convolutions
@pytest.mark.parametrize("Ci,Co,T,k,dil", [(16, 24, 50, 3, 1), (8, 8, 37, 7, 3), (12, 5, 64, 11, 5),
                                           (4, 1, 20, 7, 1), (32, 16, 9, 1, 1)])
def test_conv1d_matches_torch(ora, Ci, Co, T, k, dil):
    """conv1d.hpp:109-194 same padding (k-1)*dil/2 versus torch conv1d."""
    rng = np.random.default_rng(Ci + Co + T)
    x = rng.standard_normal((Ci, T)).astype(np.float32)
    w = f16(rng.standard_normal((Co, Ci, k)) * 0.1)
    b = (rng.standard_normal(Co) * 0.1).astype(np.float32)
    xr = ora.f16_to_f32(ora.f32_to_f16(x))
    ref = F.conv1d(torch.from_numpy(xr)[None].double(), torch.from_numpy(ora.f16_to_f32(w)).double(),
                   torch.from_numpy(b).double(), padding=(k - 1) * dil // 2, dilation=dil)[0].numpy()
    got = ora.conv1d(x, w, b, dil, round_in=True)
    np.testing.assert_allclose(got, ref, atol=1e-5, rtol=1e-5)
    got32 = ora.conv1d(x, w, b, dil, round_in=False)
    ref32 = F.conv1d(torch.from_numpy(x)[None].double(), torch.from_numpy(ora.f16_to_f32(w)).double(),
                     torch.from_numpy(b).double(), padding=(k - 1) * dil // 2, dilation=dil)[0].numpy()
    np.testing.assert_allclose(got32, ref32, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("Ci,Co,T,k,u", [(16, 8, 12, 16, 10), (8, 4, 20, 16, 8), (8, 4, 33, 8, 2),
                                         (6, 3, 40, 2, 2), (10, 6, 7, 20, 10)])
def test_convt1d_matches_torch(ora, Ci, Co, T, k, u):
    """conv1d.hpp:250-359 phase GEMM + scatter versus torch conv_transpose1d."""
    rng = np.random.default_rng(Ci * Co + T + k)
    x = rng.standard_normal((Ci, T)).astype(np.float32)
    w = f16(rng.standard_normal((Ci, Co, k)) * 0.1)
    b = (rng.standard_normal(Co) * 0.1).astype(np.float32)
    xr = ora.f16_to_f32(ora.f32_to_f16(x))
    ref = F.conv_transpose1d(torch.from_numpy(xr)[None].double(),
                             torch.from_numpy(ora.f16_to_f32(w)).double(),
                             torch.from_numpy(b).double(), stride=u, padding=(k - u) // 2)[0].numpy()
    got = ora.convt1d(x, w, b, u, round_in=True)
    assert got.shape == (Co, T * u) == ref.shape
    np.testing.assert_allclose(got, ref, atol=1e-5, rtol=1e-5)


# ------------------------------------------------------------------------ T2S
def test_greedy_sample_penalty_semantics(ora):
    """t2s_engine.cpp:1594-1636: one penalty per distinct token, EOS column
    untouched and excluded while idx < 11."""
    V = 10
    lg = np.array([0.5, -0.2, 0.3, 0.1, 0.0, -1.0, 0.2, 0.05, 0.49, 0.9], np.float32)
    hist = np.array([0, 0, 0, 1, 9, 9], np.int32)
    work = lg.copy()
    s, raw = ora.t2s_greedy_sample(work, hist, eos_allowed=False)
    assert work[0] == np.float32(0.5) / np.float32(1.35)  # once, not three times
    assert work[1] == np.float32(-0.2) * np.float32(1.35)
    assert work[9] == lg[9]  # EOS column keeps its raw value
    assert raw == 9 and s == 8
    work = lg.copy()
    s, raw = ora.t2s_greedy_sample(work, hist, eos_allowed=True)
    assert work[9] == np.float32(0.9) / np.float32(1.35) and s == 9


def test_prefill_matches_stepwise_decode(ora, gsv):
    """test_ar_unit.cpp:101-153 pattern on synthetic weights: one prefill
    block equals the same tokens decoded one by one (same slots)."""
    m = gsv.workloads.t2s_model(n_layers=2, seed=11)
    D = m["d_model"]
    cap, prefix, S = 64, 20, 9
    rng = np.random.default_rng(4)
    x0 = rng.standard_normal((S, D)).astype(np.float32)
    kv = gsv.workloads.t2s_kv_prefix(m, cap, prefix, seed=2)
    kc1, vc1 = kv[0].copy(), kv[1].copy()
    kc2, vc2 = kv[0].copy(), kv[1].copy()
    xa = x0.copy()
    for l in range(2):
        ora.t2s_prefill_layer(m, l, xa, prefix, 0, kc1[l], vc1[l])
    xb = x0.copy()
    for t in range(S):
        row = xb[t].copy()
        for l in range(2):
            ora.t2s_decode_layer(m, l, row, prefix + t, kc2[l], vc2[l])
        xb[t] = row
    # prefill rounds activations of all projections to fp16, decode keeps
    # W2 on fp32 activations: agreement at the reference's 5e-3 AMX level.
    np.testing.assert_allclose(xa, xb, atol=5e-3 * np.abs(xb).max())
