"""GPU parity for the tensor-core GEMM (a3, a6, a9) through the C-ABI.

Gates (stated per test):
  * the reference's own gemm test (test_kern.cpp:145-196):
        |acc - got| <= 1e-4 (1 + |acc|)  against an fp64 dot of the fp16 inputs;
  * the AMX-vs-FMLAL gate (test_kern.cpp:282-320): cos >= 0.9999, max|d|/max|ref| <= 1e-3;
  * the north-star bound for fused fp16-output GEMMs: max relative error <= 1e-2.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def h(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.float16)).cuda()


def f(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def rand16(rng, shape, scale):
    return (rng.uniform(-1, 1, size=shape).astype(np.float32) * scale).astype(np.float16).view(np.uint16)


def exact(a, b):
    return a.view(np.float16).astype(np.float64) @ b.view(np.float16).astype(np.float64).T


GEMM_SHAPES = [(8, 1024, 1024), (32, 4096, 1024), (14, 768, 768), (96, 200, 9),
               (2048, 50, 1024), (17, 31, 7), (1, 1, 1), (64, 3, 1536)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_f16_reference_cases(dev, M, N, K):
    """test_kern.cpp:145-196 shapes and tolerance (odd K runs the CUDA-core kernel)."""
    rng = np.random.default_rng(M * 7 + N * 13 + K)
    a, b = rand16(rng, (M, K), 0.5), rand16(rng, (N, K), 0.5)
    got = dev.gemm_f16(h(a), h(b)).cpu().numpy().astype(np.float64)
    acc = exact(a, b)
    bad = np.abs(acc - got) > 1e-4 * (1.0 + np.abs(acc))
    assert not bad.any(), f"{bad.sum()} mismatches, worst {np.abs(acc - got).max():.3g}"
    assert dev.device_status() == 0


EDGE = [(1, 16, 64), (127, 17, 64), (129, 33, 72), (300, 64, 16), (300, 48, 32), (256, 128, 128),
        (200, 200, 520), (513, 256, 256), (130, 384, 1024), (64, 1000, 512), (1000, 24, 24)]


@pytest.mark.parametrize("M,N,K", EDGE)
def test_gemm_edges_match_oracle(dev, ora, M, N, K):
    rng = np.random.default_rng(M + 31 * N + 7 * K)
    a, b = rand16(rng, (M, K), 1.0), rand16(rng, (N, K), 0.05)
    got = dev.gemm_f16(h(a), h(b)).cpu().numpy()
    ref = ora.gemm_f16x_fmlal(a, b)
    acc = exact(a, b)
    assert np.all(np.abs(acc - got) <= 1e-4 * (1.0 + np.abs(acc)))
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()


def test_gemm_config1_ffn_up(dev, ora):
    """Y = ReLU(X W^T + b), X[128,512] U(-1,1), W[2048,512] N(0,0.02),
    b N(0,0.01), fp16 output; max relative error <= 1e-2 against the oracle."""
    x, w, b = dev.workloads.gemm_ffn_up()
    yh = torch.empty(128, 2048, dtype=torch.float16, device="cuda")
    dev.gemm_ex(h(x), h(w), bias=f(b), act=dev.ACT_RELU, c_f16=yh)
    got = yh.float().cpu().numpy()
    ref = ora.linear_f16(ora.f16_to_f32(x), w, b, ora.ACT_RELU)
    err = np.abs(got - ref)
    assert err.max() <= 1e-2 * np.abs(ref).max()
    # fp16 rounding of the output is the only loss beyond fp32 reordering
    assert np.all(err <= 2.0 ** -10 * np.abs(ref) + 1e-4)


@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_gemm_fused_epilogue(dev, ora, act):
    rng = np.random.default_rng(100 + act)
    M, N, K = 300, 384, 256
    a, w = rand16(rng, (M, K), 1.0), rand16(rng, (N, K), 0.05)
    bias = rng.standard_normal(N).astype(np.float32) * 0.1
    res = rng.standard_normal((M, N)).astype(np.float32)
    c = torch.empty(M, N, device="cuda")
    c16 = torch.empty(M, N, dtype=torch.float16, device="cuda")
    dev.gemm_ex(h(a), h(w), bias=f(bias), residual=f(res), act=act, slope=0.1, c=c, c_f16=c16)
    ref = ora.linear_f16(ora.f16_to_f32(a), w, bias, act, 0.1) + res
    got = c.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max()
    np.testing.assert_array_equal(c16.cpu().numpy(), got.astype(np.float16))


@pytest.mark.parametrize("M,N,K", [(64, 1536, 512), (64, 512, 2048), (7, 1025, 512),
                                   (128, 2048, 512), (256, 640, 4096)])
def test_gemm_few_rows_fused_epilogue(dev, ora, M, N, K):
    """Decode-step shapes (M = batch): the split-K cluster kernel with bias,
    ReLU, residual and both output precisions against the oracle."""
    rng = np.random.default_rng(M + N + K)
    a, w = rand16(rng, (M, K), 1.0), rand16(rng, (N, K), 0.05)
    bias = rng.standard_normal(N).astype(np.float32) * 0.1
    res = rng.standard_normal((M, N)).astype(np.float32)
    c = torch.empty(M, N, device="cuda")
    c16 = torch.empty(M, N, dtype=torch.float16, device="cuda")
    dev.gemm_ex(h(a), h(w), bias=f(bias), residual=f(res), act=1, c=c, c_f16=c16)
    ref = ora.linear_f16(ora.f16_to_f32(a), w, bias, 1) + res
    got = c.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max()
    np.testing.assert_array_equal(c16.cpu().numpy(), got.astype(np.float16))
    assert dev.device_status() == 0


def test_gemm_strided_operands(dev, ora):
    """Leading dimensions larger than K (sub-matrix views, e.g. per-head slices)."""
    rng = np.random.default_rng(5)
    M, N, K, lda, ldb = 200, 96, 64, 192, 136
    A = rand16(rng, (M, lda), 1.0)
    B = rand16(rng, (N, ldb), 0.1)
    ta, tb = h(A)[:, 32:32 + K], h(B)[:, 8:8 + K]
    c = torch.empty(M, N, device="cuda")
    dev.gemm_ex(ta, tb, c=c)
    ref = exact(np.ascontiguousarray(A[:, 32:32 + K]), np.ascontiguousarray(B[:, 8:8 + K]))
    assert np.abs(c.cpu().numpy() - ref).max() <= 1e-4 * (1 + np.abs(ref).max())


@pytest.mark.parametrize("name", ["bert", "hubert"])
def test_gemm_encoder_shapes_vs_torch_fp32(dev, name):
    """Config 4 FFN-up shape per encoder against a torch fp32 GEMM of the same
    fp16 values (AMX gate: cos >= 0.9999, max|d|/max|ref| <= 1e-3)."""
    e = dev.workloads.ENCODERS[name]
    M, H, Fd = e["batch"] * e["seq"], e["hidden"], e["ffn"]
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(M, H, device="cuda", generator=g).half()
    w = (torch.randn(Fd, H, device="cuda", generator=g) * 0.02).half()
    got = dev.gemm_f16(x, w)
    ref = x.float() @ w.float().T
    d = (got - ref).abs().max().item() / ref.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got.flatten().double(), ref.flatten().double(), dim=0)
    assert d <= 1e-3 and cos.item() >= 0.9999
    assert dev.device_status() == 0


# ------------------------------------------------------------------ a5 sgemm
def test_sgemm_matches_naive_loop(dev, ora):
    """test_accel.cpp:102-133: NN with NaN in C (beta = 0 must not read it) and TT
    with alpha = 2, beta = 1; |d| <= 1e-5."""
    rng = np.random.default_rng(7)
    M, N, K = 5, 7, 3
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    C = torch.full((M, N), float("nan"), device="cuda")
    dev.sgemm("N", "N", M, N, K, 1.0, f(A), K, f(B), N, 0.0, C, N)
    np.testing.assert_allclose(C.cpu().numpy(), A.astype(np.float64) @ B, atol=1e-5)
    P = rng.uniform(-1, 1, (K, M)).astype(np.float32)
    Q = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    C = torch.full((M, N), 0.5, device="cuda")
    dev.sgemm("T", "T", M, N, K, 2.0, f(P), M, f(Q), K, 1.0, C, N)
    np.testing.assert_allclose(C.cpu().numpy(), 2.0 * (P.T.astype(np.float64) @ Q.T) + 0.5,
                               atol=1e-5)


@pytest.mark.parametrize("ta,tb,M,N,K", [("N", "T", 17, 128, 96), ("N", "N", 300, 129, 257),
                                         ("T", "N", 64, 65, 1000), ("T", "T", 1, 1025, 512)])
def test_sgemm_against_oracle(dev, ora, ta, tb, M, N, K):
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((K, M) if ta == "T" else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tb == "T" else (K, N)).astype(np.float32)
    lda, ldb = A.shape[1], B.shape[1]
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    ref = C0.copy()
    ora.sgemm(ta, tb, M, N, K, 0.5, A, lda, B, ldb, 2.0, ref, N)
    C = f(C0)
    dev.sgemm(ta, tb, M, N, K, 0.5, f(A), lda, f(B), ldb, 2.0, C, N)
    np.testing.assert_allclose(C.cpu().numpy(), ref, atol=1e-4, rtol=1e-5)


# ------------------------------------------- grouped GEMM, registered weights
def test_gemm_grouped_equals_individual_calls(dev, ora):
    """gsvk_gemm_grouped_f16 (amx_batch_run's role): independent problems with
    their own shapes and epilogues, each bit-identical to its own gemm_ex call."""
    rng = np.random.default_rng(11)
    shapes = [(64, 1536, 512, 0), (300, 384, 256, 1), (7, 1025, 512, 2), (129, 33, 72, 3)]
    probs, singles = [], []
    for M, N, K, act in shapes:
        a, w = h(rand16(rng, (M, K), 1.0)), h(rand16(rng, (N, K), 0.05))
        bias = f(rng.standard_normal(N).astype(np.float32) * 0.1)
        c1 = torch.empty(M, N, device="cuda")
        c2 = torch.empty(M, N, device="cuda")
        probs.append(dict(a=a, b=w, bias=bias, act=act, slope=0.1, c=c1))
        singles.append((a, w, bias, act, c2))
    dev.gemm_grouped(probs)
    for (a, w, bias, act, c2), p in zip(singles, probs):
        dev.gemm_ex(a, w, bias=bias, act=act, slope=0.1, c=c2)
        assert torch.equal(p["c"], c2)
        ref = ora.linear_f16(ora.f16_to_f32(a.cpu().numpy().view(np.uint16)),
                             w.cpu().numpy().view(np.uint16), bias.cpu().numpy(), act, 0.1)
        assert np.abs(c2.cpu().numpy() - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
    assert dev.device_status() == 0


def test_gemm_grouped_rejects_a_bad_group_before_launching(dev):
    a, w = h(np.zeros((8, 64), np.uint16)), h(np.zeros((16, 64), np.uint16))
    c = torch.full((8, 16), 7.0, device="cuda")
    with pytest.raises(dev.GsvkError):
        dev.gemm_grouped([dict(a=a, b=w, c=c), dict(a=a, b=w)])  # second has no output
    assert torch.all(c == 7.0)  # nothing ran


def test_registered_weights_match_pointer_calls(dev):
    """gsvk_weights_register (amx_pack's role): GEMM and GEMV through the handle
    equal the pointer entry points bit for bit, for host and device sources."""
    rng = np.random.default_rng(12)
    N, K, M = 2048, 512, 64
    w = rand16(rng, (N, K), 0.02)
    x = h(rand16(rng, (M, K), 1.0))
    bias = f(rng.standard_normal(N).astype(np.float32) * 0.01)
    wd = h(w)
    for src in (w, wd):
        reg = dev.Weights(src)
        c1 = torch.empty(M, N, device="cuda")
        c2 = torch.empty(M, N, device="cuda")
        reg.gemm(x, bias=bias, act=dev.ACT_RELU, c=c1)
        dev.gemm_ex(x, wd, bias=bias, act=dev.ACT_RELU, c=c2)
        assert torch.equal(c1, c2)
        xv = torch.randn(K, device="cuda")
        y1 = torch.empty(N, device="cuda")
        reg.gemv(xv, y1)
        y2 = dev.gemv_f16w_f32acc(wd, xv)
        assert torch.equal(y1, y2)
        reg.close()
    assert dev.device_status() == 0


@pytest.mark.parametrize("batch,M,N,K,shared_w", [(16, 128, 2048, 512, False), (5, 100, 300, 72, False),
                                                   (3, 1, 96, 64, True), (4, 257, 130, 136, True)])
def test_gemm_batched_matches_reference(dev, ora, batch, M, N, K, shared_w):
    """gsvk_gemm_f16_batched: independent problems in one launch (strided
    batch), each within the GEMM tolerance of the fp64 reference; the
    residual and fp16 output follow the problem stride."""
    rng = np.random.default_rng(batch * 1000 + M)
    a = h(rand16(rng, (batch, M, K), 1.0))
    w = h(rand16(rng, (N, K) if shared_w else (batch, N, K), 0.05))
    bias = f(rng.standard_normal(N).astype(np.float32) * 0.1)
    res = f(rng.standard_normal((batch, M, N)).astype(np.float32))
    c = torch.empty(batch, M, N, device="cuda")
    c16 = torch.empty(batch, M, N, dtype=torch.float16, device="cuda")
    dev.gemm_batched(a, w, bias=bias, residual=res, act=dev.ACT_RELU, c=c, c_f16=c16)
    an = a.cpu().numpy().view(np.uint16)
    wn = w.cpu().numpy().view(np.uint16)
    for i in range(batch):
        wi = wn if shared_w else wn[i]
        ref = ora.linear_f16(ora.f16_to_f32(an[i]), wi, bias.cpu().numpy(), 1, 0.0) + res[i].cpu().numpy()
        got = c[i].cpu().numpy()
        assert np.abs(got - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max()), f"problem {i}"
        np.testing.assert_array_equal(c16[i].cpu().numpy(), got.astype(np.float16))
    assert dev.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 520, 128), (1024, 768, 512), (517, 2304, 768)])
def test_gemm_pair_kernel_matches_one_sm(dev, ora, M, N, K):
    """The two-SM (cta_group::2) kernel and the one-SM kernel agree within
    the GEMM tolerance of the fp64 reference, on ragged shapes too, with the
    full epilogue (bias, GELU, residual, fp32 and fp16 outputs)."""
    rng = np.random.default_rng(M + N + K)
    a = h(rand16(rng, (M, K), 1.0))
    w = h(rand16(rng, (N, K), 0.05))
    bias = f(rng.standard_normal(N).astype(np.float32) * 0.1)
    res = f(rng.standard_normal((M, N)).astype(np.float32))
    out = {}
    try:
        for mode in (dev.PAIR_NEVER, dev.PAIR_ALWAYS):
            dev.gemm_set_pair(mode)
            c = torch.empty(M, N, device="cuda")
            c16 = torch.empty(M, N, dtype=torch.float16, device="cuda")
            dev.gemm_ex(a, w, bias=bias, residual=res, act=dev.ACT_GELU_ERF, c=c, c_f16=c16)
            out[mode] = (c.cpu().numpy(), c16.cpu().numpy())
    finally:
        dev.gemm_set_pair(dev.PAIR_AUTO)
    ref = ora.linear_f16(ora.f16_to_f32(a.cpu().numpy().view(np.uint16)), w.cpu().numpy().view(np.uint16),
                         bias.cpu().numpy(), dev.ACT_GELU_ERF, 0.0) + res.cpu().numpy()
    for mode, (c, c16) in out.items():
        assert np.abs(c - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max()), f"mode={mode}"
        np.testing.assert_array_equal(c16, c.astype(np.float16))
    assert dev.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(300, 520, 128), (517, 2304, 768), (1000, 776, 256), (260, 1002, 64)])
def test_gemm_pair_bulk_copy_epilogue(dev, ora, M, N, K):
    """A single fp16 output (bias + GELU) or a single fp32 output (bias +
    residual, alpha) leaves the two-SM kernel through swizzled shared-memory
    tiles and TMA bulk stores, which clip at M and N.  Those outputs are
    bit-identical to the same kernel's per-lane stores (taken when both
    outputs are requested) and within the GEMM tolerance of the oracle.
    N = 1002 has row pitches that are not 16-byte multiples: per-lane stores."""
    rng = np.random.default_rng(3 * M + N + K)
    a = h(rand16(rng, (M, K), 1.0))
    w = h(rand16(rng, (N, K), 0.05))
    bias = f(rng.standard_normal(N).astype(np.float32) * 0.1)
    res = f(rng.standard_normal((M, N)).astype(np.float32))
    a_np = ora.f16_to_f32(a.cpu().numpy().view(np.uint16))
    w_np = w.cpu().numpy().view(np.uint16)
    dev.gemm_set_pair(dev.PAIR_ALWAYS)
    try:
        # fp16 output alone vs both outputs
        c16 = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        dev.gemm_ex(a, w, bias=bias, act=dev.ACT_GELU_ERF, c_f16=c16)
        both32 = torch.empty(M, N, device="cuda")
        both16 = torch.empty(M, N, dtype=torch.float16, device="cuda")
        dev.gemm_ex(a, w, bias=bias, act=dev.ACT_GELU_ERF, c=both32, c_f16=both16)
        # fp32 output alone (+ residual, alpha) vs both outputs
        c32 = torch.full((M, N), float("nan"), device="cuda")
        dev.gemm_ex(a, w, bias=bias, residual=res, alpha=0.5, c=c32)
        r32 = torch.empty(M, N, device="cuda")
        r16 = torch.empty(M, N, dtype=torch.float16, device="cuda")
        dev.gemm_ex(a, w, bias=bias, residual=res, alpha=0.5, c=r32, c_f16=r16)
        # fp32 output alone, no residual
        p32 = torch.full((M, N), float("nan"), device="cuda")
        dev.gemm_ex(a, w, c=p32)
        torch.cuda.synchronize()
    finally:
        dev.gemm_set_pair(dev.PAIR_AUTO)
    assert dev.device_status() == 0
    np.testing.assert_array_equal(c16.cpu().numpy(), both16.cpu().numpy())
    np.testing.assert_array_equal(c32.cpu().numpy(), r32.cpu().numpy())
    gelu = ora.linear_f16(a_np, w_np, bias.cpu().numpy(), dev.ACT_GELU_ERF, 0.0)
    assert np.abs(c16.cpu().numpy().astype(np.float32) - gelu).max() <= 1e-2 * max(1.0, np.abs(gelu).max())
    lin = ora.linear_f16(a_np, w_np, None, dev.ACT_NONE, 0.0)
    ref = 0.5 * lin + bias.cpu().numpy() + res.cpu().numpy()
    assert np.abs(c32.cpu().numpy() - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
    assert np.abs(p32.cpu().numpy() - lin).max() <= 1e-4 * max(1.0, np.abs(lin).max())


def test_gemm_uses_pair_follows_the_mode(dev):
    """The kernel query: encoder-sized problems take the two-SM kernel under
    the default rule, few-row and short problems do not; the mode switch
    forces either way (the query launches nothing)."""
    try:
        assert dev.gemm_uses_pair(4096, 1024, 4096) and dev.gemm_uses_pair(8000, 3072, 768)
        assert not dev.gemm_uses_pair(2048, 1024, 1024)  # tile rounds tie, short K
        assert not dev.gemm_uses_pair(64, 4096, 1024)    # few rows: split-K kernel
        assert not dev.gemm_uses_pair(4096, 4096, 1000)  # K not a multiple of 64
        dev.gemm_set_pair(dev.PAIR_ALWAYS)
        assert dev.gemm_uses_pair(2048, 1024, 1024)
        dev.gemm_set_pair(dev.PAIR_NEVER)
        assert not dev.gemm_uses_pair(4096, 1024, 4096)
    finally:
        dev.gemm_set_pair(dev.PAIR_AUTO)


@pytest.mark.parametrize("M,N,K", [(300, 520, 128), (1000, 64, 256), (517, 136, 64), (300, 16, 32),
                                   (4100, 1000, 64), (260, 68, 64)])
def test_one_sm_bulk_copy_epilogue_matches_per_row_stores(dev, M, N, K):
    """The one-SM kernel's bulk-copy epilogue writes the same bits as its
    per-row stores (bias, GELU, residual, fp32 and fp16 outputs; wide and
    narrow tiles, ragged M and N).  N = 68 has an fp16 row pitch that is not a
    16-byte multiple: per-row stores in both runs."""
    rng = np.random.default_rng(M * 5 + N + K)
    a = h(rand16(rng, (M, K), 1.0))
    w = h(rand16(rng, (N, K), 0.05))
    bias = f(rng.standard_normal(N).astype(np.float32) * 0.1)
    res = f(rng.standard_normal((M, N)).astype(np.float32))
    out = {}
    dev.gemm_set_pair(dev.PAIR_NEVER)
    try:
        for bulk in (False, True):
            dev.gemm_set_bulk_epilogue(bulk)
            c = torch.full((M, N), float("nan"), device="cuda")
            c16 = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
            dev.gemm_ex(a, w, bias=bias, residual=res, act=dev.ACT_GELU_ERF, alpha=0.75, c=c, c_f16=c16)
            o16 = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
            dev.gemm_ex(a, w, bias=bias, act=dev.ACT_GELU_ERF, c_f16=o16)
            out[bulk] = (c.cpu().numpy(), c16.cpu().numpy(), o16.cpu().numpy())
    finally:
        dev.gemm_set_bulk_epilogue(True)
        dev.gemm_set_pair(dev.PAIR_AUTO)
    for i in range(3):
        np.testing.assert_array_equal(out[True][i], out[False][i])
    assert np.isfinite(out[True][0]).all()
    assert dev.device_status() == 0


# ------------------------------------------------- a7 gemm_nt_f16w, a11 chains
@pytest.mark.parametrize("T,out_,in_", [(17, 128, 96), (1, 1536, 512), (64, 2048, 512),
                                        (5, 33, 131), (300, 512, 2048)])
def test_gemm_nt_f16w_matches_oracle_sgemm(dev, ora, T, out_, in_):
    """accel::gemm_nt_f16w: bit-identical to the oracle's sgemm on the exactly
    widened weights (one fp32 FMA chain per output in k order), and within
    1e-5 of the row peak of the GEMV rows (test_accel.cpp:120-143)."""
    rng = np.random.default_rng(T * 7 + out_)
    w = (rng.standard_normal((out_, in_), dtype=np.float32) * 0.05).astype(np.float16).view(np.uint16)
    x = rng.standard_normal((T, in_), dtype=np.float32)
    y = dev.gemm_nt_f16w(torch.from_numpy(x).cuda(),
                         torch.from_numpy(w.view(np.float16)).cuda()).cpu().numpy()
    w32 = ora.f16_to_f32(w)
    ref = np.zeros((T, out_), np.float32)
    ora.sgemm("N", "T", T, out_, in_, 1.0, x, in_, w32, in_, 0.0, ref, out_)
    np.testing.assert_array_equal(y, ref)
    for t in range(min(T, 4)):
        row = ora.gemv_f16w_f32acc(w, x[t])
        assert np.abs(y[t] - row).max() <= 1e-5 * np.abs(row).max()


def test_gemm_chain_matches_links_one_by_one(dev):
    """amx_chain_run analogue: three chains of four links, each link reading
    the fp16 output of the link before it, listed out of order: the chain
    submission gives the same bits as calling the links in order."""
    M, N, K = 48, 128, 128
    rng = np.random.default_rng(3)
    a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda().half()
    ws = [torch.from_numpy(rng.standard_normal((N, K), dtype=np.float32) * 0.08).cuda().half()
          for _ in range(4)]

    def build():
        acts = [[torch.empty(M, N, dtype=torch.float16, device="cuda") for _ in range(4)]
                for _ in range(3)]
        outs = [[torch.empty(M, N, device="cuda") for _ in range(4)] for _ in range(3)]
        links = []
        for d in (3, 1, 0, 2):
            for c in range(3):
                links.append((c, d, dict(a=a if d == 0 else acts[c][d - 1], b=ws[d],
                                          act=dev.ACT_RELU if c == 1 else dev.ACT_NONE,
                                          c=outs[c][d], c_f16=acts[c][d])))
        return links, outs

    links, outs = build()
    dev.gemm_chain_run(links)
    ref_links, ref_outs = build()
    for c, d, g in sorted(ref_links, key=lambda t: (t[0], t[1])):
        dev.gemm_ex(**g)
    torch.cuda.synchronize()
    for c in range(3):
        for d in range(4):
            assert torch.equal(outs[c][d], ref_outs[c][d]), (c, d)
    with pytest.raises(dev.GsvkError):
        dev.gemm_chain_run([links[0], links[0]])
