"""CPU tests of the oracle itself: it must agree with an independent fp64
product (numpy), reproduce the reference's known-answer vector, and catch a
planted error.  Pins against the reference's own cuBLAS build live in
test_golden.py (fixtures made on a GPU box by tests/golden/make_golden.py)."""
import numpy as np
import pytest

from oracle import oracle

RNG = np.random.default_rng(1234)


def _rand(*shape):
    return RNG.standard_normal(shape).astype(np.float32)


def test_readme_known_answer():
    # README.md:41-55: [[1,2,3],[4,5,6]] x [[1..4],[5..8],[9..12]] (M=2, K=3, N=4)
    a = np.array([1, 2, 3, 4, 5, 6], np.float32).reshape(2, 3)
    b = np.arange(1, 13, dtype=np.float32).reshape(3, 4)
    c = oracle.gemm_f64(a, b)
    assert c.tolist() == [[38, 44, 50, 56], [83, 98, 113, 128]]


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (17, 33, 31), (64, 10, 129), (5, 128, 3)])
def test_gemm_matches_numpy_f64(ta, tb, M, N, K):
    A = _rand(K, M) if ta else _rand(M, K)
    B = _rand(N, K) if tb else _rand(K, N)
    opA = A.astype(np.float64).T if ta else A.astype(np.float64)
    opB = B.astype(np.float64).T if tb else B.astype(np.float64)
    ref = opA @ opB
    got = oracle.gemm_f64(A, B, transA=bool(ta), transB=bool(tb))
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


def test_gemm_non_finite_operands_follow_ieee():
    """The oracle's sequential fp64 sum gives the IEEE class of every element
    for Inf / NaN operands (the reference the non-finite GPU tests compare
    with), checked against an element-by-element fp64 sum in Python."""
    A = _rand(9, 12)
    B = _rand(12, 7)
    A[2, 3], A[4, 5], A[6, 1] = np.inf, -np.inf, np.nan
    B[3, 2], B[8, 6] = -np.inf, np.nan
    B[5, 4] = 0.0  # -Inf * 0 = NaN in row 4
    got = oracle.gemm_f64(A, B)
    exp = np.empty((9, 7))
    with np.errstate(invalid="ignore", over="ignore"):
        for i in range(9):
            for j in range(7):
                acc = 0.0
                for k in range(12):
                    acc += float(A[i, k]) * float(B[k, j])
                exp[i, j] = acc
    for cls in (np.isnan, np.isposinf, np.isneginf):
        np.testing.assert_array_equal(cls(got), cls(exp))
    fin = np.isfinite(exp)
    np.testing.assert_allclose(got[fin], exp[fin], rtol=1e-12, atol=1e-12)
    assert np.isnan(got[4, 4]) and np.isnan(got[6]).all() and np.isinf(got[2, 0])


def test_gemm_batch_bias_relu_rows():
    A = _rand(3, 20, 7)
    B = _rand(3, 7, 9)
    bias = _rand(9)
    ref = np.maximum(A.astype(np.float64) @ B.astype(np.float64) + bias, 0)
    got = oracle.gemm_f64(A, B, bias=bias, relu=True)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)
    rows = [0, 19, 5]
    sub = oracle.gemm_f64(A, B, bias=bias, relu=True, rows=rows)
    np.testing.assert_allclose(sub, ref[:, rows, :], rtol=1e-12, atol=1e-12)


def test_linear_layout_matches_reference_semantics():
    # launch_linear: out[B, out_f] = x[B, in_f] . w[out_f, in_f]^T + bias  (matmul.cu:54-67)
    x, w, b = _rand(6, 5), _rand(4, 5), _rand(4)
    got = oracle.gemm_f64(x, w, transB=True, bias=b)
    np.testing.assert_allclose(got, x.astype(np.float64) @ w.astype(np.float64).T + b, rtol=1e-12)


def test_metric_zero_on_exact_and_detects_planted_error():
    A, B = _rand(32, 16), _rand(16, 24)
    ref = oracle.gemm_f64(A, B)
    exact = ref.astype(np.float32)
    e, _ = oracle.max_rel_err(A, B, exact, ref)
    assert e < 1e-7  # only the final fp32 rounding
    planted = exact.copy()
    planted[7, 11] += 1e-3 * np.linalg.norm(A[7]) * np.linalg.norm(B[:, 11])
    e2, where = oracle.max_rel_err(A, B, planted, ref)
    assert e2 > 9e-4 and where == (0, 7, 11)
    nan = exact.copy()
    nan[3, 3] = np.nan
    assert oracle.max_rel_err(A, B, nan, ref)[0] == np.inf


def test_metric_on_rows_and_batches():
    A, B = _rand(2, 40, 8), _rand(2, 8, 12)
    rows = [3, 39]
    ref = oracle.gemm_f64(A, B, rows=rows)
    full = (A.astype(np.float64) @ B.astype(np.float64)).astype(np.float32)
    e, _ = oracle.max_rel_err(A, B, full, ref, rows=rows)
    assert e < 1e-7
    full[1, 39, 0] += 1.0
    e2, where = oracle.max_rel_err(A, B, full, ref, rows=rows)
    assert where == (1, 39, 0) and e2 > 1e-2


def test_cpu_baseline_loop():
    A, B = _rand(33, 17), _rand(17, 29)
    C = np.zeros((33, 29), np.float32)
    used = oracle.sgemm_f32_cpu(A, B, C, threads=2)
    assert used >= 1
    ref = oracle.gemm_f64(A, B)
    e, _ = oracle.max_rel_err(A, B, C, ref)
    assert e < 1e-6
    C2 = np.zeros_like(C)
    oracle.sgemm_f32_cpu(A, B, C2, row0=10, nrows=5)
    np.testing.assert_array_equal(C2[10:15], C[10:15])
    assert not C2[:10].any() and not C2[15:].any()


def test_mlp_oracle_against_finite_differences():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((4, 6))
    ws = [rng.standard_normal((5, 6)), rng.standard_normal((3, 5))]
    bs = [rng.standard_normal(5), rng.standard_normal(3)]
    out = oracle.mlp_forward_backward(x, ws, bs)

    def loss(ws_, bs_):
        return oracle.mlp_forward_backward(x, ws_, bs_)["y"].sum()

    eps = 1e-6
    for l in range(2):
        for idx in [(0, 0), (1, 2), (2, 4)]:
            if idx[0] >= ws[l].shape[0]:
                continue
            wp = [w.copy() for w in ws]
            wp[l][idx] += eps
            wm = [w.copy() for w in ws]
            wm[l][idx] -= eps
            fd = (loss(wp, bs) - loss(wm, bs)) / (2 * eps)
            assert abs(fd - out["dW"][l][idx]) < 1e-5 * max(1, abs(fd))
        bp = [b.copy() for b in bs]
        bp[l][0] += eps
        bm = [b.copy() for b in bs]
        bm[l][0] -= eps
        fd = (loss(ws, bp) - loss(ws, bm)) / (2 * eps)
        assert abs(fd - out["db"][l][0]) < 1e-5 * max(1, abs(fd))
