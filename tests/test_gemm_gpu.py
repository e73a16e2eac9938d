"""Parity of the sm_100a GEMM kernels with the fp64 oracle, through the C ABI.

Tolerance (the path's stated bound): for every checked element
    |C - C_ref| / (||op(A)_i,:|| * ||op(B)_:,j|| + |bias_j|) <= 2e-6
with C_ref the fp64-accumulated product of the same fp32 inputs.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle

TOL = 2e-6

pytestmark = pytest.mark.gpu


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _check(A, B, C, *, ta=False, tb=False, bias=None, relu=False, rows=None, tol=TOL):
    ref = oracle.gemm_f64(A, B, transA=ta, transB=tb, bias=bias, relu=relu, rows=rows)
    err, where = oracle.max_rel_err(A, B, C, ref, transA=ta, transB=tb, bias=bias, rows=rows)
    assert err <= tol, f"max rel err {err:.3e} at {where}"
    return err


def _rand(rng, *shape, dist="normal"):
    if dist == "uniform":
        return (rng.random(shape, dtype=np.float32) * 2 - 1).astype(np.float32)
    return rng.standard_normal(shape, dtype=np.float32)


@pytest.fixture(scope="module")
def jst():
    import jstorch_b200
    jstorch_b200.load()
    return jstorch_b200


KERNELS = ["ffma", "tc3xtf32"]


def test_readme_known_answer_through_host_matmul(jst):
    # README.md:41-55: torch.matmul(a, b, 2, 3, 4) -> [38, 44, 50, 56, 83, 98, 113, 128]
    a = np.array([1, 2, 3, 4, 5, 6], np.float32)
    b = np.arange(1, 13, dtype=np.float32)
    c = jst.torch.matmul(a, b, 2, 3, 4)
    assert c.dtype == np.float32 and c.tolist() == [38, 44, 50, 56, 83, 98, 113, 128]


@pytest.mark.parametrize("kernel", KERNELS)
def test_readme_known_answer_each_kernel(jst, kernel):
    a = _dev(np.array([[1, 2, 3], [4, 5, 6]], np.float32))
    b = _dev(np.arange(1, 13, dtype=np.float32).reshape(3, 4))
    c = jst.gemm(a, b, kernel=kernel).cpu().numpy()
    assert c.tolist() == [[38, 44, 50, 56], [83, 98, 113, 128]]


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (3, 17, 31), (33, 127, 129), (128, 256, 64), (129, 257, 65),
                                   (200, 300, 1000), (512, 512, 512)])
def test_layouts_odd_shapes(jst, kernel, ta, tb, M, N, K):
    rng = np.random.default_rng(M * 131 + N * 7 + K + 1000 * ta + 2000 * tb)
    A = _rand(rng, K, M) if ta else _rand(rng, M, K)
    B = _rand(rng, N, K) if tb else _rand(rng, K, N)
    a, b = _dev(A), _dev(B)
    av = a.t() if ta else a  # transposed views reach the kernels as TN / NT operands
    bv = b.t() if tb else b
    C = jst.gemm(av, bv, kernel=kernel).cpu().numpy()
    _check(A, B, C, ta=bool(ta), tb=bool(tb))


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("relu", [False, True])
def test_bias_relu_epilogue(jst, kernel, relu):
    rng = np.random.default_rng(5)
    X, W, b = _rand(rng, 300, 200), _rand(rng, 130, 200), _rand(rng, 130)
    C = jst.gemm(_dev(X), _dev(W).t(), bias=_dev(b), relu=relu, kernel=kernel).cpu().numpy()
    _check(X, W, C, tb=True, bias=b, relu=relu)
    if relu:
        assert (C >= 0).all()


@pytest.mark.parametrize("kernel", KERNELS)
def test_strided_batched(jst, kernel):
    rng = np.random.default_rng(9)
    A, B = _rand(rng, 5, 70, 40), _rand(rng, 5, 40, 90)
    C = jst.gemm(_dev(A), _dev(B), kernel=kernel).cpu().numpy()
    _check(A, B, C)


@pytest.mark.parametrize("kernel", KERNELS)
def test_leading_dimension_and_unaligned_views(jst, kernel):
    import torch
    rng = np.random.default_rng(11)
    big = _rand(rng, 100, 75)          # ld 75: not a multiple of 4
    A = big[3:90, 1:70]                # unaligned base, ld 75
    B = _rand(rng, 69, 50)
    a = _dev(big)[3:90, 1:70]
    C = jst.gemm(a, _dev(B), kernel=kernel).cpu().numpy()
    _check(np.ascontiguousarray(A), B, C)
    assert a.stride() == (75, 1)
    torch.cuda.synchronize()


@pytest.mark.parametrize("kernel", KERNELS)
def test_k_zero_and_empty(jst, kernel):
    import torch
    a = torch.empty((4, 0), device="cuda")
    b = torch.empty((0, 6), device="cuda")
    bias = _dev(np.arange(6, dtype=np.float32) - 2)
    c = jst.gemm(a, b, bias=bias, relu=True, kernel=kernel).cpu().numpy()
    assert c.tolist() == [[0, 0, 0, 1, 2, 3]] * 4
    e = jst.gemm(torch.empty((0, 5), device="cuda"), torch.zeros((5, 3), device="cuda"), kernel=kernel)
    assert e.shape == (0, 3)


def test_reference_launchers(jst):
    """launch_matmul / launch_bmm / launch_linear keep the reference signatures
    (native/ops/matmul.cu:28,40,54) and results."""
    import torch
    lib = jst.load()
    rng = np.random.default_rng(3)
    A, B = _rand(rng, 96, 80), _rand(rng, 80, 112)
    a, b = _dev(A), _dev(B)
    c = torch.empty((96, 112), device="cuda")
    lib.launch_matmul(a.data_ptr(), b.data_ptr(), c.data_ptr(), 96, 80, 112, None)
    assert lib.jst_get_last_status() == 0
    _check(A, B, c.cpu().numpy())

    A3, B3 = _rand(rng, 4, 33, 20), _rand(rng, 4, 20, 45)
    a3, b3 = _dev(A3), _dev(B3)  # keep the device tensors alive across the async launch
    c3 = torch.empty((4, 33, 45), device="cuda")
    lib.launch_bmm(a3.data_ptr(), b3.data_ptr(), c3.data_ptr(), 4, 33, 20, 45, None)
    assert lib.jst_get_last_status() == 0
    _check(A3, B3, c3.cpu().numpy())

    X, W, bias = _rand(rng, 256, 784), _rand(rng, 1024, 784), _rand(rng, 1024)
    y = torch.empty((256, 1024), device="cuda")
    x_d, w_d, b_d = _dev(X), _dev(W), _dev(bias)
    lib.launch_linear(x_d.data_ptr(), w_d.data_ptr(), b_d.data_ptr(), y.data_ptr(), 256, 784, 1024, None)
    assert lib.jst_get_last_status() == 0
    _check(X, W, y.cpu().numpy(), tb=True, bias=bias)
    lib.launch_linear(x_d.data_ptr(), w_d.data_ptr(), None, y.data_ptr(), 256, 784, 1024, None)
    _check(X, W, y.cpu().numpy(), tb=True)
    assert jst.device_error() == 0


def test_host_matmul_config1(jst):
    """Config 1: 512^3 through torch.matmul(a, b, 512, 512, 512) on host arrays."""
    from jstorch_b200 import synth
    A, B = synth.config1()
    C = jst.torch.matmul(A.reshape(-1), B.reshape(-1), 512, 512, 512).reshape(512, 512)
    _check(A, B, C)


def test_config3_sampled_rows(jst):
    """Config 3 (8192^3, N(0,1)): both kernels, 96 sampled rows x all columns."""
    import torch
    from jstorch_b200 import synth
    A, B = synth.config3()
    a, b = _dev(A), _dev(B)
    rows = np.sort(np.random.default_rng(0).choice(8192, 96, replace=False)).astype(np.int32)
    rows[0], rows[-1] = 0, 8191
    ref = oracle.gemm_f64(A, B, rows=rows)
    for kernel in KERNELS:
        c = jst.gemm(a, b, kernel=kernel)
        C = c[torch.from_numpy(rows).long().cuda()].cpu().numpy()
        full = np.zeros((8192, 8192), np.float32)
        full[rows] = C
        err, where = oracle.max_rel_err(A, B, full, ref, rows=rows)
        assert err <= TOL, (kernel, err, where)
        del c
    assert jst.device_error() == 0


def test_config4_batched_attention_shapes(jst):
    from jstorch_b200 import synth
    q, kt, p, v = synth.config4()
    for kernel in KERNELS:
        s = jst.gemm(_dev(q), _dev(kt), kernel=kernel).cpu().numpy()
        _check(q, kt, s)
        o = jst.gemm(_dev(p), _dev(v), kernel=kernel).cpu().numpy()
        _check(p, v, o)


def test_kernel_choice_heuristic(jst):
    assert jst.select_kernel(8192, 8192, 8192) == "tc3xtf32"
    assert jst.select_kernel(2048, 2048, 2048) == "tc3xtf32"
    assert jst.select_kernel(512, 64, 512, batch=64) == "tc3xtf32"
    assert jst.select_kernel(512, 512, 512) == "ffma"
    assert jst.select_kernel(256, 1024, 784) == "ffma"
    assert jst.select_kernel(256, 10, 1024) == "ffma"
    assert jst.select_kernel(2, 4, 3) == "ffma"
    # a narrow side of 16..63 goes to the tensor cores once the product is large
    assert jst.select_kernel(32, 3136, 2304, batch=32) == "tc3xtf32"
    assert jst.select_kernel(4096, 48, 8192, batch=8) == "tc3xtf32"
    assert jst.select_kernel(32, 3136, 2304) == "ffma"
    assert jst.select_kernel(8, 3136, 2304, batch=64) == "ffma"


@pytest.mark.parametrize("pinned", [False, True])
def test_host_matmul_pipelined_chunks(jst, pinned):
    """Large host-array products take the blocked path (H2D of A row blocks
    and B column panels, block GEMMs, D2H of C blocks, overlapped on three
    streams); ragged last blocks in both directions and both pageable and
    pinned host buffers must give the same product."""
    import torch
    rng = np.random.default_rng(21)
    M, K, N = 2500, 300, 2300  # 3 x 3 blocks: rows 1024, 1024, 452; columns 1024, 1024, 252
    assert jst.select_kernel(M, N, K) == "tc3xtf32"  # the pipelined path is the tensor-core one
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32)
    if pinned:
        a_h = torch.from_numpy(A).pin_memory()
        b_h = torch.from_numpy(B).pin_memory()
        c_h = torch.full((M, N), float("nan")).pin_memory()
        from jstorch_b200.gemm import matmul_host_ptr
        matmul_host_ptr(a_h.data_ptr(), b_h.data_ptr(), c_h.data_ptr(), M, K, N)
        C = c_h.numpy()
    else:
        C = jst.torch.matmul(A, B, M, K, N).reshape(M, N)
    rows = np.array([0, 1, 1023, 1024, 2047, 2048, 2499], np.int32)
    ref = oracle.gemm_f64(A, B, rows=rows)
    err, where = oracle.max_rel_err(A, B, C, ref, rows=rows)
    assert err <= TOL, (err, where)
    assert np.isfinite(C).all()


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False)])
@pytest.mark.parametrize("M,N,K,batch", [(256, 1024, 1024, 1), (256, 10, 1024, 1), (10, 1024, 256, 1),
                                         (512, 512, 512, 1), (100, 70, 999, 3), (64, 64, 130, 1)])
def test_ffma_split_k(jst, ta, tb, M, N, K, batch):
    """Shapes whose 64 x 64 tiles cannot fill the SMs run with K split into
    slices and a fixed-order reduce: checked against the oracle with the
    bias + ReLU epilogue, and bit-identical from run to run."""
    import torch
    rng = np.random.default_rng(M + 3 * N + 7 * K + batch)
    A = _rand(rng, batch, M, K)
    B = _rand(rng, batch, K, N)
    bias = _rand(rng, N)
    a = _dev(np.ascontiguousarray(A.transpose(0, 2, 1))).transpose(1, 2) if ta else _dev(A)
    b = _dev(np.ascontiguousarray(B.transpose(0, 2, 1))).transpose(1, 2) if tb else _dev(B)
    if batch == 1:
        a, b = a[0], b[0]
    c1 = jst.gemm(a, b, bias=_dev(bias), relu=True, kernel="ffma")
    c2 = jst.gemm(a, b, bias=_dev(bias), relu=True, kernel="ffma")
    torch.cuda.synchronize()
    C1 = c1.cpu().numpy().reshape(batch, M, N)
    np.testing.assert_array_equal(C1, c2.cpu().numpy().reshape(batch, M, N))
    for i in range(batch):
        _check(A[i], B[i], C1[i], bias=bias, relu=True)


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("M,N,K,batch", [(300, 520, 96, 1), (64, 4096, 576, 3), (256, 1024, 1024, 1)])
def test_row_bias_epilogue(jst, kernel, relu, M, N, K, batch):
    """bias[i] per row (JST_EPI_BIAS_ROW*), the convolution bias layout, incl. split-K and batches."""
    import torch
    rng = np.random.default_rng(M + N + K + relu)
    A = _rand(rng, batch, M, K)
    B = _rand(rng, batch, K, N)
    rb = _rand(rng, M)
    a, b = (_dev(A), _dev(B)) if batch > 1 else (_dev(A[0]), _dev(B[0]))
    c = jst.gemm(a, b, row_bias=_dev(rb), relu=relu, kernel=kernel)
    plain = jst.gemm(a, b, kernel=kernel)
    torch.cuda.synchronize()
    C = c.cpu().numpy().reshape(batch, M, N)
    P = plain.cpu().numpy().reshape(batch, M, N) + rb[None, :, None]
    np.testing.assert_array_equal(C, np.maximum(P, 0) if relu else P)


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False)])
@pytest.mark.parametrize("M,N,K,batch", [(256, 2304, 8192, 1), (128, 300, 20000, 1), (200, 256, 4100, 2)])
def test_tc_split_k(jst, ta, tb, M, N, K, batch):
    """Tensor-core GEMMs with few output tiles and a long K run split into
    K slices plus the fixed-order reduce: bias + ReLU epilogue, oracle bound,
    bit-identical reruns."""
    import torch
    rng = np.random.default_rng(M + N + K + batch + 2 * ta + tb)
    A = _rand(rng, batch, M, K)
    B = _rand(rng, batch, K, N)
    bias = _rand(rng, N)
    a = _dev(np.ascontiguousarray(A.transpose(0, 2, 1))).transpose(1, 2) if ta else _dev(A)
    b = _dev(np.ascontiguousarray(B.transpose(0, 2, 1))).transpose(1, 2) if tb else _dev(B)
    if batch == 1:
        a, b = a[0], b[0]
    c1 = jst.gemm(a, b, bias=_dev(bias), relu=True, kernel="tc3xtf32")
    c2 = jst.gemm(a, b, bias=_dev(bias), relu=True, kernel="tc3xtf32")
    torch.cuda.synchronize()
    C1 = c1.cpu().numpy().reshape(batch, M, N)
    np.testing.assert_array_equal(C1, c2.cpu().numpy().reshape(batch, M, N))
    rows = np.arange(0, M, 7)
    for i in range(batch):
        _check(A[i], B[i], C1[i], bias=bias, relu=True, rows=rows)


@pytest.mark.parametrize("kernel", KERNELS)
def test_broadcast_operand(jst, kernel):
    """A batch stride of 0 (one operand shared by the whole batch, as the
    convolution weights) through jst_gemm_ex."""
    import torch
    rng = np.random.default_rng(17)
    M, N, K, batch = 256, 1024, 576, 6
    W = _rand(rng, M, K)
    X = _rand(rng, batch, K, N)
    w, x = _dev(W), _dev(X)
    c = torch.empty((batch, M, N), device="cuda")
    d = _lib_desc(w, x, c, M, N, K, batch, strideA=0, strideB=K * N, kernel=kernel)
    jst._lib.check(jst._lib.load().jst_gemm_ex(ctypes.byref(d)))
    torch.cuda.synchronize()
    C = c.cpu().numpy()
    for i in range(batch):
        _check(W, X[i], C[i])
    W2 = _rand(rng, batch, K, M)  # B broadcast, A transposed per batch
    d = _lib_desc(_dev(W2), _dev(X[0]), c, M, N, K, batch, strideA=K * M, strideB=0, transA=1, lda=M, kernel=kernel)
    jst._lib.check(jst._lib.load().jst_gemm_ex(ctypes.byref(d)))
    torch.cuda.synchronize()
    C = c.cpu().numpy()
    for i in range(batch):
        _check(W2[i], X[0], C[i], ta=True)


def _lib_desc(a, b, c, M, N, K, batch, *, strideA, strideB, transA=0, lda=None, kernel="auto"):
    from jstorch_b200 import _lib
    d = _lib.GemmDesc()
    _lib.load().jst_gemm_desc_init(ctypes.byref(d), M, N, K, a.data_ptr(), b.data_ptr(), c.data_ptr())
    d.batch = batch
    d.transA = transA
    if lda is not None:
        d.lda = lda
    d.strideA, d.strideB, d.strideC = strideA, strideB, M * N
    d.kernel = _lib.KERNELS[kernel]
    return d


@pytest.mark.parametrize("M,N,K,batch,bcast", [
    (512, 64, 512, 8, False),     # narrow tile (64), config 4's output GEMM shape
    (300, 100, 97, 2, False),     # 128-wide tile, ragged M / N / K
    (512, 512, 64, 4, False),     # short K: 128-wide tile, config 4's scores shape
    (256, 64, 40000, 1, False),   # narrow tile with split-K
    (384, 128, 256, 5, True),     # broadcast A
])
def test_in_kernel_a_split_matches_plane_path(jst, M, N, K, batch, bcast):
    """Narrow tiles split K-major A inside the kernel.  A 16-byte-misaligned
    copy of A cannot be loaded that way and goes through the split pass: both
    must give bit-identical C, and both meet the oracle bound."""
    import torch
    from jstorch_b200 import _lib
    rng = np.random.default_rng(M + N + K)
    A = _rand(rng, 1 if bcast else batch, M, K)
    B = _rand(rng, batch, K, N)
    c_fast = torch.empty((batch, M, N), device="cuda")
    c_ref = torch.empty((batch, M, N), device="cuda")
    a_al = _dev(A)
    buf = torch.empty(A.size + 1, device="cuda")
    a_mis = buf[1:].view(A.shape)  # base 4 bytes past a 16-byte boundary
    a_mis.copy_(a_al)
    b = _dev(B)
    for a, c in ((a_al, c_fast), (a_mis, c_ref)):
        d = _lib.GemmDesc()
        _lib.load().jst_gemm_desc_init(ctypes.byref(d), M, N, K, a.data_ptr(), b.data_ptr(), c.data_ptr())
        d.batch = batch
        d.strideA, d.strideB, d.strideC = (0 if bcast else M * K), K * N, M * N
        d.kernel = _lib.KERNEL_TC3XTF32
        _lib.check(_lib.load().jst_gemm_ex(ctypes.byref(d)))
    torch.cuda.synchronize()
    C = c_fast.cpu().numpy()
    np.testing.assert_array_equal(C, c_ref.cpu().numpy())
    for i in range(batch):
        _check(A[0 if bcast else i], B[i], C[i], rows=np.arange(0, M, 5))


def _non_finite_operands(rng, M, N, K):
    A = _rand(rng, M, K)
    B = _rand(rng, K, N)
    A[3, 5], A[7, 11], A[9, 2] = np.inf, -np.inf, np.nan
    B[4, 13], B[6, N - 1] = np.inf, np.nan
    return A, B


def _check_non_finite(A, B, C):
    """Every element has the IEEE class of the exact product (the oracle's
    sequential fp64 sum over the same fp32 inputs): +Inf, -Inf and NaN where
    it has them; the elements whose row of A and column of B are all finite
    keep the path's bound."""
    ref = oracle.gemm_f64(A, B)
    for cls in (np.isnan, np.isposinf, np.isneginf):
        np.testing.assert_array_equal(cls(C), cls(ref))
    r = np.flatnonzero(np.isfinite(A).all(axis=1))
    c = np.flatnonzero(np.isfinite(B).all(axis=0))
    _check(A[r], B[:, c], C[np.ix_(r, c)], rows=np.arange(0, r.size, 3))


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("M,N,K", [
    (512, 1024, 512),   # 128 x 256 tile, operands split by the split passes
    (256, 64, 512),     # narrow tile, A split inside the kernel
    (128, 300, 20000),  # split-K slices and the reduce
])
def test_non_finite_operands(jst, kernel, M, N, K):
    """Inf and NaN operands (matmul.cu:11-37: cuBLAS fp32 GEMM, whose
    products and sums follow IEEE): a row of A holding +-Inf gives +-Inf by
    the signs of the matching row of B, NaN gives NaN, and an infinite row
    meeting an infinite column of the opposite sign gives NaN.  The 3xTF32
    cross terms of an infinite operand are Inf * 0 = NaN; the kernel returns
    the hi * hi accumulator wherever that is non-finite."""
    import torch
    rng = np.random.default_rng(M + N + K)
    A, B = _non_finite_operands(rng, M, N, K)
    c = jst.gemm(_dev(A), _dev(B), kernel=kernel)
    torch.cuda.synchronize()
    _check_non_finite(A, B, c.cpu().numpy())


def test_non_finite_operands_host_pipeline(jst):
    """The same through torch.matmul on host arrays (the blocked, pipelined
    tensor-core path)."""
    rng = np.random.default_rng(5)
    M, K, N = 2500, 300, 2300
    assert jst.select_kernel(M, N, K) == "tc3xtf32"
    A, B = _non_finite_operands(rng, M, N, K)
    A[2400, 7] = np.inf  # in the ragged last row block
    _check_non_finite(A, B, jst.torch.matmul(A, B, M, K, N).reshape(M, N))


@pytest.mark.parametrize("kernel,M,N,K", [
    ("ffma", 256, 1024, 1024),     # FFMA with split-K and the reduce
    ("tc3xtf32", 1024, 1024, 1024),  # operand splits, then the tensor-core kernel
    ("tc3xtf32", 256, 512, 4096),  # tensor cores with split-K and the reduce
])
def test_operands_written_by_the_previous_kernel(jst, kernel, M, N, K):
    """A GEMM queued right behind kernels that write its operands, and
    followed at once by a kernel that reads C, with no synchronisation in
    between: every launch of the path that is a programmatic dependent waits
    for the previous grid, so each product sees the values just written."""
    import torch
    a = torch.empty((M, K), device="cuda")
    b = torch.empty((K, N), device="cuda")
    c = torch.empty((M, N), device="cuda")
    checks = []
    for v in (1.0, 2.0, 3.0, 4.0):
        a.fill_(v)
        b.fill_(0.5)
        jst.gemm(a, b, out=c, kernel=kernel)
        checks.append((c == v * 0.5 * K).all())  # exact: every product and sum is representable
    assert all(bool(x) for x in checks)


@pytest.mark.parametrize("M,N,K,batch", [(20, 5000, 1000, 48), (3000, 40, 2000, 24)])
def test_narrow_side_on_tensor_cores_matches_oracle(jst, M, N, K, batch):
    """A narrow M or N (16..63) with a large product runs on the tensor-core
    kernel with a partly filled tile; every element is checked."""
    import torch
    assert jst.select_kernel(M, N, K, batch=batch) == "tc3xtf32"
    rng = np.random.default_rng(M + N)
    A = rng.standard_normal((batch, M, K), dtype=np.float32)
    B = rng.standard_normal((batch, K, N), dtype=np.float32)
    c = jst.gemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    err, where = oracle.max_rel_err(A, B, c.cpu().numpy(), oracle.gemm_f64(A, B))
    assert err <= TOL, (err, where)


def _gemm_desc(a, b, c, M, N, K, batch, *, ta=False, tb=False, sa=None, sb=None, ldc=None, sc=None):
    from jstorch_b200 import _lib
    d = _lib.GemmDesc()
    _lib.load().jst_gemm_desc_init(ctypes.byref(d), M, N, K, a.data_ptr(), b.data_ptr(), c.data_ptr())
    d.transA, d.transB = int(ta), int(tb)
    d.lda = M if ta else K
    d.ldb = K if tb else N
    d.ldc = ldc if ldc is not None else N
    d.batch = batch
    d.strideA = M * K if sa is None else sa
    d.strideB = K * N if sb is None else sb
    d.strideC = M * d.ldc if sc is None else sc
    d.kernel = _lib.KERNEL_TC3XTF32
    return d


@pytest.mark.parametrize("M,N,K,batch,ta,tb,bcast_a", [
    (512, 512, 64, 64, False, False, False),    # config 4 scores: 1024 tiles of 128 x 128, K = 4 slabs
    (512, 64, 512, 80, False, False, False),    # config 4's output shape, 320 tiles of 128 x 64
    (300, 100, 97, 100, False, False, False),   # ragged M / N / K, 128-wide tiles
    (1000, 60, 333, 40, False, False, False),   # ragged, 64-wide tiles
    (256, 128, 200, 150, True, False, False),   # A stored [K, M]: A planes from the split pass
    (384, 96, 130, 100, False, True, False),    # B stored [N, K]
    (128, 128, 288, 300, False, False, True),   # broadcast A (a convolution's weights)
    (512, 128, 3, 100, False, False, False),    # K below one 16-wide k-slab (zero-filled tail)
])
def test_persistent_narrow_tiles_match_one_tile_kernel(jst, M, N, K, batch, ta, tb, bcast_a):
    """At least one narrow output tile per SM runs the persistent kernel (one
    CTA per SM walking tiles, double-buffered accumulators).  One batch entry
    alone has too few tiles for it and runs the one-tile-per-CTA kernel: both
    do the same arithmetic, so C must match bit for bit; and the batched
    result meets the oracle bound."""
    import torch
    from jstorch_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(M * 3 + N + K)
    A = _rand(rng, 1 if bcast_a else batch, *((K, M) if ta else (M, K)))
    B = _rand(rng, batch, *((N, K) if tb else (K, N)))
    a, b = _dev(A), _dev(B)
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    d = _gemm_desc(a, b, c, M, N, K, batch, ta=ta, tb=tb, sa=0 if bcast_a else None)
    _lib.check(lib.jst_gemm_ex(ctypes.byref(d)))
    for i in (0, batch // 2, batch - 1):  # one entry at a time: the one-tile kernel
        ci = torch.full((1, M, N), float("nan"), device="cuda")
        ai = a[0 if bcast_a else i:(0 if bcast_a else i) + 1]
        di = _gemm_desc(ai, b[i:i + 1], ci, M, N, K, 1, ta=ta, tb=tb)
        _lib.check(lib.jst_gemm_ex(ctypes.byref(di)))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(c[i].cpu().numpy(), ci[0].cpu().numpy())
    C = c.cpu().numpy()
    assert np.isfinite(C).all()
    for i in range(0, batch, max(1, batch // 6)):
        _check(A[0 if bcast_a else i], B[i], C[i], ta=ta, tb=tb, rows=np.arange(0, M, 7))


@pytest.mark.parametrize("epi", ["bias_relu", "row_bias", "mask"])
def test_persistent_narrow_tiles_epilogues(jst, epi):
    import torch
    from jstorch_b200 import _lib
    lib = _lib.load()
    M, N, K, batch = 260, 120, 72, 100
    rng = np.random.default_rng(7)
    A, B = _rand(rng, batch, M, K), _rand(rng, batch, K, N)
    a, b = _dev(A), _dev(B)
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    d = _gemm_desc(a, b, c, M, N, K, batch)
    if epi == "bias_relu":
        bias = _rand(rng, N)
        db = _dev(bias)
        d.bias, d.epilogue = db.data_ptr(), _lib.EPI_BIAS | _lib.EPI_RELU
    elif epi == "row_bias":
        bias = _rand(rng, M)
        db = _dev(bias)
        d.bias, d.epilogue = db.data_ptr(), 8  # JST_EPI_BIAS_ROW
    else:
        aux = _rand(rng, batch, M, N)
        daux = _dev(aux)
        d.aux, d.ld_aux, d.stride_aux, d.epilogue = daux.data_ptr(), N, M * N, 4  # JST_EPI_MASK
    _lib.check(lib.jst_gemm_ex(ctypes.byref(d)))
    torch.cuda.synchronize()
    C = c.cpu().numpy().astype(np.float64)
    for i in (0, 17, batch - 1):
        ref = oracle.gemm_f64(A[i], B[i])
        if epi == "bias_relu":
            ref = np.maximum(ref + bias[None, :], 0.0)
            err, w = oracle.max_rel_err(A[i], B[i], C[i], ref, bias=bias)
        elif epi == "row_bias":
            ref = ref + bias[:, None]
            mag = np.sqrt(np.square(A[i].astype(np.float64)).sum(1))[:, None] * \
                np.sqrt(np.square(B[i].astype(np.float64)).sum(0))[None, :] + np.abs(bias)[:, None]
            err = float(np.max(np.abs(C[i] - ref) / mag))
        else:
            ref = ref * (aux[i] > 0)
            err, w = oracle.max_rel_err(A[i], B[i], C[i], ref)
        assert err <= TOL, (epi, i, err)


def test_persistent_narrow_tiles_unaligned_ldc(jst):
    """C rows not 16-byte aligned (ldc odd) take the element-store path, an
    aligned C the TMA-store path: same values bit for bit, padding columns
    untouched, and the oracle bound."""
    import torch
    from jstorch_b200 import _lib
    lib = _lib.load()
    M, N, K, batch, ldc = 256, 100, 64, 150, 101
    rng = np.random.default_rng(9)
    A, B = _rand(rng, batch, M, K), _rand(rng, batch, K, N)
    a, b = _dev(A), _dev(B)
    cbuf = torch.full((batch * M * ldc,), float("nan"), device="cuda")
    d = _gemm_desc(a, b, cbuf, M, N, K, batch, ldc=ldc)
    _lib.check(lib.jst_gemm_ex(ctypes.byref(d)))
    c_al = torch.full((batch, M, 104), float("nan"), device="cuda")  # ldc 104: 16-byte rows
    d2 = _gemm_desc(a, b, c_al, M, N, K, batch, ldc=104)
    _lib.check(lib.jst_gemm_ex(ctypes.byref(d2)))
    torch.cuda.synchronize()
    C = cbuf.cpu().numpy().reshape(batch, M, ldc)
    C2 = c_al.cpu().numpy()
    assert np.isnan(C[:, :, N:]).all() and np.isnan(C2[:, :, N:]).all()  # the padding columns are untouched
    np.testing.assert_array_equal(C[:, :, :N], C2[:, :, :N])
    for i in (0, batch - 1):
        _check(A[i], B[i], C[i, :, :N], rows=np.arange(0, M, 3))


def test_persistent_narrow_tiles_broadcast_b(jst):
    """B shared by every batch entry (stride 0): its planes are split once and
    every tile of every batch reads them."""
    import torch
    from jstorch_b200 import _lib
    lib = _lib.load()
    M, N, K, batch = 384, 96, 150, 120
    rng = np.random.default_rng(11)
    A, B = _rand(rng, batch, M, K), _rand(rng, K, N)
    a, b = _dev(A), _dev(B)
    c = torch.full((batch, M, N), float("nan"), device="cuda")
    d = _gemm_desc(a, b, c, M, N, K, batch, sb=0)
    _lib.check(lib.jst_gemm_ex(ctypes.byref(d)))
    torch.cuda.synchronize()
    C = c.cpu().numpy()
    for i in (0, 59, batch - 1):
        _check(A[i], B, C[i], rows=np.arange(0, M, 5))


@pytest.mark.parametrize("K", [1000, 1024])
def test_wide_tiles_over_two_waves_and_two_bands(jst, K):
    """2304 x 2304 output in 128 x 256 tiles: 162 one-CTA-per-SM tiles, so
    CTAs 148-161 form a second wave that walks K downwards, and the two tile
    rows past the first band of 16 walk their columns backwards.  K = 1000
    ends on a partial k-slab, which those CTAs load first (zero-filled past
    K).  Rows from both bands and every wave are checked against the fp64
    oracle, and a second run must give the same bits."""
    import torch
    rng = np.random.default_rng(K)
    M = N = 2304
    A = _rand(rng, M, K)
    B = _rand(rng, K, N)
    a, b = _dev(A), _dev(B)
    c1 = jst.gemm(a, b, kernel="tc3xtf32")
    c2 = jst.gemm(a, b, kernel="tc3xtf32")
    torch.cuda.synchronize()
    C = c1.cpu().numpy()
    np.testing.assert_array_equal(C, c2.cpu().numpy())
    rows = np.unique(np.concatenate([np.arange(0, M, 37), np.arange(2048, M, 7), [M - 1]]))
    _check(A, B, C, rows=rows)
