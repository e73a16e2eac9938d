"""jst_gemm_tc_noalloc: the tensor-core GEMM for callers that cannot call
cudaMalloc (a host whose device memory belongs to another allocator, an
embedder with a fixed memory budget, latency-critical code that cannot afford
the device-wide synchronisation cudaMalloc / cudaFree may cause).  It keeps its
scratch in a fixed 64 MiB device array instead of allocating.

Checked through the C ABI against jst_gemm_ex (the allocating entry point,
tensor-core kernel forced) on two calls in a row with different shapes and
inputs, so the second call runs on scratch the first one left behind; on a
shape that splits K (the partials live in the same array); with the device's
free memory unchanged across calls; with a timed-out wait (raised from the
host) reported by jst_device_error(); and captured into a CUDA graph, whose
replays on new inputs match the fp64 oracle and a direct call bit for bit.  This file is collected last on
purpose; it also passes when run on its own.
"""
import ctypes

import numpy as np
import pytest

from jstorch_b200 import _lib
from oracle import oracle

TOL = 2e-6  # the bound every GEMM test in this suite uses

pytestmark = pytest.mark.gpu


def _desc(a, b, c, M, N, K, *, transB=False, bias=None, relu=False, batch=1, stream=0):
    d = _lib.GemmDesc()
    d.transA, d.transB = 0, int(transB)
    d.M, d.N, d.K = M, N, K
    d.A, d.lda, d.strideA = a.data_ptr(), K, M * K
    d.B, d.ldb, d.strideB = b.data_ptr(), (K if transB else N), N * K
    d.C, d.ldc, d.strideC = c.data_ptr(), N, M * N
    d.batch = batch
    d.bias = bias.data_ptr() if bias is not None else None
    d.epilogue = (_lib.EPI_BIAS if bias is not None else 0) | (_lib.EPI_RELU if relu else 0)
    d.kernel = _lib.KERNEL_TC3XTF32
    d.stream = stream
    return d


def _run_pair(M, N, K, seed, *, transB=False, with_bias=False, relu=False, batch=1):
    import torch
    lib = _lib.load()
    rng = np.random.default_rng(seed)
    shape_a = (batch, M, K) if batch > 1 else (M, K)
    shape_b = ((batch,) if batch > 1 else ()) + ((N, K) if transB else (K, N))
    A = rng.standard_normal(shape_a, dtype=np.float32)
    B = rng.standard_normal(shape_b, dtype=np.float32)
    bias_h = rng.standard_normal(N, dtype=np.float32) if with_bias else None
    a, b = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    bias = torch.from_numpy(bias_h).cuda() if with_bias else None
    c_free = torch.full((batch, M, N), float("nan"), device="cuda")
    c_ref = torch.full((batch, M, N), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    d = _desc(a, b, c_free, M, N, K, transB=transB, bias=bias, relu=relu, batch=batch, stream=stream)
    _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))
    d2 = _desc(a, b, c_ref, M, N, K, transB=transB, bias=bias, relu=relu, batch=batch, stream=stream)
    _lib.check(lib.jst_gemm_ex(ctypes.byref(d2)))
    torch.cuda.synchronize()
    got = c_free.cpu().numpy()
    want = c_ref.cpu().numpy()
    assert np.isfinite(got).all()
    # agreement with the allocating entry point, in the suite's metric ...
    ref64 = want.astype(np.float64)
    err_vs_ex, where = oracle.max_rel_err(A, B, got if batch > 1 else got[0], ref64 if batch > 1 else ref64[0],
                                          transB=transB, bias=bias_h)
    assert err_vs_ex <= TOL, (err_vs_ex, where)
    # ... and with the fp64 oracle
    ref = oracle.gemm_f64(A, B, transB=transB, bias=bias_h, relu=relu)
    err, where = oracle.max_rel_err(A, B, got if batch > 1 else got[0], ref, transB=transB, bias=bias_h)
    assert err <= TOL, (err, where)


def test_noalloc_two_calls_in_a_row_match_allocating_entry_point():
    # first call: sets the device up and fills the scratch
    _run_pair(640, 896, 1000, seed=1, transB=True, with_bias=True, relu=True)
    # second call: other shape and inputs on the scratch the first call left behind
    _run_pair(333, 517, 250, seed=2, batch=3)


def test_noalloc_rejects_requests_beyond_the_fixed_scratch():
    import torch
    lib = _lib.load()
    a = torch.zeros((2048, 2049), device="cuda")
    b = torch.zeros((2049, 2048), device="cuda")
    c = torch.zeros((2048, 2048), device="cuda")
    d = _desc(a, b, c, 2048, 2048, 2049)  # K rounds up to 2052: just over 64 MiB of planes
    rc = lib.jst_gemm_tc_noalloc(ctypes.byref(d))
    assert rc == 1
    assert b"scratch" in lib.jst_last_error()
    d = _desc(a, b, c, 2048, 2048, 2048)  # exactly 64 MiB: accepted
    b2 = torch.zeros((2048, 2048), device="cuda")
    d.B = b2.data_ptr()
    d.lda = 2049
    _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))
    torch.cuda.synchronize()
    assert float(c.abs().max()) == 0.0


def test_noalloc_split_k_shape_matches_oracle():
    # 2 output tiles and K = 8192: the kernel splits K into slices whose
    # partials also live in the fixed scratch
    _run_pair(256, 256, 8192, seed=3)
    _run_pair(256, 256, 8192, seed=4, with_bias=True, relu=True)


def test_noalloc_calls_leave_free_device_memory_unchanged():
    import torch
    lib = _lib.load()
    rng = np.random.default_rng(5)
    M, N, K = 512, 768, 1536
    a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32)).cuda()
    c = torch.empty((M, N), device="cuda")
    d = _desc(a, b, c, M, N, K, stream=torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))  # the module (and its array) is resident from here
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, (free0, free1)
    ref = oracle.gemm_f64(a.cpu().numpy(), b.cpu().numpy())
    err, where = oracle.max_rel_err(a.cpu().numpy(), b.cpu().numpy(), c.cpu().numpy(), ref)
    assert err <= TOL, (err, where)


def test_noalloc_timeout_word_is_reported_by_device_error():
    # A kernel whose bounded wait gives up ORs a flag into the entry point's
    # own error word; the flag is planted from the host here (no GPU stall).
    import torch
    lib = _lib.load()
    a = torch.ones((128, 256), device="cuda")
    b = torch.ones((256, 128), device="cuda")
    c = torch.empty((128, 128), device="cuda")
    d = _desc(a, b, c, 128, 128, 256, stream=torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))
    assert lib.jst_device_error() == 0
    _lib.check(lib.jst_test_set_device_error(1))
    # a later call does not wipe the flag before the caller has seen it
    _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))
    assert lib.jst_device_error() == 1
    assert lib.jst_device_error() == 0  # read and cleared
    torch.cuda.synchronize()
    assert float(c.min()) == 256.0 and float(c.max()) == 256.0
    assert lib.jst_test_set_device_error(2) == 1  # JST_ERR_ARG


@pytest.mark.parametrize("M,N,K", [(512, 640, 768), (256, 256, 8192)])
def test_noalloc_call_captured_in_a_cuda_graph_replays_on_new_inputs(M, N, K):
    # The entry point's main use: after one warm-up call (module load, symbol
    # addresses, kernel attributes) a call is captured into a CUDA graph; each
    # replay then runs on whatever the captured input buffers hold.  The second
    # shape splits K, so the graph also holds the partials' reduction.
    import torch
    lib = _lib.load()
    rng = np.random.default_rng(M + K)
    a = torch.empty((M, K), device="cuda")
    b = torch.empty((K, N), device="cuda")
    c = torch.full((M, N), float("nan"), device="cuda")
    a.copy_(torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)))
    b.copy_(torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32)))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        d = _desc(a, b, c, M, N, K, stream=side.cuda_stream)
        _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        d = _desc(a, b, c, M, N, K, stream=torch.cuda.current_stream().cuda_stream)
        _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d)))
    try:
        for _ in range(2):
            A = rng.standard_normal((M, K), dtype=np.float32)
            B = rng.standard_normal((K, N), dtype=np.float32)
            a.copy_(torch.from_numpy(A))
            b.copy_(torch.from_numpy(B))
            c.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            got = c.cpu().numpy()
            ref = oracle.gemm_f64(A, B)
            err, where = oracle.max_rel_err(A, B, got, ref)
            assert err <= TOL, (err, where)
            # the replay gives exactly what a direct call gives on the same inputs
            c_direct = torch.full((M, N), float("nan"), device="cuda")
            d2 = _desc(a, b, c_direct, M, N, K, stream=torch.cuda.current_stream().cuda_stream)
            _lib.check(lib.jst_gemm_tc_noalloc(ctypes.byref(d2)))
            torch.cuda.synchronize()
            assert torch.equal(c, c_direct)
        assert lib.jst_device_error() == 0
    finally:
        del graph
