"""Tensor.fromBuffer / toArray / toFloat32Array through the pinned,
double-buffered staging (reference: tensor.cpp:740-800, napi.cpp:17-30,
235-238, 702-707): byte-exact round trips at sizes around the staging chunk,
strided read-back, page-locked sources and destinations, and ordering with
the GEMM on the core stream."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CHUNK = (8 << 20) // 4  # floats per staging chunk


@pytest.fixture(scope="module")
def core():
    from jstorch_b200 import _core
    return _core


@pytest.mark.parametrize("n", [0, 1, 1000, 65536, 65537, CHUNK - 1, CHUNK, CHUNK + 1, 2 * CHUNK + 3, 7 * CHUNK // 2])
def test_roundtrip_exact(core, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    x[: min(n, 4)] = [np.inf, -0.0, np.nan, 1e-45][: min(n, 4)]  # specials survive bit for bit
    t = core.Tensor.fromBuffer(x, [n])
    y = t.toArray()
    assert y.shape == (n,)
    assert np.array_equal(y.view(np.uint32), x.view(np.uint32))
    f = t.toFloat32Array()
    assert f.ndim == 1 and f.dtype == np.float32 and np.array_equal(f.view(np.uint32), x.view(np.uint32))


def test_many_tensors_back_to_back(core):
    """Several uploads in a row reuse the two staging chunks; every tensor
    keeps its own contents (no staging chunk overwritten before its DMA)."""
    rng = np.random.default_rng(3)
    xs = [rng.standard_normal(3 * CHUNK + 17 * i).astype(np.float32) for i in range(5)]
    ts = [core.Tensor.fromBuffer(x) for x in xs]
    for x, t in zip(xs, ts):
        np.testing.assert_array_equal(t.toArray(), x)


def test_strided_readback_and_shape(core):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3000, 1200)).astype(np.float32)  # 13.7 MiB: two chunks
    t = core.Tensor.fromBuffer(x)
    np.testing.assert_array_equal(t.transpose().toArray(), x.T)
    np.testing.assert_array_equal(t.transpose().toFloat32Array(), x.T.reshape(-1))


def test_pinned_source(core):
    import torch
    n = 5 * CHUNK // 2
    expect = np.random.default_rng(5).standard_normal(n).astype(np.float32)
    src = torch.empty(n, dtype=torch.float32, pin_memory=True)
    src.copy_(torch.from_numpy(expect))
    t = core.Tensor.fromBuffer(src.numpy())  # page-locked: one direct DMA
    src.zero_()  # the call waited for its DMA, so the tensor keeps the old values
    np.testing.assert_array_equal(t.toArray(), expect)


def test_ordering_with_gemm(core):
    """fromBuffer -> matmul -> toArray in stream order, with no explicit
    synchronisation in between (the last upload DMAs may still be running
    when matmul is enqueued)."""
    from oracle import oracle
    rng = np.random.default_rng(6)
    A = rng.standard_normal((1024, 2048)).astype(np.float32)  # 8 MiB: exactly one chunk
    B = rng.standard_normal((2048, 1536)).astype(np.float32)  # 12 MiB: two chunks
    C = core.Tensor.fromBuffer(A).matmul(core.Tensor.fromBuffer(B)).toArray()
    ref = oracle.gemm_f64(A, B, rows=np.arange(0, 1024, 37))
    err, _ = oracle.max_rel_err(A, B, C, ref, rows=np.arange(0, 1024, 37))
    assert err <= 2e-6


def test_c_abi_copies_on_torch_buffers():
    """jst_copy_h2d / jst_copy_d2h directly: odd byte counts, a pageable numpy
    source and destination, and a stream other than the legacy one."""
    import torch
    from jstorch_b200 import _lib
    lib = _lib.load()
    s = torch.cuda.Stream()
    for nbytes in (1, 4097, 3 * (8 << 20) + 5):
        src = np.random.default_rng(nbytes).integers(0, 256, nbytes, dtype=np.uint8)
        dev = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        _lib.check(lib.jst_copy_h2d(dev.data_ptr(), src.ctypes.data, nbytes, s.cuda_stream))
        back = np.empty(nbytes, dtype=np.uint8)
        _lib.check(lib.jst_copy_d2h(back.ctypes.data, dev.data_ptr(), nbytes, s.cuda_stream))
        assert np.array_equal(back, src)
