"""Several host threads driving the library at once, each on its own CUDA
stream: tensor-core and FFMA GEMMs (split-K included, so the stream-ordered
workspace pool is shared), host-array matmuls (shared staging, serialised by
the library) and the pinned host copies.  Every result is checked."""
import threading

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 2e-6


def _worker(idx, errors):
    import torch

    import jstorch_b200
    from jstorch_b200 import _core
    try:
        rng = np.random.default_rng(100 + idx)
        s = torch.cuda.Stream()
        shapes = [(1024, 1024, 1024, "tc3xtf32"), (256, 1024, 784, "ffma"), (300, 520, 96, "auto"),
                  (128, 64, 20000, "tc3xtf32")]
        with torch.cuda.stream(s):
            for it in range(6):
                M, N, K, kern = shapes[(idx + it) % len(shapes)]
                A = rng.standard_normal((M, K), dtype=np.float32)
                B = rng.standard_normal((K, N), dtype=np.float32)
                a, b = torch.from_numpy(A).cuda(non_blocking=False), torch.from_numpy(B).cuda()
                c = jstorch_b200.gemm(a, b, kernel=kern)
                s.synchronize()
                rows = np.arange(0, M, max(1, M // 16))
                ref = oracle.gemm_f64(A, B, rows=rows)
                err, _ = oracle.max_rel_err(A, B, c.cpu().numpy(), ref, rows=rows)
                if err > TOL:
                    errors.append((idx, it, "gemm", err))
            # host-array path (library staging, one call at a time per device)
            A = rng.standard_normal((64, 48), dtype=np.float32)
            B = rng.standard_normal((48, 80), dtype=np.float32)
            C = jstorch_b200.torch.matmul(A, B, 64, 48, 80).reshape(64, 80)
            err, _ = oracle.max_rel_err(A, B, C, oracle.gemm_f64(A, B))
            if err > TOL:
                errors.append((idx, "host", err))
            # staged host copies
            x = rng.standard_normal(3 * (1 << 21) + idx).astype(np.float32)
            back = _core.Tensor.fromBuffer(x).toArray()
            if not np.array_equal(back, x):
                errors.append((idx, "hostio"))
    except Exception as e:  # noqa: BLE001 -- reported by the test
        errors.append((idx, repr(e)))


def test_threads_on_separate_streams():
    import jstorch_b200
    errors = []
    threads = [threading.Thread(target=_worker, args=(i, errors)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in threads), "a worker did not finish"
    assert not errors, errors
    assert jstorch_b200.device_error() == 0


@pytest.mark.parametrize("M,K,N", [(640, 384, 512), (4096, 1024, 2048)])  # direct and pipelined host paths
def test_host_async_calls_on_two_streams_take_turns(M, K, N):
    """Two jst_matmul_host_async calls with different inputs, enqueued back to
    back on two streams with pinned buffers, share the device's staging
    buffer: the second waits on the GPU for the first, and both C are right."""
    import torch

    import jstorch_b200
    rng = np.random.default_rng(M + N)
    ins = [(rng.standard_normal((M, K), dtype=np.float32), rng.standard_normal((K, N), dtype=np.float32))
           for _ in range(2)]
    pinned = [(torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory(),
               torch.full((M, N), float("nan")).pin_memory()) for A, B in ins]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for (a, b, c), st in zip(pinned, streams):
        jstorch_b200.matmul_host_async(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, K, N, st)
    torch.cuda.synchronize()
    for (A, B), (_, _, c) in zip(ins, pinned):
        rows = np.arange(0, M, max(1, M // 32))
        err, where = oracle.max_rel_err(A, B, c.numpy(), oracle.gemm_f64(A, B, rows=rows), rows=rows)
        assert err <= TOL, (err, where)
