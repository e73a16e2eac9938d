"""Host core (Tensor / GradTensor / nn mirror) on the GPU, against the oracle.

Covers the reference's Tensor.matmul (tensor.cpp:630-654) in its 2-D x 2-D,
3-D x 3-D and 2-D x 1-D forms, Tensor.linear (:658-671), the transposed-view
operands of nn.Linear and its backward, the bias add / ReLU / sum ops, the
backward engine, and configuration 2 (the 784-1024-1024-10 MLP, batch 256,
one forward + backward).

GEMM results use the path's bound: |C - C_ref| / (||A_i|| ||B_j|| + |bias_j|)
<= 2e-6 against the fp64 product of the same fp32 inputs.  Sums over the batch
(bias gradients) use |s - s_ref| <= 2e-6 * sum_i |g_i|.
"""
import numpy as np
import pytest

from oracle import oracle

TOL = 2e-6
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def core():
    from jstorch_b200 import _core
    return _core


def _chk(A, B, C, **kw):
    ref = oracle.gemm_f64(A, B, **{k: v for k, v in kw.items() if k in ("transA", "transB", "bias", "relu")})
    err, where = oracle.max_rel_err(A, B, C, ref, **{k: v for k, v in kw.items() if k in ("transA", "transB", "bias")})
    assert err <= TOL, (err, where)


def _sum_ok(g, s):
    ref = g.astype(np.float64).sum(axis=0)
    scale = np.abs(g.astype(np.float64)).sum(axis=0) + 1e-30
    assert (np.abs(s - ref) <= TOL * scale).all(), np.max(np.abs(s - ref) / scale)


def test_from_buffer_to_array_roundtrip(core):
    x = np.arange(12, dtype=np.float32).reshape(3, 4)
    t = core.Tensor.fromBuffer(x, [3, 4])
    assert t.shape == [3, 4] and t.isContiguous()
    np.testing.assert_array_equal(t.toArray(), x)
    tt = t.transpose()
    assert tt.shape == [4, 3] and not tt.isContiguous()
    np.testing.assert_array_equal(tt.toArray(), x.T)  # strided read-back (tensor.cpp:782-799)
    with pytest.raises(RuntimeError):
        core.Tensor.fromBuffer(x, [5, 5])


def test_readme_vector_through_tensor_matmul(core):
    a = core.Tensor.fromBuffer(np.array([1, 2, 3, 4, 5, 6], np.float32), [2, 3])
    b = core.Tensor.fromBuffer(np.arange(1, 13, dtype=np.float32), [3, 4])
    assert a.matmul(b).toArray().tolist() == [[38, 44, 50, 56], [83, 98, 113, 128]]


@pytest.mark.parametrize("M,K,N", [(256, 784, 1024), (33, 17, 65), (512, 512, 512)])
def test_matmul_transposed_views_without_copies(core, M, K, N):
    rng = np.random.default_rng(M + K + N)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32)
    G = rng.standard_normal((M, N), dtype=np.float32)
    x, w, g = (core.Tensor.fromBuffer(v) for v in (X, W, G))
    n0 = core.stridedCopies()
    y = x.matmul(w.transpose())          # NT: nn.Linear forward
    gx = g.matmul(w)                     # NN: grad input
    gw = x.transpose().matmul(g)         # TN: grad weight (as W^T)
    assert core.stridedCopies() == n0    # no contiguous() materialisation
    _chk(X, W, y.toArray(), transB=True)
    _chk(G, W, gx.toArray())
    _chk(X, G, gw.toArray(), transA=True)


def test_matmul_forms_and_errors(core):
    rng = np.random.default_rng(2)
    A3, B3 = rng.standard_normal((4, 30, 20), dtype=np.float32), rng.standard_normal((4, 20, 40), dtype=np.float32)
    c3 = core.Tensor.fromBuffer(A3).matmul(core.Tensor.fromBuffer(B3)).toArray()
    _chk(A3, B3, c3)
    A, v = rng.standard_normal((50, 70), dtype=np.float32), rng.standard_normal(70, dtype=np.float32)
    mv = core.Tensor.fromBuffer(A).matmul(core.Tensor.fromBuffer(v)).toArray()
    assert mv.shape == (50,)
    _chk(A, v.reshape(70, 1), mv.reshape(50, 1))
    with pytest.raises(RuntimeError, match="shape mismatch"):
        core.Tensor.fromBuffer(A).matmul(core.Tensor.fromBuffer(A))
    with pytest.raises(RuntimeError, match="unsupported dims"):
        core.Tensor.fromBuffer(A3).matmul(core.Tensor.fromBuffer(A))
    # a non-transposable view goes through contiguous() first
    big = core.Tensor.fromBuffer(rng.standard_normal((4, 20, 30), dtype=np.float32))
    n0 = core.stridedCopies()
    perm = big.transpose(0, 2)  # [30, 20, 4]: batch stride 1, not a GEMM layout
    out = perm.matmul(core.Tensor.fromBuffer(rng.standard_normal((30, 4, 5), dtype=np.float32)))
    assert core.stridedCopies() == n0 + 1 and out.shape == [30, 20, 5]


def test_linear_with_and_without_bias(core):
    rng = np.random.default_rng(4)
    X = rng.standard_normal((256, 784), dtype=np.float32)
    W = rng.standard_normal((1024, 784), dtype=np.float32)
    b = rng.standard_normal(1024, dtype=np.float32)
    x, w, bt = core.Tensor.fromBuffer(X), core.Tensor.fromBuffer(W), core.Tensor.fromBuffer(b)
    _chk(X, W, x.linear(w, bt).toArray(), transB=True, bias=b)
    _chk(X, W, x.linear(w).toArray(), transB=True)
    with pytest.raises(RuntimeError, match="shape mismatch"):
        x.linear(core.Tensor.fromBuffer(np.ascontiguousarray(W[:, :100])))


def test_add_relu_sum(core):
    rng = np.random.default_rng(6)
    Z = rng.standard_normal((64, 48), dtype=np.float32)
    b = rng.standard_normal(48, dtype=np.float32)
    z, bt = core.Tensor.fromBuffer(Z), core.Tensor.fromBuffer(b)
    np.testing.assert_array_equal(z.add(bt).toArray(), Z + b)
    np.testing.assert_array_equal(bt.add(z).toArray(), Z + b)
    np.testing.assert_array_equal(z.add(z).toArray(), Z + Z)
    np.testing.assert_array_equal(z.relu().toArray(), np.maximum(Z, 0))
    _sum_ok(Z, z.sum(0).toArray())
    _sum_ok(Z.T, z.sum(1).toArray())
    assert z.sum(0, True).shape == [1, 48]
    with pytest.raises(RuntimeError, match="broadcast"):
        z.add(core.Tensor.fromBuffer(rng.standard_normal(7, dtype=np.float32)))


def test_backward_engine_accumulates(core):
    """y = x.W + x.W (x used twice): W.grad = 2 x^T . ones (autograd.hpp:56-58)."""
    rng = np.random.default_rng(8)
    X, W = rng.standard_normal((8, 5), dtype=np.float32), rng.standard_normal((5, 3), dtype=np.float32)
    x = core.GradTensor(core.Tensor.fromBuffer(X), False)
    w = core.GradTensor(core.Tensor.fromBuffer(W), True)
    y = x.matmul(w).add(x.matmul(w))
    y.backward()
    assert x.grad is None
    ref = 2 * X.astype(np.float64).T @ np.ones((8, 3))
    np.testing.assert_allclose(w.grad.toArray(), ref, rtol=1e-6, atol=1e-5)


def _mlp(core):
    from jstorch_b200 import nn, synth
    x, ws, bs = synth.config2()
    model = nn.Sequential(nn.Linear(784, 1024), nn.ReLU(), nn.Linear(1024, 1024), nn.ReLU(), nn.Linear(1024, 10))
    state = {}
    for i, (w, b) in zip((0, 2, 4), zip(ws, bs)):
        state[f"{i}.weight"] = core.Tensor.fromBuffer(w)
        state[f"{i}.bias"] = core.Tensor.fromBuffer(b)
    model.load_state_dict(state)
    model._init_grad()
    return model, x, ws, bs


def test_config2_mlp_forward_backward(core):
    """Configuration 2: nn.Linear 784->1024->1024->10 with ReLU, batch 256;
    one forward and backward with loss = sum(y).  Every GEMM of the pass is
    checked against the fp64 product of the GPU's own inputs to that GEMM
    (forward NT, grad-input NN, grad-weight TN), the ReLU masks and bias
    gradients exactly / to the sum bound, and the whole pass against the
    oracle's fp64 forward + backward."""
    model, X, Ws, Bs = _mlp(core)
    layers = list(model._modules.values())
    x = core.GradTensor(core.Tensor.fromBuffer(X), False)
    n0 = core.stridedCopies()
    acts = [x]
    for m in layers:
        acts.append(m(acts[-1]))
    y = acts[-1]
    y.backward()
    assert core.stridedCopies() == n0, "the nn.Linear path must not materialise transposes"
    A = [a.toArray() for a in acts]  # x, z1, h1, z2, h2, y
    G = [a.grad.toArray() if a.grad is not None else None for a in acts]
    params = model.parameters()
    Wg = [params[i].grad.toArray() for i in (0, 2, 4)]
    bg = [params[i].grad.toArray() for i in (1, 3, 5)]

    # forward: z = h.W^T + b per layer (NT with bias epilogue through the core), relu exact
    for l, (hi, zi) in enumerate([(0, 1), (2, 3), (4, 5)]):
        _chk(A[hi], Ws[l], A[zi], transB=True, bias=Bs[l])
    np.testing.assert_array_equal(A[2], np.maximum(A[1], 0))
    np.testing.assert_array_equal(A[4], np.maximum(A[3], 0))

    # backward, layer by layer on the GPU's own upstream gradients
    gz = [G[1], G[3], G[5]]
    np.testing.assert_array_equal(G[5], np.ones_like(A[5]))  # default upstream (napi.cpp:975-977)
    for l, hi in enumerate([0, 2, 4]):
        # dW^T = h^T . gz  (TN); the stored W.grad is its transpose (autograd.hpp:536)
        _chk(A[hi], gz[l], Wg[l].T, transA=True)
        _sum_ok(gz[l], bg[l])
        if l > 0:
            _chk(gz[l], Ws[l], G[hi])  # grad input: gz . W  (NN)
            np.testing.assert_array_equal(gz[l - 1], np.where(A[hi - 1] > 0, G[hi], 0.0).astype(np.float32))

    # end to end against the oracle's fp64 pass
    ref = oracle.mlp_forward_backward(X, Ws, Bs)
    rel = lambda a, b: np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
    assert rel(A[5], ref["y"]) < 1e-5
    for l in range(3):
        assert rel(Wg[l], ref["dW"][l]) < 1e-4, (l, rel(Wg[l], ref["dW"][l]))
        assert rel(bg[l], ref["db"][l]) < 1e-4, (l, rel(bg[l], ref["db"][l]))
    # masks agree wherever the pre-activation is not within rounding of zero
    for zi, zr in ((1, ref["z"][0]), (3, ref["z"][1])):
        clear = np.abs(zr) > 1e-4 * np.abs(zr).max()
        assert ((A[zi] > 0) == (zr > 0))[clear].all()
