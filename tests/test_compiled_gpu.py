"""CompiledGraph (reference: native/core/autograd.hpp:856-1498, MATMUL case
:1134; binding native/binding/napi.cpp:1488-1830) and the GEMM mask epilogue
it fuses the ReLU backward into.

The compiled pass must give what the eager GradTensor pass gives on the same
tensors: the first run executes eagerly, the second captures a CUDA graph,
later runs replay it; all three are compared with the eager pass and with
the fp64 oracle.
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


@pytest.mark.parametrize("kernel", ["tc3xtf32", "ffma"])
@pytest.mark.parametrize("M,N,K", [(256, 784, 1024), (200, 300, 96), (1, 5, 7)])
def test_mask_epilogue(kernel, M, N, K):
    """out = (g . W) * (h > 0): the grad-input GEMM with the ReLU backward fused."""
    import torch
    from jstorch_b200 import gemm

    if kernel == "tc3xtf32" and min(M, N) < 8:
        pytest.skip("tiny shapes run on FFMA")
    rng = np.random.default_rng(M * 7 + N + K)
    G = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((K, N), dtype=np.float32)
    H = rng.standard_normal((M, N), dtype=np.float32)
    H[rng.random((M, N)) < 0.1] = 0.0  # exact zeros are masked (x > 0 is false)
    g, w, h = (torch.from_numpy(v).cuda() for v in (G, W, H))
    out = gemm(g, w, mask=h, kernel=kernel)
    plain = gemm(g, w, kernel=kernel)
    torch.cuda.synchronize()
    o, p = out.cpu().numpy(), plain.cpu().numpy()
    np.testing.assert_array_equal(o, np.where(H > 0, p, 0.0).astype(np.float32))
    ref = oracle.gemm_f64(G, W) * (H > 0)
    err, where = oracle.max_rel_err(G, W, o, ref)
    assert err <= TOL, (err, where)
    # transposed operand (TN) and a batched form
    gt = torch.from_numpy(np.ascontiguousarray(G.T)).cuda()
    out2 = gemm(gt.t(), w, mask=h, kernel=kernel)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out2.cpu().numpy(), o)
    with pytest.raises(ValueError):
        gemm(g, w, mask=h, relu=True)


def test_mask_epilogue_batched():
    import torch
    from jstorch_b200 import gemm

    rng = np.random.default_rng(11)
    G = rng.standard_normal((3, 130, 70), dtype=np.float32)
    W = rng.standard_normal((3, 70, 260), dtype=np.float32)
    H = rng.standard_normal((3, 130, 260), dtype=np.float32)
    for kernel in ("tc3xtf32", "ffma"):
        out = gemm(*(torch.from_numpy(v).cuda() for v in (G, W)), mask=torch.from_numpy(H).cuda(), kernel=kernel)
        plain = gemm(*(torch.from_numpy(v).cuda() for v in (G, W)), kernel=kernel)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), np.where(H > 0, plain.cpu().numpy(), 0.0))


def _tape(core, n_layers, relu_last=False, bias=True):
    """Record Sequential(Linear, ReLU, ..., Linear) the way nn.Linear builds it
    (src/nn.js:105-110: x.matmul(W.transpose()).add(b))."""
    g = core.CompiledGraph()
    h = g.input()
    for l in range(n_layers):
        w = g.param()
        b = g.param() if bias else None
        h = g.matmul(h, g.transpose(w))
        if b is not None:
            h = g.add(h, b)
        if l < n_layers - 1 or relu_last:
            h = g.relu(h)
    g.setOutput(h)
    return g


def _eager(core, X, params, n_layers, relu_last=False, bias=True):
    x = core.GradTensor(core.Tensor.fromBuffer(X), False)
    ps = [core.GradTensor(p, True) for p in params]
    h, i = x, 0
    for l in range(n_layers):
        w = ps[i]; i += 1
        h = h.matmul(w.transpose())
        if bias:
            h = h.add(ps[i]); i += 1
        if l < n_layers - 1 or relu_last:
            h = h.relu()
    h.backward()
    return h.toArray(), [p.grad.toArray() for p in ps]


def _config2_params(core):
    from jstorch_b200 import synth
    X, Ws, Bs = synth.config2()
    params = []
    for w, b in zip(Ws, Bs):
        params += [core.Tensor.fromBuffer(w), core.Tensor.fromBuffer(b)]
    return X, Ws, Bs, params


def test_compiled_config2_matches_eager_and_oracle(core):
    """Configuration 2 (784-1024-1024-10 MLP, batch 256): eager run, capture,
    replays -- each identical to the eager GradTensor pass, and within the
    path's bound of the fp64 oracle."""
    X, Ws, Bs, params = _config2_params(core)
    y_ref, g_ref = _eager(core, X, params, 3)
    g = _tape(core, 3)
    x = core.Tensor.fromBuffer(X)
    ref = oracle.mlp_forward_backward(X, Ws, Bs)
    rel = lambda a, b: np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
    for run in range(4):
        y, grads = g.run(x, params)
        assert g.fused
        assert g.replaying == (run >= 1)
        ya = y.toArray()
        np.testing.assert_array_equal(ya, y_ref)
        assert len(grads) == 6
        for a, b in zip(grads, g_ref):
            np.testing.assert_allclose(a.toArray(), b, rtol=1e-6, atol=1e-5 * np.abs(b).max())
        assert rel(ya, ref["y"]) < 1e-5
        for l in range(3):
            assert rel(grads[2 * l].toArray(), ref["dW"][l]) < 1e-4
            assert rel(grads[2 * l + 1].toArray(), ref["db"][l]) < 1e-4
    # 3 forward GEMMs, 3 dW GEMMs, 2 dX GEMMs, 3 bias sums, plus at most one
    # split-K reduce per GEMM; no bias-add, ReLU or mask kernels
    assert 11 <= g.kernelsPerRun <= 19, g.kernelsPerRun


def test_compiled_new_input_values_and_batch(core):
    """Replays read the new input; a new batch size re-captures."""
    X, Ws, Bs, params = _config2_params(core)
    g = _tape(core, 3)
    rng = np.random.default_rng(5)
    for batch in (256, 256, 256, 64, 64, 64):
        Xb = rng.standard_normal((batch, 784), dtype=np.float32)
        y, grads = g.run(core.Tensor.fromBuffer(Xb), params)
        y_ref, g_ref = _eager(core, Xb, params, 3)
        np.testing.assert_array_equal(y.toArray(), y_ref)
        for a, b in zip(grads, g_ref):
            np.testing.assert_allclose(a.toArray(), b, rtol=1e-6, atol=1e-5 * np.abs(b).max())


@pytest.mark.parametrize("relu_last,bias", [(True, True), (False, False)])
def test_compiled_variants_large_layers(core, relu_last, bias):
    """Layers big enough for the tensor-core kernel (graph-captured workspace),
    a ReLU on the last layer, and Linear without bias."""
    rng = np.random.default_rng(9)
    dims = [512, 2048, 1024]
    params, Ws, Bs = [], [], []
    for i in range(2):
        W = (rng.standard_normal((dims[i + 1], dims[i])) / np.sqrt(dims[i])).astype(np.float32)
        B = rng.standard_normal(dims[i + 1]).astype(np.float32) if bias else np.zeros(dims[i + 1], np.float32)
        Ws.append(W); Bs.append(B)
        params.append(core.Tensor.fromBuffer(W))
        if bias:
            params.append(core.Tensor.fromBuffer(B))
    X = rng.standard_normal((1024, 512), dtype=np.float32)
    y_ref, g_ref = _eager(core, X, params, 2, relu_last, bias)
    g = _tape(core, 2, relu_last, bias)
    for run in range(3):
        y, grads = g.run(core.Tensor.fromBuffer(X), params)
        assert g.fused
        np.testing.assert_allclose(y.toArray(), y_ref, rtol=1e-6, atol=1e-6 * np.abs(y_ref).max())
        for a, b in zip(grads, g_ref):
            np.testing.assert_allclose(a.toArray(), b, rtol=1e-5, atol=1e-5 * np.abs(b).max())


def test_compiled_unrecognised_tape_runs_eagerly(core):
    """A tape that is not a Linear chain (here x . W without transpose, W used
    twice) runs through GradTensor and still returns output and gradients."""
    rng = np.random.default_rng(3)
    X = rng.standard_normal((16, 8), dtype=np.float32)
    W = rng.standard_normal((8, 8), dtype=np.float32)
    g = core.CompiledGraph()
    x = g.input()
    w = g.param()
    h = g.matmul(g.matmul(x, w), w)
    g.setOutput(h)
    y, grads = g.run(core.Tensor.fromBuffer(X), [core.Tensor.fromBuffer(W)])
    assert not g.fused
    np.testing.assert_allclose(y.toArray(), X.astype(np.float64) @ W @ W, rtol=1e-5, atol=1e-4)
    ones = np.ones((16, 8))
    dW = (X.astype(np.float64).T @ ones @ W.T) + (X.astype(np.float64) @ W).T @ ones
    np.testing.assert_allclose(grads[0].toArray(), dW, rtol=1e-5, atol=1e-4)


def test_compiled_errors(core):
    g = _tape(core, 1)
    rng = np.random.default_rng(1)
    W = core.Tensor.fromBuffer(rng.standard_normal((4, 6), dtype=np.float32))
    b = core.Tensor.fromBuffer(rng.standard_normal(4, dtype=np.float32))
    with pytest.raises(RuntimeError, match="number of parameters"):
        g.run(core.Tensor.fromBuffer(rng.standard_normal((3, 6), dtype=np.float32)), [W])
    with pytest.raises(RuntimeError, match="input must be"):
        g.run(core.Tensor.fromBuffer(rng.standard_normal((3, 5), dtype=np.float32)), [W, b])
    with pytest.raises(RuntimeError, match="bad slot"):
        core.CompiledGraph().relu(3)
