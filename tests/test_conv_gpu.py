"""The eight im2col-GEMM convolution launchers (include/jstorch_conv.h,
reference native/ops/conv.cu:324-627) against the fp64 oracle.

Bound: the path's GEMM metric, per output element
    |y - y_ref| <= 2e-6 * (||A_i|| ||B_j|| + |b|)
with A_i, B_j the row and column of the im2col GEMM that produce the element
(a filter and an input patch; for the weight gradients a grad_output channel
and a column row over batch x pixels).  For a transposed convolution an
output element sums several GEMM elements (col2im), and the bound is the
sum of theirs.  The norms are computed with the oracle's own convolutions
of squared inputs."""
import numpy as np
import pytest

from oracle import oracle

TOL = 2e-6
pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def _host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy().astype(np.float64)


def _ok(got, ref, mag):
    err = np.abs(got - ref) / (mag + 1e-30)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.max(err, initial=0.0) <= TOL, float(np.max(err))


def _bound_conv2d(x, w, b, s, p, d, g):
    """||w_o|| * ||patch|| (+ |b_o|): the patch norm is a conv of x^2 with ones."""
    Co, Cig, kH, kW = w.shape
    patch2 = oracle.conv2d_f64(np.square(x, dtype=np.float64), np.ones((Co, Cig, kH, kW)), None, s, p, d, g)
    wn2 = np.square(w.astype(np.float64)).reshape(Co, -1).sum(1)
    out = np.sqrt(patch2 * wn2[None, :, None, None])
    return out + (np.abs(b)[None, :, None, None] if b is not None else 0.0)


def _bound_conv2d_bw(x, go, k, s, p, d, g):
    """||go_o|| over (b, pixel) times ||col row (c, tap)|| over (b, pixel)."""
    col2 = oracle.conv2d_backward_weight_f64(np.square(x, dtype=np.float64), np.ones(go.shape), k, s, p, d, g)
    gn2 = np.square(go.astype(np.float64)).sum(axis=(0, 2, 3))
    return np.sqrt(col2 * gn2[:, None, None, None])


def _bound_conv_transpose2d(x, w, b, s, p, d, g, op):
    """sum over the taps landing on an output element of ||w[:, co, tap]|| * ||x[b, :, pixel]||
    (per group): a transposed conv of the pixel norms with the tap norms."""
    B, Ci, H, W = x.shape
    Cig = Ci // g
    xn = np.sqrt(np.square(x.astype(np.float64)).reshape(B, g, Cig, H, W).sum(2))       # [B, g, H, W]
    wn = np.sqrt(np.square(w.astype(np.float64)).reshape(g, Cig, *w.shape[1:]).sum(1))  # [g, Co_g, kH, kW]
    out = oracle.conv_transpose2d_f64(xn, wn, None, s, p, d, g, (op, op))
    return out + np.abs(b)[None, :, None, None]


def _bound_conv_transpose2d_bw(x, go, k, s, p, d, g):
    """||x_ci|| over (b, pixel) times ||im2col(go) row (co, tap)|| over (b, pixel)."""
    col2 = oracle.conv_transpose2d_backward_weight_f64(np.ones(x.shape), np.square(go, dtype=np.float64), k, s, p,
                                                       d, g)
    xn2 = np.square(x.astype(np.float64)).sum(axis=(0, 2, 3))
    return np.sqrt(col2 * xn2[:, None, None, None])


CASES2D = [
    # B, Ci, Co, H, W, k, stride, padding, dilation, groups
    (2, 3, 8, 16, 15, (3, 3), (1, 1), (1, 1), (1, 1), 1),
    (3, 8, 12, 11, 9, (3, 2), (2, 1), (0, 2), (1, 2), 4),
    (4, 16, 32, 14, 14, (1, 1), (1, 1), (0, 0), (1, 1), 1),   # direct: no im2col
    (2, 6, 6, 9, 10, (5, 3), (3, 2), (2, 1), (2, 1), 6),      # depthwise-like
    (1, 5, 7, 1, 40, (1, 4), (1, 3), (0, 2), (1, 2), 1),      # H = 1
    (16, 64, 128, 32, 32, (3, 3), (1, 1), (1, 1), (1, 1), 1),  # large enough for the tensor-core kernel
    (32, 128, 128, 32, 32, (3, 3), (1, 1), (1, 1), (1, 1), 2),  # tensor cores, two groups
    (16, 64, 128, 63, 64, (3, 3), (2, 2), (1, 1), (1, 1), 1),  # tensor cores, stride 2, ragged pixel count
]


@pytest.mark.parametrize("case", CASES2D)
@pytest.mark.parametrize("with_bias", [True, False])
def test_conv2d_forward(case, with_bias):
    from jstorch_b200 import conv
    B, Ci, Co, H, W, k, s, p, d, g = case
    rng = np.random.default_rng(sum(case[:5]) + with_bias)
    x = rng.standard_normal((B, Ci, H, W)).astype(np.float32)
    w = rng.standard_normal((Co, Ci // g, *k)).astype(np.float32)
    b = rng.standard_normal(Co).astype(np.float32) if with_bias else None
    y = _host(conv.conv2d(_dev(x), _dev(w), _dev(b) if with_bias else None, s, p, d, g))
    _ok(y, oracle.conv2d_f64(x, w, b, s, p, d, g), _bound_conv2d(x, w, b, s, p, d, g))


@pytest.mark.parametrize("case", CASES2D)
def test_conv2d_backward_weight(case):
    from jstorch_b200 import conv
    B, Ci, Co, H, W, k, s, p, d, g = case
    rng = np.random.default_rng(sum(case[:5]) + 11)
    x = rng.standard_normal((B, Ci, H, W)).astype(np.float32)
    Ho, Wo = oracle.conv_out_size(H, k[0], s[0], p[0], d[0]), oracle.conv_out_size(W, k[1], s[1], p[1], d[1])
    go = rng.standard_normal((B, Co, Ho, Wo)).astype(np.float32)
    gw = _host(conv.conv2d_backward_weight(_dev(x), _dev(go), k, s, p, d, g))
    _ok(gw, oracle.conv2d_backward_weight_f64(x, go, k, s, p, d, g), _bound_conv2d_bw(x, go, k, s, p, d, g))


@pytest.mark.parametrize("case", CASES2D)
@pytest.mark.parametrize("op", [0, 1])
def test_conv_transpose2d_forward_and_backward_weight(case, op):
    from jstorch_b200 import conv
    B, Ci, Co, H, W, k, s, p, d, g = case
    if op >= max(s[0], d[0]) or op >= max(s[1], d[1]):
        pytest.skip("output padding must be smaller than stride or dilation")
    rng = np.random.default_rng(sum(case[:5]) + 23 + op)
    x = rng.standard_normal((B, Ci, H, W)).astype(np.float32)
    w = rng.standard_normal((Ci, Co // g, *k)).astype(np.float32)
    b = rng.standard_normal(Co).astype(np.float32)
    y = _host(conv.conv_transpose2d(_dev(x), _dev(w), _dev(b), s, p, op, d, g))
    ref = oracle.conv_transpose2d_f64(x, w, b, s, p, d, g, (op, op))
    _ok(y, ref, _bound_conv_transpose2d(x, w, b, s, p, d, g, op))
    go = rng.standard_normal(ref.shape).astype(np.float32)
    gw = _host(conv.conv_transpose2d_backward_weight(_dev(x), _dev(go), k, s, p, d, g))
    _ok(gw, oracle.conv_transpose2d_backward_weight_f64(x, go, k, s, p, d, g),
        _bound_conv_transpose2d_bw(x, go, k, s, p, d, g))


CASES1D = [
    # B, C_in, C_out, L, K, stride, padding, dilation, groups
    (2, 3, 5, 50, 3, 1, 1, 1, 1),
    (4, 8, 8, 33, 5, 2, 2, 2, 2),
    (1, 4, 12, 17, 1, 1, 0, 1, 4),
]


@pytest.mark.parametrize("case", CASES1D)
def test_conv1d_paths(case):
    """The 1-D launchers against the 2-D oracle with H = 1 (conv.cu:324-400, 495-598)."""
    from jstorch_b200 import conv
    B, Ci, Co, L, K, s, p, d, g = case
    rng = np.random.default_rng(sum(case))
    x = rng.standard_normal((B, Ci, L)).astype(np.float32)
    w = rng.standard_normal((Co, Ci // g, K)).astype(np.float32)
    b = rng.standard_normal(Co).astype(np.float32)
    x4, w4 = x[:, :, None, :], w[:, :, None, :]
    S, P, D = (1, s), (0, p), (1, d)
    y = _host(conv.conv1d(_dev(x), _dev(w), _dev(b), s, p, d, g))
    _ok(y, oracle.conv2d_f64(x4, w4, b, S, P, D, g)[:, :, 0], _bound_conv2d(x4, w4, b, S, P, D, g)[:, :, 0])
    go = rng.standard_normal(y.shape).astype(np.float32)
    gw = _host(conv.conv1d_backward_weight(_dev(x), _dev(go), K, s, p, d, g))
    go4 = go[:, :, None, :]
    _ok(gw, oracle.conv2d_backward_weight_f64(x4, go4, (1, K), S, P, D, g)[:, :, 0],
        _bound_conv2d_bw(x4, go4, (1, K), S, P, D, g)[:, :, 0])
    # transposed: weight [C_in, C_out/g, K]
    wt = rng.standard_normal((Ci, Co // g, K)).astype(np.float32)
    wt4 = wt[:, :, None, :]
    yt = _host(conv.conv_transpose1d(_dev(x), _dev(wt), _dev(b), s, p, 0, d, g))
    _ok(yt, oracle.conv_transpose2d_f64(x4, wt4, b, S, P, D, g)[:, :, 0],
        _bound_conv_transpose2d(x4, wt4, b, S, P, D, g, 0)[:, :, 0])
    got = rng.standard_normal(yt.shape).astype(np.float32)
    got4 = got[:, :, None, :]
    gwt = _host(conv.conv_transpose1d_backward_weight(_dev(x), _dev(got), K, s, p, d, g))
    _ok(gwt, oracle.conv_transpose2d_backward_weight_f64(x4, got4, (1, K), S, P, D, g)[:, :, 0],
        _bound_conv_transpose2d_bw(x4, got4, (1, K), S, P, D, g)[:, :, 0])


def test_direct_1x1_leaves_col_buf_untouched():
    """A 1 x 1, stride-1, unpadded conv2d reads the input as its column matrix."""
    import torch
    from jstorch_b200 import _lib
    rng = np.random.default_rng(1)
    x = _dev(rng.standard_normal((2, 8, 5, 7)))
    w = _dev(rng.standard_normal((4, 8, 1, 1)))
    out = torch.empty((2, 4, 5, 7), device="cuda")
    col = torch.full((2 * 8 * 35,), 7.0, device="cuda")
    _lib.load().launch_conv2d(x.data_ptr(), w.data_ptr(), None, out.data_ptr(), col.data_ptr(), 2, 8, 5, 7, 4, 1, 1,
                              1, 1, 0, 0, 1, 1, 1, 5, 7, torch.cuda.current_stream().cuda_stream)
    _lib.check_last()
    torch.cuda.synchronize()
    assert bool((col == 7.0).all())
    X, Wt = x.cpu().numpy(), w.cpu().numpy()
    one = (1, 1)
    _ok(out.cpu().numpy().astype(np.float64), oracle.conv2d_f64(X, Wt), _bound_conv2d(X, Wt, None, one, (0, 0), one, 1))


GOLDEN_CONV = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "ref_conv_int.npz"


@pytest.mark.parametrize("kernel_path", ["auto"])
def test_launchers_reproduce_reference_outputs_exactly(kernel_path):
    """The fixtures of tests/golden/ref_conv_int.npz hold the reference's own
    conv.cu launchers' outputs on integer-valued inputs (exact there).  Each of
    this library's launchers, on the same inputs and geometry, must return the
    same values bit for bit: small integers are exact in the 3xTF32 split and
    in the FFMA kernel's fp32 accumulation."""
    from jstorch_b200 import conv
    gd = np.load(GOLDEN_CONV)
    names = sorted({k.split("__")[0] for k in gd.files})
    assert len(names) == 9
    for name in names:
        B, Ci, H, W, Co, kH, kW, sH, sW, pH, pW, dH, dW, g, opH, opW = [int(v) for v in gd[f"{name}__params"]]
        one_d = H == 1 and kH == 1
        x = gd[f"{name}__x"]
        want = gd[f"{name}__out"]
        if "bw" in name:
            go = gd[f"{name}__go"]
            if one_d:
                fn = conv.conv_transpose1d_backward_weight if name.startswith("convT") else conv.conv1d_backward_weight
                got = fn(_dev(x[:, :, 0]), _dev(go[:, :, 0]), kW, sW, pW, dW, g)
            else:
                fn = conv.conv_transpose2d_backward_weight if name.startswith("convT") else conv.conv2d_backward_weight
                got = fn(_dev(x), _dev(go), (kH, kW), (sH, sW), (pH, pW), (dH, dW), g)
        else:
            w = gd[f"{name}__w"]
            b = _dev(gd[f"{name}__bias"]) if f"{name}__bias" in gd.files else None
            if one_d:
                if name.startswith("convT"):
                    got = conv.conv_transpose1d(_dev(x[:, :, 0]), _dev(w[:, :, 0]), b, sW, pW, opW, dW, g)
                else:
                    got = conv.conv1d(_dev(x[:, :, 0]), _dev(w[:, :, 0]), b, sW, pW, dW, g)
            elif name.startswith("convT"):
                got = conv.conv_transpose2d(_dev(x), _dev(w), b, (sH, sW), (pH, pW), (opH, opW), (dH, dW), g)
            else:
                got = conv.conv2d(_dev(x), _dev(w), b, (sH, sW), (pH, pW), (dH, dW), g)
        got = _host(got).astype(np.float32).reshape(want.shape)
        np.testing.assert_array_equal(got, want, err_msg=name)
