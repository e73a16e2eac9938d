"""Pins the convolution restatements of the oracle (oracle.conv2d_f64 and
friends, restating native/ops/conv.cu) against an independent
implementation: torch's fp64 CPU convolutions and their autograd weight
gradients.  CPU only."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle

CASES = [
    # B, Ci, Co, H, W, k, stride, padding, dilation, groups
    (2, 3, 4, 9, 11, (3, 3), (1, 1), (1, 1), (1, 1), 1),
    (1, 4, 6, 8, 8, (3, 2), (2, 1), (0, 2), (1, 2), 2),
    (3, 6, 6, 7, 10, (1, 1), (1, 1), (0, 0), (1, 1), 3),
    (2, 2, 5, 12, 5, (5, 3), (3, 2), (2, 1), (2, 1), 1),
    (1, 8, 8, 1, 17, (1, 4), (1, 3), (0, 2), (1, 2), 4),  # a 1-D case (H = 1)
]


@pytest.mark.parametrize("case", CASES)
def test_conv2d_and_weight_grad(case):
    B, Ci, Co, H, W, k, s, p, d, g = case
    rng = np.random.default_rng(sum(case[:5]))
    x = rng.standard_normal((B, Ci, H, W))
    w = rng.standard_normal((Co, Ci // g, *k))
    b = rng.standard_normal(Co)
    xt = torch.from_numpy(x)
    wt = torch.from_numpy(w).requires_grad_(True)
    y = F.conv2d(xt, wt, torch.from_numpy(b), stride=s, padding=p, dilation=d, groups=g)
    ours = oracle.conv2d_f64(x, w, b, s, p, d, g)
    np.testing.assert_allclose(ours, y.detach().numpy(), rtol=1e-12, atol=1e-12)
    go = rng.standard_normal(y.shape)
    y.backward(torch.from_numpy(go))
    gw = oracle.conv2d_backward_weight_f64(x, go, k, s, p, d, g)
    np.testing.assert_allclose(gw, wt.grad.numpy(), rtol=1e-12, atol=1e-11)


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("op", [(0, 0), (1, 0)])
def test_conv_transpose2d_and_weight_grad(case, op):
    B, Ci, Co, H, W, k, s, p, d, g = case
    if op[0] >= max(s[0], d[0]):
        pytest.skip("output padding must be smaller than stride or dilation")
    rng = np.random.default_rng(sum(case[:5]) + 7)
    x = rng.standard_normal((B, Ci, H, W))
    w = rng.standard_normal((Ci, Co // g, *k))
    b = rng.standard_normal(Co)
    wt = torch.from_numpy(w).requires_grad_(True)
    y = F.conv_transpose2d(torch.from_numpy(x), wt, torch.from_numpy(b), stride=s, padding=p, output_padding=op,
                           dilation=d, groups=g)
    ours = oracle.conv_transpose2d_f64(x, w, b, s, p, d, g, op)
    np.testing.assert_allclose(ours, y.detach().numpy(), rtol=1e-12, atol=1e-12)
    go = rng.standard_normal(y.shape)
    y.backward(torch.from_numpy(go))
    gw = oracle.conv_transpose2d_backward_weight_f64(x, go, k, s, p, d, g)
    np.testing.assert_allclose(gw, wt.grad.numpy(), rtol=1e-12, atol=1e-11)


def test_output_sizes():
    # tensor.cpp:469-470 and :484-485
    assert oracle.conv_out_size(32, 3, 1, 1, 1) == 32
    assert oracle.conv_out_size(32, 3, 2, 1, 1) == 16
    assert oracle.conv_out_size(10, 3, 1, 0, 2) == 6
    assert oracle.conv_transpose_out_size(16, 4, 2, 1, 1) == 32
    assert oracle.conv_transpose_out_size(5, 3, 2, 0, 1, 1) == 12

