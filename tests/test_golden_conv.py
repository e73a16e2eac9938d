"""Pins of the convolution oracle against the reference itself (CPU only).

tests/golden/ref_conv_int.npz was produced by tests/golden/make_conv_golden.py,
which ran the reference's own native/ops/conv.cu (built unmodified into
oracle/_ref/; im2col / col2im kernels and cuBLAS sgemm with TF32 math) on a
B200 with integer-valued inputs, where TF32 and fp32 accumulation are exact.
The oracle's fp64 restatements (oracle.conv2d_f64 and friends; 1-D as 2-D
with H = 1) must reproduce every output bit for bit: that pins their layouts
-- batch-outer columns, grouped weights, stride / padding / dilation, the
transposed convolution's col2im and output padding, the bias -- to the
reference's launchers (conv.cu:324-627)."""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "ref_conv_int.npz"
NAMES = ["conv2d_g2", "conv2d_1x1", "convT2d_g2", "conv2d_bw_g2", "convT2d_bw_g2", "conv1d_g2", "convT1d_g2",
         "conv1d_bw_g2", "convT1d_bw_g2"]


@pytest.fixture(scope="module")
def golden():
    if not GOLDEN.exists():
        pytest.fail(f"missing golden fixture {GOLDEN}; regenerate with tests/golden/make_conv_golden.py on a GPU box")
    return np.load(GOLDEN)


@pytest.mark.parametrize("name", NAMES)
def test_oracle_reproduces_reference_conv_launcher(golden, name):
    p = [int(v) for v in golden[f"{name}__params"]]
    B, Ci, H, W, Co, kH, kW, sH, sW, pH, pW, dH, dW, g, opH, opW = p
    with_bias = f"{name}__bias" in golden.files
    x = golden[f"{name}__x"]
    out = golden[f"{name}__out"]
    geo = dict(stride=(sH, sW), padding=(pH, pW), dilation=(dH, dW), groups=g)
    if "bw" not in name:
        w = golden[f"{name}__w"]
        bias = golden[f"{name}__bias"] if with_bias else None
        if name.startswith("convT"):
            ref = oracle.conv_transpose2d_f64(x, w, bias, output_padding=(opH, opW), **geo)
        else:
            ref = oracle.conv2d_f64(x, w, bias, **geo)
    else:
        go = golden[f"{name}__go"]
        fn = oracle.conv_transpose2d_backward_weight_f64 if name.startswith("convT") else \
            oracle.conv2d_backward_weight_f64
        ref = fn(x, go, (kH, kW), **geo)
    assert ref.shape == out.shape, (ref.shape, out.shape)
    assert np.isfinite(out).all()
    np.testing.assert_array_equal(ref, out)
