"""Pins of the oracle against the reference itself (CPU-only test).

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py,
which ran the reference's own native/ops/matmul.cu (cuBLAS sgemm, TF32
tensor-op math; built unmodified into oracle/_ref/) on a B200.  For the
integer-valued cases TF32 is exact, so the oracle must reproduce the
reference's output bit for bit; that pins the layout conventions (row-major
NN, packed batch strides, x.w^T + bias).  The float case pins agreement to
within the reference's TF32 error.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    p = GOLDEN / name
    if not p.exists():
        pytest.fail(f"missing golden fixture {p}; regenerate with tests/golden/make_golden.py on a GPU box")
    return np.load(p)


def test_reference_readme_vector():
    d = _load("ref_readme.npz")
    assert d["c"].tolist() == [[38, 44, 50, 56], [83, 98, 113, 128]]
    np.testing.assert_array_equal(oracle.gemm_f64(d["a"], d["b"]), d["c"])


def test_reference_matmul_integer_exact():
    d = _load("ref_matmul_int.npz")
    np.testing.assert_array_equal(oracle.gemm_f64(d["a"], d["b"]), d["c"])


def test_reference_bmm_integer_exact():
    d = _load("ref_bmm_int.npz")
    np.testing.assert_array_equal(oracle.gemm_f64(d["a"], d["b"]), d["c"])


def test_reference_linear_integer_exact():
    d = _load("ref_linear_int.npz")
    np.testing.assert_array_equal(oracle.gemm_f64(d["x"], d["w"], transB=True, bias=d["bias"]), d["y_bias"])
    np.testing.assert_array_equal(oracle.gemm_f64(d["x"], d["w"], transB=True), d["y"])


def test_reference_float_within_tf32():
    d = _load("ref_matmul_float.npz")
    ref = oracle.gemm_f64(d["a"], d["b"])
    err, _ = oracle.max_rel_err(d["a"], d["b"], d["c"], ref)
    # single-pass TF32 (10-bit mantissa inputs): agreement to ~2^-11 relative
    assert err < 2e-3, err
    assert err > 0.0  # the reference's TF32 math is not the exact fp32 product
