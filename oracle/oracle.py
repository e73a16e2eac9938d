"""Python side of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only to check results or to time the CPU baseline; the
product (jstorch_b200) never calls it.

  gemm_f64 / max_rel_err / sgemm_f32_cpu   ctypes wrappers of oracle.c
  mlp_forward_backward                     fp64 restatement of one forward +
                                           backward of the reference's
                                           nn.Linear / ReLU / Sequential MLP

Reference citations are relative to the JsTorch project root.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libref_matmul.so"

_lib = None


def build() -> None:
    """Compile liboracle.so (gcc) if it is missing or stale."""
    src = HERE / "oracle.c"
    if LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= src.stat().st_mtime:
        return
    subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True, capture_output=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIB_PATH))
        vp, ci, cl, cll = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_longlong
        lib.jo_gemm_rows_f64.restype = ci
        lib.jo_gemm_rows_f64.argtypes = [ci, ci, ci, ci, ci, vp, cl, cll, vp, cl, cll, ci, vp, ci, vp, ci, vp]
        lib.jo_max_rel_err.restype = ctypes.c_double
        lib.jo_max_rel_err.argtypes = [ci, ci, ci, ci, ci, vp, cl, cll, vp, cl, cll, ci, vp, vp, cl, cll, vp, vp,
                                       ci, vp]
        lib.jo_sgemm_f32_cpu.restype = ci
        lib.jo_sgemm_f32_cpu.argtypes = [ci, ci, ci, vp, vp, vp, ci, ci, ci]
        lib.jo_max_threads.restype = ci
        lib.jo_max_threads.argtypes = []
        _lib = lib
    return _lib


def _ptr(x: np.ndarray | None):
    return None if x is None else x.ctypes.data


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def _layout(x: np.ndarray, trans: bool):
    """(stored 2-D/3-D array, ld, batch stride) of an operand stored row-major."""
    x = _f32(x)
    ld = x.shape[-1]
    bstride = x.shape[-1] * x.shape[-2] if x.ndim == 3 else 0
    return x, ld, bstride


def gemm_f64(A: np.ndarray, B: np.ndarray, *, transA: bool = False, transB: bool = False,
             bias: np.ndarray | None = None, relu: bool = False, rows=None) -> np.ndarray:
    """fp64-accumulated op(A) op(B) [+ bias] [relu] on selected rows.

    A is stored [M,K] ([K,M] if transA), optionally with a leading batch dim;
    B is stored [K,N] ([N,K] if transB).  Follows native/ops/matmul.cu:28-37
    (NN, beta 0), :40-50 (packed batch strides), :54-67 (x w^T + bias) and
    native/ops/kernels.cuh:50 (relu after the bias, nn.js:105-110 + :547).
    Returns [batch?, nrows, N] float64.
    """
    A, lda, sA = _layout(A, transA)
    B, ldb, sB = _layout(B, transB)
    M = A.shape[-1] if transA else A.shape[-2]
    K = A.shape[-2] if transA else A.shape[-1]
    N = B.shape[-2] if transB else B.shape[-1]
    Kb = B.shape[-1] if transB else B.shape[-2]
    assert K == Kb, (K, Kb)
    batch = max(A.shape[0] if A.ndim == 3 else 1, B.shape[0] if B.ndim == 3 else 1)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    nrows = M if rows_arr is None else rows_arr.size
    out = np.empty((batch, nrows, N), dtype=np.float64)
    bias_arr = None if bias is None else _f32(bias)
    rc = load().jo_gemm_rows_f64(int(transA), int(transB), M, N, K, _ptr(A), lda, sA, _ptr(B), ldb, sB, batch,
                                 _ptr(bias_arr), int(relu), _ptr(rows_arr), nrows, out.ctypes.data)
    assert rc == 0
    return out if (A.ndim == 3 or B.ndim == 3) else out[0]


def max_rel_err(A, B, C_test, C_ref, *, transA=False, transB=False, bias=None, rows=None):
    """max |C - C_ref| / (||op(A)_i,:|| ||op(B)_:,j|| + |bias_j|) over the rows
    C_ref was computed on.  Returns (err, (batch, row, col) of the worst)."""
    A, lda, sA = _layout(A, transA)
    B, ldb, sB = _layout(B, transB)
    C_test = _f32(C_test)
    M = A.shape[-1] if transA else A.shape[-2]
    K = A.shape[-2] if transA else A.shape[-1]
    N = B.shape[-2] if transB else B.shape[-1]
    batch = max(A.shape[0] if A.ndim == 3 else 1, B.shape[0] if B.ndim == 3 else 1)
    ref = np.ascontiguousarray(C_ref, dtype=np.float64)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    nrows = M if rows_arr is None else rows_arr.size
    worst = np.zeros(3, dtype=np.int32)
    bias_arr = None if bias is None else _f32(bias)
    e = load().jo_max_rel_err(int(transA), int(transB), M, N, K, _ptr(A), lda, sA, _ptr(B), ldb, sB, batch,
                              _ptr(bias_arr), C_test.ctypes.data, N, M * N if C_test.ndim == 3 else 0,
                              ref.ctypes.data, _ptr(rows_arr), nrows, worst.ctypes.data)
    return float(e), tuple(int(v) for v in worst)


def sgemm_f32_cpu(A: np.ndarray, B: np.ndarray, C: np.ndarray, row0: int = 0, nrows: int | None = None,
                  threads: int = 0) -> int:
    """The CPU baseline: fp32 i-k-j triple loop on rows [row0, row0+nrows) of C
    (OpenMP over rows); returns the thread count used."""
    M, K = A.shape
    N = B.shape[1]
    nrows = M - row0 if nrows is None else nrows
    assert A.flags.c_contiguous and B.flags.c_contiguous and C.flags.c_contiguous
    assert A.dtype == B.dtype == C.dtype == np.float32
    return load().jo_sgemm_f32_cpu(M, N, K, A.ctypes.data, B.ctypes.data, C.ctypes.data, row0, nrows, threads)


def max_threads() -> int:
    return load().jo_max_threads()


# --------------------------------------------------------------------- MLP
def mlp_forward_backward(x: np.ndarray, weights: list, biases: list) -> dict:
    """One forward + backward of Sequential(Linear, ReLU, Linear, ReLU, ..., Linear)
    with loss = sum(y), restated in fp64.

      Linear.forward   y = x.matmul(W.transpose()).add(b)      src/nn.js:105-110
      ReLU.forward     relu(x)                                 src/nn.js:547
      backward seed    upstream = ones(shape(y))               native/binding/napi.cpp:975-977
      matmul_ grads    {g . b^T, a^T . g}                       native/core/autograd.hpp:439
                       with b = W^T:  dX = g . W,  d(W^T) = X^T . g
      transpose_ grad  dW = (d(W^T))^T                         autograd.hpp:532-538
      add_ grads       unbroadcast(g, [out]) = g.sum(0)         autograd.hpp:324-342
      relu_ grad       g * (x > 0)  (0 at x == 0)              autograd.hpp:127-134

    Returns fp64 arrays: 'z' (pre-activations), 'h' (layer inputs), 'y',
    'dW', 'db' (per layer) and 'dh' (gradient w.r.t. each layer input).
    """
    h = [np.asarray(x, dtype=np.float64)]
    z = []
    L = len(weights)
    for l, (W, b) in enumerate(zip(weights, biases)):
        zl = h[-1] @ np.asarray(W, dtype=np.float64).T + np.asarray(b, dtype=np.float64)
        z.append(zl)
        if l < L - 1:
            h.append(np.where(zl > 0, zl, 0.0))
    y = z[-1]
    g = np.ones_like(y)
    dW, db, dh = [None] * L, [None] * L, [None] * L
    for l in range(L - 1, -1, -1):
        W = np.asarray(weights[l], dtype=np.float64)
        db[l] = g.sum(axis=0)
        dW[l] = (h[l].T @ g).T
        dh[l] = g @ W
        if l > 0:
            g = dh[l] * (z[l - 1] > 0)
    return {"z": z, "h": h, "y": y, "dW": dW, "db": db, "dh": dh}
