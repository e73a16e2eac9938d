"""Python side of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only to check results or to time the CPU baseline; the
product (jstorch_b200) never calls it.

  gemm_f64 / max_rel_err / sgemm_f32_cpu   ctypes wrappers of oracle.c
  mlp_forward_backward                     fp64 restatement of one forward +
                                           backward of the reference's
                                           nn.Linear / ReLU / Sequential MLP
  conv2d_f64 / conv_transpose2d_f64 /      fp64 restatements of the im2col-GEMM
  conv2d_backward_weight_f64 /             convolution launchers (1-D = 2-D
  conv_transpose2d_backward_weight_f64     with H = 1), tap by tap
  gru_forward_f64                          fp64 restatement of the reference's GRU
  gru_backward_f64                         its gradients (what GradTensor computes)

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


# ------------------------------------------------------------- convolutions
# Restated from native/ops/conv.cu with the tensor shapes of native/core/tensor.cpp:
#   im2col            conv.cu:202-220   col[b, c*kk + kh*kW + kw, ho*Wo + wo] =
#                                       x[b, c, ho*sH - pH + kh*dH, wo*sW - pW + kw*dW] (0 outside)
#   conv2d            conv.cu:402-434   out[b, g] = W_g . col[b, g] (+ bias[co])
#   conv_transpose2d  conv.cu:436-466   col[b, g] = W_g^T . x[b, g]; out = col2im(col) (+ bias)
#   col2im            conv.cu:223-247   out[b, c, h, w] = sum of col entries whose tap maps to (h, w)
#   backward weight   conv.cu:530-563   gw_g = sum_b go[b, g] . col[b, g]^T
#                     conv.cu:600-627   gw_g = sum_b x[b, g] . im2col(go)[b, g]^T
#   output sizes      tensor.cpp:469-470 (conv), 484-485 (transposed)
# Each product is accumulated in fp64 tap by tap (no col matrix is formed).


def conv_out_size(n, k, s, p, d):
    """tensor.cpp:469: (n + 2p - d(k-1) - 1) / s + 1."""
    return (n + 2 * p - d * (k - 1) - 1) // s + 1


def conv_transpose_out_size(n, k, s, p, d, op=0):
    """tensor.cpp:484: (n - 1)s - 2p + d(k-1) + op + 1."""
    return (n - 1) * s - 2 * p + d * (k - 1) + op + 1


def _pad_to(x, pH, pW, need_h, need_w):
    """Zero-pad H by pH before and W by pW before, and after so that the
    padded extents are at least need_h x need_w."""
    H, W = x.shape[2], x.shape[3]
    return np.pad(x, ((0, 0), (0, 0), (pH, max(0, need_h - H - pH)), (pW, max(0, need_w - W - pW))))


def _taps(xp, kh, kw, dH, dW, sH, sW, Ho, Wo):
    """xp[:, :, kh*dH + ho*sH, kw*dW + wo*sW] for ho < Ho, wo < Wo."""
    return xp[:, :, kh * dH: kh * dH + sH * (Ho - 1) + 1: sH, kw * dW: kw * dW + sW * (Wo - 1) + 1: sW]


def conv2d_f64(x, w, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1):
    """Convolution (conv.cu:402-434): x [B, Ci, H, W], w [Co, Ci/g, kH, kW],
    bias [Co] or None -> [B, Co, Ho, Wo] in fp64."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    B, Ci, H, W = x.shape
    Co, Cig, kH, kW = w.shape
    (sH, sW), (pH, pW), (dH, dW) = stride, padding, dilation
    Ho, Wo = conv_out_size(H, kH, sH, pH, dH), conv_out_size(W, kW, sW, pW, dW)
    Cog = Co // groups
    xp = _pad_to(x, pH, pW, (Ho - 1) * sH + (kH - 1) * dH + 1, (Wo - 1) * sW + (kW - 1) * dW + 1)
    out = np.zeros((B, Co, Ho, Wo))
    for g in range(groups):
        xg = xp[:, g * Cig:(g + 1) * Cig]
        wg = w[g * Cog:(g + 1) * Cog]
        for kh in range(kH):
            for kw in range(kW):
                out[:, g * Cog:(g + 1) * Cog] += np.einsum(
                    "bchw,oc->bohw", _taps(xg, kh, kw, dH, dW, sH, sW, Ho, Wo), wg[:, :, kh, kw], optimize=True)
    if bias is not None:
        out += np.asarray(bias, np.float64)[None, :, None, None]
    return out


def conv_transpose2d_f64(x, w, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1,
                         output_padding=(0, 0)):
    """Transposed convolution (conv.cu:436-466): x [B, Ci, Hi, Wi],
    w [Ci, Co/g, kH, kW] -> [B, Co, Ho, Wo] in fp64: input pixel (hi, wi)
    scatters into output (hi*sH - pH + kh*dH, wi*sW - pW + kw*dW)."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    B, Ci, Hi, Wi = x.shape
    _, Cog, kH, kW = w.shape
    (sH, sW), (pH, pW), (dH, dW) = stride, padding, dilation
    Co = Cog * groups
    Cig = Ci // groups
    Ho = conv_transpose_out_size(Hi, kH, sH, pH, dH, output_padding[0])
    Wo = conv_transpose_out_size(Wi, kW, sW, pW, dW, output_padding[1])
    Hc = max(Ho + pH, (Hi - 1) * sH + (kH - 1) * dH + 1)
    Wc = max(Wo + pW, (Wi - 1) * sW + (kW - 1) * dW + 1)
    canvas = np.zeros((B, Co, Hc, Wc))
    for g in range(groups):
        xg = x[:, g * Cig:(g + 1) * Cig]
        wg = w[g * Cig:(g + 1) * Cig]
        for kh in range(kH):
            for kw in range(kW):
                canvas[:, g * Cog:(g + 1) * Cog, kh * dH: kh * dH + sH * (Hi - 1) + 1: sH,
                       kw * dW: kw * dW + sW * (Wi - 1) + 1: sW] += np.einsum("bchw,co->bohw", xg, wg[:, :, kh, kw], optimize=True)
    out = canvas[:, :, pH:pH + Ho, pW:pW + Wo].copy()
    if bias is not None:
        out += np.asarray(bias, np.float64)[None, :, None, None]
    return out


def conv2d_backward_weight_f64(x, go, kernel, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1):
    """Weight gradient of conv2d (conv.cu:530-563): x [B, Ci, H, W],
    go [B, Co, Ho, Wo] -> [Co, Ci/g, kH, kW] in fp64."""
    x = np.asarray(x, np.float64)
    go = np.asarray(go, np.float64)
    B, Ci, H, W = x.shape
    _, Co, Ho, Wo = go.shape
    kH, kW = kernel
    (sH, sW), (pH, pW), (dH, dW) = stride, padding, dilation
    Cig, Cog = Ci // groups, Co // groups
    xp = _pad_to(x, pH, pW, (Ho - 1) * sH + (kH - 1) * dH + 1, (Wo - 1) * sW + (kW - 1) * dW + 1)
    gw = np.zeros((Co, Cig, kH, kW))
    for g in range(groups):
        xg = xp[:, g * Cig:(g + 1) * Cig]
        gg = go[:, g * Cog:(g + 1) * Cog]
        for kh in range(kH):
            for kw in range(kW):
                gw[g * Cog:(g + 1) * Cog, :, kh, kw] = np.einsum(
                    "bohw,bchw->oc", gg, _taps(xg, kh, kw, dH, dW, sH, sW, Ho, Wo), optimize=True)
    return gw


def conv_transpose2d_backward_weight_f64(x, go, kernel, stride=(1, 1), padding=(0, 0), dilation=(1, 1), groups=1):
    """Weight gradient of conv_transpose2d (conv.cu:600-627): x [B, Ci, Hi, Wi],
    go [B, Co, Ho, Wo] -> [Ci, Co/g, kH, kW] in fp64; im2col of go over the
    input grid: go[b, co, hi*sH - pH + kh*dH, wi*sW - pW + kw*dW] (0 outside)."""
    x = np.asarray(x, np.float64)
    go = np.asarray(go, np.float64)
    B, Ci, Hi, Wi = x.shape
    _, Co, Ho, Wo = go.shape
    kH, kW = kernel
    (sH, sW), (pH, pW), (dH, dW) = stride, padding, dilation
    Cig, Cog = Ci // groups, Co // groups
    gp = _pad_to(go, pH, pW, (Hi - 1) * sH + (kH - 1) * dH + 1, (Wi - 1) * sW + (kW - 1) * dW + 1)
    gw = np.zeros((Ci, Cog, kH, kW))
    for g in range(groups):
        xg = x[:, g * Cig:(g + 1) * Cig]
        gg = gp[:, g * Cog:(g + 1) * Cog]
        for kh in range(kH):
            for kw in range(kW):
                gw[g * Cig:(g + 1) * Cig, :, kh, kw] = np.einsum(
                    "bchw,bohw->co", xg, _taps(gg, kh, kw, dH, dW, sH, sW, Hi, Wi), optimize=True)
    return gw


# --------------------------------------------------------------------- GRU
def gru_forward_f64(x, params, hidden, num_layers=1, bidirectional=False, h0=None):
    """The reference GRU (src/nn.js:451-536) in fp64, batch_first = False.

    x [seq, batch, in]; params: dict with the PyTorch names weight_ih_l{l}[_reverse]
    [3H, in], weight_hh_l{l} [3H, H], bias_ih_l{l}, bias_hh_l{l} [3H];
    h0 [layers*dirs, batch, H] or None (zeros, nn.js:494).
      _cell          nn.js:477-485  gi = x W_ih^T + b_ih, gh = h W_hh^T + b_hh,
                                    r = sig(gi_r + gh_r), z = sig(gi_z + gh_z),
                                    n = tanh(gi_n + r gh_n), h' = (1 - z) n + z h
      _run_direction nn.js:487-511  reverse walks t = seq-1..0, output row t stays at t
      forward        nn.js:513-535  layer input = previous output (directions
                                    concatenated on features), h_n stacked per layer/direction
    Returns (output [seq, batch, H*dirs], h_n [layers*dirs, batch, H])."""
    x = np.asarray(x, np.float64)
    seq, batch = x.shape[0], x.shape[1]
    sig = lambda v: 1.0 / (1.0 + np.exp(-v))
    dirs = 2 if bidirectional else 1
    inp = x
    hn = []
    for l in range(num_layers):
        outs = []
        for d in range(dirs):
            sfx = "_reverse" if d else ""
            wih = np.asarray(params[f"weight_ih_l{l}{sfx}"], np.float64)
            whh = np.asarray(params[f"weight_hh_l{l}{sfx}"], np.float64)
            bih = np.asarray(params[f"bias_ih_l{l}{sfx}"], np.float64)
            bhh = np.asarray(params[f"bias_hh_l{l}{sfx}"], np.float64)
            H = hidden
            h = np.zeros((batch, H)) if h0 is None else np.asarray(h0[l * dirs + d], np.float64)
            out = np.zeros((seq, batch, H))
            steps = range(seq - 1, -1, -1) if d else range(seq)
            for t in steps:
                gi = inp[t] @ wih.T + bih
                gh = h @ whh.T + bhh
                r = sig(gi[:, :H] + gh[:, :H])
                z = sig(gi[:, H:2 * H] + gh[:, H:2 * H])
                n = np.tanh(gi[:, 2 * H:] + r * gh[:, 2 * H:])
                h = (1 - z) * n + z * h
                out[t] = h
            outs.append(out)
            hn.append(h)
        inp = np.concatenate(outs, axis=2)
    return inp, np.stack(hn)


def gru_backward_f64(x, params, hidden, num_layers=1, bidirectional=False, h0=None, dout=None, dh_n=None):
    """Gradients of the reference GRU (src/nn.js:451-536) in fp64, for the loss
    L = sum(dout * output) + sum(dh_n * h_n), batch_first = False.

    What the reference's GradTensor computes when the GRU's parameters require
    grad (nn.js:442-444): its backward sweep (native/core/autograd.hpp:40-65)
    through the cell's two matmuls ({g . b^T, a^T . g}, autograd.hpp:433-441,
    with b = W^T so dW = g^T . a), the bias adds (unbroadcast = sum over the
    batch, autograd.hpp:324-342), the slices, sigmoid (s' = s (1 - s)), tanh
    (t' = 1 - t^2), the products and the (1 - z) term, composed per step:
        g = dL/dh' ;  dn = g (1 - z) ;  dz = g (h - n) ;  dh = g z + dgh . W_hh
        da_n = dn (1 - n^2) ; da_r = da_n gh_n r (1 - r) ; da_z = dz z (1 - z)
        dgi = (da_r, da_z, da_n) ;  dgh = (da_r, da_z, da_n r)
    Returns (grads {param name: fp64 array}, dx [seq, batch, in], dh0 [layers*dirs,
    batch, H] or None)."""
    x = np.asarray(x, np.float64)
    seq, batch = x.shape[0], x.shape[1]
    H = hidden
    sig = lambda v: 1.0 / (1.0 + np.exp(-v))
    dirs = 2 if bidirectional else 1
    # forward, keeping every step's gate values and the state it started from
    inps, tapes = [], []
    inp = x
    for l in range(num_layers):
        outs, tl = [], []
        for d in range(dirs):
            sfx = "_reverse" if d else ""
            wih = np.asarray(params[f"weight_ih_l{l}{sfx}"], np.float64)
            whh = np.asarray(params[f"weight_hh_l{l}{sfx}"], np.float64)
            bih = np.asarray(params[f"bias_ih_l{l}{sfx}"], np.float64)
            bhh = np.asarray(params[f"bias_hh_l{l}{sfx}"], np.float64)
            h = np.zeros((batch, H)) if h0 is None else np.asarray(h0[l * dirs + d], np.float64)
            out = np.zeros((seq, batch, H))
            tape = {}
            for t in (range(seq - 1, -1, -1) if d else range(seq)):
                gi = inp[t] @ wih.T + bih
                gh = h @ whh.T + bhh
                r = sig(gi[:, :H] + gh[:, :H])
                z = sig(gi[:, H:2 * H] + gh[:, H:2 * H])
                n = np.tanh(gi[:, 2 * H:] + r * gh[:, 2 * H:])
                tape[t] = (r, z, n, gh[:, 2 * H:], h)
                h = (1 - z) * n + z * h
                out[t] = h
            outs.append(out)
            tl.append(tape)
        inps.append(inp)
        tapes.append(tl)
        inp = np.concatenate(outs, axis=2)
    # backward, last layer first
    g_out = np.zeros((seq, batch, H * dirs)) if dout is None else np.asarray(dout, np.float64)
    grads = {}
    dh0 = np.zeros((num_layers * dirs, batch, H)) if h0 is not None else None
    for l in range(num_layers - 1, -1, -1):
        inp = inps[l]
        dinp = np.zeros_like(inp)
        for d in range(dirs):
            sfx = "_reverse" if d else ""
            wih = np.asarray(params[f"weight_ih_l{l}{sfx}"], np.float64)
            whh = np.asarray(params[f"weight_hh_l{l}{sfx}"], np.float64)
            gw_ih, gw_hh = np.zeros_like(wih), np.zeros_like(whh)
            gb_ih, gb_hh = np.zeros(3 * H), np.zeros(3 * H)
            dh = np.zeros((batch, H)) if dh_n is None else np.asarray(dh_n[l * dirs + d], np.float64).copy()
            for t in (range(seq) if d else range(seq - 1, -1, -1)):
                r, z, n, ghn, hp = tapes[l][d][t]
                gt = dh + g_out[t, :, d * H:(d + 1) * H]
                dn = gt * (1 - z)
                dz = gt * (hp - n)
                dan = dn * (1 - n * n)
                dar = dan * ghn * r * (1 - r)
                daz = dz * z * (1 - z)
                dgi = np.concatenate([dar, daz, dan], axis=1)
                dgh = np.concatenate([dar, daz, dan * r], axis=1)
                gw_ih += dgi.T @ inp[t]
                gw_hh += dgh.T @ hp
                gb_ih += dgi.sum(0)
                gb_hh += dgh.sum(0)
                dinp[t] += dgi @ wih
                dh = gt * z + dgh @ whh
            if dh0 is not None:
                dh0[l * dirs + d] = dh
            grads[f"weight_ih_l{l}{sfx}"] = gw_ih
            grads[f"weight_hh_l{l}{sfx}"] = gw_hh
            grads[f"bias_ih_l{l}{sfx}"] = gb_ih
            grads[f"bias_hh_l{l}{sfx}"] = gb_hh
        g_out = dinp
    return grads, g_out, dh0
