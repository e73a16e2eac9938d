"""Python face of the C ABI: GEMMs on device tensors and the host-array
`torch.matmul(a, b, M, K, N)` of the reference's README.

Device memory, streams and tensor views come from PyTorch (plumbing only);
every product is computed by libjstorch_gemm.so's own sm_100a kernels.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib


def _operand(x, name: str):
    """(trans, ld, batch_stride, rows, cols) of a 2-D or 3-D fp32 CUDA tensor.

    A row-major view gives trans=0; a transposed view (unit stride along the
    rows) gives trans=1, so `W.t()` reaches the kernels as an NT/TN operand
    without a copy.  Other strides are rejected.
    """
    import torch

    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if x.dtype != torch.float32:
        raise TypeError(f"{name} must be float32 (got {x.dtype})")
    if not x.is_cuda:
        raise ValueError(f"{name} must live on a CUDA device")
    if x.dim() not in (2, 3):
        raise ValueError(f"{name} must be 2-D or 3-D")
    rows, cols = x.shape[-2], x.shape[-1]
    s0, s1 = x.stride(-2), x.stride(-1)
    bstride = x.stride(0) if x.dim() == 3 else 0
    if s1 == 1 and (rows == 1 or s0 >= cols):
        return 0, max(s0 if rows > 1 else cols, 1), bstride, rows, cols
    if s0 == 1 and (cols == 1 or s1 >= rows):
        return 1, max(s1 if cols > 1 else rows, 1), bstride, rows, cols
    if cols == 1 and s0 >= 1:
        return 0, s0, bstride, rows, cols
    if rows == 1 and s1 >= 1:
        return 1, s1, bstride, rows, cols
    raise ValueError(f"{name}: unsupported strides {tuple(x.stride())} for shape {tuple(x.shape)}")


def gemm(a, b, out=None, *, bias=None, row_bias=None, relu: bool = False, mask=None, kernel: str = "auto",
         stream=None):
    """out = relu?(a @ b + bias) with a: [M,K] or [B,M,K], b: [K,N] or [B,K,N].

    bias has N elements (one per column); row_bias, exclusive with it, has M
    (one per row: a convolution's output channels).
    mask (a contiguous float32 tensor of out's shape) selects the ReLU-backward
    epilogue instead: out = (a @ b) * (mask > 0); it excludes bias and relu.
    Transposed views of either operand are consumed in place (NT / TN forms).
    Runs asynchronously on `stream` (default: torch's current stream).
    """
    import torch

    ta, lda, sa, M, K = _operand(a, "a")
    tb, ldb, sb, Kb, N = _operand(b, "b")
    if K != Kb:
        raise ValueError(f"matmul shape mismatch: a is [.., {M}, {K}], b is [.., {Kb}, {N}]")
    batched = a.dim() == 3 or b.dim() == 3
    batch = a.shape[0] if a.dim() == 3 else (b.shape[0] if b.dim() == 3 else 1)
    if a.dim() == 3 and b.dim() == 3 and a.shape[0] != b.shape[0]:
        raise ValueError("batch sizes differ")
    shape = (batch, M, N) if batched else (M, N)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=a.device)
    elif tuple(out.shape) != shape or not out.is_contiguous() or out.dtype != torch.float32:
        raise ValueError(f"out must be a contiguous float32 tensor of shape {shape}")
    if bias is not None:
        if bias.dtype != torch.float32 or bias.numel() != N or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous float32 tensor with N elements")
    if row_bias is not None:
        if bias is not None:
            raise ValueError("bias and row_bias are exclusive")
        if row_bias.dtype != torch.float32 or row_bias.numel() != M or not row_bias.is_contiguous():
            raise ValueError("row_bias must be a contiguous float32 tensor with M elements")
    if mask is not None:
        if bias is not None or row_bias is not None or relu:
            raise ValueError("mask excludes bias and relu")
        if tuple(mask.shape) != shape or not mask.is_contiguous() or mask.dtype != torch.float32:
            raise ValueError(f"mask must be a contiguous float32 tensor of shape {shape}")
    d = _lib.GemmDesc()
    d.transA, d.transB = ta, tb
    d.M, d.N, d.K = M, N, K
    d.A, d.lda, d.strideA = a.data_ptr(), lda, sa
    d.B, d.ldb, d.strideB = b.data_ptr(), ldb, sb
    d.C, d.ldc, d.strideC = out.data_ptr(), N, M * N
    d.batch = batch
    d.bias = bias.data_ptr() if bias is not None else None
    d.epilogue = (_lib.EPI_BIAS if bias is not None else 0) | (_lib.EPI_RELU if relu else 0)
    if row_bias is not None:
        d.bias = row_bias.data_ptr()
        d.epilogue = _lib.EPI_BIAS_ROW_RELU if relu else _lib.EPI_BIAS_ROW
    if mask is not None:
        d.epilogue = _lib.EPI_MASK
        d.aux, d.ld_aux, d.stride_aux = mask.data_ptr(), N, M * N
    d.kernel = _lib.KERNELS[kernel]
    st = stream if stream is not None else torch.cuda.current_stream(a.device)
    d.stream = st.cuda_stream
    with torch.cuda.device(a.device):
        _lib.check(_lib.load().jst_gemm_ex(ctypes.byref(d)))
    return out


def select_kernel(M: int, N: int, K: int, batch: int = 1) -> str:
    """Name of the kernel the shape heuristic picks for a packed NN GEMM."""
    d = _lib.GemmDesc()
    lib = _lib.load()
    lib.jst_gemm_desc_init(ctypes.byref(d), M, N, K, 16, 16, 16)
    d.batch = batch
    d.strideA, d.strideB, d.strideC = M * K, K * N, M * N
    k = lib.jst_gemm_select_kernel(ctypes.byref(d))
    return {_lib.KERNEL_TC3XTF32: "tc3xtf32", _lib.KERNEL_FFMA: "ffma"}.get(k, "invalid")


def matmul_host(a: np.ndarray, b: np.ndarray, M: int, K: int, N: int) -> np.ndarray:
    """torch.matmul(a, b, M, K, N) of the reference README (README.md:60-72).

    a, b: row-major float32 arrays with M*K and K*N elements (any shape);
    returns a new float32 array of M*N elements, C = A x B.
    """
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    if a.size != M * K or b.size != K * N:
        raise ValueError(f"expected {M * K} and {K * N} elements, got {a.size} and {b.size}")
    c = np.empty(M * N, dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    _lib.check(_lib.load().jst_matmul_host(a.ctypes.data_as(fp), b.ctypes.data_as(fp), c.ctypes.data_as(fp),
                                           M, K, N))
    return c


def matmul_host_ptr(a_ptr: int, b_ptr: int, c_ptr: int, M: int, K: int, N: int) -> None:
    """jst_matmul_host on raw host addresses (e.g. pinned torch CPU tensors)."""
    fp = ctypes.POINTER(ctypes.c_float)
    _lib.check(_lib.load().jst_matmul_host(ctypes.cast(a_ptr, fp), ctypes.cast(b_ptr, fp),
                                           ctypes.cast(c_ptr, fp), M, K, N))


def matmul_host_async(a_ptr: int, b_ptr: int, c_ptr: int, M: int, K: int, N: int, stream) -> None:
    """jst_matmul_host_async: enqueue H2D, GEMM and D2H on `stream` (a torch
    CUDA stream); host buffers should be pinned for the copies to be async."""
    fp = ctypes.POINTER(ctypes.c_float)
    _lib.check(_lib.load().jst_matmul_host_async(ctypes.cast(a_ptr, fp), ctypes.cast(b_ptr, fp),
                                                 ctypes.cast(c_ptr, fp), M, K, N, stream.cuda_stream))


def device_error() -> int:
    """Synchronise and return (and clear) the kernels' device error word."""
    return _lib.load().jst_device_error()
