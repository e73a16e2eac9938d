"""ctypes binding of libjstorch_gemm.so (the C ABI in include/jstorch_gemm.h).

The library is loaded from this package directory only.  There is no CPU or
library fallback: if the shared object is missing, or no sm_100 device is
present, every entry point raises.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libjstorch_gemm.so"
HEADER = PKG.parent / "include" / "jstorch_gemm.h"
CONV_HEADER = PKG.parent / "include" / "jstorch_conv.h"
RNN_HEADER = PKG.parent / "include" / "jstorch_rnn.h"

JST_OK = 0
STATUS_NAMES = {
    0: "JST_OK", 1: "JST_ERR_ARG", 2: "JST_ERR_ALIGN", 3: "JST_ERR_CUDA", 4: "JST_ERR_NCCL",
    5: "JST_ERR_TIMEOUT", 6: "JST_ERR_UNSUPPORTED", 7: "JST_ERR_NOMEM", 8: "JST_ERR_NO_DEVICE",
}
EPI_NONE, EPI_BIAS, EPI_RELU, EPI_BIAS_RELU, EPI_MASK = 0, 1, 2, 3, 4
EPI_BIAS_ROW, EPI_BIAS_ROW_RELU = 8, 10
KERNEL_AUTO, KERNEL_TC3XTF32, KERNEL_FFMA = 0, 1, 2
KERNELS = {"auto": KERNEL_AUTO, "tc3xtf32": KERNEL_TC3XTF32, "ffma": KERNEL_FFMA}


class JstError(RuntimeError):
    """A non-OK jst_status returned by the native library."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class GemmDesc(ctypes.Structure):
    """Mirror of `jst_gemm_desc` (field order and C types must match)."""
    _fields_ = [
        ("transA", ctypes.c_int), ("transB", ctypes.c_int),
        ("M", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int),
        ("A", ctypes.c_void_p), ("lda", ctypes.c_int64), ("strideA", ctypes.c_int64),
        ("B", ctypes.c_void_p), ("ldb", ctypes.c_int64), ("strideB", ctypes.c_int64),
        ("C", ctypes.c_void_p), ("ldc", ctypes.c_int64), ("strideC", ctypes.c_int64),
        ("batch", ctypes.c_int),
        ("bias", ctypes.c_void_p),
        ("epilogue", ctypes.c_int),
        ("kernel", ctypes.c_int),
        ("stream", ctypes.c_void_p),
        ("aux", ctypes.c_void_p), ("ld_aux", ctypes.c_int64), ("stride_aux", ctypes.c_int64),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run `python -m jstorch_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    fp = ctypes.POINTER(ctypes.c_float)
    vp = ctypes.c_void_p
    ci = ctypes.c_int
    lib.jst_last_error.restype = ctypes.c_char_p
    lib.jst_last_error.argtypes = []
    lib.jst_get_last_status.restype = ci
    lib.jst_get_last_status.argtypes = []
    lib.jst_gemm_desc_init.restype = None
    lib.jst_gemm_desc_init.argtypes = [ctypes.POINTER(GemmDesc), ci, ci, ci, vp, vp, vp]
    lib.jst_gemm_ex.restype = ci
    lib.jst_gemm_ex.argtypes = [ctypes.POINTER(GemmDesc)]
    lib.jst_gemm_select_kernel.restype = ci
    lib.jst_gemm_select_kernel.argtypes = [ctypes.POINTER(GemmDesc)]
    lib.jst_gemm_tc_noalloc.restype = ci
    lib.jst_gemm_tc_noalloc.argtypes = [ctypes.POINTER(GemmDesc)]
    lib.launch_matmul.restype = None
    lib.launch_matmul.argtypes = [vp, vp, vp, ci, ci, ci, vp]
    lib.launch_bmm.restype = None
    lib.launch_bmm.argtypes = [vp, vp, vp, ci, ci, ci, ci, vp]
    lib.launch_linear.restype = None
    lib.launch_linear.argtypes = [vp, vp, vp, vp, ci, ci, ci, vp]
    lib.jst_matmul_host.restype = ci
    lib.jst_matmul_host.argtypes = [fp, fp, fp, ci, ci, ci]
    lib.jst_matmul_host_async.restype = ci
    lib.jst_matmul_host_async.argtypes = [fp, fp, fp, ci, ci, ci, vp]
    lib.jst_copy_h2d.restype = ci
    lib.jst_copy_h2d.argtypes = [vp, vp, ctypes.c_size_t, vp]
    lib.jst_copy_d2h.restype = ci
    lib.jst_copy_d2h.argtypes = [vp, vp, ctypes.c_size_t, vp]
    lib.jst_device_error.restype = ci
    lib.jst_device_error.argtypes = []
    lib.jst_test_set_device_error.restype = ci
    lib.jst_test_set_device_error.argtypes = [ci]
    lib.jst_release_caches.restype = None
    lib.jst_release_caches.argtypes = []
    lib.jst_launch_count.restype = ctypes.c_int64
    lib.jst_launch_count.argtypes = []
    lib.jst_profile_enable.restype = ci
    lib.jst_profile_enable.argtypes = [ci]
    lib.jst_profile_read.restype = ci
    lib.jst_profile_read.argtypes = [ctypes.POINTER(KernelStat), ci]
    # convolution launchers (include/jstorch_conv.h): 5 pointers, then ints, then the stream
    conv1d_args = [vp] * 5 + [ci] * 10 + [vp]
    conv2d_args = [vp] * 5 + [ci] * 16 + [vp]
    for name in ("launch_conv1d", "launch_conv_transpose1d"):
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = conv1d_args
    for name in ("launch_conv2d", "launch_conv_transpose2d"):
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = conv2d_args
    for name in ("launch_conv1d_backward_weight", "launch_conv_transpose1d_backward_weight"):
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = [vp] * 4 + [ci] * 10 + [vp]
    for name in ("launch_conv2d_backward_weight", "launch_conv_transpose2d_backward_weight"):
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = [vp] * 4 + [ci] * 16 + [vp]
    lib.jst_gru_layer_forward.restype = ci
    lib.jst_gru_layer_forward.argtypes = [vp, ci, ci, ci, ci, vp, vp, vp, vp, vp, ci, vp, ctypes.c_int64, vp, vp]
    lib.jst_gru_layer_forward_train.restype = ci
    lib.jst_gru_layer_forward_train.argtypes = [vp, ci, ci, ci, ci, vp, vp, vp, vp, vp, ci, vp, ctypes.c_int64, vp,
                                                vp, vp]
    lib.jst_gru_layer_backward.restype = ci
    lib.jst_gru_layer_backward.argtypes = ([vp, ci, ci, ci, ci, vp, vp, vp, ci, vp, ctypes.c_int64, vp, vp,
                                            ctypes.c_int64, vp] + [vp] * 6 + [ci, vp])
    _lib = lib
    return lib


class KernelStat(ctypes.Structure):
    """Mirror of `jst_kernel_stat`."""
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int64), ("total_ms", ctypes.c_double)]


def profile_enable(on: bool = True) -> None:
    check(load().jst_profile_enable(1 if on else 0))


def profile_read() -> dict:
    """{kernel family: (launches, total device ms)} since profile_enable()."""
    buf = (KernelStat * 16)()
    n = load().jst_profile_read(buf, 16)
    if n < 0:
        check(-n)
    return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms)) for i in range(min(n, 16))}


def launch_count() -> int:
    return int(load().jst_launch_count())


def check(status: int) -> None:
    """Raise JstError for a non-OK status, with the library's message."""
    if status != JST_OK:
        msg = load().jst_last_error().decode(errors="replace")
        raise JstError(status, msg)


def check_last() -> None:
    """Raise if the last void launcher on this thread failed."""
    check(load().jst_get_last_status())


def header_functions(header: Path = HEADER) -> list[str]:
    """Names of every function a public header declares."""
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*([A-Za-z_][A-Za-z0-9_]*)\s*\(",
                       text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "while", "return", "sizeof")))
