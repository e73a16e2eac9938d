"""CPU checks of the C ABI boundary: the library loads, exports every function
include/jstorch_gemm.h declares, keeps the reference launcher names, and
validates arguments without touching a GPU."""
import ctypes
import subprocess

import pytest

from jstorch_b200 import _lib

REFERENCE_LAUNCHERS = ["launch_matmul", "launch_bmm", "launch_linear"]


def test_library_is_built_for_sm100a_only():
    from jstorch_b200 import build
    assert _lib.LIB_PATH.exists(), "run python -m jstorch_b200.build"
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert all("arch=" not in f for f in build.NVFLAGS if f not in build.ARCH)


def test_every_header_function_is_exported():
    names = _lib.header_functions()
    for n in REFERENCE_LAUNCHERS + ["jst_gemm_ex", "jst_matmul_host", "jst_last_error"]:
        assert n in names
    lib = _lib.load()
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/jstorch_gemm.h but not exported"
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in nm.splitlines() if " T " in line}
    for n in names:
        assert n in exported, n


CONV_LAUNCHERS = ["launch_conv1d", "launch_conv_transpose1d", "launch_conv2d", "launch_conv_transpose2d",
                  "launch_conv1d_backward_weight", "launch_conv2d_backward_weight",
                  "launch_conv_transpose1d_backward_weight", "launch_conv_transpose2d_backward_weight"]


def test_conv_header_matches_reference_names_and_is_exported():
    names = _lib.header_functions(_lib.CONV_HEADER)
    assert sorted(names) == sorted(CONV_LAUNCHERS)  # conv.cu:324-627, the eight im2col-GEMM sites
    lib = _lib.load()
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in nm.splitlines() if " T " in line}
    for n in names:
        assert hasattr(lib, n) and n in exported, n


def test_conv_argument_validation_without_gpu():
    """Bad geometry is rejected on the host before anything is launched."""
    lib = _lib.load()
    # groups that do not divide the channels
    lib.launch_conv2d(16, 16, None, 16, 16, 1, 3, 8, 8, 4, 3, 3, 1, 1, 1, 1, 1, 1, 2, 8, 8, None)
    assert lib.jst_get_last_status() == 1 and b"groups" in lib.jst_last_error()
    # stride 0
    lib.launch_conv1d(16, 16, None, 16, 16, 1, 4, 8, 4, 3, 0, 1, 1, 1, 8, None)
    assert lib.jst_get_last_status() == 1
    lib.launch_conv2d_backward_weight(16, 16, 16, 16, 1, 4, 8, 8, 4, 0, 3, 1, 1, 1, 1, 1, 1, 1, 8, 8, None)
    assert lib.jst_get_last_status() == 1


def test_copy_entry_points_validate_without_gpu():
    lib = _lib.load()
    assert lib.jst_copy_h2d(None, None, 16, None) == 1  # JST_ERR_ARG: null pointers
    assert lib.jst_copy_d2h(None, None, 16, None) == 1
    assert b"null" in lib.jst_last_error()


def test_desc_layout_matches_c():
    # jst_gemm_desc_init writes through the C struct; the ctypes mirror must
    # read back the same fields
    lib = _lib.load()
    d = _lib.GemmDesc()
    lib.jst_gemm_desc_init(ctypes.byref(d), 3, 5, 7, 0x1000, 0x2000, 0x3000)
    assert (d.M, d.N, d.K) == (3, 5, 7)
    assert (d.A, d.B, d.C) == (0x1000, 0x2000, 0x3000)
    assert (d.lda, d.ldb, d.ldc) == (7, 5, 5)
    assert (d.strideA, d.strideB, d.strideC) == (21, 35, 15)
    assert d.batch == 1 and d.epilogue == 0 and d.kernel == 0 and d.stream is None


@pytest.mark.parametrize("field,value", [("M", -1), ("batch", 0), ("transA", 2), ("epilogue", 9), ("epilogue", 5), ("kernel", 7),
                                         ("lda", 2), ("ldc", 1)])
def test_argument_validation_without_gpu(field, value):
    lib = _lib.load()
    d = _lib.GemmDesc()
    lib.jst_gemm_desc_init(ctypes.byref(d), 4, 4, 4, 0x1000, 0x2000, 0x3000)
    setattr(d, field, value)
    rc = lib.jst_gemm_ex(ctypes.byref(d))
    assert rc == 1, (rc, lib.jst_last_error())
    assert lib.jst_get_last_status() == 1
    assert lib.jst_last_error()
    with pytest.raises(_lib.JstError):
        _lib.check(rc)


def test_bias_epilogue_requires_bias():
    lib = _lib.load()
    d = _lib.GemmDesc()
    lib.jst_gemm_desc_init(ctypes.byref(d), 4, 4, 4, 0x1000, 0x2000, 0x3000)
    d.epilogue = _lib.EPI_BIAS
    assert lib.jst_gemm_ex(ctypes.byref(d)) == 1


def test_no_device_is_an_error_not_a_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    d = _lib.GemmDesc()
    lib.jst_gemm_desc_init(ctypes.byref(d), 4, 4, 4, 0x1000, 0x2000, 0x3000)
    assert lib.jst_gemm_ex(ctypes.byref(d)) == 8  # JST_ERR_NO_DEVICE


def test_rnn_header_exported_and_validates_without_gpu():
    names = _lib.header_functions(_lib.RNN_HEADER)
    assert names == ["jst_gru_layer_backward", "jst_gru_layer_forward", "jst_gru_layer_forward_train"]
    lib = _lib.load()
    for n in names:
        assert hasattr(lib, n)
    # ld_out < hidden and a negative size are rejected on the host
    assert lib.jst_gru_layer_forward(16, 2, 2, 4, 8, 16, 16, None, None, None, 0, 16, 4, None, None) == 1
    assert lib.jst_gru_layer_forward(16, -1, 2, 4, 8, 16, 16, None, None, None, 0, 16, 8, None, None) == 1
    # training entry points: a null saved buffer, an unknown accumulate bit
    # and a negative size are rejected on the host
    assert lib.jst_gru_layer_forward_train(16, 2, 2, 4, 8, 16, 16, None, None, None, 0, 16, 8, None, None,
                                           None) == 1
    bw = lambda acc, seq=2: lib.jst_gru_layer_backward(16, seq, 2, 4, 8, 16, 16, None, 0, 16, 8, 16, 16, 8, None,
                                                       None, None, None, None, None, None, acc, None)
    assert bw(8) == 1
    assert bw(0, seq=-1) == 1
