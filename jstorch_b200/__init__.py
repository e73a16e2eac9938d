"""jstorch_b200 -- B200 (sm_100a) replacement for JsTorch's fp32 matmul path.

Native libraries: libjstorch_gemm.so (C ABI in include/jstorch_gemm.h,
jstorch_conv.h, jstorch_rnn.h) and libjstorch_dist.so (include/jstorch_dist.h).
Python surface, mirroring the reference's JS surface for this path:

    jstorch_b200.torch.matmul(a, b, M, K, N)   host float32 arrays in and out
    jstorch_b200.gemm(a, b, bias=, relu=)       device tensors, NN/NT/TN views,
                                                row bias, ReLU-backward mask
    jstorch_b200.conv                           the im2col-GEMM convolutions
    jstorch_b200.rnn.GRU                        the GRU module (forward)
    jstorch_b200.loader                         the .bin model format
    jstorch_b200.dist.Comm                      row- / batch-sharded GEMMs over GPUs
    jstorch_b200._core                          Tensor, GradTensor, CompiledGraph
    jstorch_b200.nn                             Linear, ReLU, Sequential
"""
from __future__ import annotations

from types import SimpleNamespace

from ._lib import JstError, load  # noqa: F401
from .gemm import device_error, gemm, matmul_host, matmul_host_async, select_kernel  # noqa: F401

# `import { torch } from '@alex000291/jstorch'; torch.matmul(a, b, M, K, N)`
torch = SimpleNamespace(matmul=matmul_host)

__all__ = ["gemm", "matmul_host", "matmul_host_async", "select_kernel", "device_error", "torch", "JstError", "load"]
