"""Convolutions through the im2col-GEMM launchers of libjstorch_gemm.so
(include/jstorch_conv.h) on torch CUDA tensors.

Mirrors the reference's Tensor methods that allocate the output and the
column buffer and call those launchers (native/core/tensor.cpp:687-724 for
conv1d / conv_transpose1d, :478-494 for conv_transpose2d, :841-868 and
:989-1018 for the backward-weight forms).  conv2d calls launch_conv2d (the
reference's Tensor::conv2d went to cuDNN instead, tensor.cpp:464-476).
All tensors are float32, contiguous and on the current CUDA device; every
call runs on torch's current stream.
"""
from __future__ import annotations

from . import _lib

__all__ = ["conv1d", "conv_transpose1d", "conv2d", "conv_transpose2d", "conv1d_backward_weight",
           "conv2d_backward_weight", "conv_transpose1d_backward_weight", "conv_transpose2d_backward_weight"]


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def _check(*ts):
    import torch
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("tensors must be contiguous float32 CUDA tensors")


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _empty(*shape, like):
    import torch
    return torch.empty(shape, dtype=torch.float32, device=like.device)


def conv2d(x, w, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """x [B, Ci, H, W], w [Co, Ci/groups, kH, kW] -> [B, Co, Ho, Wo] (launch_conv2d, conv.cu:402)."""
    _check(x, w, bias)
    (sH, sW), (pH, pW), (dH, dW) = _pair(stride), _pair(padding), _pair(dilation)
    B, Ci, H, W = x.shape
    Co, _, kH, kW = w.shape
    Ho = (H + 2 * pH - dH * (kH - 1) - 1) // sH + 1
    Wo = (W + 2 * pW - dW * (kW - 1) - 1) // sW + 1
    out = _empty(B, Co, Ho, Wo, like=x)
    col = _empty(max(B * Ci * kH * kW * Ho * Wo, 1), like=x)
    _lib.load().launch_conv2d(_ptr(x), _ptr(w), _ptr(bias), _ptr(out), _ptr(col), B, Ci, H, W, Co, kH, kW, sH, sW,
                              pH, pW, dH, dW, groups, Ho, Wo, _stream())
    _lib.check_last()
    return out


def conv_transpose2d(x, w, bias=None, stride=1, padding=0, output_padding=0, dilation=1, groups=1):
    """x [B, Ci, Hi, Wi], w [Ci, Co/groups, kH, kW] -> [B, Co, Ho, Wo]
    (tensor.cpp:478-494 -> launch_conv_transpose2d, conv.cu:436)."""
    _check(x, w, bias)
    (sH, sW), (pH, pW), (oH, oW), (dH, dW) = _pair(stride), _pair(padding), _pair(output_padding), _pair(dilation)
    B, Ci, Hi, Wi = x.shape
    _, Cog, kH, kW = w.shape
    Co = Cog * groups
    Ho = (Hi - 1) * sH - 2 * pH + dH * (kH - 1) + oH + 1
    Wo = (Wi - 1) * sW - 2 * pW + dW * (kW - 1) + oW + 1
    out = _empty(B, Co, Ho, Wo, like=x)
    col = _empty(max(B * Co * kH * kW * Hi * Wi, 1), like=x)
    _lib.load().launch_conv_transpose2d(_ptr(x), _ptr(w), _ptr(bias), _ptr(out), _ptr(col), B, Ci, Hi, Wi, Co, kH,
                                        kW, sH, sW, pH, pW, dH, dW, groups, Ho, Wo, _stream())
    _lib.check_last()
    return out


def conv1d(x, w, bias=None, stride=1, padding=0, dilation=1, groups=1):
    """x [B, C_in, L_in], w [C_out, C_in/groups, K] -> [B, C_out, L_out] (tensor.cpp:687-705)."""
    _check(x, w, bias)
    B, C_in, L_in = x.shape
    C_out, _, K = w.shape
    L_out = (L_in + 2 * padding - dilation * (K - 1) - 1) // stride + 1
    out = _empty(B, C_out, L_out, like=x)
    col = _empty(max(B * C_in * K * L_out, 1), like=x)
    _lib.load().launch_conv1d(_ptr(x), _ptr(w), _ptr(bias), _ptr(out), _ptr(col), B, C_in, L_in, C_out, K, stride,
                              padding, dilation, groups, L_out, _stream())
    _lib.check_last()
    return out


def conv_transpose1d(x, w, bias=None, stride=1, padding=0, output_padding=0, dilation=1, groups=1):
    """x [B, C_in, L_in], w [C_in, C_out/groups, K] -> [B, C_out, L_out] (tensor.cpp:708-724)."""
    _check(x, w, bias)
    B, C_in, L_in = x.shape
    _, Cog, K = w.shape
    C_out = Cog * groups
    L_out = (L_in - 1) * stride - 2 * padding + dilation * (K - 1) + output_padding + 1
    out = _empty(B, C_out, L_out, like=x)
    col = _empty(max(B * C_out * K * L_in, 1), like=x)
    _lib.load().launch_conv_transpose1d(_ptr(x), _ptr(w), _ptr(bias), _ptr(out), _ptr(col), B, C_in, L_in, C_out, K,
                                        stride, padding, dilation, groups, L_out, _stream())
    _lib.check_last()
    return out


def conv1d_backward_weight(x, go, K, stride=1, padding=0, dilation=1, groups=1):
    """x [B, C_in, L_in], grad_output [B, C_out, L_out] -> [C_out, C_in/groups, K] (tensor.cpp:841-854)."""
    _check(x, go)
    B, C_in, L_in = x.shape
    C_out, L_out = go.shape[1], go.shape[2]
    gw = _empty(C_out, C_in // groups, K, like=x)
    col = _empty(max(B * C_in * K * L_out, 1), like=x)
    _lib.load().launch_conv1d_backward_weight(_ptr(x), _ptr(go), _ptr(gw), _ptr(col), B, C_in, L_in, C_out, K,
                                              stride, padding, dilation, groups, L_out, _stream())
    _lib.check_last()
    return gw


def conv2d_backward_weight(x, go, kernel, stride=1, padding=0, dilation=1, groups=1):
    """x [B, Ci, H, W], grad_output [B, Co, Ho, Wo] -> [Co, Ci/groups, kH, kW] (tensor.cpp:856-868)."""
    _check(x, go)
    (kH, kW), (sH, sW), (pH, pW), (dH, dW) = _pair(kernel), _pair(stride), _pair(padding), _pair(dilation)
    B, Ci, H, W = x.shape
    Co, Ho, Wo = go.shape[1], go.shape[2], go.shape[3]
    gw = _empty(Co, Ci // groups, kH, kW, like=x)
    col = _empty(max(B * Ci * kH * kW * Ho * Wo, 1), like=x)
    _lib.load().launch_conv2d_backward_weight(_ptr(x), _ptr(go), _ptr(gw), _ptr(col), B, Ci, H, W, Co, kH, kW, sH,
                                              sW, pH, pW, dH, dW, groups, Ho, Wo, _stream())
    _lib.check_last()
    return gw


def conv_transpose1d_backward_weight(x, go, K, stride=1, padding=0, dilation=1, groups=1):
    """x [B, C_in, L_in], grad_output [B, C_out, L_out] -> [C_in, C_out/groups, K] (tensor.cpp:989-1003)."""
    _check(x, go)
    B, C_in, L_in = x.shape
    C_out, L_out = go.shape[1], go.shape[2]
    gw = _empty(C_in, C_out // groups, K, like=x)
    col = _empty(max(B * C_out * K * L_in, 1), like=x)
    _lib.load().launch_conv_transpose1d_backward_weight(_ptr(x), _ptr(go), _ptr(gw), _ptr(col), B, C_in, L_in, C_out,
                                                        K, stride, padding, dilation, groups, L_out, _stream())
    _lib.check_last()
    return gw


def conv_transpose2d_backward_weight(x, go, kernel, stride=1, padding=0, dilation=1, groups=1):
    """x [B, Ci, Hi, Wi], grad_output [B, Co, Ho, Wo] -> [Ci, Co/groups, kH, kW] (tensor.cpp:1005-1018)."""
    _check(x, go)
    (kH, kW), (sH, sW), (pH, pW), (dH, dW) = _pair(kernel), _pair(stride), _pair(padding), _pair(dilation)
    B, Ci, Hi, Wi = x.shape
    Co, Ho, Wo = go.shape[1], go.shape[2], go.shape[3]
    gw = _empty(Ci, Co // groups, kH, kW, like=x)
    col = _empty(max(B * Co * kH * kW * Hi * Wi, 1), like=x)
    _lib.load().launch_conv_transpose2d_backward_weight(_ptr(x), _ptr(go), _ptr(gw), _ptr(col), B, Ci, Hi, Wi, Co,
                                                        kH, kW, sH, sW, pH, pW, dH, dW, groups, Ho, Wo, _stream())
    _lib.check_last()
    return gw
