"""Make tests/golden/ref_conv_int.npz by running the REFERENCE's own
convolution launchers on a GPU.

The reference's native/ops/conv.cu is compiled unmodified from its source
tree into oracle/_ref/libref_conv.so (`make -C oracle ref REF_SRC=...`).  Its
eight im2col-GEMM launchers (conv.cu:324-627: im2col / col2im kernels and one
cuBLAS sgemm per image and group with TF32 tensor-op math, beta = 1
accumulation for the weight gradients) are called here on seeded
integer-valued inputs in [-4, 4]: every product and partial sum is then a
small integer that TF32 inputs and fp32 accumulation represent exactly, so
the saved outputs are the exact results and pin the oracle's restatement of
the launchers' layouts (batch-outer col, grouped weights, stride / padding /
dilation, transposed-conv col2im, output padding through Ho / Wo, bias)
bit for bit.

Usage (needs a B200 and the built oracle/_ref library):
    python tests/golden/make_conv_golden.py --out tests/golden
"""
from __future__ import annotations

import argparse
import ctypes
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

# name: (kind, B, Ci, H, W, Co, kH, kW, sH, sW, pH, pW, dH, dW, groups, opH, opW, bias)
# kind: conv | convT | conv_bw | convT_bw; 1-D cases have H = kH = 1, s/p/d along W only
CASES = {
    "conv2d_g2": ("conv", 2, 4, 7, 6, 6, 3, 2, 2, 1, 1, 0, 1, 2, 2, 0, 0, True),
    "conv2d_1x1": ("conv", 3, 5, 4, 5, 7, 1, 1, 1, 1, 0, 0, 1, 1, 1, 0, 0, False),
    "convT2d_g2": ("convT", 2, 4, 5, 4, 6, 3, 3, 2, 2, 1, 0, 1, 1, 2, 1, 0, True),
    "conv2d_bw_g2": ("conv_bw", 2, 4, 7, 6, 6, 3, 2, 2, 1, 1, 0, 1, 2, 2, 0, 0, False),
    "convT2d_bw_g2": ("convT_bw", 2, 4, 5, 4, 6, 3, 3, 2, 2, 1, 0, 1, 1, 2, 1, 0, False),
    "conv1d_g2": ("conv", 2, 4, 1, 11, 6, 1, 3, 1, 2, 0, 1, 1, 2, 2, 0, 0, True),
    "convT1d_g2": ("convT", 2, 4, 1, 6, 6, 1, 3, 1, 2, 0, 1, 1, 1, 2, 0, 1, True),
    "conv1d_bw_g2": ("conv_bw", 2, 4, 1, 11, 6, 1, 3, 1, 2, 0, 1, 1, 2, 2, 0, 0, False),
    "convT1d_bw_g2": ("convT_bw", 2, 4, 1, 6, 6, 1, 3, 1, 2, 0, 1, 1, 1, 2, 0, 1, False),
}


def out_size(n, k, s, p, d):
    return (n + 2 * p - d * (k - 1) - 1) // s + 1


def t_out_size(n, k, s, p, d, op):
    return (n - 1) * s - 2 * p + d * (k - 1) + op + 1


def main() -> None:
    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    args = ap.parse_args()
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_conv.so"))
    vp, ci = ctypes.c_void_p, ctypes.c_int
    lib.launch_conv1d.argtypes = [vp] * 5 + [ci] * 10 + [vp]
    lib.launch_conv_transpose1d.argtypes = [vp] * 5 + [ci] * 10 + [vp]
    lib.launch_conv2d.argtypes = [vp] * 5 + [ci] * 16 + [vp]
    lib.launch_conv_transpose2d.argtypes = [vp] * 5 + [ci] * 16 + [vp]
    for n in ("launch_conv1d_backward_weight", "launch_conv_transpose1d_backward_weight"):
        getattr(lib, n).argtypes = [vp] * 4 + [ci] * 10 + [vp]
    for n in ("launch_conv2d_backward_weight", "launch_conv_transpose2d_backward_weight"):
        getattr(lib, n).argtypes = [vp] * 4 + [ci] * 16 + [vp]
    rng = np.random.default_rng(20261202)

    def ints(*shape):
        return rng.integers(-4, 5, size=shape).astype(np.float32)

    def dev(x):
        return torch.from_numpy(np.ascontiguousarray(x)).cuda()

    saved = {}
    for name, c in CASES.items():
        kind, B, Ci, H, W, Co, kH, kW, sH, sW, pH, pW, dH, dW, g, opH, opW, with_bias = c
        one_d = H == 1 and kH == 1
        if kind in ("conv", "conv_bw"):
            Ho, Wo = out_size(H, kH, sH, pH, dH), out_size(W, kW, sW, pW, dW)
            w_shape = (Co, Ci // g, kH, kW)
            col = B * Ci * kH * kW * Ho * Wo
        else:
            Ho, Wo = t_out_size(H, kH, sH, pH, dH, opH), t_out_size(W, kW, sW, pW, dW, opW)
            w_shape = (Ci, Co // g, kH, kW)
            col = B * Co * kH * kW * H * W
        x = ints(B, Ci, H, W)
        colbuf = torch.empty(col, device="cuda")
        rec = {"x": x, "params": np.array(c[1:17], np.int64)}
        if kind in ("conv", "convT"):
            w = ints(*w_shape)
            bias = ints(Co) if with_bias else None
            out = torch.full((B, Co, Ho, Wo), float("nan"), device="cuda")
            dx, dw_ = dev(x), dev(w)
            db = dev(bias) if with_bias else None
            bp = db.data_ptr() if with_bias else None
            if one_d:
                fn = lib.launch_conv1d if kind == "conv" else lib.launch_conv_transpose1d
                fn(dx.data_ptr(), dw_.data_ptr(), bp, out.data_ptr(), colbuf.data_ptr(), B, Ci, W, Co, kW, sW, pW,
                   dW, g, Wo, None)
            else:
                fn = lib.launch_conv2d if kind == "conv" else lib.launch_conv_transpose2d
                fn(dx.data_ptr(), dw_.data_ptr(), bp, out.data_ptr(), colbuf.data_ptr(), B, Ci, H, W, Co, kH, kW, sH,
                   sW, pH, pW, dH, dW, g, Ho, Wo, None)
            rec["w"] = w
            if with_bias:
                rec["bias"] = bias
        else:
            go = ints(B, Co, Ho, Wo)
            out = torch.full(w_shape, float("nan"), device="cuda")
            dx, dgo = dev(x), dev(go)
            if one_d:
                fn = (lib.launch_conv1d_backward_weight if kind == "conv_bw"
                      else lib.launch_conv_transpose1d_backward_weight)
                fn(dx.data_ptr(), dgo.data_ptr(), out.data_ptr(), colbuf.data_ptr(), B, Ci, W, Co, kW, sW, pW, dW, g,
                   Wo, None)
            else:
                fn = (lib.launch_conv2d_backward_weight if kind == "conv_bw"
                      else lib.launch_conv_transpose2d_backward_weight)
                fn(dx.data_ptr(), dgo.data_ptr(), out.data_ptr(), colbuf.data_ptr(), B, Ci, H, W, Co, kH, kW, sH, sW,
                   pH, pW, dH, dW, g, Ho, Wo, None)
            rec["go"] = go
        torch.cuda.synchronize()
        rec["out"] = out.cpu().numpy()
        for k, v in rec.items():
            saved[f"{name}__{k}"] = v
    dst = Path(args.out) / "ref_conv_int.npz"
    np.savez(dst, **saved)
    print(f"wrote {dst} ({len(CASES)} cases)")


if __name__ == "__main__":
    main()
