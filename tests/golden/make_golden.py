"""Make the golden fixtures of tests/golden/ by running the REFERENCE's own
GEMM build on a GPU.

The reference's native/ops/matmul.cu is compiled unmodified from its source
tree into oracle/_ref/libref_matmul.so (`make -C oracle ref`).  Its three
launchers (launch_matmul, launch_bmm, launch_linear; cuBLAS sgemm with TF32
tensor-op math) are called here on seeded inputs and the inputs and outputs
are saved as .npz files.

Integer-valued inputs in [-8, 8] make every product and partial sum an exact
small integer, which TF32 math and fp32 accumulation represent exactly, so for
those cases the reference's output is the exact product and pins the oracle's
layout conventions (row-major NN, packed batch strides, x.w^T + bias) bit for
bit.  One random-float case records how far the reference's TF32 math sits
from the fp64 product.

Usage (needs a B200 and the built oracle/_ref library):
    python tests/golden/make_golden.py --out tests/golden
"""
from __future__ import annotations

import argparse
import ctypes
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def main() -> None:
    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(Path(__file__).resolve().parent))
    args = ap.parse_args()
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    lib_path = ROOT / "oracle" / "_ref" / "libref_matmul.so"
    lib = ctypes.CDLL(str(lib_path))
    vp, ci = ctypes.c_void_p, ctypes.c_int
    lib.launch_matmul.argtypes = [vp, vp, vp, ci, ci, ci, vp]
    lib.launch_bmm.argtypes = [vp, vp, vp, ci, ci, ci, ci, vp]
    lib.launch_linear.argtypes = [vp, vp, vp, vp, ci, ci, ci, vp]
    rng = np.random.default_rng(20261201)

    def ints(*shape):
        return rng.integers(-8, 9, size=shape).astype(np.float32)

    def dev(x):
        return torch.from_numpy(np.ascontiguousarray(x)).cuda()

    # README.md:41-55 through the reference launcher
    a = np.array([1, 2, 3, 4, 5, 6], np.float32).reshape(2, 3)
    b = np.arange(1, 13, dtype=np.float32).reshape(3, 4)
    da, db = dev(a), dev(b)
    dc = torch.empty((2, 4), device="cuda")
    lib.launch_matmul(da.data_ptr(), db.data_ptr(), dc.data_ptr(), 2, 3, 4, None)
    torch.cuda.synchronize()
    np.savez(out / "ref_readme.npz", a=a, b=b, c=dc.cpu().numpy())

    # launch_matmul, integer inputs, odd shape
    M, K, N = 37, 53, 29
    a, b = ints(M, K), ints(K, N)
    da, db = dev(a), dev(b)
    dc = torch.empty((M, N), device="cuda")
    lib.launch_matmul(da.data_ptr(), db.data_ptr(), dc.data_ptr(), M, K, N, None)
    torch.cuda.synchronize()
    np.savez(out / "ref_matmul_int.npz", a=a, b=b, c=dc.cpu().numpy())

    # launch_bmm, integer inputs
    Bt, M, K, N = 3, 17, 19, 23
    a, b = ints(Bt, M, K), ints(Bt, K, N)
    da, db = dev(a), dev(b)
    dc = torch.empty((Bt, M, N), device="cuda")
    lib.launch_bmm(da.data_ptr(), db.data_ptr(), dc.data_ptr(), Bt, M, K, N, None)
    torch.cuda.synchronize()
    np.savez(out / "ref_bmm_int.npz", a=a, b=b, c=dc.cpu().numpy())

    # launch_linear with and without bias, integer inputs
    Bs, fin, fout = 13, 31, 21
    x, w, bias = ints(Bs, fin), ints(fout, fin), ints(fout)
    dx, dw, dbias = dev(x), dev(w), dev(bias)
    dy = torch.empty((Bs, fout), device="cuda")
    lib.launch_linear(dx.data_ptr(), dw.data_ptr(), dbias.data_ptr(), dy.data_ptr(), Bs, fin, fout, None)
    torch.cuda.synchronize()
    y_bias = dy.cpu().numpy()
    lib.launch_linear(dx.data_ptr(), dw.data_ptr(), None, dy.data_ptr(), Bs, fin, fout, None)
    torch.cuda.synchronize()
    np.savez(out / "ref_linear_int.npz", x=x, w=w, bias=bias, y_bias=y_bias, y=dy.cpu().numpy())

    # launch_matmul, random floats U[-1,1): the reference's TF32 distance from fp64
    M, K, N = 64, 96, 80
    a = (rng.random((M, K), dtype=np.float32) * 2 - 1)
    b = (rng.random((K, N), dtype=np.float32) * 2 - 1)
    da, db = dev(a), dev(b)
    dc = torch.empty((M, N), device="cuda")
    lib.launch_matmul(da.data_ptr(), db.data_ptr(), dc.data_ptr(), M, K, N, None)
    torch.cuda.synchronize()
    np.savez(out / "ref_matmul_float.npz", a=a, b=b, c=dc.cpu().numpy())
    print(f"wrote fixtures to {out}")


if __name__ == "__main__":
    main()
