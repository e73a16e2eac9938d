"""Seeded synthetic inputs for the benchmark configurations.

The reference has no seedable generator (Tensor.randn advances a hidden
curand seed counter, native/core/tensor.cpp:753-758), so the inputs of every
configuration come from numpy's PCG64 generator, documented here:

  * a matrix is generated in blocks of BLOCK_ROWS rows; block i of matrix
    `tag` in configuration `seed` uses np.random.default_rng([seed, tag, i]),
    so any row range (one rank's shard) is reproducible on its own and the
    full matrix does not depend on how it is sharded;
  * "uniform" is U[-1, 1) (rng.random(float32) * 2 - 1);
  * "normal" is N(0, std^2) (rng.standard_normal(float32) * std).
"""
from __future__ import annotations

import numpy as np

BLOCK_ROWS = 1024

# tags
A, B, X, W1, W2, W3 = 0, 1, 2, 3, 4, 5


def matrix(seed: int, tag: int, rows: int, cols: int, dist: str, std: float = 1.0,
           row0: int = 0) -> np.ndarray:
    """Rows [row0, row0 + rows) of the (seed, tag) matrix with `cols` columns."""
    out = np.empty((rows, cols), dtype=np.float32)
    r = row0
    while r < row0 + rows:
        blk = r // BLOCK_ROWS
        b0 = blk * BLOCK_ROWS
        rng = np.random.default_rng([seed, tag, blk])
        n = BLOCK_ROWS
        if dist == "uniform":
            vals = rng.random((n, cols), dtype=np.float32)
            vals *= 2.0
            vals -= 1.0
        elif dist == "normal":
            vals = rng.standard_normal((n, cols), dtype=np.float32)
            if std != 1.0:
                vals *= np.float32(std)
        else:
            raise ValueError(dist)
        lo = r - b0
        hi = min(BLOCK_ROWS, row0 + rows - b0)
        out[r - row0:r - row0 + (hi - lo)] = vals[lo:hi]
        r = b0 + hi
    return out


def kaiming_uniform(seed: int, tag: int, out_f: int, in_f: int) -> np.ndarray:
    """W [out_f, in_f] ~ U(-sqrt(6/fan_in), sqrt(6/fan_in)) (ReLU gain)."""
    bound = np.float32(np.sqrt(6.0 / in_f))
    return matrix(seed, tag, out_f, in_f, "uniform") * bound


# --- the five BASELINE configurations -------------------------------------
def config1():
    """512^3 NN GEMM, U[-1,1), seed 0."""
    return matrix(0, A, 512, 512, "uniform"), matrix(0, B, 512, 512, "uniform")


def config2():
    """MLP 784-1024-1024-10, batch 256: x ~ N(0,1), Kaiming-uniform W, zero b, seed 1."""
    x = matrix(1, X, 256, 784, "normal")
    dims = [(1024, 784), (1024, 1024), (10, 1024)]
    ws = [kaiming_uniform(1, t, o, i) for t, (o, i) in zip((W1, W2, W3), dims)]
    bs = [np.zeros(o, dtype=np.float32) for o, _ in dims]
    return x, ws, bs


def config3(rows: int = 8192, row0: int = 0):
    """8192^3 NN GEMM, N(0,1), seed 2 (rows of A selectable for sharding)."""
    return matrix(2, A, rows, 8192, "normal", row0=row0), matrix(2, B, 8192, 8192, "normal")


def config4():
    """batch 64 of [512x64].[64x512] and [512x512].[512x64], N(0, 1/8) (std 1/sqrt(8)), seed 3."""
    std = 1.0 / np.sqrt(8.0)
    q = matrix(3, A, 64 * 512, 64, "normal", std).reshape(64, 512, 64)
    kt = matrix(3, B, 64 * 64, 512, "normal", std).reshape(64, 64, 512)
    p = matrix(3, X, 64 * 512, 512, "normal", std).reshape(64, 512, 512)
    v = matrix(3, W1, 64 * 512, 64, "normal", std).reshape(64, 512, 64)
    return q, kt, p, v


def config5(rows: int = 65536, row0: int = 0):
    """M=65536, K=N=8192, U[-1,1), seed 4; rows of A selectable per rank."""
    return matrix(4, A, rows, 8192, "uniform", row0=row0), matrix(4, B, 8192, 8192, "uniform")
