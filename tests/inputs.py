"""Seeded synthetic inputs for the matmul path (the reference ships no
datasets or golden tensors for it).

Generator: numpy PCG64 (np.random.default_rng(seed)); uniform values are
rng.uniform(lo, hi) in float64 rounded to float32, normal values are
rng.standard_normal() in float64 rounded to float32 (scaled by std).  Each
tensor of a workload draws from one generator in the order listed, so the
same seed gives the same bits on every host with this numpy.
"""
from __future__ import annotations

import numpy as np


def uniform(rng, shape, lo=-1.0, hi=1.0):
    return rng.uniform(lo, hi, size=shape).astype(np.float32)


def normal(rng, shape, std=1.0):
    return (rng.standard_normal(size=shape) * std).astype(np.float32)


def cfg_square(n=512, seed=0):
    """C[n,n] = A[n,n] . B[n,n], A and B ~ U[-1,1] (seed 0 at n=512)."""
    rng = np.random.default_rng(seed)
    return uniform(rng, (n, n)), uniform(rng, (n, n))


def cfg_broadcast(seed=1):
    """A[32,128,64] . B[64,128] (B broadcast over the batch); A, B, dC ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    a = normal(rng, (32, 128, 64))
    b = normal(rng, (64, 128))
    dc = normal(rng, (32, 128, 128))
    return a, b, dc


def cfg_linear(m=4096, k=1024, n=4096, seed=2):
    """Y = X . W^T + b with X[m,k] ~ N(0,1), W[n,k] ~ U(-1/32, 1/32), dY ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    x = normal(rng, (m, k))
    w = uniform(rng, (n, k), -1.0 / 32, 1.0 / 32)
    dy = normal(rng, (m, n))
    return x, w, dy


def ragged_integer(M=259, K=300, N=277):
    """Integer-valued operands of the reference's ragged test (tests/test_ops.cpp:99-103)."""
    i = np.arange(M * K, dtype=np.int64)
    a = (((i * 3 + 1) % 11) - 5).astype(np.float32).reshape(M, K)
    j = np.arange(K * N, dtype=np.int64)
    b = (((j * 7 + 2) % 13) - 6).astype(np.float32).reshape(K, N)
    return a, b
