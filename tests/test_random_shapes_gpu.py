"""A seeded sweep over random GEMM problems on the GPU through the C ABI:
sizes from 1 to a few hundred (ragged tiles, rows that are not a multiple of
4), transposed operands, batch dims with and without broadcasting (B broadcast
over a batch folds into M; some shapes must not fold), 1-D operands, and
problems small enough for the split-K 3xTF32 path.  Exact mode must equal the
oracle bit for bit, forward and MatmulBackward; TF32 and 3xTF32 must stay
within 1e-2 and 1e-5 relative Frobenius error of the float64 product."""
import numpy as np
import pytest

import inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tlcuda  # noqa: E402

DEV = "cuda:0"
TOL = {"tf32": 1e-2, "3xtf32": 1e-5}


def dev(x):
    return torch.from_numpy(np.array(x, dtype=np.float32, order="C", copy=True)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


def rel_fro(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


def problem(seed):
    """Shapes (A, B), whether each is read transposed, from one seed."""
    rng = np.random.default_rng(seed)
    dim = lambda: int(rng.choice([1, 3, 5, 7, 8, 13, 31, 32, 33, 64, 100, 127, 128, 129, 200, 277, 300]))
    M, N, K = dim(), dim(), dim()
    kind = int(rng.integers(0, 5))
    if kind == 0:    # plain 2-D
        ba, bb = (), ()
    elif kind == 1:  # batched A, broadcast B (folds into M when A is K-major)
        ba, bb = (int(rng.integers(2, 9)),), ()
    elif kind == 2:  # both batched
        n = int(rng.integers(2, 6))
        ba, bb = (n,), (n,)
    elif kind == 3:  # two-sided broadcast
        ba, bb = (int(rng.integers(2, 4)), 1), (1, int(rng.integers(2, 4)))
    else:            # 1-D operand on one side
        if rng.integers(0, 2):
            return (K,), (K, N), False, bool(rng.integers(0, 2)), seed
        return (M, K), (K,), bool(rng.integers(0, 2)), False, seed
    ta, tb = bool(rng.integers(0, 2)), bool(rng.integers(0, 2))
    return ba + (M, K), bb + (K, N), ta, tb, seed


CASES = [problem(s) for s in range(40)]


def operands(sa, sb, ta, tb, seed):
    rng = np.random.default_rng(1000 + seed)
    a = inputs.normal(rng, sa)
    b = inputs.normal(rng, sb)
    # a transposed operand is stored transposed and read through a view
    A = dev(np.swapaxes(a, -1, -2)).transpose(-1, -2) if ta and a.ndim >= 2 else dev(a)
    B = dev(np.swapaxes(b, -1, -2)).transpose(-1, -2) if tb and b.ndim >= 2 else dev(b)
    return a, b, A, B


@pytest.mark.parametrize("sa,sb,ta,tb,seed", CASES)
def test_random_exact(sa, sb, ta, tb, seed):
    a, b, A, B = operands(sa, sb, ta, tb, seed)
    ref = O.matmul(a, b)
    got = host(tlcuda.matmul(A, B))
    assert bits_equal(got, ref)
    g = inputs.normal(np.random.default_rng(2000 + seed), ref.shape)
    da, db = tlcuda.matmul_backward(dev(g), A, B)
    oa, ob = O.matmul_backward(g, a, b)
    assert bits_equal(host(da), oa) and bits_equal(host(db), ob)


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
@pytest.mark.parametrize("sa,sb,ta,tb,seed", CASES)
def test_random_tensor_cores(mode, sa, sb, ta, tb, seed):
    a, b, A, B = operands(sa, sb, ta, tb, seed)
    ref = np.matmul(np.asarray(a, np.float64), np.asarray(b, np.float64))
    got = host(tlcuda.matmul(A, B, mode=mode))
    assert got.shape == ref.shape and rel_fro(got, ref) <= TOL[mode]
    # the same call twice gives the same bits (fixed split and reduction orders)
    assert bits_equal(host(tlcuda.matmul(A, B, mode=mode)), got)
