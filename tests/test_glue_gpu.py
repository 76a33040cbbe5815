"""The glue around the GEMMs on the GPU through the C ABI, against the oracle:
tl::add with broadcasting, tl::scale, SoftmaxBackward, sum_to and the fused
GEMM epilogue (scale, then bias) bit for bit; tl::softmax within the stated
tolerance (CUDA's expf is not the C library's)."""
import numpy as np
import pytest

import inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tlcuda  # noqa: E402

DEV = "cuda:0"
# tl::softmax: |gpu - reference| <= SOFTMAX_RTOL * |reference| per element
SOFTMAX_RTOL = 2e-6


def dev(x):
    return torch.from_numpy(np.array(x, dtype=np.float32, order="C", copy=True)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


ADD_SHAPES = [((4, 3, 5), (5,)), ((4, 1, 5), (3, 1)), ((2, 3), (2, 3)), ((6,), (1,)),
              ((2, 1, 4, 1), (3, 1, 5)), ((4096, 4096), (4096,)), ((), (3, 2)), ((0, 3), (3,)),
              # inner dims that are multiples of 4 take the row-wise float4 path: b one value
              # per row, and b a contiguous run under a broadcast outer dim
              ((8, 16), (8, 1)), ((3, 5, 12), (5, 12)), ((2, 64, 8), (64, 1))]


@pytest.mark.parametrize("sa,sb", ADD_SHAPES)
def test_add_broadcast(sa, sb):
    rng = np.random.default_rng(len(sa) * 5 + len(sb))
    a, b = inputs.normal(rng, sa), inputs.normal(rng, sb)
    assert bits_equal(host(tlcuda.add_tensors(dev(a), dev(b))), O.add_bcast(a, b))
    assert bits_equal(host(tlcuda.add_tensors(dev(b), dev(a))), O.add_bcast(b, a))


def test_add_strided_and_errors():
    rng = np.random.default_rng(2)
    a = inputs.normal(rng, (7, 5))
    b = inputs.normal(rng, (7,))
    at = dev(a).t()  # [5, 7] transposed view
    assert bits_equal(host(tlcuda.add_tensors(at, dev(b))), O.add_bcast(a.T, b))
    with pytest.raises(tlcuda.TLCError, match="Incompatible dimensions for broadcasting"):
        tlcuda.add_tensors(dev(np.ones((3, 4))), dev(np.ones((2, 4))),
                           out=torch.empty((3, 4), device=DEV))


@pytest.mark.parametrize("s", [0.125, -3.0, 1.0 / 8.0, 1e-30])
@pytest.mark.parametrize("shape", [(33, 17), (32, 64)])  # (32, 64): the row-wise float4 path
def test_scale(s, shape):
    x = inputs.normal(np.random.default_rng(11), shape)
    assert bits_equal(host(tlcuda.scale(dev(x), s)), O.scale(x, s))
    assert bits_equal(host(tlcuda.scale(dev(x).t(), s)), O.scale(x.T, s))


# row lengths covering every register bucket (<= 32, 64, 128, 256, 512, 1024) and the
# streaming kernel above 1024
SOFTMAX_SHAPES = [(1,), (7,), (5, 7), (2, 9), (3, 4, 64), (2, 100), (3, 200), (2, 512), (192, 33),
                  (4, 1000), (3, 4096), (6, 1),
                  # enough rows for the thread-per-row kernels (float4 and scalar rows)
                  (24, 1024, 64), (19000, 37)]


def softmax_close(got, ref):
    both_zero = (got == 0) & (ref == 0)
    ok = both_zero | (np.abs(got.astype(np.float64) - ref) <= SOFTMAX_RTOL * np.abs(ref.astype(np.float64)))
    return bool(np.all(ok | (np.isnan(got) & np.isnan(ref))))


@pytest.mark.parametrize("shape", SOFTMAX_SHAPES)
def test_softmax_and_backward(shape):
    rng = np.random.default_rng(sum(shape) + 1)
    x = inputs.normal(rng, shape) * np.float32(4.0)
    g = inputs.normal(rng, shape)
    y = host(tlcuda.softmax(dev(x)))
    assert softmax_close(y, O.softmax(x))
    # backward from the same y: bit-identical to the oracle (reference v4 build order)
    dx = host(tlcuda.softmax_backward(dev(g), dev(y)))
    assert bits_equal(dx, O.softmax_backward(g, y))


def test_softmax_edge_rows():
    x = np.array([[0.0, 0.0, 0.0], [-np.inf, 1.0, 2.0], [1e30, -1e30, 0.0], [-5.0, -5.0, -4.0],
                  [np.nan, 1.0, 2.0], [1.0, np.nan, 2.0], [-np.inf, -np.inf, -np.inf]], np.float32)
    assert softmax_close(host(tlcuda.softmax(dev(x))), O.softmax(x))
    # a strided (transposed) input is read as the reference reads input.contiguous()
    z = inputs.normal(np.random.default_rng(8), (40, 3))
    assert softmax_close(host(tlcuda.softmax(dev(z).t())), O.softmax(z.T))
    with pytest.raises(tlcuda.TLCError, match="at least 1D"):
        tlcuda.softmax(dev(np.float32(1.0)), out=torch.empty((), device=DEV))


@pytest.mark.parametrize("shape,target", [((32, 64, 128), (64, 128)), ((4, 3, 5), (5,)),
                                          ((4, 3, 5), (1, 5)), ((4, 3, 5), (4, 1, 5)),
                                          ((4096, 4096), (4096,)), ((7,), (7,)),
                                          ((1000, 100), (100,)), ((4, 300, 40), (4, 1, 40))])
def test_sum_to(shape, target):
    x = inputs.normal(np.random.default_rng(len(shape) + len(target)), shape)
    assert bits_equal(host(tlcuda.sum_to(dev(x), target)), O.sum_to(x, target))


# ---- the fused GEMM epilogue -------------------------------------------------------------

LAYOUTS = [(False, False), (True, False), (False, True), (True, True)]


def T(t, flag):
    return t.transpose(-1, -2) if flag else t


@pytest.mark.parametrize("M,N,K", [(132, 260, 36), (300, 124, 1004), (129, 130, 131), (5, 7, 0),
                                   (64, 512, 96)])
@pytest.mark.parametrize("ta,tb", LAYOUTS)
def test_matmul_fused_exact(M, N, K, ta, tb):
    rng = np.random.default_rng(M + N * 3 + K * 7)
    a = inputs.normal(rng, (K, M) if ta else (M, K))
    b = inputs.normal(rng, (N, K) if tb else (K, N))
    bias = inputs.normal(rng, (N,))
    an, bn = (a.T if ta else a), (b.T if tb else b)
    c = O.matmul(an, bn)
    A, B = T(dev(a), ta), T(dev(b), tb)
    # Linear: add(matmul(x, W), b)
    got = host(tlcuda.matmul_fused(A, B, 1.0, dev(bias), mode="exact"))
    assert bits_equal(got, O.add_bcast(c, bias))
    # attention scores: scale(matmul(q, k^T), 1/sqrt(d))
    s = float(np.float32(1.0 / np.sqrt(64.0)))
    got = host(tlcuda.matmul_fused(A, B, s, None, mode="exact"))
    assert bits_equal(got, O.scale(c, s))
    # both, in that order
    got = host(tlcuda.matmul_fused(A, B, -0.75, dev(bias), mode="exact"))
    assert bits_equal(got, O.add_bcast(O.scale(c, -0.75), bias))


def test_matmul_fused_batched_broadcast():
    rng = np.random.default_rng(31)
    x = inputs.normal(rng, (4, 33, 68))
    w = inputs.normal(rng, (68, 260))
    bias = inputs.normal(rng, (260,))
    got = host(tlcuda.matmul_fused(dev(x), dev(w), 1.0, dev(bias), mode="exact"))
    assert bits_equal(got, O.add_bcast(O.matmul(x, w), bias))
    with pytest.raises(tlcuda.TLCError, match="bias must be a 1-D tensor of length N"):
        tlcuda.matmul_fused(dev(x), dev(w), 1.0, dev(np.ones((259,), np.float32)))


@pytest.mark.parametrize("mode,tol", [("tf32", 1e-2), ("3xtf32", 1e-5)])
def test_matmul_fused_tensor_cores(mode, tol):
    rng = np.random.default_rng(5)
    x = inputs.normal(rng, (512, 384))
    w = inputs.normal(rng, (640, 384))  # X . W^T with W [out, in]
    bias = inputs.normal(rng, (640,))
    ref = (x.astype(np.float64) @ w.T.astype(np.float64)) * 0.5 + bias
    got = host(tlcuda.matmul_fused(dev(x), dev(w).t(), 0.5, dev(bias), mode=mode)).astype(np.float64)
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= tol
