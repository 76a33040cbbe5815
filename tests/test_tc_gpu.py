"""Tensor-core modes on the GPU through the C ABI: TF32 within 1e-2 and
3xTF32 within 1e-5 relative Frobenius error, against the float64 product of
the same float32 operands and against the reference's own result (the
oracle), over every operand layout, ragged tiles, batching, broadcasting,
1-D operands and the backward pass; plus the bounded-wait failure path."""
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


def rel_fro(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


def f64_matmul(a, b):
    """float64 product of float32 operands with tl::matmul's shape rules."""
    a64 = np.asarray(a, np.float64)
    b64 = np.asarray(b, np.float64)
    return np.matmul(a64, b64)


def T(t, flag):
    return t.transpose(-1, -2) if flag else t


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
@pytest.mark.parametrize("M,N,K", [(128, 256, 32), (1, 1, 1), (7, 9, 13), (129, 257, 33),
                                   (300, 277, 259), (256, 128, 1024), (64, 64, 4096)])
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_layouts_and_tails(mode, M, N, K, ta, tb):
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    a = inputs.normal(rng, (K, M) if ta else (M, K))
    b = inputs.normal(rng, (N, K) if tb else (K, N))
    an, bn = (a.T if ta else a), (b.T if tb else b)
    got = host(tlcuda.matmul(T(dev(a), ta), T(dev(b), tb), mode=mode))
    assert rel_fro(got, f64_matmul(an, bn)) <= TOL[mode]
    assert rel_fro(got, O.matmul(an, bn)) <= TOL[mode]


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_golden_cases(golden, mode):
    for case in ["r_2d", "r_ta", "r_tb", "r_tab", "r_batch", "r_bcast", "r_vecmat", "r_matvec",
                 "r_vecvec", "r_k1"]:
        a, b = dev(golden[f"{case}.a"]), dev(golden[f"{case}.b"])
        ta, tb = bool(golden[f"{case}.ta"]), bool(golden[f"{case}.tb"])
        got = host(tlcuda.matmul(T(a, ta), T(b, tb), mode=mode))
        assert rel_fro(got, golden[f"{case}.c"]) <= TOL[mode], case
        da, db = tlcuda.matmul_backward(dev(golden[f"{case}.g"]), T(a, ta), T(b, tb), mode=mode)
        da = T(torch.from_numpy(host(da)), ta).numpy()
        db = T(torch.from_numpy(host(db)), tb).numpy()
        assert rel_fro(da, golden[f"{case}.da"]) <= TOL[mode], case
        assert rel_fro(db, golden[f"{case}.db"]) <= TOL[mode], case
    a, b = inputs.ragged_integer()
    got = host(tlcuda.matmul(dev(a), dev(b), mode=mode))
    assert rel_fro(got, golden["ragged.c"]) <= TOL[mode]


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_broadcast_workload_fwd_bwd(mode):
    a, b, dc = inputs.cfg_broadcast()
    c = host(tlcuda.matmul(dev(a), dev(b), mode=mode))
    assert rel_fro(c, f64_matmul(a, b)) <= TOL[mode]
    da, db = tlcuda.matmul_backward(dev(dc), dev(a), dev(b), mode=mode)
    ref_da = np.matmul(dc.astype(np.float64), b.T.astype(np.float64))
    ref_db = np.einsum("bmk,bmn->kn", a.astype(np.float64), dc.astype(np.float64))
    assert rel_fro(host(da), ref_da) <= TOL[mode]
    assert rel_fro(host(db), ref_db) <= TOL[mode]


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_batched_broadcast_dims(mode):
    rng = np.random.default_rng(3)
    a = inputs.normal(rng, (2, 1, 3, 40, 36))
    b = inputs.normal(rng, (1, 4, 1, 36, 140))
    got = host(tlcuda.matmul(dev(a), dev(b), mode=mode))
    assert rel_fro(got, f64_matmul(a, b)) <= TOL[mode]


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_unaligned_operands_repacked(mode):
    rng = np.random.default_rng(4)
    big = dev(inputs.normal(rng, (70 * 131 + 3,)))
    a = big[1:1 + 70 * 131].view(70, 131)       # misaligned base, odd row pitch
    b = dev(inputs.normal(rng, (131, 45)))      # odd N: row pitch not a multiple of 4
    got = host(tlcuda.matmul(a, b, mode=mode))
    assert rel_fro(got, f64_matmul(host(a), host(b))) <= TOL[mode]


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_linear_full_size(mode):
    """Y = X . W^T (W K-major in place) at [4096,1024] x [1024,4096] and its
    backward, sampled rows against float64."""
    x, w, dy = inputs.cfg_linear()
    X, W = dev(x), dev(w)
    y = host(tlcuda.matmul(X, W.t(), mode=mode))
    rows = np.arange(0, 4096, 128)
    assert rel_fro(y[rows], x[rows].astype(np.float64) @ w.T.astype(np.float64)) <= TOL[mode]
    dx, dwt = tlcuda.matmul_backward(dev(dy), X, W.t(), mode=mode)
    dx, dwt = host(dx), host(dwt)
    assert rel_fro(dx[rows], dy[rows].astype(np.float64) @ w.astype(np.float64)) <= TOL[mode]
    cols = np.arange(0, 1024, 32)
    ref = x.T[cols].astype(np.float64) @ dy.astype(np.float64)
    assert rel_fro(dwt[cols], ref) <= TOL[mode]


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
@pytest.mark.parametrize("n", [8192, 16384])
def test_square_sampled(mode, n):
    """The square sweep sizes, U[-1,1] seed 4: 16 sampled rows against float64."""
    g = torch.Generator(device=DEV).manual_seed(4)
    A = torch.rand((n, n), generator=g, device=DEV) * 2 - 1
    B = torch.rand((n, n), generator=g, device=DEV) * 2 - 1
    C = tlcuda.matmul(A, B, mode=mode)
    tlcuda.check_device_errors()
    rows = torch.arange(0, n, n // 16, device=DEV)
    a = A[rows].double().cpu().numpy()
    ref = a @ B.double().cpu().numpy()
    assert rel_fro(host(C[rows]), ref) <= TOL[mode]
    del A, B, C
    torch.cuda.empty_cache()


def test_bounded_wait_times_out_and_context_survives():
    st = tlcuda.selftest_bounded_wait(2_000_000)  # 2 ms on a barrier nothing completes
    assert st == 5, tlcuda.lib().tlc_last_error()
    # the context is still usable and the error word was cleared
    a = dev(np.ones((130, 70), np.float32))
    b = dev(np.ones((70, 140), np.float32))
    c = host(tlcuda.matmul(a, b, mode="tf32"))
    assert np.all(c == 70.0)
    tlcuda.check_device_errors()
