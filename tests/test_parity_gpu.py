"""Exact-mode parity on the GPU through the C ABI: libtl_cuda's tl::matmul and
MatmulBackward must reproduce the reference bit for bit (the golden fixtures
and the oracle), including transposed views, broadcasting, 1-D operands,
ragged tiles, empty and K == 0 inputs, and misaligned or strided views."""
import hashlib

import numpy as np
import pytest

import inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tlcuda  # noqa: E402

DEV = "cuda:0"


def dev(x):
    # np.array keeps 0-D inputs 0-D (np.ascontiguousarray would make them 1-D)
    return torch.from_numpy(np.array(x, dtype=np.float32, order="C", copy=True)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


def sha(x):
    return hashlib.sha256(np.ascontiguousarray(x, np.float32).tobytes()).hexdigest()


def T(t, flag):
    return t.transpose(-1, -2) if flag else t


def test_kats(golden):
    c = host(tlcuda.matmul(dev(golden["kat2x3.a"]), dev(golden["kat2x3.b"])))
    assert c[0, 0] == 58.0 and c[1, 1] == 154.0 and bits_equal(c, golden["kat2x3.c"])
    c = host(tlcuda.matmul(dev(golden["bcast4d.a"]), dev(golden["bcast4d.b"])))
    assert c.shape == (2, 3, 2, 4) and bits_equal(c, golden["bcast4d.c"])
    c = host(tlcuda.matmul(dev(np.ones((256, 512), np.float32)), dev(np.ones((512, 256), np.float32))))
    assert sha(c) == str(golden["heavy.c_sha"])
    a, b = inputs.ragged_integer()
    assert bits_equal(host(tlcuda.matmul(dev(a), dev(b))), golden["ragged.c"])


@pytest.mark.parametrize("lv", ["l1", "l2", "l3", "l4a", "l4b"])
def test_backward_levels(golden, lv):
    g = {k: golden[f"bwd_{lv}.{k}"] for k in ("a", "b", "g", "da", "db")}
    da, db = tlcuda.matmul_backward(dev(g["g"]), dev(g["a"]), dev(g["b"]))
    assert bits_equal(host(da), g["da"]) and bits_equal(host(db), g["db"])


@pytest.mark.parametrize("case", ["r_2d", "r_ta", "r_tb", "r_tab", "r_batch", "r_bcast",
                                  "r_vecmat", "r_matvec", "r_vecvec", "r_k1"])
def test_golden_random(golden, case):
    a, b = dev(golden[f"{case}.a"]), dev(golden[f"{case}.b"])
    ta, tb = bool(golden[f"{case}.ta"]), bool(golden[f"{case}.tb"])
    c = tlcuda.matmul(T(a, ta), T(b, tb))  # transposed views, read in place
    assert bits_equal(host(c), golden[f"{case}.c"])
    da, db = tlcuda.matmul_backward(dev(golden[f"{case}.g"]), T(a, ta), T(b, tb))
    assert bits_equal(T(torch.from_numpy(host(da)), ta).numpy(), golden[f"{case}.da"])
    assert bits_equal(T(torch.from_numpy(host(db)), tb).numpy(), golden[f"{case}.db"])


def test_broadcast_workload(golden):
    a, b, dc = inputs.cfg_broadcast()
    c = tlcuda.matmul(dev(a), dev(b))
    assert sha(host(c)) == str(golden["cfg_broadcast.c_sha"])
    da, db = tlcuda.matmul_backward(dev(dc), dev(a), dev(b))
    assert sha(host(da)) == str(golden["cfg_broadcast.da_sha"])
    assert bits_equal(host(db), golden["cfg_broadcast.db"])


def test_square512_workload(golden):
    a, b = inputs.cfg_square(512, 0)
    assert sha(host(tlcuda.matmul(dev(a), dev(b)))) == str(golden["cfg_square512.c_sha"])


RAGGED = [(1, 1, 1), (1, 7, 5), (7, 1, 9), (3, 5, 1), (129, 130, 131), (128, 128, 16),
          (127, 255, 17), (259, 277, 300), (64, 64, 1000), (5, 300, 2)]


@pytest.mark.parametrize("M,N,K", RAGGED)
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_ragged_layouts(M, N, K, ta, tb):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = inputs.normal(rng, (K, M) if ta else (M, K))
    b = inputs.normal(rng, (N, K) if tb else (K, N))
    an, bn = (a.T if ta else a), (b.T if tb else b)
    ref = O.matmul(an, bn)
    got = host(tlcuda.matmul(T(dev(a), ta), T(dev(b), tb)))
    assert bits_equal(got, ref)


# Contiguous extents that are multiples of 4 floats: every layout below is read
# by the TMA-fed exact kernel (ragged M / N / K tiles zero-filled by TMA).
ALIGNED = [(4, 4, 4), (132, 260, 36), (300, 124, 1004), (260, 132, 4), (1000, 8, 300),
           (128, 256, 2048)]


@pytest.mark.parametrize("M,N,K", ALIGNED)
@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_aligned_layouts(M, N, K, ta, tb):
    rng = np.random.default_rng(M * 5 + N * 11 + K)
    a = inputs.normal(rng, (K, M) if ta else (M, K))
    b = inputs.normal(rng, (N, K) if tb else (K, N))
    an, bn = (a.T if ta else a), (b.T if tb else b)
    got = host(tlcuda.matmul(T(dev(a), ta), T(dev(b), tb)))
    assert bits_equal(got, O.matmul(an, bn))


@pytest.mark.parametrize("tb", [False, True])
def test_aligned_batched_broadcast(tb):
    rng = np.random.default_rng(21)
    a = inputs.normal(rng, (3, 1, 132, 68))
    b = inputs.normal(rng, (1, 2, 36, 68) if tb else (1, 2, 68, 36))
    bn = np.swapaxes(b, -1, -2) if tb else b
    got = host(tlcuda.matmul(dev(a), T(dev(b), tb)))
    assert bits_equal(got, O.matmul(a, bn))
    g = inputs.normal(rng, got.shape)
    da, db = tlcuda.matmul_backward(dev(g), dev(a), T(dev(b), tb))
    oa, ob = O.matmul_backward(g, a, bn)
    assert bits_equal(host(da), oa) and bits_equal(host(db), ob)


@pytest.mark.parametrize("shape_a,shape_b,ta", [
    ((33, 7, 64), (64, 96), False),      # B broadcast, A's rows contiguous: folded into M = 231
    ((2, 3, 5, 40), (40, 24), False),    # two batch dims, merged, then folded
    ((4, 1, 9, 36), (3, 36, 20), False),  # B batched: not folded
    ((6, 40, 9), (40, 28), True),        # A read transposed (M-major): not folded
])
def test_broadcast_batch_folded_into_m(shape_a, shape_b, ta):
    """A batch dim over which B is broadcast folds into M when A's and C's rows
    run on contiguously; every output keeps its k-chain, so exact mode stays
    bit-identical and the tolerance modes stay within their bounds, forward and
    MatmulBackward."""
    rng = np.random.default_rng(sum(shape_a) + 7 * sum(shape_b))
    a = inputs.normal(rng, shape_a)
    b = inputs.normal(rng, shape_b)
    an = np.swapaxes(a, -1, -2) if ta else a
    A = T(dev(a), ta)
    got = host(tlcuda.matmul(A, dev(b)))
    assert bits_equal(got, O.matmul(an, b))
    g = inputs.normal(rng, got.shape)
    da, db = tlcuda.matmul_backward(dev(g), A, dev(b))
    oa, ob = O.matmul_backward(g, an, b)
    assert bits_equal(host(da), oa) and bits_equal(host(db), ob)
    ref = np.matmul(an.astype(np.float64), b.astype(np.float64))
    for mode, tol in (("tf32", 1e-2), ("3xtf32", 1e-5)):
        c = host(tlcuda.matmul(A, dev(b), mode=mode)).astype(np.float64)
        assert np.linalg.norm(c - ref) / np.linalg.norm(ref) <= tol


def test_empty_and_k0():
    z = tlcuda.matmul(dev(np.ones((0, 4), np.float32)), dev(np.ones((4, 3), np.float32)))
    assert tuple(z.shape) == (0, 3)
    c = host(tlcuda.matmul(dev(np.ones((3, 0), np.float32)), dev(np.ones((0, 5), np.float32))))
    assert c.shape == (3, 5) and np.all(c == 0) and not np.signbit(c).any()
    c = host(tlcuda.matmul(dev(np.ones((2, 0, 4), np.float32)), dev(np.ones((4, 3), np.float32))))
    assert c.shape == (2, 0, 3)
    # an empty batch dim against a broadcast one: an empty result (NumPy's rule)
    z = tlcuda.matmul(dev(np.ones((0, 5, 6), np.float32)), dev(np.ones((1, 6, 7), np.float32)))
    assert tuple(z.shape) == (0, 5, 7)


def test_misaligned_and_strided_views():
    rng = np.random.default_rng(5)
    big = dev(inputs.normal(rng, (4 * 130 * 131 + 3,)))
    a = big[1:1 + 130 * 131].view(130, 131)           # base not 16-byte aligned
    b = big[3:3 + 131 * 66].view(131, 66)[:, ::2]       # no unit stride: copied first
    an = host(a).copy()
    bn = host(b.contiguous()).copy()
    got = host(tlcuda.matmul(a, b))
    assert bits_equal(got, O.matmul(an, bn))
    c3 = dev(inputs.normal(rng, (6, 40, 50)))
    sub = c3[1::2]                                       # batch stride over a strided batch
    w = dev(inputs.normal(rng, (50, 30)))
    assert bits_equal(host(tlcuda.matmul(sub, w)), O.matmul(host(sub), host(w)))


def test_many_batch_dims_broadcast():
    rng = np.random.default_rng(9)
    a = inputs.normal(rng, (2, 1, 3, 1, 5, 6))
    b = inputs.normal(rng, (1, 4, 1, 2, 6, 7))
    assert bits_equal(host(tlcuda.matmul(dev(a), dev(b))), O.matmul(a, b))
    c = O.matmul(a, b)
    g = inputs.normal(rng, c.shape)
    da, db = tlcuda.matmul_backward(dev(g), dev(a), dev(b))
    oa, ob = O.matmul_backward(g, a, b)
    assert bits_equal(host(da), oa) and bits_equal(host(db), ob)


def test_accumulate_grad():
    rng = np.random.default_rng(10)
    a, b = inputs.normal(rng, (8, 9)), inputs.normal(rng, (9, 10))
    g = inputs.normal(rng, (8, 10))
    prev_a, prev_b = inputs.normal(rng, (8, 9)), inputs.normal(rng, (9, 10))
    da, db = dev(prev_a), dev(prev_b)
    tlcuda.matmul_backward(dev(g), dev(a), dev(b), da=da, db=db, accumulate=True)
    oa, ob = O.matmul_backward(g, a, b)
    assert bits_equal(host(da), O.add(prev_a, oa)) and bits_equal(host(db), O.add(prev_b, ob))


def test_host_buffer_form(golden):
    a, b = inputs.ragged_integer()
    assert bits_equal(tlcuda.matmul_host(a, b), golden["ragged.c"])
    g = {k: golden[f"r_bcast.{k}"] for k in ("a", "b", "g", "da", "db", "c")}
    assert bits_equal(tlcuda.matmul_host(g["a"], g["b"]), g["c"])
    da, db = tlcuda.matmul_backward_host(g["g"], g["a"], g["b"])
    assert bits_equal(da, g["da"]) and bits_equal(db, g["db"])
    x = np.asfortranarray(inputs.normal(np.random.default_rng(1), (33, 20)))  # strided host view
    w = inputs.normal(np.random.default_rng(2), (20, 9))
    assert bits_equal(tlcuda.matmul_host(x, w), O.matmul(x, w))


def test_errors_on_device():
    a = dev(np.ones((3, 4), np.float32))
    with pytest.raises(tlcuda.TLCInvalidArgument) as e:
        tlcuda.matmul(a, dev(np.ones((5, 6), np.float32)))
    assert e.value.msg == "Incompatible dimensions for matmul"


def test_full_size_linear_sampled_rows():
    """Y = X . W^T at [4096,1024] x [1024,4096] (W read in place as a K-major
    view): every element of 64 sampled rows equals the oracle bit for bit."""
    x, w, dy = inputs.cfg_linear()
    X, W = dev(x), dev(w)
    y = host(tlcuda.matmul(X, W.t()))
    rows = np.arange(0, 4096, 64)
    ref = O.gemm2d(np.ascontiguousarray(x[rows]), w.T)
    assert bits_equal(y[rows], ref)
    # backward at full size, sampled: dX = dY . W, dW^T = X^T . dY
    dxa, dwt = tlcuda.matmul_backward(dev(dy), X, W.t())
    dxa, dwt = host(dxa), host(dwt)
    assert bits_equal(dxa[rows], O.gemm2d(np.ascontiguousarray(dy[rows]), w))
    cols = np.arange(0, 1024, 64)
    ref_dwt = O.gemm2d(np.ascontiguousarray(x.T[cols]), dy)
    assert bits_equal(dwt[cols], ref_dwt)


def test_full_size_batched_sampled():
    """[64,2048,2048] . [64,2048,2048], U[-1,1] seed 4: sampled rows of a few
    batches equal the oracle bit for bit; a checksum of row checksums is
    stable across two runs."""
    g = torch.Generator(device=DEV).manual_seed(4)
    A = torch.rand((64, 2048, 2048), generator=g, device=DEV) * 2 - 1
    B = torch.rand((64, 2048, 2048), generator=g, device=DEV) * 2 - 1
    C = tlcuda.matmul(A, B)
    C2 = tlcuda.matmul(A, B)
    torch.cuda.synchronize()
    assert torch.equal(C, C2)
    for bi in (0, 31, 63):
        a = host(A[bi, ::256]).copy()
        b = host(B[bi])
        assert bits_equal(host(C[bi, ::256]), O.gemm2d(a, b))
    del A, B, C, C2
    torch.cuda.empty_cache()


@pytest.mark.parametrize("shape_a,shape_b", [
    ((40, 512, 512), (40, 512, 512)),    # chunks of batch entries
    ((32, 1024, 512), (512, 256)),       # batch chunks, B shared by every entry
    ((4100, 2048), (2048, 2048)),        # one GEMM: chunks of 256 rows of A and C
])
@pytest.mark.parametrize("pinned", [False, True])
def test_host_buffer_pipelined(shape_a, shape_b, pinned):
    """Problems above 64 MB go through the chunked upload / GEMM / download
    pipeline; the result must equal the device-resident call bit for bit."""
    g = torch.Generator(device=DEV).manual_seed(31)
    A = torch.rand(shape_a, generator=g, device=DEV) * 2 - 1
    B = torch.rand(shape_b, generator=g, device=DEV) * 2 - 1
    ref = host(tlcuda.matmul(A, B))
    ha, hb = A.cpu(), B.cpu()
    if pinned:
        ha, hb = ha.pin_memory(), hb.pin_memory()
    out = torch.empty(ref.shape, dtype=torch.float32, pin_memory=pinned)
    tlcuda.matmul_host(ha, hb, out=out)
    assert bits_equal(out.numpy(), ref)
    got = tlcuda.matmul_host(ha, hb, mode="tf32")
    denom = np.linalg.norm(ref.astype(np.float64))
    assert np.linalg.norm(got.astype(np.float64) - ref) / denom <= 1e-2
