"""flash_attention (src/ops.cpp:1040-1137) and FlashAttentionBackward
(src/autograd.cpp:575-669).

CPU: the oracle's restatement (64 x 64 tiles, online softmax, the Release
build's rounding of each dot over d) equals the reference compiled from its
sources bit for bit, forward and backward, on tile-crossing and ragged shapes;
the library's argument checks.
GPU: tlc_flash_attention / _backward against the oracle (exact mode: the
FFMA forward kernel; tf32: the tensor-core forward, checked to the TF32
tolerance).  The reference's own
bar for flash attention is 1e-4 per element against the materialised softmax
path (tests/test_ops.cpp:651-704); the device path keeps to
|gpu - oracle| <= FA_ATOL + FA_RTOL * |oracle| per element (CUDA's expf and
logf are not the C library's, the softmax sums and the dots run in another
order).  The tensor-core modes of the backward: relative Frobenius error
against an fp64 torch reference within the GEMM tolerances (1e-2 TF32, 1e-5
3xTF32)."""
import math

import numpy as np
import pytest

import inputs
from oracle import oracle as O

FA_ATOL = 1e-5
FA_RTOL = 1e-4

# (heads, S, d): heads () is the reference's one-head [S, d]
CASES = [((), 80, 16), ((), 64, 64), ((), 1, 8), ((), 130, 33), ((), 65, 100), ((), 200, 7),
         ((), 70, 128), ((2, 3), 97, 64), ((4,), 256, 32)]


def case_data(heads, S, d, seed):
    rng = np.random.default_rng(seed)
    shape = tuple(heads) + (S, d)
    q, k, v, g = (inputs.normal(rng, shape) for _ in range(4))
    return q, k, v, g, np.float32(1.0 / math.sqrt(d))


def ref():
    try:
        return O.tlref()
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")


@pytest.mark.parametrize("heads,S,d", [c for c in CASES if c[0] == ()] + [((), 70, 24), ((), 70, 12)])
def test_oracle_matches_reference(heads, S, d):
    R = ref()
    q, k, v, g, sc = case_data(heads, S, d, 5)
    o_r, dq_r, dk_r, dv_r = R.flash_attention(q, k, v, sc, grad=g)
    o, lse = O.flash_attention(q, k, v, sc)
    assert np.array_equal(o, o_r)
    dq, dk, dv = O.flash_attention_backward(g, q, k, v, o, lse, sc)
    assert np.array_equal(dq, dq_r) and np.array_equal(dk, dk_r) and np.array_equal(dv, dv_r)


def test_oracle_against_materialised_softmax():
    """The reference's own check (tests/test_ops.cpp:651-669), on the oracle:
    flash attention within 1e-4 of softmax(Q.K^T * scale).V in float64."""
    q, k, v, _, sc = case_data((), 80, 16, 6)
    o, _ = O.flash_attention(q, k, v, sc)
    t = q.astype(np.float64) @ k.T.astype(np.float64) * float(sc)
    p = np.exp(t - t.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    assert np.abs(o - p @ v.astype(np.float64)).max() <= 1e-4


def test_library_argument_checks():
    """Shape and layout checks run on the host before any device work."""
    import tlcuda
    L = tlcuda.lib()
    q = np.ones((4, 8), np.float32)

    def call(k, out, lse=None):
        vq, vk, vo = tlcuda.view_of(q), tlcuda.view_of(k), tlcuda.view_of(out)
        vl = tlcuda.view_of(lse) if lse is not None else None
        return L.tlc_flash_attention(tlcuda.ctypes.byref(vq), tlcuda.ctypes.byref(vk),
                                     tlcuda.ctypes.byref(vk), 1.0, tlcuda.ctypes.byref(vo),
                                     tlcuda.ctypes.byref(vl) if vl else None, 0, None)

    assert call(np.ones((4, 9), np.float32), np.ones((4, 8), np.float32)) == 1
    assert "shapes differ" in L.tlc_last_error().decode()
    assert call(np.ones((8, 4), np.float32).T, np.ones((4, 8), np.float32)) == 1
    assert "contiguous" in L.tlc_last_error().decode()
    assert call(q, np.ones((4, 8), np.float32), np.ones((5,), np.float32)) == 1
    assert "lse" in L.tlc_last_error().decode()
    big = np.ones((2, 129), np.float32)
    vb = tlcuda.view_of(big)
    st = L.tlc_flash_attention(*(tlcuda.ctypes.byref(vb) for _ in range(3)), 1.0,
                               tlcuda.ctypes.byref(vb), None, 0, None)
    assert st == 2 and "head dim above 128" in L.tlc_last_error().decode()


# ---- GPU ----------------------------------------------------------------------------------


def close(gpu, want):
    err = np.abs(gpu.astype(np.float64) - want)
    return bool(np.all(err <= FA_ATOL + FA_RTOL * np.abs(want))), float(err.max())


@pytest.mark.gpu
@pytest.mark.parametrize("heads,S,d", CASES)
def test_device_forward_and_backward(heads, S, d):
    torch = pytest.importorskip("torch")
    import tlcuda
    q, k, v, g, sc = case_data(heads, S, d, 21)
    Q, K, V, G = (torch.from_numpy(a).cuda() for a in (q, k, v, g))
    out, lse = tlcuda.flash_attention(Q, K, V, sc)
    torch.cuda.synchronize()
    o_o, l_o = O.flash_attention(q, k, v, sc)
    ok, e = close(out.cpu().numpy(), o_o)
    assert ok, f"O max err {e}"
    ok, e = close(lse.cpu().numpy(), l_o)
    assert ok, f"L max err {e}"
    dq, dk, dv = tlcuda.flash_attention_backward(G, Q, K, V, out, lse, sc, mode="exact")
    torch.cuda.synchronize()
    for name, got, want in zip("QKV", (dq, dk, dv), O.flash_attention_backward(g, q, k, v, o_o, l_o, sc)):
        ok, e = close(got.cpu().numpy(), want)
        assert ok, f"d{name} max err {e}"


@pytest.mark.gpu
def test_device_unaligned_operands():
    """Operands 4 bytes off a 16-byte boundary take the scalar tile loads."""
    torch = pytest.importorskip("torch")
    import tlcuda
    q, k, v, _, sc = case_data((), 100, 64, 22)
    flat = torch.zeros(3 * q.size + 1, device="cuda")
    views = []
    for i, a in enumerate((q, k, v)):
        t = flat[1 + i * q.size:1 + (i + 1) * q.size].view(q.shape)
        t.copy_(torch.from_numpy(a))
        views.append(t)
    for mode in ("exact", "tf32"):  # tf32 too: unaligned operands take the FFMA kernel
        out, _ = tlcuda.flash_attention(*views, sc, mode=mode)
        ok, e = close(out.cpu().numpy(), O.flash_attention(q, k, v, sc)[0])
        assert ok, (mode, e)


@pytest.mark.gpu
def test_device_matches_materialised_path():
    """The reference's own test (tests/test_ops.cpp:651-704) on the device:
    flash forward and backward within 1e-4 of the materialised path through
    the same library (scaled GEMM, softmax, GEMM; their backward nodes)."""
    torch = pytest.importorskip("torch")
    import tlcuda
    q, k, v, _, sc = case_data((), 80, 16, 23)
    Q, K, V = (torch.from_numpy(a).cuda() for a in (q, k, v))
    G = torch.ones((80, 16), device="cuda")  # backward() seeds ones
    sc_ = tlcuda.matmul_fused(Q, K.t(), float(sc), None, mode="exact")
    P = tlcuda.softmax(sc_)
    ref_o = tlcuda.matmul(P, V, mode="exact")
    dP, dV_ref = tlcuda.matmul_backward(G, P, V, mode="exact")
    dS = tlcuda.softmax_backward(dP, P)
    dS = tlcuda.scale(dS, float(sc))
    dQ_ref, dKt_ref = tlcuda.matmul_backward(dS, Q, K.t(), mode="exact")
    out, lse = tlcuda.flash_attention(Q, K, V, sc)
    dq, dk, dv = tlcuda.flash_attention_backward(G, Q, K, V, out, lse, sc, mode="exact")
    torch.cuda.synchronize()
    for got, want in ((out, ref_o), (dq, dQ_ref), (dk, dKt_ref.t()), (dv, dV_ref)):
        assert (got - want).abs().max().item() <= 1e-4


# TF32 forward (tensor-core kernel): relative Frobenius error of O and L
# against the oracle / fp64 within the TF32 tolerance
TF32_TOL = 1e-2
TF32_CASES = [((), 80, 64), ((2, 3), 300, 64), ((4,), 1000, 32), ((2,), 129, 48), ((), 1, 64),
              ((), 64, 40), ((3,), 257, 64)]


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("heads,S,d", TF32_CASES)
def test_device_tf32_forward(heads, S, d):
    """mode tf32: the tensor-core forward (32 <= d <= 64) against the oracle."""
    torch = pytest.importorskip("torch")
    import tlcuda
    q, k, v, _, sc = case_data(heads, S, d, 25)
    Q, K, V = (torch.from_numpy(a).cuda() for a in (q, k, v))
    launches = tlcuda.launch_count()
    out, lse = tlcuda.flash_attention(Q, K, V, sc, mode="tf32")
    assert tlcuda.lib().tlc_check_device_errors() == 0  # no bounded wait gave up
    assert tlcuda.launch_count() == launches + 1
    o_o, l_o = O.flash_attention(q, k, v, sc)
    assert rel(out.cpu().numpy(), o_o) <= TF32_TOL
    # L = m + log(l) is a log-sum of scores: its TF32 error is absolute (the
    # scores' rounding), so it is bounded against max(1, |L|), not |L| alone
    dl = np.abs(lse.cpu().numpy().astype(np.float64) - l_o)
    assert dl.max() <= TF32_TOL * max(1.0, float(np.abs(l_o).max()))
    assert np.isfinite(out.cpu().numpy()).all()


@pytest.mark.gpu
@pytest.mark.parametrize("heads,S,d", TF32_CASES)
def test_device_tf32_backward(heads, S, d):
    """mode tf32: the fused tensor-core backward (prep + dK/dV + dQ kernels,
    32 <= d <= 64) against the oracle, relative Frobenius error per gradient."""
    torch = pytest.importorskip("torch")
    import tlcuda
    q, k, v, g, sc = case_data(heads, S, d, 26)
    Q, K, V, G = (torch.from_numpy(a).cuda() for a in (q, k, v, g))
    o_o, l_o = O.flash_attention(q, k, v, sc)
    Oo, Lo = torch.from_numpy(o_o).cuda(), torch.from_numpy(l_o).cuda()
    launches = tlcuda.launch_count()
    dq, dk, dv = tlcuda.flash_attention_backward(G, Q, K, V, Oo, Lo, sc, mode="tf32")
    assert tlcuda.lib().tlc_check_device_errors() == 0  # no bounded wait gave up
    assert tlcuda.launch_count() == launches + 3
    for name, got, want in zip("QKV", (dq, dk, dv), O.flash_attention_backward(g, q, k, v, o_o, l_o, sc)):
        got = got.cpu().numpy()
        if S == 1 and name in "QK":
            # one key: P = 1 and dP = D, so dS = 0 and dQ = dK = 0 exactly; the
            # device's dP - D is a TF32 rounding, bounded by |dO| |V| |K or Q| * scale
            other = k if name == "Q" else q
            bound = TF32_TOL * float(sc) * np.linalg.norm(g) * np.linalg.norm(v) * np.linalg.norm(other)
            assert np.linalg.norm(got) <= bound, (name, np.linalg.norm(got), bound)
            continue
        e = rel(got, want)
        assert e <= TF32_TOL, (name, e)


@pytest.mark.gpu
def test_device_tf32_backward_low_scores():
    """Rows whose scores all lie far below zero (L << 0): keys past S must not
    turn exp(-L) into inf * 0 in the dQ kernel."""
    torch = pytest.importorskip("torch")
    import tlcuda
    S, d = 100, 64
    rng = np.random.default_rng(27)
    q = inputs.normal(rng, (S, d))
    k = -np.abs(q[:, :1]) * 0 + inputs.normal(rng, (S, d))
    v, g = inputs.normal(rng, (S, d)), inputs.normal(rng, (S, d))
    q = q * 0 + 1.0  # every query the same, keys shifted so all scores are << 0
    k = (k - 30.0).astype(np.float32)
    q = q.astype(np.float32)
    sc = np.float32(0.125)
    o_o, l_o = O.flash_attention(q, k, v, sc)
    assert l_o.max() < -50
    Q, K, V, G, Oo, Lo = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v, g, o_o, l_o))
    dq, dk, dv = tlcuda.flash_attention_backward(G, Q, K, V, Oo, Lo, sc, mode="tf32")
    assert tlcuda.lib().tlc_check_device_errors() == 0
    # Scores near -240: TF32's relative rounding (~5e-4) of each score is an
    # absolute error of ~0.1 in the exponent, ~10 % in P, for any TF32 path.
    # What this case checks is that the result stays finite (without the
    # masking, padded keys give 0 * inf = NaN); the bound only catches garbage.
    for name, got, want in zip("QKV", (dq, dk, dv), O.flash_attention_backward(g, q, k, v, o_o, l_o, sc)):
        got = got.cpu().numpy()
        assert np.isfinite(got).all(), name
        assert rel(got, want) <= 0.5, (name, rel(got, want))


@pytest.mark.gpu
@pytest.mark.parametrize("mode,tol", [("exact", 1e-5), ("3xtf32", 1e-5), ("tf32", 1e-2)])
def test_device_large_against_fp64(mode, tol):
    """A multi-head case too large for the oracle: 8 heads of S = 2048, d = 64,
    against torch's fp64 materialised attention and its autograd; the forward
    in the same mode (tf32: the tensor-core kernel)."""
    torch = pytest.importorskip("torch")
    import tlcuda
    g = torch.Generator(device="cuda").manual_seed(24)
    Q, K, V, G = (torch.randn((8, 2048, 64), generator=g, device="cuda") for _ in range(4))
    sc = 0.125
    out, lse = tlcuda.flash_attention(Q, K, V, sc, mode=mode)
    dq, dk, dv = tlcuda.flash_attention_backward(G, Q, K, V, out, lse, sc, mode=mode)
    Qd, Kd, Vd = (t.double().requires_grad_() for t in (Q, K, V))
    ref = torch.softmax(Qd @ Kd.transpose(1, 2) * sc, -1) @ Vd
    ref.backward(G.double())

    def trel(a, b):
        return ((a.double() - b).norm() / b.norm()).item()
    ftol = 1e-6 if mode != "tf32" else TF32_TOL
    assert trel(out, ref.detach()) <= ftol
    lse_ref = torch.logsumexp(Qd.detach() @ Kd.detach().transpose(1, 2) * sc, -1)
    assert trel(lse, lse_ref) <= ftol
    for got, want in ((dq, Qd.grad), (dk, Kd.grad), (dv, Vd.grad)):
        assert trel(got, want) <= tol, (mode, trel(got, want))


@pytest.mark.gpu
def test_device_empty_and_zero_dim():
    torch = pytest.importorskip("torch")
    import tlcuda
    z = torch.empty((3, 0, 16), device="cuda")
    out, lse = tlcuda.flash_attention(z, z, z, 0.25)
    assert out.shape == (3, 0, 16) and lse.shape == (3, 0)
    dq, dk, dv = tlcuda.flash_attention_backward(z, z, z, z, out, lse, 0.25)
    assert dq.shape == (3, 0, 16)
    # d = 0: out is empty, L = log(S) (every score 0)
    e = torch.empty((5, 0), device="cuda")
    out, lse = tlcuda.flash_attention(e, e, e, 1.0)
    torch.cuda.synchronize()
    assert out.shape == (5, 0)
    assert torch.allclose(lse, torch.full((5,), math.log(5.0), device="cuda"))
