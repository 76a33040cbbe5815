"""Parity at every workload of the matmul path, in every precision mode, at
full size on the GPU (through the C ABI), against the oracle.

Bars, per mode:
  exact   bit-identical to the oracle (the reference's per-element ascending-k
          fmaf chain, src/ops.cpp:242-268) on every sampled element;
  tf32    relative Frobenius error <= 1e-2 against float64 and against the oracle;
  3xtf32  relative Frobenius error <= 1e-5 against float64 and against the oracle.
Full-size products are checked on sampled rows (or sampled heads): every
element of a sampled row is compared, and the rows are spread over the whole
output, so every tile row, k-block and batch stride of the launch is covered.

Workloads (seeded synthetic inputs, the reference has no datasets):
  square512   C[512,512] = A.B, A, B ~ U[-1,1] seed 0 (bench_matmul's shape)
  broadcast   A[32,128,64] . B[64,128], N(0,1) seed 1, forward + MatmulBackward
  attention   batch 16, seq 512, d_model 768, 12 heads of 64 (src/nn.cpp:401-445):
              QKV [8192,768].[768,2304], scores [192,512,64].[192,64,512] with the
              1/8 scale fused, softmax, context [192,512,512].[192,512,64],
              out-proj [8192,768].[768,768]; activations N(0,1), weights N(0,0.02)
  squares     M = N = K in {4096, 8192, 16384}, U[-1,1] seed 4
  batched     [64,2048,2048] . [64,2048,2048], U[-1,1] seed 4
"""
import numpy as np
import pytest

import inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tlcuda  # noqa: E402

DEV = "cuda:0"
MODES = ["exact", "tf32", "3xtf32"]
TOL = {"tf32": 1e-2, "3xtf32": 1e-5}
# tl::softmax on the device: |gpu - reference| <= 2e-6 * |reference| per element
# (CUDA's expf is not the C library's); a context GEMM fed by it is held to 1e-5.
SOFTMAX_CHAIN_TOL = 1e-5


def dev(x):
    return torch.from_numpy(np.array(x, dtype=np.float32, order="C", copy=True)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


def ndiff(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return int((x.view(np.uint32) != y.view(np.uint32)).sum())


def rel_fro(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


def check(mode, got, oracle_rows, f64_rows, what):
    """The per-mode bar on one block of sampled output."""
    if mode == "exact":
        assert bits_equal(got, oracle_rows), f"{what}: {ndiff(got, oracle_rows)} floats differ"
    else:
        e64, eor = rel_fro(got, f64_rows), rel_fro(got, oracle_rows)
        assert e64 <= TOL[mode], (what, "vs float64", e64)
        assert eor <= TOL[mode], (what, "vs oracle", eor)


def free():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


# ---- square512 ------------------------------------------------------------------------

@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_square512_tensor_core_modes(mode):
    """All 262144 outputs of the 512^3 product (exact mode: test_parity_gpu's sha)."""
    a, b = inputs.cfg_square(512, 0)
    got = host(tlcuda.matmul(dev(a), dev(b), mode=mode))
    check(mode, got, O.gemm2d(a, b), O.gemm2d_f64(a, b), "square512")


# ---- broadcast -----------------------------------------------------------------------

@pytest.mark.parametrize("mode", MODES)
def test_broadcast_against_oracle(mode):
    """Forward and MatmulBackward (dB summed over the batch in the reference's
    order) against the oracle's tl::matmul / MatmulBackward."""
    a, b, dc = inputs.cfg_broadcast()
    c = host(tlcuda.matmul(dev(a), dev(b), mode=mode))
    da, db = tlcuda.matmul_backward(dev(dc), dev(a), dev(b), mode=mode)
    oc = O.matmul(a, b)
    oa, ob = O.matmul_backward(dc, a, b)
    f64c = np.matmul(a.astype(np.float64), b.astype(np.float64))
    f64a = np.matmul(dc.astype(np.float64), b.T.astype(np.float64))
    f64b = np.einsum("bmk,bmn->kn", a.astype(np.float64), dc.astype(np.float64))
    check(mode, c, oc, f64c, "broadcast C")
    check(mode, host(da), oa, f64a, "broadcast dA")
    check(mode, host(db), ob, f64b, "broadcast dB")


# ---- attention (transformer encoder block) ------------------------------------------------

def attention_inputs():
    """x [8192,768] ~ N(0,1); W_qkv [768,2304], W_o [768,768] ~ N(0,0.02);
    Q, K, V [192,512,64] ~ N(0,1); numpy PCG64 seed 3."""
    rng = np.random.default_rng(3)
    x = inputs.normal(rng, (8192, 768))
    wqkv = inputs.normal(rng, (768, 2304), 0.02)
    wo = inputs.normal(rng, (768, 768), 0.02)
    q, k, v = (inputs.normal(rng, (192, 512, 64)) for _ in range(3))
    return x, wqkv, wo, q, k, v


@pytest.fixture(scope="module")
def attn():
    return attention_inputs()


ROWS_8192 = np.arange(0, 8192, 97)          # 85 rows spread over every 128-row tile band
HEADS = (0, 1, 77, 128, 191)


@pytest.mark.parametrize("mode", MODES)
def test_attention_projections(attn, mode):
    """QKV [8192,768].[768,2304] and out-proj [8192,768].[768,768]."""
    x, wqkv, wo, *_ = attn
    X = dev(x)
    for name, w in (("qkv", wqkv), ("out_proj", wo)):
        got = host(tlcuda.matmul(X, dev(w), mode=mode))
        xs = np.ascontiguousarray(x[ROWS_8192])
        check(mode, got[ROWS_8192], O.gemm2d(xs, w), O.gemm2d_f64(xs, w), name)
    free()


@pytest.mark.parametrize("mode", MODES)
def test_attention_scores_softmax_context(attn, mode):
    """scores = (Q.K^T) * 1/8 with K^T read in place and the scale fused into
    the GEMM epilogue (tl::scale(tl::matmul(q, transpose(k)), 1/sqrt(64)),
    src/nn.cpp:423-424), P = softmax(scores) on the device, context = P.V.
    Exact mode: scores bit-identical to the oracle's scale(matmul); the
    context GEMM bit-identical to the oracle's product of the same P; the
    whole chain (oracle softmax on oracle scores) within 1e-5."""
    *_, q, k, v = attn
    Q, K, V = dev(q), dev(k), dev(v)
    S = tlcuda.matmul_fused(Q, K.transpose(1, 2), 0.125, None, mode=mode)
    P = tlcuda.softmax(S)
    C = tlcuda.matmul(P, V, mode=mode)
    s_h, p_h, c_h = (host(t[list(HEADS)]) for t in (S, P, C))
    for i, h in enumerate(HEADS):
        kt = np.ascontiguousarray(k[h].T)
        o_s = O.scale(O.gemm2d(q[h], kt), 0.125)
        f_s = O.gemm2d_f64(q[h], kt) * 0.125
        check(mode, s_h[i], o_s, f_s, f"scores head {h}")
        # the context GEMM on the device's own probabilities
        check(mode, c_h[i], O.gemm2d(p_h[i], v[h]), O.gemm2d_f64(p_h[i], v[h]), f"context head {h}")
        # the whole chain against the oracle's chain
        o_c = O.gemm2d(O.softmax(o_s), v[h])
        tol = SOFTMAX_CHAIN_TOL if mode == "exact" else TOL[mode]
        assert rel_fro(c_h[i], o_c) <= tol, (h, rel_fro(c_h[i], o_c))
    del S, P, C
    free()


# ---- squares and the batched headline ------------------------------------------------------

def uniform_dev(shape, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.rand(shape, generator=g, device=DEV) * 2 - 1


@pytest.mark.parametrize("n", [4096, 8192, 16384])
def test_square_exact_sampled(n):
    """Exact mode at the square sweep sizes: 16 sampled rows, every element
    bit-identical to the oracle's fmaf chain."""
    g = torch.Generator(device=DEV).manual_seed(4)
    A = torch.rand((n, n), generator=g, device=DEV) * 2 - 1
    B = torch.rand((n, n), generator=g, device=DEV) * 2 - 1
    C = tlcuda.matmul(A, B, mode="exact")
    tlcuda.check_device_errors()
    rows = torch.arange(n // 37, n, n // 16, device=DEV)
    a = host(A[rows])
    b = host(B)
    got = host(C[rows])
    ref = O.gemm2d(a, b)
    assert bits_equal(got, ref), f"{ndiff(got, ref)} floats differ"
    del A, B, C
    free()


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_square4096_tensor_core_modes(mode):
    A = uniform_dev((4096, 4096), 4)
    B = uniform_dev((4096, 4096), 5)
    C = tlcuda.matmul(A, B, mode=mode)
    rows = torch.arange(3, 4096, 128, device=DEV)
    a, b = host(A[rows]), host(B)
    check(mode, host(C[rows]), O.gemm2d(a, b), O.gemm2d_f64(a, b), "square4096")
    del A, B, C
    free()


def test_batched_3xtf32_split_pipeline_same_bits():
    """A large batched 3xTF32 product splits its lo planes chunk by chunk on a
    side stream ahead of the GEMMs (4 chunks of 16 entries here).  Each entry
    must come out with the bits of a launch that splits everything first:
    sub-batches of 7 entries (too few to be chunked), across chunk boundaries,
    and a broadcast A (split whole, with the first chunk)."""
    g = torch.Generator(device=DEV).manual_seed(9)
    A = torch.rand((64, 2048, 2048), generator=g, device=DEV) * 2 - 1
    B = torch.rand((64, 2048, 2048), generator=g, device=DEV) * 2 - 1
    C = tlcuda.matmul(A, B, mode="3xtf32")
    for b0 in (0, 13, 45, 57):  # 13..19 and 45..51 cross chunk boundaries
        Cs = tlcuda.matmul(A[b0:b0 + 7], B[b0:b0 + 7], mode="3xtf32")
        assert torch.equal(C[b0:b0 + 7], Cs), b0
    del C, Cs
    A2 = A[5].clone()
    C = tlcuda.matmul(A2, B[:16], mode="3xtf32")
    for b0 in (0, 9):
        Cs = tlcuda.matmul(A2, B[b0:b0 + 7], mode="3xtf32")
        assert torch.equal(C[b0:b0 + 7], Cs), b0
    tlcuda.check_device_errors()
    rows = torch.arange(1, 2048, 256, device=DEV)
    a, b = host(A2[rows]), host(B[11])
    check("3xtf32", host(C[11, rows]), O.gemm2d(a, b), O.gemm2d_f64(a, b), "broadcast A, entry 11")
    del A, B, A2, C, Cs
    free()


def test_batched_3xtf32_split_pipeline_in_cuda_graph():
    """The chunked split runs on a side stream joined by events; captured into
    a CUDA graph (the side stream joins the capture through its first event
    wait), every replay recomputes the lo planes from the current inputs and
    gives the eager call's bits."""
    g = torch.Generator(device=DEV).manual_seed(10)
    A = torch.rand((16, 2048, 2048), generator=g, device=DEV) * 2 - 1
    B = torch.rand((16, 2048, 2048), generator=g, device=DEV) * 2 - 1
    eager = tlcuda.matmul(A, B, mode="3xtf32")
    out = torch.empty_like(eager)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        tlcuda.matmul(A, B, mode="3xtf32", out=out)
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    A.mul_(-0.75)  # new inputs: the replay must split them again
    graph.replay()
    eager2 = tlcuda.matmul(A, B, mode="3xtf32")
    torch.cuda.synchronize()
    assert torch.equal(out, eager2) and not torch.equal(out, eager)
    tlcuda.check_device_errors()
    del graph, A, B, eager, eager2, out
    free()


@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
def test_batched_headline_tensor_core_modes(mode):
    """[64,2048,2048] . [64,2048,2048] (the headline workload): 8 sampled rows
    of each of 6 batch entries against float64 and the oracle, and a second
    call gives the same bits (no dependence on launch order)."""
    g = torch.Generator(device=DEV).manual_seed(4)
    A = torch.rand((64, 2048, 2048), generator=g, device=DEV) * 2 - 1
    B = torch.rand((64, 2048, 2048), generator=g, device=DEV) * 2 - 1
    C = tlcuda.matmul(A, B, mode=mode)
    C2 = tlcuda.matmul(A, B, mode=mode)
    tlcuda.check_device_errors()
    assert torch.equal(C, C2)
    for bi in (0, 1, 17, 31, 62, 63):
        rows = torch.arange(bi % 7, 2048, 256, device=DEV)
        a = host(A[bi, rows])
        b = host(B[bi])
        check(mode, host(C[bi, rows]), O.gemm2d(a, b), O.gemm2d_f64(a, b), f"batch {bi}")
    del A, B, C, C2
    free()
