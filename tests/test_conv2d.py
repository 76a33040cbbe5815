"""conv2d (src/ops.cpp:1443-1548) and Conv2dBackward (src/autograd.cpp:386-517).

CPU: the oracle's restatement (im2col, gemm_blocked's chain, col2im in the
reference's loop order, the (n, oh, ow) bias chain) equals the reference
library compiled from its sources, bit for bit, forward and backward.
GPU: libtl_cuda's im2col + batched GEMM path (tlc_conv2d / _backward) equals
the oracle bit for bit in exact mode; TF32 / 3xTF32 within their GEMM
tolerances; the reference's error texts."""
import numpy as np
import pytest

import inputs
from oracle import oracle as O

# (N, C_in, H, W, C_out, k, stride, padding, groups)
CASES = [
    (2, 3, 8, 8, 4, 3, 1, 1, 1),
    (1, 4, 7, 9, 6, 3, 2, 0, 2),
    (3, 6, 5, 5, 6, 1, 1, 0, 3),
    (2, 2, 6, 6, 4, 5, 2, 2, 1),
    (1, 8, 10, 10, 8, 3, 1, 1, 8),   # depthwise
    (2, 3, 4, 4, 2, 3, 3, 0, 1),     # stride larger than the step the kernel needs
    (1, 1, 2, 2, 1, 3, 2, 0, 1),     # input smaller than the kernel: (2 - 3) / 2 + 1 = 1 (C++ division)
    # widths that are multiples of 4 take the vectorised im2col / col2im kernels
    (2, 4, 12, 16, 8, 3, 2, 1, 2),   # stride 2, padding, groups
    (1, 3, 9, 12, 4, 1, 1, 0, 1),    # 1x1
    (2, 2, 8, 8, 2, 5, 1, 2, 1),     # 5x5, padding 2
]


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


def case_data(case, seed):
    N, C, H, W, Co, k, s, p, g = case
    rng = np.random.default_rng(seed)
    x = inputs.normal(rng, (N, C, H, W))
    w = inputs.normal(rng, (Co, C // g, k, k))
    b = inputs.normal(rng, (Co,))
    return x, w, b, s, p, g


def ref():
    try:
        return O.tlref()
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference(case):
    R = ref()
    x, w, b, s, p, g = case_data(case, 7)
    y = O.conv2d(x, w, b, s, p, g)
    go = inputs.normal(np.random.default_rng(8), y.shape)
    y_r, dx_r, dw_r, db_r = R.conv2d(x, w, b, s, p, g, grad=go)
    assert bits_equal(y, y_r)
    dx, dw, db = O.conv2d_backward(go, x, w, s, p, g)
    assert bits_equal(dx, dx_r) and bits_equal(dw, dw_r) and bits_equal(db, db_r)


def test_reference_errors():
    R = ref()
    x = np.ones((1, 4, 5, 5), np.float32)
    for w, g, msg in [(np.ones((4, 4, 3, 3), np.float32), 0, "conv2d: groups must be > 0"),
                      (np.ones((4, 4, 3, 3), np.float32), 3, "conv2d: groups doesn't divide C_in"),
                      (np.ones((3, 2, 3, 3), np.float32), 2, "conv2d: groups doesn't divide C_out"),
                      (np.ones((4, 3, 3, 3), np.float32), 2,
                       "conv2d: weight.sizes()[1] must equal C_in / groups"),
                      (np.ones((4, 4, 9, 3), np.float32), 1, "Tensor size must be positive integer"),
                      (np.ones((4, 4, 9, 9), np.float32), 1, "reshape: negative dims not allowed")]:
        with pytest.raises(ValueError) as e:
            R.conv2d(x, w, None, 1, 0, g)
        assert str(e.value) == msg


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_device_conv2d_exact(case):
    torch = pytest.importorskip("torch")
    import tlcuda
    x, w, b, s, p, g = case_data(case, 11)
    X, Wt, B = (torch.from_numpy(a).cuda() for a in (x, w, b))
    y = tlcuda.conv2d(X, Wt, B, s, p, g, mode="exact")
    torch.cuda.synchronize()
    assert bits_equal(y.cpu().numpy(), O.conv2d(x, w, b, s, p, g))
    go = inputs.normal(np.random.default_rng(12), tuple(y.shape))
    dx, dw, db = tlcuda.conv2d_backward(torch.from_numpy(go).cuda(), X, Wt, s, p, g, mode="exact")
    torch.cuda.synchronize()
    ox, ow_, ob = O.conv2d_backward(go, x, w, s, p, g)
    assert bits_equal(dx.cpu().numpy(), ox)
    assert bits_equal(dw.cpu().numpy(), ow_)
    assert bits_equal(db.cpu().numpy(), ob)


@pytest.mark.gpu
@pytest.mark.parametrize("mode,tol", [("tf32", 1e-2), ("3xtf32", 1e-5)])
@pytest.mark.parametrize("case", [(4, 32, 28, 28, 64, 3, 1, 1, 1), (2, 64, 30, 30, 64, 3, 1, 1, 1),
                                  (2, 16, 17, 23, 48, 3, 1, 0, 1), (2, 8, 15, 15, 12, 5, 1, 2, 2),
                                  # implicit GEMM (stride 1, output rows a multiple of 8 wide):
                                  # forward and input gradient without a column buffer
                                  (2, 64, 16, 16, 64, 3, 1, 1, 1), (2, 32, 20, 24, 48, 3, 1, 1, 1),
                                  (1, 4, 10, 8, 8, 3, 1, 1, 1), (2, 64, 12, 16, 64, 3, 1, 1, 2),
                                  (1, 16, 12, 16, 16, 5, 1, 2, 1), (2, 32, 8, 8, 16, 1, 1, 0, 1),
                                  (2, 64, 56, 56, 64, 3, 1, 1, 1),
                                  # weight gradient as the split-K implicit GEMM with two
                                  # 128-row tiles of output channels
                                  (1, 8, 10, 16, 160, 3, 1, 1, 1)]
                         # float64 torch needs the padded input at least as large as the kernel
                         + [c for c in CASES if min(c[2], c[3]) + 2 * c[7] >= c[5]])
def test_device_conv2d_tensor_cores(mode, tol, case):
    """The tensor-core modes against float64 over the reference's shapes,
    strides, paddings and groups: at stride 1 with output rows a multiple of 8
    wide the implicit GEMMs (forward, input gradient, weight gradient),
    otherwise im2col + batched tcgen05 GEMMs and col2im."""
    torch = pytest.importorskip("torch")
    import tlcuda
    x, w, b, s, p, g = case_data(case, 13)
    X, Wt, B = (torch.from_numpy(a).cuda() for a in (x, w, b))
    ref64 = torch.nn.functional.conv2d(X.double(), Wt.double(), B.double(), s, p, 1, g)
    y = tlcuda.conv2d(X, Wt, B, s, p, g, mode=mode).double()
    assert ((y - ref64).norm() / ref64.norm()).item() <= tol
    go = torch.randn(tuple(y.shape), device="cuda")
    Xd, Wd = X.double().requires_grad_(), Wt.double().requires_grad_()
    torch.nn.functional.conv2d(Xd, Wd, None, s, p, 1, g).backward(go.double())
    dx, dw, db = tlcuda.conv2d_backward(go, X, Wt, s, p, g, mode=mode)
    assert ((dx.double() - Xd.grad).norm() / Xd.grad.norm()).item() <= tol
    assert ((dw.double() - Wd.grad).norm() / Wd.grad.norm()).item() <= tol
    # the bias gradient is a plain sum: in these modes a tree, not the reference's chain
    db64 = go.double().sum(dim=(0, 2, 3))
    assert ((db.double() - db64).norm() / db64.norm()).item() <= 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["tf32", "3xtf32"])
@pytest.mark.parametrize("case", [(2, 64, 12, 16, 48, 3, 1, 1, 1), (3, 32, 9, 24, 40, 3, 1, 1, 1)])
def test_backward_gradient_subsets(mode, case):
    """Every subset of (d_input, d_weight, d_bias): the implicit backward
    shares one preparation launch between the gradients (NHWC copies, flipped
    weights, and the bias partial sums taken from dO's transpose when d_input
    is requested), so each subset takes a different launch plan.  d_input and
    d_weight must equal the all-three call bit for bit; d_bias is a tree sum
    in these modes, within 1e-5 of float64."""
    torch = pytest.importorskip("torch")
    import itertools
    import tlcuda
    x, w, b, s, p, g = case_data(case, 29)
    X, Wt = (torch.from_numpy(a).cuda() for a in (x, w))
    y = tlcuda.conv2d(X, Wt, None, s, p, g, mode=mode)
    go = torch.randn(tuple(y.shape), device="cuda", generator=torch.Generator("cuda").manual_seed(7))
    full = tlcuda.conv2d_backward(go, X, Wt, s, p, g, mode=mode)
    db64 = go.double().sum(dim=(0, 2, 3))
    for need in itertools.product((False, True), repeat=3):
        if not any(need):
            continue
        got = tlcuda.conv2d_backward(go, X, Wt, s, p, g, mode=mode, need=need)
        torch.cuda.synchronize()
        for k in range(2):
            if need[k]:
                assert torch.equal(got[k].view(torch.int32), full[k].view(torch.int32)), (need, k)
            else:
                assert got[k] is None
        if need[2]:
            assert ((got[2].double() - db64).norm() / db64.norm()).item() <= 1e-5, need


def test_library_errors_match_reference():
    """The shape checks run on the host (tlc_conv2d_shape): the reference's texts."""
    import tlcuda
    x = np.ones((1, 4, 5, 5), np.float32)
    for w, g, msg in [(np.ones((4, 4, 3, 3), np.float32), 0, "conv2d: groups must be > 0"),
                      (np.ones((4, 4, 3, 3), np.float32), 3, "conv2d: groups doesn't divide C_in"),
                      (np.ones((3, 2, 3, 3), np.float32), 2, "conv2d: groups doesn't divide C_out"),
                      (np.ones((4, 3, 3, 3), np.float32), 2,
                       "conv2d: weight.sizes()[1] must equal C_in / groups"),
                      (np.ones((4, 4, 9, 3), np.float32), 1, "Tensor size must be positive integer"),
                      (np.ones((4, 4, 9, 9), np.float32), 1, "reshape: negative dims not allowed")]:
        vx, vw = tlcuda.view_of(x), tlcuda.view_of(w)
        sz = (tlcuda.ctypes.c_int64 * 4)()
        st = tlcuda.lib().tlc_conv2d_shape(tlcuda.ctypes.byref(vx), tlcuda.ctypes.byref(vw), 1, 0, g, sz)
        assert st == 1 and tlcuda.lib().tlc_last_error().decode() == msg
