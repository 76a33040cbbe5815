"""The oracle of the glue around the GEMMs (add with broadcasting, scale,
softmax and SoftmaxBackward, sum_to), pinned bit for bit against the
reference library compiled from its own sources (oracle/_ref):
src/ops.cpp:74-103 (add), :963-983 (scale), :985-1037 (softmax),
src/autograd.cpp:228-256 (SoftmaxBackward), :24-36 (sum_to).

A planted mistake in the oracle (one ulp in one softmax output) must be
caught by the same comparison."""
import os

import numpy as np
import pytest

import inputs
from oracle import oracle as O

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


def refs(builds=("libtlref_v3.so", "libtlref_v4.so")):
    out = []
    for lib in builds:
        path = os.path.join(REF_DIR, lib)
        if not os.path.exists(path):
            continue
        if lib.endswith("v4.so") and "avx512f" not in O._cpu_flags():
            continue
        out.append(O.TLRef(path))
    if not out:
        pytest.skip("oracle/_ref not built")
    return out


def _have(lib):
    path = os.path.join(REF_DIR, lib)
    return os.path.exists(path) and (not lib.endswith("v4.so") or "avx512f" in O._cpu_flags())


SOFTMAX_SHAPES = [(1,), (7,), (5, 7), (2, 9), (3, 13), (3, 4, 64), (2, 512), (192, 33), (4, 1000),
                  (2, 37)]


@pytest.mark.parametrize("shape", SOFTMAX_SHAPES)
def test_softmax_matches_reference(shape):
    rng = np.random.default_rng(sum(shape))
    x = inputs.normal(rng, shape) * np.float32(4.0)
    g = inputs.normal(rng, shape)
    y_o = O.softmax(x)
    # The reference's SoftmaxBackward rounds its row dot product as its build
    # vectorised it: blocks of 8 (x86-64-v4) or 4 (x86-64-v3) rounded products,
    # the tail fused.  accumulate_grad then adds the result to 0.
    for lib, vec in (("libtlref_v3.so", 4), ("libtlref_v4.so", 8)):
        dx_o = O.softmax_backward(g, y_o, vec) + np.float32(0.0)
        for R in refs((lib,)) if _have(lib) else []:
            y_r, dx_r = R.softmax(x, g)
            assert bits_equal(y_o, y_r)
            assert bits_equal(dx_o, dx_r)


def test_softmax_edge_rows():
    x = np.array([[0.0, 0.0, 0.0], [-np.inf, 1.0, 2.0], [1e30, -1e30, 0.0], [-5.0, -5.0, -4.0]],
                 np.float32)
    for R in refs():
        assert bits_equal(O.softmax(x), R.softmax(x))


def test_backward_rounding_is_pinned_to_the_build():
    # the other build's rounding differs somewhere: the pin is not vacuous
    rng = np.random.default_rng(4)
    x = inputs.normal(rng, (64, 37)) * np.float32(4.0)
    g = inputs.normal(rng, (64, 37))
    y = O.softmax(x)
    assert not bits_equal(O.softmax_backward(g, y, 4), O.softmax_backward(g, y, 8))


def test_planted_mistake_is_caught():
    x = inputs.normal(np.random.default_rng(3), (4, 9))
    bad = O.softmax(x).copy()
    bad[2, 5] = np.nextafter(bad[2, 5], np.float32(1))
    for R in refs():
        assert not bits_equal(bad, R.softmax(x))


ADD_SHAPES = [((4, 3, 5), (5,)), ((4, 1, 5), (3, 1)), ((2, 3), (2, 3)), ((6,), (1,)),
              ((2, 1, 4, 1), (3, 1, 5)), ((128, 256), (256,)), ((), (3, 2))]


@pytest.mark.parametrize("sa,sb", ADD_SHAPES)
def test_add_broadcast_matches_reference(sa, sb):
    rng = np.random.default_rng(len(sa) * 7 + len(sb))
    a, b = inputs.normal(rng, sa), inputs.normal(rng, sb)
    for R in refs():
        assert bits_equal(O.add_bcast(a, b), R.add(a, b))
        assert bits_equal(O.add_bcast(b, a), R.add(b, a))


def test_add_broadcast_error():
    a, b = np.ones((3, 4), np.float32), np.ones((2, 4), np.float32)
    with pytest.raises(ValueError, match="Incompatible dimensions for broadcasting"):
        O.add_bcast(a, b)
    for R in refs():
        with pytest.raises(ValueError, match="Incompatible dimensions for broadcasting"):
            R.add(a, b)


@pytest.mark.parametrize("s", [0.125, -3.0, 1.0 / np.sqrt(64.0), 1e-30])
def test_scale_matches_reference(s):
    x = inputs.normal(np.random.default_rng(11), (17, 33))
    for R in refs():
        assert bits_equal(O.scale(x, s), R.scale(x, s))
