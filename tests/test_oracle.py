"""The oracle (oracle/) pinned against the reference: the golden fixtures the
reference library produced (tests/golden/make_golden.py) and, where
oracle/_ref is built, the reference library itself on further cases.
CPU only."""
import os

import numpy as np
import pytest

import inputs
from oracle import oracle as O

REF_DIR = os.path.join(os.path.dirname(O.__file__), "_ref")


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


def sha(x):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(x, np.float32).tobytes()).hexdigest()


def T(x, t):
    return np.swapaxes(x, -1, -2) if t else x


def test_kat_2x3(golden):
    # tests/test_ops.cpp:21-32
    c = O.matmul(golden["kat2x3.a"], golden["kat2x3.b"])
    assert c[0, 0] == 58.0 and c[1, 1] == 154.0
    assert bits_equal(c, golden["kat2x3.c"])


def test_broadcast_4d(golden):
    # tests/test_ops.cpp:56-76
    c = O.matmul(golden["bcast4d.a"], golden["bcast4d.b"])
    assert c.shape == (2, 3, 2, 4)
    assert bits_equal(c, golden["bcast4d.c"])


def test_heavy_ones(golden):
    # tests/test_ops.cpp:78-89
    c = O.matmul(np.ones((256, 512), np.float32), np.ones((512, 256), np.float32))
    assert np.all(c == 512.0)
    assert sha(c) == str(golden["heavy.c_sha"])


def test_ragged_integer(golden):
    # tests/test_ops.cpp:91-114 (integer-valued, every element exact)
    a, b = inputs.ragged_integer()
    c = O.matmul(a, b)
    assert bits_equal(c, golden["ragged.c"])
    assert np.array_equal(c.astype(np.float64), a.astype(np.float64) @ b.astype(np.float64))


@pytest.mark.parametrize("lv", ["l1", "l2", "l3", "l4a", "l4b"])
def test_matmul_backward_levels(golden, lv):
    # tests/test_autograd.cpp:150-261
    g = {k: golden[f"bwd_{lv}.{k}"] for k in ("a", "b", "g", "da", "db")}
    da, db = O.matmul_backward(g["g"], g["a"], g["b"])
    assert bits_equal(da, g["da"]) and bits_equal(db, g["db"])


@pytest.mark.parametrize("case", ["r_2d", "r_ta", "r_tb", "r_tab", "r_batch", "r_bcast",
                                  "r_vecmat", "r_matvec", "r_vecvec", "r_k1"])
def test_random_cases(golden, case):
    a, b = golden[f"{case}.a"], golden[f"{case}.b"]
    ta, tb = bool(golden[f"{case}.ta"]), bool(golden[f"{case}.tb"])
    c = O.matmul(T(a, ta), T(b, tb))
    assert bits_equal(c, golden[f"{case}.c"])
    da, db = O.matmul_backward(golden[f"{case}.g"], T(a, ta), T(b, tb))
    # gradients of the stored leaves: transpose back through TransposeBackward
    assert bits_equal(T(da, ta), golden[f"{case}.da"])
    assert bits_equal(T(db, tb), golden[f"{case}.db"])


def test_broadcast_workload(golden):
    a, b, dc = inputs.cfg_broadcast()
    c = O.matmul(a, b)
    assert sha(c) == str(golden["cfg_broadcast.c_sha"])
    da, db = O.matmul_backward(dc, a, b)
    assert sha(da) == str(golden["cfg_broadcast.da_sha"])
    assert bits_equal(db, golden["cfg_broadcast.db"])


def test_square512_workload(golden):
    a, b = inputs.cfg_square(512, 0)
    c = O.matmul(a, b)
    assert sha(c) == str(golden["cfg_square512.c_sha"])


def test_error_messages(golden_meta):
    for name, (sa, sb) in {"k_mismatch": ((3, 4), (5, 6)),
                           "bcast_mismatch": ((2, 3, 4), (3, 4, 5))}.items():
        with pytest.raises(ValueError) as e:
            O.matmul(np.ones(sa, np.float32), np.ones(sb, np.float32))
        assert str(e.value) == golden_meta["errors"][name]


def test_oracle_error_model():
    # A planted mistake in the oracle must be caught by the comparison.
    a, b = inputs.cfg_square(64, 3)
    good = O.matmul(a, b)
    bad = O.gemm2d(a, b).copy()
    bad[3, 5] = np.nextafter(bad[3, 5], np.float32(np.inf))
    assert not bits_equal(good, bad)


@pytest.mark.skipif(not os.path.isdir(REF_DIR), reason="oracle/_ref not built")
@pytest.mark.parametrize("lib", ["libtlref_v3.so", "libtlref_v4.so"])
def test_oracle_matches_reference_library(lib):
    path = os.path.join(REF_DIR, lib)
    if not os.path.exists(path):
        pytest.skip(f"{lib} not built")
    if lib.endswith("v4.so"):
        flags = O._cpu_flags()
        if "avx512f" not in flags:
            pytest.skip("host has no AVX-512")
    R = O.TLRef(path)
    rng = np.random.default_rng(123)
    shapes = [((300, 1024), (1024, 277)), ((5, 64, 33), (33, 70)), ((1, 3, 8, 9), (2, 1, 9, 4)),
              ((257, 258), (258, 259))]
    for sa, sb in shapes:
        a, b = inputs.normal(rng, sa), inputs.uniform(rng, sb)
        assert bits_equal(R.matmul(a, b), O.matmul(a, b))
    a, b = inputs.normal(rng, (70, 40)), inputs.normal(rng, (50, 40))  # X . W^T
    assert bits_equal(R.matmul(a, b, False, True), O.matmul(a, b.T))
    g = inputs.normal(rng, (70, 50))
    ra, rb = R.matmul_backward(a, b, g, False, True)
    oa, ob = O.matmul_backward(g, a, b.T)
    assert bits_equal(ra, oa) and bits_equal(rb, ob.T)
    a, b, g = inputs.normal(rng, (6, 1, 7, 5)), inputs.normal(rng, (3, 5, 4)), None
    c = R.matmul(a, b)
    g = inputs.normal(rng, c.shape)
    ra, rb = R.matmul_backward(a, b, g)
    oa, ob = O.matmul_backward(g, a, b)
    assert bits_equal(ra, oa) and bits_equal(rb, ob)
