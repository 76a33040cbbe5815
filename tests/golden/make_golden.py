"""Generates tests/golden/*.npz by running the reference library itself
(oracle/_ref/libtlref_*.so: the reference's own src/*.cpp compiled by
oracle/Makefile, driven through oracle/ref_shim.cpp).

Run in the build container (it needs the reference sources to build
oracle/_ref):   make -C oracle ref && python tests/golden/make_golden.py

Each case stores its inputs when they are small, or the recipe to rebuild
them from tests/inputs.py when they are not, plus the reference outputs (or,
for large outputs, their SHA-256 and a few full rows).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.dirname(HERE))

from oracle import oracle as O  # noqa: E402
import inputs  # noqa: E402


def sha(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x, np.float32).tobytes()).hexdigest()


def main():
    R = O.tlref()
    out = {}
    meta = {"generator": "reference library (oracle/_ref) " + os.path.basename(R.path), "cases": {}}

    def put(name, **arrs):
        for k, v in arrs.items():
            out[f"{name}.{k}"] = np.asarray(v)

    # tests/test_ops.cpp:21-32: [[1,2,3],[4,5,6]] . [[7,8],[9,10],[11,12]]
    a = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    b = np.arange(7, 13, dtype=np.float32).reshape(3, 2)
    put("kat2x3", a=a, b=b, c=R.matmul(a, b))

    # tests/test_ops.cpp:56-76: ones[2,3,2,2] . 0.5[2,4] -> 1.0, shape [2,3,2,4]
    a = np.ones((2, 3, 2, 2), np.float32)
    b = np.full((2, 4), 0.5, np.float32)
    put("bcast4d", a=a, b=b, c=R.matmul(a, b))

    # tests/test_ops.cpp:78-89: ones[256,512] . ones[512,256] -> 512
    a = np.ones((256, 512), np.float32)
    b = np.ones((512, 256), np.float32)
    c = R.matmul(a, b)
    put("heavy", c_sha=np.array(sha(c)), c_row0=c[0], shape=np.array(c.shape))

    # tests/test_ops.cpp:91-114: ragged integer-valued [259,300] . [300,277]
    a, b = inputs.ragged_integer()
    c = R.matmul(a, b)
    put("ragged", c=c)

    # tests/test_autograd.cpp:150-261: MatmulBackward levels 1-4b
    lv = {}
    a = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    b = np.arange(1, 7, dtype=np.float32).reshape(3, 2)
    lv["l1"] = (a, b, np.ones((2, 2), np.float32))
    lv["l2"] = (np.ones((2, 2, 3), np.float32), np.ones((2, 3, 2), np.float32),
                np.ones((2, 2, 2), np.float32))
    lv["l3"] = (np.ones((2, 3, 4), np.float32), np.ones((4, 2), np.float32),
                np.ones((2, 3, 2), np.float32))
    lv["l4a"] = (np.ones(4, np.float32), np.ones((4, 3), np.float32), np.ones(3, np.float32))
    lv["l4b"] = (np.ones((3, 4), np.float32), np.ones(4, np.float32), np.ones(3, np.float32))
    for k, (a, b, g) in lv.items():
        da, db = R.matmul_backward(a, b, g)
        put(f"bwd_{k}", a=a, b=b, g=g, da=da, db=db)

    # Seeded random cases (small enough to store whole).
    rng = np.random.default_rng(11)
    small = {
        "r_2d": ((37, 53), (53, 29), False, False),
        "r_ta": ((53, 37), (53, 29), True, False),     # A given as [K, M], used transposed
        "r_tb": ((37, 53), (29, 53), False, True),     # B given as [N, K]: the Linear X.W^T form
        "r_tab": ((53, 37), (29, 53), True, True),
        "r_batch": ((3, 17, 40), (3, 40, 19), False, False),
        "r_bcast": ((2, 1, 9, 12), (4, 12, 5), False, False),
        "r_vecmat": ((33,), (33, 7), False, False),
        "r_matvec": ((6, 33), (33,), False, False),
        "r_vecvec": ((33,), (33,), False, False),
        "r_k1": ((20, 1), (1, 21), False, False),
    }
    for k, (sa, sb, ta, tb) in small.items():
        a = inputs.normal(rng, sa)
        b = inputs.normal(rng, sb)
        c = R.matmul(a, b, ta, tb)
        g = inputs.normal(rng, c.shape)
        da, db = R.matmul_backward(a, b, g, ta, tb)
        put(k, a=a, b=b, ta=np.array(ta), tb=np.array(tb), c=c, g=g, da=da, db=db)

    # The broadcast workload A[32,128,64] . B[64,128], fwd + bwd (seed 1).
    a, b, dc = inputs.cfg_broadcast()
    c = R.matmul(a, b)
    da, db = R.matmul_backward(a, b, dc)
    put("cfg_broadcast", c_sha=np.array(sha(c)), da_sha=np.array(sha(da)), db=db,
        c_rows=c[:, 0, :], da_rows=da[:, 0, :])

    # The square workload C[512,512] = A . B, A, B ~ U[-1,1] seed 0.
    a, b = inputs.cfg_square(512, 0)
    c = R.matmul(a, b)
    put("cfg_square512", c_sha=np.array(sha(c)), c_rows=c[::64])

    # Error messages (src/ops.cpp:622, :635, :66).
    errs = {}
    for name, (sa, sb) in {"k_mismatch": ((3, 4), (5, 6)),
                           "bcast_mismatch": ((2, 3, 4), (3, 4, 5))}.items():
        try:
            R.matmul(np.ones(sa, np.float32), np.ones(sb, np.float32))
            errs[name] = None
        except ValueError as e:
            errs[name] = str(e)
    meta["errors"] = errs
    meta["cases"] = sorted({k.split(".")[0] for k in out})

    np.savez_compressed(os.path.join(HERE, "reference_matmul.npz"), **out)
    with open(os.path.join(HERE, "reference_matmul.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(out), "arrays;", os.path.getsize(os.path.join(HERE, "reference_matmul.npz")),
          "bytes")


if __name__ == "__main__":
    main()
