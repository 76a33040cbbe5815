"""The C ABI without a GPU: libtl_cuda loads, exports every entry point that
include/*.h declares, and its host-only logic (shape rules and errors of
tl::matmul, partition helpers, mode parsing) matches the reference."""
import ctypes
import glob
import os
import re
import subprocess

import numpy as np
import pytest

import tlcuda
from oracle import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(tlc_\w+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_library_built_and_loads():
    assert os.path.exists(tlcuda.LIB_PATH), "run python torchlite-cpp_b200/build.py"
    L = tlcuda.lib()
    assert L.tlc_version() >= 100


def test_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 25
    L = ctypes.CDLL(tlcuda.LIB_PATH)
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", tlcuda.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\bT (tlc_\w+)", out))
    assert names <= exported
    # the Python binding declares a signature for each of them
    assert names <= set(tlcuda.SIGNATURES), names - set(tlcuda.SIGNATURES)


def test_kernels_are_sm100a():
    out = subprocess.run(["cuobjdump", "--list-elf", tlcuda.LIB_PATH], capture_output=True,
                         text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


SHAPES = [((2, 3), (3, 2)), ((2, 3, 2, 2), (2, 4)), ((4,), (4, 3)), ((3, 4), (4,)), ((4,), (4,)),
          ((2, 1, 5, 7), (3, 7, 4)), ((7, 1, 3), (1, 3, 2)), ((0, 3), (3, 5)), ((3, 0), (0, 5))]


@pytest.mark.parametrize("sa,sb", SHAPES)
def test_matmul_shape_matches_reference(sa, sb):
    a, b = np.zeros(sa, np.float32), np.zeros(sb, np.float32)
    assert tlcuda.matmul_shape(a, b) == O.matmul(a, b).shape


@pytest.mark.parametrize("sa,sb,msg", [
    ((3, 4), (5, 6), "Incompatible dimensions for matmul"),
    ((2, 3, 4), (3, 4, 5), "Incompatible dimensions for broadcasting"),
    ((5,), (4,), "Incompatible dimensions for matmul"),
])
def test_matmul_shape_errors(sa, sb, msg, golden_meta):
    a, b = np.zeros(sa, np.float32), np.zeros(sb, np.float32)
    with pytest.raises(tlcuda.TLCInvalidArgument) as e:
        tlcuda.matmul_shape(a, b)
    assert e.value.msg == msg
    with pytest.raises(ValueError) as e2:
        O.matmul(a, b)
    assert str(e2.value) == msg


def test_zero_dim_operand_error():
    a = np.zeros((), np.float32)
    b = np.zeros((3, 2), np.float32)
    with pytest.raises(tlcuda.TLCInvalidArgument) as e:
        tlcuda.matmul_shape(a, b)
    assert e.value.msg == "matmul: requires at least 1D tensors"


def test_shard_helpers():
    for count, world in [(64, 8), (65, 8), (3, 8), (0, 4), (64, 3)]:
        got = [tlcuda.shard_range(count, world, r) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == count
        assert all(got[i][1] == got[i + 1][0] for i in range(world - 1))
        sizes = [e - b for b, e in got]
        assert max(sizes) - min(sizes) <= 1
    for N, world, align in [(8192, 8, 256), (4096, 3, 128), (1000, 8, 16)]:
        got = [tlcuda.shard_cols(N, world, r, align) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == N
        assert all(b % align == 0 for b, _ in got)


def test_modes():
    L = tlcuda.lib()
    assert L.tlc_mode_from_string(b"exact") == 0
    assert L.tlc_mode_from_string(b"TF32") == 1
    assert L.tlc_mode_from_string(b"3xtf32") == 2
    assert L.tlc_mode_from_string(b"fp16") == -1
    assert L.tlc_status_string(5) == b"kernel wait timed out"


def test_group_argument_errors_without_a_gpu():
    """tlc_group_create rejects an empty device list before touching a GPU."""
    L = tlcuda.lib()
    g = ctypes.c_void_p()
    assert L.tlc_group_create((ctypes.c_int * 1)(0), 0, ctypes.byref(g)) == 1
    assert "1 to 64 devices" in L.tlc_last_error().decode()
    assert L.tlc_group_destroy(None) == 0
    n = ctypes.c_int(0)
    assert L.tlc_group_size(None, ctypes.byref(n), None) == 1
