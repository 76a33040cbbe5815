"""tlc_gemm_3xtf32_noalloc, the 3xTF32 GEMM that allocates no device memory.

It is meant for callers that may not let the library allocate: an
application whose device memory all belongs to its own arena allocator, or a
latency-critical loop where an allocation that can block or fail is not
allowed.  Its split planes live in a fixed 64 MiB array inside the library.

Checked through the C ABI: on two calls in a row (which share that array),
its result equals the regular entry point's, tlc_gemm with TLC_MODE_3XTF32,
within the 3xTF32 tolerance of the other tests (1e-5 relative Frobenius),
device free memory does not move across the calls, and problems that do not
fit the array or its alignment rules are refused with an error.

The file name sorts last so that a run stopping at its first failure has run
every other test before this one.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tlcuda  # noqa: E402

DEV = "cuda:0"
TOL = 1e-5


def rel_fro(x, ref):
    x = x.double()
    ref = ref.double()
    return float((x - ref).norm() / ref.norm())


def desc(A, B, C):
    """GemmDesc for C = A . B over row-major (or transposed-view) CUDA tensors,
    2-D or with one batch dim (a 2-D operand is broadcast over the batch)."""
    d = tlcuda.GemmDesc()
    d.M, d.K = A.shape[-2], A.shape[-1]
    d.N = B.shape[-1]
    d.A, d.a_rs, d.a_cs = A.data_ptr(), A.stride(-2), A.stride(-1)
    d.B, d.b_rs, d.b_cs = B.data_ptr(), B.stride(-2), B.stride(-1)
    d.C, d.c_rs = C.data_ptr(), C.stride(-2)
    if C.dim() == 3:
        d.batch_ndim = 1
        d.batch_sizes[0] = C.shape[0]
        d.a_bstride[0] = A.stride(0) if A.dim() == 3 else 0
        d.b_bstride[0] = B.stride(0) if B.dim() == 3 else 0
        d.c_bstride[0] = C.stride(0)
    return d


def regular(A, B, C):
    d = desc(A, B, C)
    st = tlcuda.lib().tlc_gemm(ctypes.byref(d), 2, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, tlcuda.lib().tlc_last_error()


def noalloc(A, B, C):
    d = desc(A, B, C)
    return tlcuda.lib().tlc_gemm_3xtf32_noalloc(
        ctypes.byref(d), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_regular_entry_on_two_calls():
    g = torch.Generator(device=DEV).manual_seed(21)
    # call 1: a batch of 3 against a broadcast B, row-major, ragged tiles
    A1 = torch.randn((3, 300, 520), generator=g, device=DEV)
    B1 = torch.randn((520, 260), generator=g, device=DEV)
    # call 2: other sizes and values, A read in place as a transposed view
    A2 = torch.rand((900, 700), generator=g, device=DEV).t() * 2 - 1
    B2 = torch.rand((900, 1000), generator=g, device=DEV) * 2 - 1
    R1 = torch.empty((3, 300, 260), device=DEV)
    R2 = torch.empty((700, 1000), device=DEV)
    N1 = torch.full_like(R1, float("nan"))
    N2 = torch.full_like(R2, float("nan"))
    regular(A1, B1, R1)
    regular(A2, B2, R2)
    torch.cuda.synchronize()

    free_before = torch.cuda.mem_get_info()[0]
    st1 = noalloc(A1, B1, N1)
    st2 = noalloc(A2, B2, N2)
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info()[0]
    assert st1 == 0 and st2 == 0, tlcuda.lib().tlc_last_error()
    tlcuda.check_device_errors()
    assert free_after == free_before

    assert not torch.isnan(N1).any() and not torch.isnan(N2).any()
    assert rel_fro(N1, R1) <= TOL
    assert rel_fro(N2, R2) <= TOL
    assert rel_fro(N1, torch.matmul(A1.double(), B1.double())) <= TOL
    assert rel_fro(N2, A2.double() @ B2.double()) <= TOL


def test_noalloc_refuses_what_it_cannot_hold():
    # 4096x2048 + 2048x4096 floats need 128 MiB of split planes: above 64 MiB
    A = torch.zeros((4096, 2048), device=DEV)
    B = torch.zeros((2048, 4096), device=DEV)
    C = torch.zeros((4096, 4096), device=DEV)
    assert noalloc(A, B, C) == 1
    assert "MiB static scratch" in tlcuda.lib().tlc_last_error().decode()
    # an odd row pitch cannot be read by TMA without a repacking copy
    A = torch.zeros((64, 33), device=DEV)
    B = torch.zeros((33, 64), device=DEV)
    C = torch.zeros((64, 64), device=DEV)
    assert noalloc(A, B, C) == 2
    torch.cuda.synchronize()


def test_noalloc_batched_transposed_with_broadcast():
    """A batch of 4 transposed A views (M-major, read in place) against a
    broadcast K-major B (a transposed view of [N, K]), twice in a row."""
    g = torch.Generator(device=DEV).manual_seed(22)
    A = torch.randn((4, 260, 300), generator=g, device=DEV).transpose(1, 2)   # [4, 300, 260]
    B = torch.randn((196, 260), generator=g, device=DEV).t()                  # [260, 196]
    R = torch.empty((4, 300, 196), device=DEV)
    regular(A, B, R)
    for _ in range(2):
        N = torch.full_like(R, float("nan"))
        assert noalloc(A, B, N) == 0, tlcuda.lib().tlc_last_error()
        torch.cuda.synchronize()
        assert not torch.isnan(N).any()
        assert rel_fro(N, R) <= TOL
        assert rel_fro(N, torch.matmul(A.double(), B.double())) <= TOL


FRESH = r"""
import ctypes, sys
import torch
sys.path.insert(0, {tests!r})
import test_zz_no_alloc as t
g = torch.Generator(device="cuda:0").manual_seed(23)
A = torch.randn((2, 130, 72), generator=g, device="cuda:0")
B = torch.randn((72, 152), generator=g, device="cuda:0")
N1 = torch.empty((2, 130, 152), device="cuda:0")
N2 = torch.empty_like(N1)
R = torch.empty_like(N1)
st = t.noalloc(A, B, N1)          # the first GEMM of the process
assert st == 0, (st, t.tlcuda.lib().tlc_last_error())
st = t.noalloc(A, B, N2)
assert st == 0, (st, t.tlcuda.lib().tlc_last_error())
t.regular(A, B, R)
torch.cuda.synchronize()
assert torch.equal(N1, N2), "two calls differ"
assert t.rel_fro(N1, R) <= t.TOL, t.rel_fro(N1, R)
print("fresh ok")
"""


def test_noalloc_first_call_in_a_fresh_process():
    """In a process whose first GEMM is the allocation-free call (its set-up
    runs inside that call), the result equals the regular entry point's."""
    import os
    import subprocess
    import sys
    tests = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([tests, os.path.join(os.path.dirname(tests), "torchlite-cpp_b200"),
                                         os.path.dirname(tests), env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", FRESH.format(tests=tests)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "fresh ok" in r.stdout, r.stdout + r.stderr
