"""The reference library's own callers of tl::matmul on the GPU path.

oracle/_ref/ref_callers_{v3,v4} is linked from the reference's objects
(nn::Linear, MultiHeadAttention, MatmulBackward and the ops they use, compiled
from the reference's sources) with tl::matmul redirected by the linker to
torchlite-cpp_b200/integration/reference_matmul_gpu.cpp, which runs every
product through libtl_cuda's host-buffer entry point.  The driver program
(tests/integration/ref_callers_main.cpp) runs Linear forward/backward on 2-D
and batched inputs, MultiHeadAttention forward/backward, a broadcast batched
matmul and an X.W^T product on seeded inputs and writes every output and
gradient as float32.

oracle/_ref/ref_callers_cpu_{v3,v4} links the same objects and driver with
the reference's own CPU matmul, so the two runs differ only in where the
products are computed.  Exact mode must give identical bits (the reference's
src/ops.cpp:605-699 matmul and src/autograd.cpp:341-384 backward, unmodified
callers in src/nn.cpp:77-83 and src/nn.cpp:401-445); TF32 and 3xTF32 are held
to relative Frobenius errors of 1e-2 and 1e-5 over the whole output.  The
"encoder" scenario runs the reference's MultiHeadAttention at the full
transformer-encoder size (batch 16, seq 512, d_model 768, 12 heads) forward
and backward the same way.

tests/integration/device_callers_main.cpp runs the same scenarios on the
device-resident C++ tl:: layer (torchlite-cpp_b200/host: Linear with the
bias add fused into its GEMM, attention with the 1/sqrt(d) scale fused and
the softmax and its backward on the GPU); its outputs must equal the
reference's bit for bit, except the attention block, which carries the
softmax's few-ulp difference (CUDA's expf) and is held to 1e-5.
"""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "oracle", "_ref")


def _binary(cpu=False):
    flags = O._cpu_flags()
    v4 = {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl"} <= flags
    name = ("ref_callers_cpu_" if cpu else "ref_callers_") + ("v4" if v4 else "v3")
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built (needs the reference sources)")
    return path


def _run(tmp_path, name, env_extra, cpu=False, scenario=None, timeout=300):
    out = tmp_path / f"{name}.bin"
    env = dict(os.environ)
    env.update(env_extra)
    cmd = [_binary(cpu), str(out)] + ([scenario] if scenario else [])
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout + r.stderr
    fields = r.stdout.split()
    launches = int(fields[fields.index("launches") + 1])
    return np.fromfile(out, dtype=np.float32), launches


def _compare(got, ref, tol):
    assert got.shape == ref.shape
    if tol == 0.0:
        assert got.tobytes() == ref.tobytes(), (
            f"{int((got.view(np.uint32) != ref.view(np.uint32)).sum())} floats differ")
    else:
        d = got.astype(np.float64) - ref
        rel = np.linalg.norm(d) / np.linalg.norm(ref.astype(np.float64))
        assert rel <= tol, rel


def test_reference_callers_cpu_run(tmp_path):
    """The reference-only binary runs without a GPU and launches nothing."""
    y, launches = _run(tmp_path, "cpu", {}, cpu=True)
    assert launches == 0
    assert y.size == sum(int(np.prod(shp)) for _, shapes in SEGMENTS for shp in shapes)
    assert np.isfinite(y).all() and np.abs(y).max() > 0


@pytest.mark.gpu
@pytest.mark.parametrize("mode,tol", [("exact", 0.0), ("tf32", 1e-2), ("3xtf32", 1e-5)])
def test_reference_callers_on_gpu(tmp_path, mode, tol):
    ref, n0 = _run(tmp_path, "cpu", {}, cpu=True)
    got, n1 = _run(tmp_path, mode, {"TL_GEMM_MODE": mode})
    assert n0 == 0
    assert n1 > 0, "no kernel of libtl_cuda ran: the matmuls did not reach the GPU"
    _compare(got, ref, tol)


@pytest.fixture(scope="module")
def encoder_reference(tmp_path_factory):
    ref, n0 = _run(tmp_path_factory.mktemp("enc"), "cpu", {}, cpu=True, scenario="encoder",
                   timeout=900)
    assert n0 == 0
    return ref


# y [16,512,768], dx [16,512,768], dW_q [768,768], dW_v [768,768]
ENCODER_FLOATS = 2 * 16 * 512 * 768 + 2 * 768 * 768


@pytest.mark.gpu
@pytest.mark.parametrize("mode,tol", [("exact", 0.0), ("tf32", 1e-2), ("3xtf32", 1e-5)])
def test_reference_encoder_attention_full_size(tmp_path, encoder_reference, mode, tol):
    """The reference's own MultiHeadAttention at batch 16, seq 512, d_model 768,
    12 heads, forward + backward, every product through libtl_cuda (the
    projections [8192,768].[768,768], scores on transposed views, the context
    product and all their MatmulBackward products)."""
    got, n1 = _run(tmp_path, mode, {"TL_GEMM_MODE": mode}, scenario="encoder", timeout=900)
    assert n1 > 0, "no kernel of libtl_cuda ran: the matmuls did not reach the GPU"
    assert got.size == ENCODER_FLOATS
    _compare(got, encoder_reference, tol)


# (scenario, shapes of its outputs in dump order) of both callers programs
SEGMENTS = [
    ("linear", [(129, 257), (129, 300), (300, 257), (257,)]),
    ("linear_batched", [(4, 33, 50), (4, 33, 70), (70, 50)]),
    ("attention", [(2, 40, 96), (2, 40, 96), (96, 96), (96, 96)]),
    ("broadcast_matmul", [(3, 20, 25), (3, 20, 30), (30, 25)]),
    ("x_wt", [(65, 31), (65, 48), (31, 48)]),
    ("conv2d", [(2, 6, 5, 6), (2, 4, 9, 11), (6, 2, 3, 3), (6,)]),
]
DEVICE_BIN = os.path.join(ROOT, "torchlite-cpp_b200", "lib", "tl_device_callers")


@pytest.mark.gpu
def test_device_layer_runs_the_reference_callers(tmp_path):
    if not os.path.exists(DEVICE_BIN):
        pytest.skip("tl_device_callers not built")
    ref, _ = _run(tmp_path, "cpu", {}, cpu=True)
    out = tmp_path / "device.bin"
    r = subprocess.run([DEVICE_BIN, str(out)], capture_output=True, text=True, timeout=300,
                       env={k: v for k, v in os.environ.items() if k != "TL_GEMM_MODE"})
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.fromfile(out, dtype=np.float32)
    assert got.shape == ref.shape
    off = 0
    for name, shapes in SEGMENTS:
        for shp in shapes:
            n = int(np.prod(shp))
            g, e = got[off:off + n], ref[off:off + n]
            off += n
            if name == "attention":
                rel = np.linalg.norm(g.astype(np.float64) - e) / np.linalg.norm(e.astype(np.float64))
                assert rel <= 1e-5, (name, shp, rel)
            else:
                assert g.tobytes() == e.tobytes(), (
                    name, shp, int((g.view(np.uint32) != e.view(np.uint32)).sum()))
    assert off == got.size
