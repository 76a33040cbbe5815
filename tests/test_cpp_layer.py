"""The C++ tl:: layer (torchlite-cpp_b200/host): tl::Tensor with device
storage, tl::matmul and MatmulBackward over libtl_cuda.  Its tests
(host/tests/test_matmul.cpp) restate the reference's own matmul and
MatmulBackward tests in C++; the shape / exception part needs no GPU."""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(REPO, "torchlite-cpp_b200", "lib", "tl_tests")


def _run(*args):
    assert os.path.exists(BIN), "run python torchlite-cpp_b200/build.py"
    r = subprocess.run([BIN, *args], capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout + r.stderr


def test_cpp_layer_shape_errors():
    rc, out = _run("--cpu")
    assert rc == 0, out
    assert "errors ok" in out


@pytest.mark.gpu
def test_cpp_layer_on_gpu():
    rc, out = _run()
    assert rc == 0, out
    assert "all tl:: tests passed" in out


@pytest.mark.gpu
def test_cpp_layer_multi_gpu_group():
    """tl::matmul and MatmulBackward through the device group (TL_NUM_GPUS=2),
    bit-identical to the single-GPU entry points; skipped below two GPUs."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, TL_NUM_GPUS="2"))
    out = r.stdout + r.stderr
    assert r.returncode == 0, out
    assert "multi-GPU group ok" in out
