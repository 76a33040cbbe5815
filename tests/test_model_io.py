"""TLMD model files straight to and from device memory (tlc_load_tlmd /
tlc_save_tlmd) against the reference's load_model / save_model
(src/model_io.cpp:7-94), compiled from its sources (oracle/_ref).

CPU: the format restated below writes the reference's bytes; the library's
header and shape checks fail with the reference's messages before any
device work.  GPU: files written from device tensors equal the reference's
byte for byte; files the reference wrote load into device tensors exactly,
including tensors larger than one staging chunk, 0-D and empty ones."""
import os
import struct

import numpy as np
import pytest

import inputs
from oracle import oracle as O

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def write_tlmd(path, arrays):
    """The TLMD format: "TLMD", int32 1, int64 count, per tensor int64 ndim,
    int64 shape[ndim], float32 data (little-endian)."""
    with open(path, "wb") as f:
        f.write(b"TLMD" + struct.pack("<i", 1) + struct.pack("<q", len(arrays)))
        for a in arrays:
            a = np.array(a, dtype=np.float32, order="C", copy=True)  # keeps 0-D
            f.write(struct.pack("<q", a.ndim) + struct.pack(f"<{a.ndim}q", *a.shape))
            f.write(a.tobytes())


def ref():
    try:
        return O.tlref()
    except FileNotFoundError:
        pytest.skip("oracle/_ref not built")


def tensors(rng):
    return [inputs.normal(rng, (4, 8)), inputs.normal(rng, (8,)), inputs.normal(rng, (8, 2)),
            inputs.normal(rng, (2,)), np.array(3.5, np.float32), np.zeros((0, 5), np.float32)]


def test_format_matches_reference(tmp_path):
    R = ref()
    ts = tensors(np.random.default_rng(1))
    R.save_model(tmp_path / "ref.tl", ts)
    write_tlmd(tmp_path / "ours.tl", ts)
    assert (tmp_path / "ref.tl").read_bytes() == (tmp_path / "ours.tl").read_bytes()
    back = R.load_model(tmp_path / "ours.tl", [t.shape for t in ts])
    assert all(np.array_equal(a, b) for a, b in zip(back, ts))


def _expect(fn, msg):
    with pytest.raises(Exception) as e:
        fn()
    assert msg in str(e.value), str(e.value)


def test_header_errors_match_reference(tmp_path):
    """Errors the library reports before touching a device: same texts as the reference."""
    import tlcuda
    R = ref()
    ts = tensors(np.random.default_rng(2))
    shapes = [t.shape for t in ts]
    good = tmp_path / "good.tl"
    write_tlmd(good, ts)
    bad_magic = tmp_path / "magic.tl"
    bad_magic.write_bytes(b"XLMD" + good.read_bytes()[4:])
    bad_version = tmp_path / "version.tl"
    bad_version.write_bytes(b"TLMD" + struct.pack("<i", 2) + good.read_bytes()[8:])
    host = [np.empty(s, np.float32) for s in shapes]
    cases = [
        (tmp_path / "missing.tl", host, f"load_model: cannot open file: {tmp_path / 'missing.tl'}"),
        (bad_magic, host, f"load_model: no TLMD magic header in {bad_magic}"),
        (bad_version, host, "load_model: unsupported version"),
        (good, host[:-1], "load_model: tensor count mismatch"),
        (good, [np.empty((4, 8, 1), np.float32)] + host[1:], "load_model: ndim mismatch"),
        (good, [np.empty((4, 9), np.float32)] + host[1:], "load_model: shape mismatch"),
    ]
    for path, dst, msg in cases:
        _expect(lambda: tlcuda.load_tlmd(path, dst), msg)
        _expect(lambda: R.load_model(path, [d.shape for d in dst]), msg)


@pytest.mark.gpu
def test_device_round_trip_and_reference_files(tmp_path):
    torch = pytest.importorskip("torch")
    import tlcuda
    R = ref()
    rng = np.random.default_rng(3)
    ts = tensors(rng) + [inputs.normal(rng, (5, 1000, 1000))]  # 20 MB: more than one chunk
    dev = [torch.from_numpy(np.array(t, copy=True)).cuda() for t in ts]
    tlcuda.save_tlmd(tmp_path / "dev.tl", dev)
    R.save_model(tmp_path / "ref.tl", ts)
    assert (tmp_path / "dev.tl").read_bytes() == (tmp_path / "ref.tl").read_bytes()
    # strided device sources are written as the reference writes p->contiguous()
    w = torch.from_numpy(inputs.normal(rng, (6, 9))).cuda()
    tlcuda.save_tlmd(tmp_path / "t.tl", [w.t()])
    R.save_model(tmp_path / "t_ref.tl", [w.cpu().numpy().T])
    assert (tmp_path / "t.tl").read_bytes() == (tmp_path / "t_ref.tl").read_bytes()
    # a reference-written file straight into device tensors
    out = [torch.full(tuple(t.shape), -1.0, device="cuda") for t in ts]
    tlcuda.load_tlmd(tmp_path / "ref.tl", out)
    torch.cuda.synchronize()
    for o, t in zip(out, ts):
        assert np.array_equal(o.cpu().numpy(), t)
    # a shape mismatch after earlier tensors loaded, and a file that ends early
    wrong = [torch.empty(tuple(t.shape), device="cuda") for t in ts]
    wrong[2] = torch.empty((8, 3), device="cuda")
    _expect(lambda: tlcuda.load_tlmd(tmp_path / "ref.tl", wrong), "load_model: shape mismatch")
    cut = tmp_path / "cut.tl"
    cut.write_bytes((tmp_path / "ref.tl").read_bytes()[:-1000])
    _expect(lambda: tlcuda.load_tlmd(cut, [torch.empty(tuple(t.shape), device="cuda") for t in ts]),
            "load_model: file truncated")
