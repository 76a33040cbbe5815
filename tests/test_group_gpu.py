"""Device groups (tlc_group_*): one tl::matmul over several GPUs from one
process, through the C ABI.

Every split keeps each output element's additions on one GPU, so results must
equal the single-device entry points bit for bit in exact mode (and the
oracle), and stay within the mode's tolerance of them otherwise.  The dB of a
broadcast B, summed over the batch by a chain across the GPUs, must equal the
oracle's sequential sum_to bit for bit.  On a box with one GPU the group
lists that device more than once, which runs the same splits, worker threads,
copies and chain on it; with two or more GPUs a group of distinct devices
also runs the NCCL broadcast and the copies between devices.
"""
import numpy as np
import pytest

import inputs
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import tlcuda  # noqa: E402

TOL = {"tf32": 1e-2, "3xtf32": 1e-5}


def groups():
    n = torch.cuda.device_count()
    out = [[0, 0], [0, 0, 0]]
    if n >= 2:
        out.append(list(range(n)))
    return out


GROUPS = groups()


def bits_equal(x, y):
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return x.shape == y.shape and np.array_equal(x.view(np.uint32), y.view(np.uint32))


def rel_fro(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(x - ref) / max(np.linalg.norm(ref), 1e-300))


def same(mode, got, ref):
    if mode == "exact":
        assert bits_equal(got, ref), int((np.asarray(got).view(np.uint32) != ref.view(np.uint32)).sum())
    else:
        assert rel_fro(got, ref) <= TOL[mode]


@pytest.fixture(scope="module", params=range(len(GROUPS)), ids=lambda i: "x".join(map(str, GROUPS[i])))
def group(request):
    g = tlcuda.Group(GROUPS[request.param])
    yield g
    g.close()


@pytest.mark.parametrize("mode", ["exact", "tf32", "3xtf32"])
@pytest.mark.parametrize("sa,sb", [((7, 130, 72), (7, 72, 100)),     # both batched
                                   ((5, 2, 64, 48), (48, 80)),       # broadcast B, two batch dims
                                   ((300, 260), (260, 520)),         # one product: row blocks
                                   ((9, 40, 36), (36, 20))])
def test_group_matmul_host(group, mode, sa, sb):
    rng = np.random.default_rng(len(sa) * 100 + sa[0])
    a, b = inputs.normal(rng, sa), inputs.normal(rng, sb)
    ref = tlcuda.matmul_host(a, b, mode=mode)
    got = group.matmul_host(a, b, mode=mode)
    same(mode, got, ref)
    if mode == "exact":
        assert bits_equal(got, O.matmul(a, b))


@pytest.mark.parametrize("mode", ["exact", "tf32", "3xtf32"])
@pytest.mark.parametrize("sa,sb", [((6, 33, 20), (6, 20, 28)),       # every entry independent
                                   ((7, 40, 24), (24, 36)),          # broadcast B: the dB chain
                                   ((600, 64), (64, 96))])           # one product: dA row blocks
@pytest.mark.parametrize("accumulate", [False, True])
def test_group_matmul_backward_host(group, mode, sa, sb, accumulate):
    rng = np.random.default_rng(sa[0] * 7 + len(sb))
    a, b = inputs.normal(rng, sa), inputs.normal(rng, sb)
    g = inputs.normal(rng, O.matmul(a, b).shape)
    prev_a, prev_b = inputs.normal(rng, sa), inputs.normal(rng, sb)
    da, db = (prev_a.copy(), prev_b.copy()) if accumulate else (None, None)
    da, db = group.matmul_backward_host(g, a, b, mode=mode, da=da, db=db, accumulate=accumulate)
    oa, ob = O.matmul_backward(g, a, b)
    if accumulate:
        oa, ob = O.add(prev_a, oa), O.add(prev_b, ob)
    if mode == "exact":
        assert bits_equal(da, oa) and bits_equal(db, ob)
    else:
        assert rel_fro(da, oa) <= TOL[mode] and rel_fro(db, ob) <= TOL[mode]


@pytest.mark.parametrize("mode", ["exact", "tf32"])
@pytest.mark.parametrize("sa,sb", [((8, 130, 72), (8, 72, 100)),
                                   ((6, 64, 96), (96, 40)),
                                   ((300, 200), (200, 1100))])      # one product: column blocks
def test_group_matmul_device(group, mode, sa, sb):
    rng = np.random.default_rng(sa[-1] + sb[-1])
    a, b = inputs.normal(rng, sa), inputs.normal(rng, sb)
    dev = "cuda:%d" % group.devices[0]
    A, B = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    ref = tlcuda.matmul(A, B, mode=mode).cpu().numpy()
    got = group.matmul(A, B, mode=mode)
    torch.cuda.synchronize()
    same(mode, got.cpu().numpy(), ref)
    if mode == "exact":
        assert bits_equal(got.cpu().numpy(), O.matmul(a, b))


def test_group_errors():
    with pytest.raises(tlcuda.TLCInvalidArgument):
        tlcuda.Group([torch.cuda.device_count()])
    with tlcuda.Group([0, 0]) as g:
        with pytest.raises(tlcuda.TLCInvalidArgument, match="Incompatible dimensions for matmul"):
            g.matmul_host(np.ones((3, 4), np.float32), np.ones((5, 6), np.float32))
        n, _ = g.size()
        assert n == 2
