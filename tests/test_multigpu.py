"""The multi-GPU partitioning of tl::matmul (torchlite-cpp_b200/tldist.py).

CPU: two gloo ranks run the partition plan (libtl_cuda's host-only
tlc_shard_range / tlc_shard_cols), compute their shares with the oracle,
all-gather them, and reassemble with the index rule of tlc_gather_colblocks;
the result must equal the oracle's full product bit for bit.  They also run
tldist.chained_batch_sum (the rank-to-rank chain that reduces a broadcast
operand's gradient in batch order) on oracle per-entry products, which must
equal the oracle's MatmulBackward dB bit for bit.
GPU (1 device): tlc_gather_colblocks on blocks computed per simulated rank.
GPU (2+ devices): the real NCCL path, one process per GPU.
"""
import os
import socket

import numpy as np
import pytest

import inputs
from oracle import oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def reassemble_colblocks(gathered, M, N, edges):
    """numpy restatement of tlc_gather_colblocks' index rule."""
    out = np.empty((M, N), np.float32)
    for r in range(len(edges) - 1):
        w = edges[r + 1] - edges[r]
        out[:, edges[r]:edges[r + 1]] = gathered[M * edges[r]: M * edges[r] + M * w].reshape(M, w)
    return out


def _gloo_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import tlcuda
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(7)
        # single GEMM, output column blocks (ragged N and ragged last block)
        M, K, N = 37, 53, 300
        a = inputs.normal(rng, (M, K))
        b = inputs.normal(rng, (K, N))
        edges = [tlcuda.shard_cols(N, world, r, 64)[0] for r in range(world)] + [N]
        c0, c1 = edges[rank], edges[rank + 1]
        block = O.gemm2d(a, np.ascontiguousarray(b[:, c0:c1]))
        wmax = max(edges[r + 1] - edges[r] for r in range(world))
        pad = np.zeros((M, wmax), np.float32)
        pad[:, : c1 - c0] = block
        parts = [torch.zeros((M, wmax)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(pad))
        gathered = np.concatenate([parts[r].numpy()[:, : edges[r + 1] - edges[r]].reshape(-1)
                                   for r in range(world)])
        full = reassemble_colblocks(gathered, M, N, edges)
        ok_cols = np.array_equal(full.view(np.uint32), O.gemm2d(a, b).view(np.uint32))
        # batched GEMM with broadcast B, split over the batch
        A = inputs.normal(rng, (5, 9, 11))
        B = inputs.normal(rng, (11, 6))
        b0, b1 = tlcuda.shard_range(5, world, rank)
        mine = O.matmul(A[b0:b1], B)
        sizes = [tlcuda.shard_range(5, world, r) for r in range(world)]
        per = max(e - s for s, e in sizes)
        pad = np.zeros((per, 9, 6), np.float32)
        pad[: b1 - b0] = mine
        parts = [torch.zeros((per, 9, 6)) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(pad))
        C = np.concatenate([parts[r].numpy()[: sizes[r][1] - sizes[r][0]] for r in range(world)])
        ok_batch = np.array_equal(C.view(np.uint32), O.matmul(A, B).view(np.uint32))
        # its backward: dB of the broadcast B through the order-keeping chain
        # (per-entry products from the oracle, the chain and its sends as shipped)
        import tldist
        dC = inputs.normal(np.random.default_rng(9), (5, 9, 6))
        G = O.matmul(np.ascontiguousarray(A[b0:b1].transpose(0, 2, 1)), dC[b0:b1])
        def sum0(st, init=None):
            # the oracle's sequential sum; continuing from `init` is the sum
            # of [init, entries...] from 0.0f (0 + init == init here)
            x = st.numpy() if init is None else np.concatenate([init.numpy()[None], st.numpy()])
            return torch.from_numpy(O.sum_dim(x, 0, False))
        dB = tldist.chained_batch_sum(torch.from_numpy(G), sum0=sum0).numpy()
        ref_dA, ref_dB = O.matmul_backward(dC, A, B)
        ok_bwd = np.array_equal(dB.view(np.uint32), ref_dB.view(np.uint32))
        dist.destroy_process_group()
        q.put((rank, ok_cols, ok_batch and ok_bwd, None))
    except Exception as e:  # report, do not hang the parent
        q.put((rank, False, False, repr(e)))


def test_partition_plan_gloo_two_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok_cols, ok_batch, err in res:
        assert err is None, err
        assert ok_cols and ok_batch, (rank, ok_cols, ok_batch)


@pytest.mark.gpu
def test_gather_colblocks_single_gpu():
    torch = pytest.importorskip("torch")
    import tlcuda
    rng = np.random.default_rng(8)
    M, K, N, P = 130, 70, 1000, 3
    a = inputs.normal(rng, (M, K))
    b = inputs.normal(rng, (K, N))
    A = torch.from_numpy(a).cuda()
    B = torch.from_numpy(b).cuda()
    edges = [tlcuda.shard_cols(N, P, r, 64)[0] for r in range(P)] + [N]
    blocks = [tlcuda.matmul(A, B[:, edges[r]:edges[r + 1]]) for r in range(P)]
    gathered = torch.cat([x.reshape(-1) for x in blocks])
    out = torch.empty((M, N), device="cuda")
    tlcuda.gather_colblocks(gathered, out, M, N, edges)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), O.gemm2d(a, b).view(np.uint32))


def _nccl_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import tldist
    import tlcuda
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import datetime
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        g = torch.Generator(device="cuda").manual_seed(3)
        A = torch.randn((512, 384), generator=g, device="cuda")
        B = torch.randn((384, 1000), generator=g, device="cuda")
        full = tldist.colblock_sharded_matmul(A, B, mode="exact", gather=True, align=128)
        ref = tlcuda.matmul(A, B, mode="exact")
        ok1 = torch.equal(full, ref)
        A3 = torch.randn((7, 64, 96), generator=g, device="cuda")
        B2 = torch.randn((96, 80), generator=g, device="cuda")
        C = tldist.batch_sharded_matmul(A3, B2, mode="exact", gather=True)
        ok2 = torch.equal(C, tlcuda.matmul(A3, B2, mode="exact"))
        # backward of the batch split: dA shards local, dB of the broadcast B
        # summed across ranks (exact: ordered chain, bit-identical; tf32:
        # all-reduce, within the TF32 tolerance)
        dC = torch.randn((7, 64, 80), generator=g, device="cuda")
        b0, b1 = tldist.batch_shard(7, world, rank)
        ref_dA, ref_dB = tlcuda.matmul_backward(dC, A3, B2, mode="exact")
        dA, dB = tldist.batch_sharded_matmul_backward(dC[b0:b1], A3, B2, mode="exact")
        ok2 = ok2 and torch.equal(dA, ref_dA[b0:b1]) and torch.equal(dB, ref_dB)
        dA, dB = tldist.batch_sharded_matmul_backward(dC[b0:b1], A3, B2, mode="tf32")
        rel = ((dB.double() - ref_dB.double()).norm() / ref_dB.double().norm()).item()
        ok2 = ok2 and rel < 1e-2
        torch.cuda.synchronize()
        dist.destroy_process_group()
        q.put((rank, ok1, ok2, None))
    except Exception as e:
        q.put((rank, False, False, repr(e)))


@pytest.mark.gpu
def test_nccl_two_gpus():
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok1, ok2, err in res:
        assert err is None, err
        assert ok1 and ok2, (rank, ok1, ok2)
