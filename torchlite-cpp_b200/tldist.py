"""Multi-GPU partitioning of tl::matmul over the GPUs of one node.

One process per GPU; torch.distributed (NCCL) is the plumbing.  The compute
is libtl_cuda's GEMM on each rank's share; no collective runs in the data
path of the GEMM itself.

  batch_sharded_matmul    a batched / broadcast GEMM split over its flattened
                          batch dim: rank r computes batch entries
                          [begin_r, end_r) (tlc_shard_range); broadcast
                          operands are replicated.  Optional all-gather of C.
  colblock_sharded_matmul a single GEMM split over output column blocks:
                          rank r computes C[:, c_r:c_{r+1}] = A . B[:, c_r:c_{r+1}]
                          with B's column block read in place (row stride N,
                          no repack) and A replicated.  Optional NCCL
                          all-gather of the blocks + tlc_gather_colblocks into
                          the row-major [M, N] result on every rank.

The reference library has no multi-GPU path (its only parallelism is the
std::thread row bands of gemm_mt, src/ops.cpp:569-587); this module is the
B200-node counterpart of that intra-op split.
"""
from __future__ import annotations

import tlcuda


def world():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def batch_shard(count: int, nranks: int, rank: int):
    return tlcuda.shard_range(count, nranks, rank)


def col_blocks(N: int, nranks: int, align: int = 256):
    """Column-block edges [c_0 = 0, ..., c_P = N] (tlc_shard_cols)."""
    edges = [tlcuda.shard_cols(N, nranks, r, align)[0] for r in range(nranks)]
    return edges + [N]


def batch_sharded_matmul(A, B, mode="tf32", gather=False, group=None):
    """C = A . B for A [batch, M, K] and B [batch, K, N] or [K, N] (broadcast),
    split over the batch: returns this rank's C shard [end-begin, M, N], or the
    full C on every rank if gather=True."""
    import torch
    import torch.distributed as dist
    P, r = world()
    b0, b1 = batch_shard(A.shape[0], P, r)
    Bs = B[b0:b1] if B.dim() == 3 else B
    C = tlcuda.matmul(A[b0:b1], Bs, mode=mode)
    if not gather or P == 1:
        return C
    # all_gather_into_tensor takes equal shards: pad ragged ones
    per = -(-A.shape[0] // P)
    buf = torch.zeros((per,) + tuple(C.shape[1:]), device=C.device, dtype=C.dtype)
    buf[: C.shape[0]] = C
    out = torch.empty((per * P,) + tuple(C.shape[1:]), device=C.device, dtype=C.dtype)
    dist.all_gather_into_tensor(out, buf, group=group)
    keep = []
    for q in range(P):
        s, e = batch_shard(A.shape[0], P, q)
        keep.append(torch.arange(q * per, q * per + (e - s), device=C.device))
    return out[torch.cat(keep)]


def colblock_sharded_matmul(A, B, mode="tf32", gather=False, align=256, group=None):
    """C = A . B for A [M, K] (replicated) and B [K, N] (replicated), split over
    output column blocks.  Returns this rank's block C[:, c_r:c_{r+1}]
    ([M, w_r], contiguous), or the full [M, N] on every rank if gather=True."""
    import torch
    import torch.distributed as dist
    P, r = world()
    M, N = A.shape[0], B.shape[1]
    edges = col_blocks(N, P, align)
    c0, c1 = edges[r], edges[r + 1]
    block = tlcuda.matmul(A, B[:, c0:c1], mode=mode)  # B block read in place, stride N
    if not gather or P == 1:
        return block
    wmax = max(edges[q + 1] - edges[q] for q in range(P))
    if all(edges[q + 1] - edges[q] == wmax for q in range(P)):
        gathered = torch.empty((P * M * wmax,), device=A.device, dtype=A.dtype)
        dist.all_gather_into_tensor(gathered, block.reshape(-1), group=group)
    else:  # ragged last block: gather padded blocks, then compact
        pad = torch.zeros((M, wmax), device=A.device, dtype=A.dtype)
        pad[:, : c1 - c0] = block
        tmp = torch.empty((P, M, wmax), device=A.device, dtype=A.dtype)
        dist.all_gather_into_tensor(tmp, pad, group=group)
        gathered = torch.cat([tmp[q, :, : edges[q + 1] - edges[q]].reshape(-1) for q in range(P)])
    out = torch.empty((M, N), device=A.device, dtype=A.dtype)
    tlcuda.gather_colblocks(gathered, out, M, N, edges)
    return out
