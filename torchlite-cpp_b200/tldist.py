"""Multi-GPU partitioning of tl::matmul over the GPUs of one node.

One process per GPU; torch.distributed (NCCL) is the plumbing.  The compute
is libtl_cuda's GEMM on each rank's share; no collective runs in the data
path of the GEMM itself.

  batch_sharded_matmul    a batched / broadcast GEMM split over its flattened
                          batch dim: rank r computes batch entries
                          [begin_r, end_r) (tlc_shard_range); broadcast
                          operands are replicated.  Optional all-gather of C.
  batch_sharded_matmul_backward
                          MatmulBackward of the batch-split product: dA is
                          local to each rank's entries; dB of a broadcast B
                          is summed over all entries, by a rank-to-rank
                          chain in batch order for exact mode (bit-identical
                          to the reference's sequential sum_to) or by one
                          NCCL all-reduce for the tensor-core modes.
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
    out = torch.empty((A.shape[0],) + tuple(C.shape[1:]), device=C.device, dtype=C.dtype)
    if A.shape[0] % P == 0:
        # equal shards land in place: rank q's entries are [q*per, (q+1)*per)
        dist.all_gather_into_tensor(out, C, group=group)
        return out
    # ragged shards (the first count % P ranks hold one more): every rank's
    # shard is gathered straight into its rows of `out`
    parts = [out[slice(*batch_shard(A.shape[0], P, q))] for q in range(P)]
    dist.all_gather(parts, C, group=group)
    return out


def chained_batch_sum(local_stack, sum0=None, group=None):
    """The sum over dim 0 of the stack of all ranks' entries, in global entry
    order, returned on every rank.  Rank r holds entries [begin_r, end_r) of
    the global order (tlc_shard_range), as `local_stack`.

    The reference reduces a broadcast operand's gradient with one sequential
    sum from 0.0f over the batch (sum_to -> sum, src/autograd.cpp:24-36,
    src/ops.cpp:1181-1233).  The chain keeps that order across ranks: rank r
    receives the running sum of ranks < r, continues it over its own entries
    and sends it on; the last rank broadcasts the total.  Continuing is
    ((running + e0) + e1)..., the same additions as one sequential sum.
    `sum0(stack, init=...)` sums a stack over dim 0 from `init` (from 0.0f
    when init is None; default: the library's tlc_sum_dim_from on the GPU)."""
    import torch
    import torch.distributed as dist
    if sum0 is None:
        sum0 = tlcuda.sum_dim0
    P, r = world()
    shape = tuple(local_stack.shape[1:])
    run = None
    if P > 1 and r > 0:
        run = torch.empty(shape, dtype=local_stack.dtype, device=local_stack.device)
        dist.recv(run, src=r - 1, group=group)
    total = sum0(local_stack.contiguous(), init=run)
    if P == 1:
        return total
    if r < P - 1:
        dist.send(total.contiguous(), dst=r + 1, group=group)
    out = total.contiguous() if r == P - 1 else torch.empty(shape, dtype=local_stack.dtype,
                                                           device=local_stack.device)
    dist.broadcast(out, src=P - 1, group=group)
    return out


def batch_sharded_matmul_backward(dC, A, B, mode="tf32", group=None):
    """MatmulBackward of batch_sharded_matmul(A, B): `dC` is this rank's
    shard of the upstream gradient ([end-begin, M, N]); A [batch, M, K] and B
    ([batch, K, N] or broadcast [K, N]) are the full operands, as given to the
    forward.  Returns (dA shard [end-begin, M, K], dB), where dB is this
    rank's shard for a batched B and the full [K, N] on every rank for a
    broadcast B (src/autograd.cpp:341-384: dA = dC.B^T, dB = sum_to(A^T.dC))."""
    import torch.distributed as dist
    P, r = world()
    b0, b1 = batch_shard(A.shape[0], P, r)
    A_r = A[b0:b1]
    if B.dim() == 3:  # every entry has its own B: nothing to exchange
        return tlcuda.matmul_backward(dC, A_r, B[b0:b1], mode=mode)
    dA, _ = tlcuda.matmul_backward(dC, A_r, B, mode=mode, need_b=False)
    if P == 1:
        _, dB = tlcuda.matmul_backward(dC, A_r, B, mode=mode, need_a=False)
        return dA, dB
    if mode == "exact":
        # per-entry products A_b^T.dC_b, then the order-keeping chain
        G = tlcuda.matmul(A_r.transpose(-1, -2), dC, mode=mode)
        return dA, chained_batch_sum(G, group=group)
    _, dB = tlcuda.matmul_backward(dC, A_r, B, mode=mode, need_a=False)  # local sum_to
    dist.all_reduce(dB, group=group)
    return dA, dB


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
