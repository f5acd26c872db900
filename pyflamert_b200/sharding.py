"""Work partitioning across the GPUs of one node (one process per GPU).

Two schemes, as the path needs them:

* batch sharding -- every rank holds the weights and processes a contiguous
  slice of the batch (M) rows.  No data-path collective: the quantized linear
  layer, the fp32 Gemm and the SpMM all shard this way (weak scaling).
* output-column sharding of a sparse weight -- W [N, K] is split by CSR rows
  (output channels) into equal shards of ceil(N / world) rows (the last one
  padded with empty rows), every rank computes Y[:, its columns] for the full
  batch, and one all-gather (NCCL over NVLink) assembles Y [M, N].  This is
  for weights too large to replicate.

The reference has no communication backend: its partitioner
(src/partition/graph_partitioner.cpp:111-200) only plans CommOps and runs the
partitions one after another on the CPU.
"""
from __future__ import annotations

import numpy as np


def batch_slice(M: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous rows [m0, m1) of an M-row batch for `rank`."""
    return M * rank // world, M * (rank + 1) // world


def csr_row_shard(indptr, indices, values, rank: int, world: int):
    """Rows [n0, n0 + ns) of a CSR matrix, padded with empty rows to ns =
    ceil(N / world) so that every rank's output block has the same size.
    Returns (n0, n_real, indptr_s, indices_s, values_s) with indptr rebased to 0."""
    indptr = np.asarray(indptr)
    N = indptr.size - 1
    ns = -(-N // world)
    n0 = min(N, rank * ns)
    n1 = min(N, n0 + ns)
    lo, hi = int(indptr[n0]), int(indptr[n1])
    ip = np.empty(ns + 1, dtype=indptr.dtype)
    ip[: n1 - n0 + 1] = indptr[n0:n1 + 1] - lo
    ip[n1 - n0 + 1:] = hi - lo
    return n0, n1 - n0, ip, np.asarray(indices)[lo:hi], np.asarray(values)[lo:hi]


def assemble_columns(gathered, M: int, N: int, world: int):
    """[world, M, ns] blocks (rank-major, as all_gather_into_tensor returns them)
    -> Y [M, N]: rank r's block holds columns [r*ns, r*ns + ns)."""
    ns = -(-N // world)
    g = gathered.reshape(world, M, ns)
    if hasattr(g, "permute"):
        y = g.permute(1, 0, 2).reshape(M, world * ns)
    else:
        y = np.transpose(g, (1, 0, 2)).reshape(M, world * ns)
    return y[:, :N]


class NShardSpMM:
    """Y [M, N] = X [M, K] W^T with W's rows (output channels) sharded over the
    ranks of the default process group; X is replicated."""

    def __init__(self, ctx, N: int, K: int, indptr, indices, values, rank: int, world: int):
        from . import CSR
        self.N, self.K, self.rank, self.world = int(N), int(K), rank, world
        self.ns = -(-self.N // world)
        n0, nreal, ip, ix, v = csr_row_shard(indptr, indices, values, rank, world)
        self.n0, self.nreal = n0, nreal
        self.local = CSR(ctx, self.ns, self.K, ip, ix, v)

    def __call__(self, x, out=None, gather_buf=None, local_buf=None):
        import torch
        import torch.distributed as dist
        M = x.shape[0]
        if local_buf is None:
            local_buf = torch.empty((M, self.ns), dtype=torch.float32, device=x.device)
        self.local(x, y=local_buf)
        if gather_buf is None:
            gather_buf = torch.empty((self.world * M * self.ns,), dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(gather_buf, local_buf.reshape(-1))
        y = assemble_columns(gather_buf, M, self.N, self.world)
        if out is not None:
            out.copy_(y)
            return out
        return y.contiguous()
