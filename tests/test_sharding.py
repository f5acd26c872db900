"""Host-side multi-GPU logic on CPU: the CSR row shards, the all-gather of the
per-rank output blocks and their assembly into Y, run as two gloo ranks.
The per-rank SpMM is the oracle here (no GPU in this test); on the GPU the
same shards go through pfrt_spmm (bench.py, N > 1)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from pyflamert_b200 import sharding, workloads as wl


def test_batch_slices_cover_rows():
    for M in (1, 7, 512, 8192):
        for world in (1, 2, 3, 8):
            sl = [sharding.batch_slice(M, r, world) for r in range(world)]
            assert sl[0][0] == 0 and sl[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_csr_row_shards_reassemble(world):
    from oracle import pyoracle as po
    c = wl.spmm_case(5, 101, 80, sparsity=0.8, seed=world)
    ref = po.spmm_linear(c.indptr, c.indices, c.values, c.X, c.N)
    blocks = []
    for r in range(world):
        n0, nreal, ip, ix, v = sharding.csr_row_shard(c.indptr, c.indices, c.values, r, world)
        ns = ip.size - 1
        assert ns == -(-c.N // world)
        blocks.append(po.spmm_linear(ip, ix, v, c.X, ns))
    y = sharding.assemble_columns(np.stack(blocks), 5, c.N, world)
    np.testing.assert_array_equal(y, ref)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q):
    import torch
    import torch.distributed as dist

    from oracle import pyoracle as po
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = wl.spmm_case(6, 203, 150, sparsity=0.9, seed=11)
        n0, nreal, ip, ix, v = sharding.csr_row_shard(c.indptr, c.indices, c.values, rank, world)
        local = torch.from_numpy(po.spmm_linear(ip, ix, v, c.X, ip.size - 1))
        gathered = torch.empty(world * local.numel(), dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, local.reshape(-1))
        y = sharding.assemble_columns(gathered, 6, c.N, world).contiguous().numpy()
        ref = po.spmm_linear(c.indptr, c.indices, c.values, c.X, c.N)
        result_q.put((rank, bool(np.array_equal(y, ref))))
    finally:
        dist.destroy_process_group()


def test_nshard_allgather_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
