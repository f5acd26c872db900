"""The output-channel-sharded SpMM fused with its all-gather
(pfrt_spmm_allgather): every rank's kernel sends each value of its rows of Y
to every other rank over NVLink, marked with the call's number, and unpacks
the values it receives into its own gathered output.  The
gathered Y must match pruning::sparse_matmul (src/pruning/sparse_tensor.cpp:
473-519) on the whole W, normwise <= 1e-5, on every rank, call after call
(the call counter lives on the device) and inside CUDA graph replays.

World 1 runs on one GPU (the rank's own buffers only); worlds 2 and 4
need that many GPUs and are skipped with fewer."""
import os
import socket

import numpy as np
import pytest
import torch

from tests.helpers import FP32_TOL, normwise_rel

pytestmark = pytest.mark.gpu


def _case(seed=5, N=3001, K=2048, sparsity=0.9):
    from pyflamert_b200 import workloads as wl
    return wl.spmm_case(1, N, K, sparsity=sparsity, seed=seed)


def _check_calls(sh, c, rng, graph=True):
    """Three eager calls with fresh X, then a captured call replayed with X
    changed in place between replays.  Returns the worst normwise error."""
    from oracle import pyoracle as po
    worst = 0.0
    for _ in range(3):
        X = rng.standard_normal((1, c.K)).astype(np.float32)
        y = sh(torch.from_numpy(X).cuda()).cpu().numpy()
        worst = max(worst, normwise_rel(y, po.spmm_linear(c.indptr, c.indices, c.values, X, c.N)))
    if graph:
        xg = torch.zeros((1, c.K), dtype=torch.float32, device="cuda")
        sh(xg)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                sh(xg, stream=s)
        torch.cuda.synchronize()
        for _ in range(3):
            X = rng.standard_normal((1, c.K)).astype(np.float32)
            xg.copy_(torch.from_numpy(X))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            y = sh.output().cpu().numpy()
            worst = max(worst, normwise_rel(y, po.spmm_linear(c.indptr, c.indices, c.values, X, c.N)))
        del g
    return worst


def test_world1_self_gather(ctx):
    from pyflamert_b200 import sharding
    c = _case()
    sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, 0, 1)
    try:
        assert _check_calls(sh, c, np.random.default_rng(1)) <= FP32_TOL
        ctx.check()
    finally:
        sh.close()


def test_world1_rejects_batches(ctx):
    import pyflamert_b200 as pf
    from pyflamert_b200 import sharding
    c = _case(N=64, K=32)
    sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, 0, 1)
    try:
        import ctypes as C
        x = torch.zeros((2, c.K), dtype=torch.float32, device="cuda")
        st = pf.lib().pfrt_spmm_allgather(ctx.handle, sh.local._h, 2, x.data_ptr(), c.K, C.byref(sh.peers), None)
        assert st == 5  # PFRT_ERR_UNSUPPORTED
    finally:
        sh.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    try:
        import torch.distributed as dist

        import pyflamert_b200 as pf
        from pyflamert_b200 import sharding
        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        ctx = pf.Context(rank)
        c = _case(seed=9, N=4099, K=4096)
        sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, rank, world)
        worst = _check_calls(sh, c, np.random.default_rng(7))  # same X sequence on every rank
        ctx.check()
        dist.barrier()
        sh.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, worst, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_world_n_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, worst, err = q.get(timeout=300)
        res[r] = (worst, err)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        worst, err = res[r]
        assert err is None, err
        assert worst <= FP32_TOL
