"""The output-channel-sharded SpMM fused with its all-gather
(pfrt_spmm_allgather) and the all-gather alone (pfrt_peer_allgather).
M = 1: every rank's kernel sends each value of its rows of Y to every other
rank over NVLink, marked with the call's number, and unpacks the values it
receives into its own gathered output.  M > 1: every rank computes its column
block of Y into its own output and one kernel stores the block into every
other rank's output (or, opt-in, the dense path's GEMM epilogue does).  The gathered Y must match pruning::sparse_matmul
(src/pruning/sparse_tensor.cpp:473-519) on the whole W, normwise <= 1e-5, on
every rank, call after call (the call counter lives on the device), with M
changing between calls, and inside CUDA graph replays.

World 1 runs on one GPU (the rank's own buffers only), as does the timeout
test (its peer is a local buffer nobody writes); worlds 2, 4 and 8 need that
many GPUs and are skipped with fewer."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

from tests.helpers import FP32_TOL, normwise_rel

pytestmark = pytest.mark.gpu


def _case(M=1, seed=5, N=3001, K=2048, sparsity=0.9):
    from pyflamert_b200 import workloads as wl
    return wl.spmm_case(M, N, K, sparsity=sparsity, seed=seed)


def _ref_rows(c, X, rows):
    from oracle import pyoracle as po
    return po.spmm_linear(c.indptr, c.indices, c.values, X[rows], c.N)


def _sample(M):
    return np.unique(np.r_[0:3, M // 2, M - 3:M].clip(0, M - 1))


def _check_calls(sh, c, rng, Ms=(1,), graph=True):
    """Eager calls with fresh X for each M in Ms (in order, twice), then a
    captured call of the largest M replayed with X changed in place between
    replays.  Rows of the output are sampled for M > 64.  Returns the worst
    normwise error."""
    worst = 0.0
    for M in list(Ms) * 2:
        X = rng.standard_normal((M, c.K)).astype(np.float32)
        y = sh(torch.from_numpy(X).cuda()).cpu().numpy()
        rows = _sample(M) if M > 64 else np.arange(M)
        worst = max(worst, normwise_rel(y[rows], _ref_rows(c, X, rows)))
    if graph:
        M = max(Ms)
        xg = torch.zeros((M, c.K), dtype=torch.float32, device="cuda")
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
            X = rng.standard_normal((M, c.K)).astype(np.float32)
            xg.copy_(torch.from_numpy(X))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            y = sh.output(M).cpu().numpy()
            rows = _sample(M) if M > 64 else np.arange(M)
            worst = max(worst, normwise_rel(y[rows], _ref_rows(c, X, rows)))
        del g
    return worst


def test_world1_self_gather(ctx):
    from pyflamert_b200 import sharding
    c = _case()
    sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, 0, 1, max_m=40)
    try:
        assert _check_calls(sh, c, np.random.default_rng(1), Ms=(1, 5, 40)) <= FP32_TOL
        ctx.check()
    finally:
        sh.close()


@pytest.mark.parametrize("M", [1, 64, 1024, 8192])
def test_world1_config5(ctx, M):
    """Config 5's weight (8192 x 8192, 90 % sparse) at every batch size of its
    sweep through the sharded entry at world 1."""
    from pyflamert_b200 import sharding
    c = _case(M, seed=51, N=8192, K=8192)
    sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, 0, 1, max_m=M)
    try:
        y = sh(torch.from_numpy(c.X).cuda()).cpu().numpy()
        ctx.check()
        rows = _sample(M)
        assert normwise_rel(y[rows], _ref_rows(c, c.X, rows)) <= FP32_TOL
        assert np.isfinite(y).all()
    finally:
        sh.close()


def test_world1_rejects_rows_beyond_max_m(ctx):
    import pyflamert_b200 as pf
    from pyflamert_b200 import sharding
    c = _case(N=64, K=32)
    sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, 0, 1, max_m=2)
    try:
        x = torch.zeros((3, c.K), dtype=torch.float32, device="cuda")
        st = pf.lib().pfrt_spmm_allgather(ctx.handle, sh.local._h, 3, x.data_ptr(), c.K, C.byref(sh.peers),
                                          pf._stream(None))
        assert st == 1  # PFRT_ERR_INVALID_ARGUMENT
        assert "max_m" in pf._abi.last_error()
    finally:
        sh.close()


@pytest.mark.parametrize("M", [1, 8])
def test_timeout_reported_then_reset(ctx, M):
    """A world-2 peer set whose rank 1 is a set of local buffers nobody writes:
    the call's bounded wait runs out (limit shortened through
    PFRT_PEER_WAIT_MS), pfrt_ctx_check reports PFRT_ERR_DEVICE_TIMEOUT, the
    next call reports it at once, and after pfrt_peer_reset the same state
    serves a world-1 call that matches the oracle.  All memory is local to
    this GPU; every wait is bounded."""
    import pyflamert_b200 as pf
    from pyflamert_b200 import _abi, sharding
    c = _case(M, seed=8, N=512, K=256)
    sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, 0, 1, max_m=8)
    ns = sh.ns
    fake = {k: torch.zeros(n, dtype=torch.int64, device="cuda")
            for k, n in (("recv", 2 * 2 * ns), ("y", 8 * 2 * ns), ("sig", _abi.PFRT_PEER_SIG_WORDS))}
    mine = {k: torch.zeros(n, dtype=torch.int64, device="cuda")
            for k, n in (("recv", 2 * 2 * ns), ("y", 8 * 2 * ns), ("sig", _abi.PFRT_PEER_SIG_WORDS))}
    ps = _abi.PeerSet()
    ps.rank, ps.world, ps.ns, ps.max_m = 0, 2, ns, 8
    ps.y = mine["y"].data_ptr()
    ps.state = sh.peers.state
    ps.recv[0], ps.recv[1] = mine["recv"].data_ptr(), fake["recv"].data_ptr()
    ps.y_peer[0], ps.y_peer[1] = mine["y"].data_ptr(), fake["y"].data_ptr()
    ps.sig[0], ps.sig[1] = mine["sig"].data_ptr(), fake["sig"].data_ptr()
    old = os.environ.get("PFRT_PEER_WAIT_MS")
    os.environ["PFRT_PEER_WAIT_MS"] = "200"
    try:
        x = torch.from_numpy(c.X).cuda()
        for _ in range(2):  # the second call gives up at once (the abort word is set)
            st = pf.lib().pfrt_spmm_allgather(ctx.handle, sh.local._h, M, x.data_ptr(), c.K, C.byref(ps),
                                              pf._stream(None))
            assert st == 0
            with pytest.raises(pf.PfrtError) as ei:
                ctx.check()
            assert ei.value.status == 6  # PFRT_ERR_DEVICE_TIMEOUT
        # the kernel did reach its (fake) peer: values tagged with calls 1 and 2
        # (M = 1, receive halves by parity), or its "free for call 2" word (M > 1)
        if M == 1:
            tags = fake["recv"].cpu().numpy().view(np.uint64) >> np.uint64(32)
            assert (tags[2 * ns:3 * ns] == 1).all() and (tags[0:ns] == 2).all()
        else:
            assert int(fake["sig"].cpu().numpy().view(np.uint32)[0]) == 2
        sh.reset()
        ctx.check()
        y = sh(x).cpu().numpy()
        ctx.check()
        assert normwise_rel(y, _ref_rows(c, c.X, np.arange(M))) <= FP32_TOL
    finally:
        if old is None:
            os.environ.pop("PFRT_PEER_WAIT_MS", None)
        else:
            os.environ["PFRT_PEER_WAIT_MS"] = old
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
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        ctx = pf.Context(rank)
        worst = 0.0
        # a ragged shape (the last shard padded with empty rows), every M
        c = _case(seed=9, N=4099, K=4096)
        sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, rank, world, max_m=70)
        worst = max(worst, _check_calls(sh, c, np.random.default_rng(7), Ms=(1, 3, 70)))  # same X on every rank
        ctx.check()
        # the all-gather alone: every rank writes its own block, then gathers
        y = sh.output(5)
        full = torch.arange(5 * sh.world * sh.ns, dtype=torch.float32, device="cuda").reshape(5, -1)
        blk = slice(rank * sh.ns, (rank + 1) * sh.ns)
        raw = torch.as_tensor(sharding._DeviceArray(sh._y_ptr, (sh.max_m, sh.world * sh.ns), "<f4"), device="cuda")
        raw[:5, blk].copy_(full[:, blk])
        torch.cuda.synchronize()
        sh.allgather(5)
        ctx.check()
        ok_gather = bool(torch.equal(raw[:5], full))
        sh.close()
        # config 5's weight at every M of its sweep
        c = _case(8192, seed=51, N=8192, K=8192)
        sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, rank, world, max_m=8192)
        for M in (1, 64, 1024, 8192):
            X = c.X[:M]
            yv = sh(torch.from_numpy(X).cuda()).cpu().numpy()
            rows = _sample(M)
            worst = max(worst, normwise_rel(yv[rows], _ref_rows(c, X, rows)))
        ctx.check()
        # the opt-in fused form: the dense path's GEMM epilogue stores the
        # block into every rank's output (PFRT_PEER_FUSE=1 on every rank)
        os.environ["PFRT_PEER_FUSE"] = "1"
        X = c.X[:1024]
        yv = sh(torch.from_numpy(X).cuda()).cpu().numpy()
        os.environ.pop("PFRT_PEER_FUSE")
        rows = _sample(1024)
        worst = max(worst, normwise_rel(yv[rows], _ref_rows(c, X, rows)))
        ctx.check()
        dist.barrier()
        sh.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, worst, ok_gather, None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
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
        r, worst, ok_gather, err = q.get(timeout=600)
        res[r] = (worst, ok_gather, err)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        worst, ok_gather, err = res[r]
        assert err is None, err
        assert worst <= FP32_TOL
        assert ok_gather
