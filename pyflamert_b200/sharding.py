"""Work partitioning across the GPUs of one node (one process per GPU).

Two schemes, as the path needs them:

* batch sharding -- every rank holds the weights and processes a contiguous
  slice of the batch (M) rows.  No data-path collective: the quantized linear
  layer, the fp32 Gemm and the SpMM all shard this way (weak scaling).
* output-column sharding of a sparse weight -- W [N, K] is split by CSR rows
  (output channels) into equal shards of ceil(N / world) rows (the last one
  padded with empty rows), every rank computes Y[:, its columns] for the full
  batch, and one all-gather over NVLink assembles Y [M, N] on every rank.
  This is for weights too large to replicate.  FusedNShardSpMM is the product
  path (the all-gather done by the library's own kernels over peer memory);
  NShardSpMM does the same with NCCL's all_gather_into_tensor and stays as the
  library baseline.

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


class _DeviceArray:
    """A device buffer from pfrt_malloc, exposed to torch without a copy."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class FusedNShardSpMM:
    """Output-channel-sharded SpMM with the all-gather fused into the call
    (pfrt_spmm_allgather).  M = 1: each rank's kernel sends every value of its
    rows of Y to every other rank as it computes it, and unpacks the values it
    receives into its own gathered output.  M > 1 (up to `max_m`): each rank
    computes its column block of Y into its own gathered output, and one
    kernel stores the block into every other rank's output over NVLink.  The
    output, the receive buffer, the signal words and the state live in
    library-allocated device memory; the ranks exchange CUDA IPC handles of
    their output, receive buffer and signal words once, through the default
    process group (any backend: only host objects travel).  All ranks must
    construct the object together and then make the same calls."""

    def __init__(self, ctx, N: int, K: int, indptr, indices, values, rank: int, world: int, max_m: int = 1):
        import ctypes as C

        import torch.distributed as dist

        from . import CSR, _abi, lib
        if world > _abi.PFRT_MAX_PEERS:
            raise ValueError(f"at most {_abi.PFRT_MAX_PEERS} ranks")
        if max_m < 1:
            raise ValueError("max_m must be >= 1")
        self.ctx, self.N, self.K, self.rank, self.world = ctx, int(N), int(K), rank, world
        self.max_m = int(max_m)
        self.ns = -(-self.N // world)
        n0, nreal, ip, ix, v = csr_row_shard(indptr, indices, values, rank, world)
        self.local = CSR(ctx, self.ns, self.K, ip, ix, v)
        L = lib()
        self._own = []
        ptrs = {}
        sizes = (("y", 4 * self.max_m * world * self.ns), ("recv", 8 * 2 * world * self.ns), ("state", 16),
                 ("sig", 4 * _abi.PFRT_PEER_SIG_WORDS))
        for name, nbytes in sizes:
            p = C.c_void_p()
            _abi.check(L.pfrt_malloc(ctx.handle, max(nbytes, 16), C.byref(p)), "pfrt_malloc")
            self._own.append(p.value)
            _abi.check(L.pfrt_memset(ctx.handle, p, 0, max(nbytes, 16), None), "pfrt_memset")
            ptrs[name] = p.value
        _abi.check(L.pfrt_ctx_check(ctx.handle, None), "pfrt_ctx_check")  # zeroed before anyone sees them
        shared = ("recv", "y", "sig")
        mine = []
        for name in shared:
            h = _abi.IpcHandle()
            _abi.check(L.pfrt_ipc_get_handle(ctx.handle, C.c_void_p(ptrs[name]), C.byref(h)), "pfrt_ipc_get_handle")
            mine.append(bytes(h.bytes))
        allh = [None] * world
        if world > 1:
            dist.all_gather_object(allh, mine)
        else:
            allh = [mine]
        self._opened = []
        ps = _abi.PeerSet()
        ps.rank, ps.world = rank, world
        ps.y = ptrs["y"]
        ps.state = ptrs["state"]
        ps.ns, ps.max_m = self.ns, self.max_m
        for p in range(world):
            if p == rank:
                ps.recv[p], ps.y_peer[p], ps.sig[p] = ptrs["recv"], ptrs["y"], ptrs["sig"]
                continue
            mapped = []
            for i in range(len(shared)):
                hp = _abi.IpcHandle()
                C.memmove(hp.bytes, allh[p][i], 64)
                d = C.c_void_p()
                _abi.check(L.pfrt_ipc_open(ctx.handle, C.byref(hp), C.byref(d)), "pfrt_ipc_open")
                self._opened.append(d.value)
                mapped.append(d.value)
            ps.recv[p], ps.y_peer[p], ps.sig[p] = mapped
        self.peers = ps
        self._y_ptr = ptrs["y"]
        if world > 1:
            dist.barrier()  # every rank has mapped every other rank's buffers

    def output(self, M: int = 1):
        """This rank's gathered output Y [M, N] (a view of the library buffer)."""
        import torch
        y = torch.as_tensor(_DeviceArray(self._y_ptr, (self.max_m, self.world * self.ns), "<f4"), device="cuda")
        return y[:M, : self.N]

    def __call__(self, x, stream=None, csr=None):
        """Y [M, N] = X [M, K] W^T on every rank.  `csr` (optional) is another
        upload of this rank's shard (same rows), used instead of the own one
        (benchmarks rotate copies of the weight through the same buffers)."""
        import ctypes as C

        from . import _abi, _dptr, _stream, lib
        M = int(x.shape[0])
        if x.shape[1] != self.K or M < 1 or M > self.max_m:
            raise ValueError(f"FusedNShardSpMM: X must be [M <= {self.max_m}, {self.K}]")
        if x.stride(1) != 1:
            raise ValueError("FusedNShardSpMM: X rows must be contiguous")
        w = self.local if csr is None else csr
        _abi.check(lib().pfrt_spmm_allgather(self.ctx.handle, w._h, M, _dptr(x), x.stride(0),
                                             C.byref(self.peers), _stream(stream)), "pfrt_spmm_allgather")
        return self.output(M)

    def shard_copy(self, indptr, indices, values):
        """Another upload of this rank's shard of the same W (a CSR object
        for __call__'s `csr`)."""
        from . import CSR
        n0, nreal, ip, ix, v = csr_row_shard(indptr, indices, values, self.rank, self.world)
        return CSR(self.ctx, self.ns, self.K, ip, ix, v)

    def allgather(self, M: int, stream=None):
        """The all-gather alone (pfrt_peer_allgather): every rank has written
        its own column block of the first M rows of output(); afterwards every
        rank's output holds all blocks."""
        import ctypes as C

        from . import _abi, _stream, lib
        _abi.check(lib().pfrt_peer_allgather(self.ctx.handle, int(M), C.byref(self.peers), _stream(stream)),
                   "pfrt_peer_allgather")
        return self.output(M)

    def reset(self, stream=None):
        """pfrt_peer_reset: clears this rank's state after a timeout; every
        rank calls it and the ranks synchronize before the next call."""
        import ctypes as C

        from . import _abi, _stream, lib
        _abi.check(lib().pfrt_peer_reset(self.ctx.handle, C.byref(self.peers), _stream(stream)), "pfrt_peer_reset")

    def close(self):
        import ctypes as C

        from . import lib
        L = lib()
        for d in self._opened:
            L.pfrt_ipc_close(self.ctx.handle, C.c_void_p(d))
        self._opened = []
        for d in self._own:
            L.pfrt_free(self.ctx.handle, C.c_void_p(d))
        self._own = []
        self.local.close()
