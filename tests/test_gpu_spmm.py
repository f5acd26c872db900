"""CSR SpMM on the GPU vs pruning::sparse_matmul
(src/pruning/sparse_tensor.cpp:473-519) in the pruned-Linear orientation
Y = X W^T.  Summation order differs, so parity is normwise <= 1e-5."""
import numpy as np
import pytest
import torch

import pyflamert_b200 as pf
from oracle import pyoracle as po
from pyflamert_b200 import workloads as wl
from tests.golden import cases as gcases
from tests.helpers import FP32_TOL, normwise_rel

pytestmark = pytest.mark.gpu


def gpu(ctx, c: wl.CsrCase, X=None):
    X = c.X if X is None else X
    w = pf.CSR(ctx, c.N, c.K, c.indptr, c.indices, c.values)
    y = w(torch.from_numpy(np.ascontiguousarray(X)).cuda())
    ctx.check()
    return y.cpu().numpy()


def oracle(c: wl.CsrCase, X=None):
    X = c.X if X is None else X
    return po.spmm_linear(c.indptr, c.indices, c.values, X, c.N)


@pytest.mark.parametrize("name", [n for n, c in gcases.all_cases().items() if c["kind"] == "spmm"])
def test_golden(ctx, golden, name):
    case = gcases.all_cases()[name]
    c = case["case"]
    rows = case.get("rows", c.X.shape[0])
    y = gpu(ctx, c, c.X[:rows])
    assert normwise_rel(y, golden[0][name]) <= FP32_TOL


def test_config3_full(ctx):
    c = wl.spmm_case()
    y = gpu(ctx, c)
    ref = oracle(c)
    assert normwise_rel(y, ref) <= FP32_TOL
    f64 = po.spmm_linear_f64(c.indptr, c.indices, c.values, c.X, c.N)
    assert normwise_rel(y, f64) <= 2 * normwise_rel(ref, f64) + 1e-6


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 31, 64, 130])
def test_batch_sizes(ctx, M):
    c = wl.spmm_case(M, 300, 700, sparsity=0.9, seed=M)
    assert normwise_rel(gpu(ctx, c), oracle(c)) <= FP32_TOL


@pytest.mark.parametrize("sparsity", [0.5, 0.7, 0.9, 0.95])
@pytest.mark.parametrize("M", [1, 64, 1024, 8192])
def test_config5_sweep(ctx, sparsity, M):
    """Config 5 weights (8192 x 8192); the oracle checks 8 rows of the output."""
    c = wl.spmm_case(M, 8192, 8192, sparsity=sparsity, seed=50 + int(sparsity * 100))
    y = gpu(ctx, c)
    rows = np.unique(np.r_[0:4, M - 4:M].clip(0, M - 1))
    ref = oracle(c, c.X[rows])
    assert normwise_rel(y[rows], ref) <= FP32_TOL
    assert np.isfinite(y).all()


def test_empty_rows_and_unaligned_starts(ctx):
    rng = np.random.default_rng(5)
    N, K, M = 97, 211, 6
    counts = rng.integers(0, 9, N)
    counts[::7] = 0
    indptr = np.zeros(N + 1, np.int64)
    indptr[1:] = np.cumsum(counts)
    indices = np.concatenate([np.sort(rng.choice(K, k, replace=False)) for k in counts]).astype(np.int64)
    values = rng.standard_normal(indices.size).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    c = wl.CsrCase(N, K, indptr.astype(np.int32), indices.astype(np.int32), values, X)
    y = gpu(ctx, c)
    assert normwise_rel(y, oracle(c)) <= FP32_TOL
    np.testing.assert_array_equal(y[:, counts == 0], 0.0)


def test_no_nonzeros(ctx):
    c = wl.CsrCase(5, 8, np.zeros(6, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32),
                   np.ones((3, 8), np.float32))
    np.testing.assert_array_equal(gpu(ctx, c), np.zeros((3, 5), np.float32))


def test_bad_csr_rejected_on_upload(ctx):
    with pytest.raises(pf.PfrtError, match="out of range"):
        pf.CSR(ctx, 2, 4, np.array([0, 1, 2], np.int32), np.array([0, 4], np.int32), np.ones(2, np.float32))
    with pytest.raises(pf.PfrtError, match="indptr"):
        pf.CSR(ctx, 2, 4, np.array([0, 2, 1], np.int32), np.array([0, 1], np.int32), np.ones(2, np.float32))


def test_raw_api_bad_index_is_skipped_and_reported(ctx):
    """A caller-owned device CSR with an index >= K: the kernel skips it (no
    out-of-bounds read) and pfrt_ctx_check reports PFRT_ERR_BAD_CSR."""
    indptr = torch.tensor([0, 2, 4], dtype=torch.int32, device="cuda")
    indices = torch.tensor([0, 3, 1, 99], dtype=torch.int32, device="cuda")
    values = torch.tensor([1.0, 2.0, 3.0, 4.0], dtype=torch.float32, device="cuda")
    x = torch.arange(8, dtype=torch.float32, device="cuda").reshape(2, 4)
    y = ctx.spmm_csr_raw(2, 2, 4, 4, indptr, indices, values, x)
    with pytest.raises(pf.PfrtError) as ei:
        ctx.check()
    assert ei.value.status == 2
    yy = y.cpu().numpy()
    np.testing.assert_array_equal(yy[:, 0], x.cpu().numpy() @ np.array([1, 0, 0, 2], np.float32))
    np.testing.assert_array_equal(yy[:, 1], x.cpu().numpy()[:, 1] * 3.0)
    ctx.check()  # the error was cleared


@pytest.mark.parametrize("M", [9, 40, 200])
def test_raw_api_wide_kernel(ctx, M):
    """Caller-owned device CSR with M > 8 (the transposed-X wide kernel)."""
    c = wl.spmm_case(M, 333, 517, sparsity=0.85, seed=70 + M)
    y = ctx.spmm_csr_raw(M, c.N, c.K, c.values.size, torch.from_numpy(c.indptr).cuda(),
                         torch.from_numpy(c.indices).cuda(), torch.from_numpy(c.values).cuda(),
                         torch.from_numpy(c.X).cuda())
    ctx.check()
    assert normwise_rel(y.cpu().numpy(), oracle(c)) <= FP32_TOL


@pytest.mark.parametrize("M,N,K", [(65, 100, 257), (130, 1000, 700), (64, 8, 4096), (256, 4096, 4096)])
def test_tiled_kernel(ctx, M, N, K, monkeypatch):
    """The shared-memory tiled kernel, including its tails: M not a multiple of
    64, N not a multiple of the rows per block, K not a multiple of 256."""
    monkeypatch.setenv("PFRT_SPMM_TILED", "1")
    c = wl.spmm_case(M, N, K, sparsity=0.7 if M < 256 else 0.9, seed=M + N + K)
    assert normwise_rel(gpu(ctx, c), oracle(c)) <= FP32_TOL


@pytest.mark.parametrize("kernel", ["rowwarp", "stream"])
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_small_batch_kernels(ctx, kernel, M, monkeypatch):
    """Both small-batch kernels (one warp per row; the nnz-balanced streaming
    kernel) on rows of uneven length, including empty rows at the ends."""
    monkeypatch.setenv("PFRT_SPMM_ROWWARP" if kernel == "rowwarp" else "PFRT_SPMM_STREAM", "1")
    rng = np.random.default_rng(M)
    N, K = 1500, 900
    counts = rng.integers(0, 700, N)
    counts[:3] = 0
    counts[-5:] = 0
    counts[100:140] = 0
    indptr = np.zeros(N + 1, np.int64)
    indptr[1:] = np.cumsum(counts)
    indices = np.concatenate([np.sort(rng.choice(K, k, replace=False)) for k in counts]).astype(np.int32)
    values = rng.standard_normal(indices.size).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    c = wl.CsrCase(N, K, indptr.astype(np.int32), indices, values, X)
    y = gpu(ctx, c)
    assert normwise_rel(y, oracle(c)) <= FP32_TOL
    np.testing.assert_array_equal(y[:, counts == 0], 0.0)


@pytest.mark.parametrize("dense", ["0", "1"])
@pytest.mark.parametrize("M,N,K,sparsity", [(32, 300, 700, 0.9), (130, 1000, 333, 0.5),
                                            (512, 4096, 4096, 0.9), (1024, 2048, 8192, 0.97)])
def test_large_batch_dense_and_csr_paths(ctx, dense, M, N, K, sparsity, monkeypatch):
    """Batches above 8 rows take the tensor-core GEMM on a dense copy of W or
    the tiled CSR kernel, by a cost model (dense above ~6-7 % density at
    M <= 64, and at lower density as M grows); both the dense path and the
    CSR kernels, forced in turn, match the oracle, with tails in M, N and K."""
    monkeypatch.setenv("PFRT_SPMM_DENSE", dense)
    c = wl.spmm_case(M, N, K, sparsity=sparsity, seed=M + N + K)
    y = gpu(ctx, c)
    ref = oracle(c)
    assert normwise_rel(y, ref) <= FP32_TOL
    f64 = po.spmm_linear_f64(c.indptr, c.indices, c.values, c.X, c.N)
    assert normwise_rel(y, f64) <= 2 * normwise_rel(ref, f64) + 1e-6


@pytest.mark.parametrize("M,N,K,sparsity", [(9, 300, 700, 0.9), (64, 1000, 333, 0.5), (100, 129, 4100, 0.99),
                                            (256, 4096, 4096, 0.9), (300, 2048, 2048, 0.7)])
def test_tensor_core_kernel(ctx, M, N, K, sparsity, monkeypatch):
    """The tensor-core kernel on W's compressed form (W densified in TMEM),
    forced: tails in M (slabs of 64 rows of X), N (tiles of 128 rows of W)
    and K (k-blocks of 32), and the cost model's K split."""
    monkeypatch.setenv("PFRT_SPMM_TC", "1")
    c = wl.spmm_case(M, N, K, sparsity=sparsity, seed=M + N + K + 1)
    y = gpu(ctx, c)
    ref = oracle(c)
    assert normwise_rel(y, ref) <= FP32_TOL
    f64 = po.spmm_linear_f64(c.indptr, c.indices, c.values, c.X, c.N)
    assert normwise_rel(y, f64) <= 2 * normwise_rel(ref, f64) + 1e-6


@pytest.mark.parametrize("M,N,K", [(70, 333, 1000), (30, 100, 1000), (300, 4096, 1000), (200, 129, 4100)])
def test_tensor_core_kernel_schedules(ctx, M, N, K, monkeypatch):
    """The stream-K schedule over the SMs: fewer k-blocks than SMs (one
    k-block per CTA, every unit finished by the fix-up from up to 32
    partial tiles), CTA ranges longer than a unit (whole units in the
    middle, partial pieces at both ends) and shorter ones; rows of W without
    nonzeros give exact zeros."""
    monkeypatch.setenv("PFRT_SPMM_TC", "1")
    rng = np.random.default_rng(M + N + K)
    counts, indptr, indices, values = _ragged_csr(rng, N, K, 120)
    X = rng.standard_normal((M, K)).astype(np.float32)
    c = wl.CsrCase(N, K, indptr, indices, values, X)
    y = gpu(ctx, c)
    assert normwise_rel(y, oracle(c)) <= FP32_TOL
    np.testing.assert_array_equal(y[:, counts == 0], 0.0)


def test_tensor_core_kernel_duplicate_columns_fall_back(ctx, monkeypatch):
    """A CSR row that stores a column twice (the reference sums both) cannot
    use the compressed form; the call falls back to another path and still
    matches the oracle."""
    monkeypatch.setenv("PFRT_SPMM_TC", "1")
    rng = np.random.default_rng(3)
    N, K, M = 40, 96, 33
    indptr = np.arange(0, 4 * N + 1, 4, dtype=np.int32)
    indices = rng.integers(0, K, 4 * N).astype(np.int32)
    indices[1] = indices[0]  # row 0 stores one column twice
    values = rng.standard_normal(4 * N).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    c = wl.CsrCase(N, K, indptr, indices, values, X)
    assert normwise_rel(gpu(ctx, c), oracle(c)) <= FP32_TOL


def test_dense_path_reuses_copy_and_keeps_empty_rows_zero(ctx, monkeypatch):
    """The dense copy is built once per CSR and reused; rows of W with no
    nonzeros still give exact zeros."""
    monkeypatch.setenv("PFRT_SPMM_DENSE", "1")
    rng = np.random.default_rng(9)
    N, K, M = 257, 129, 96
    counts = rng.integers(0, 60, N)
    counts[::5] = 0
    indptr = np.zeros(N + 1, np.int64)
    indptr[1:] = np.cumsum(counts)
    indices = np.concatenate([np.sort(rng.choice(K, k, replace=False)) for k in counts]).astype(np.int32)
    values = rng.standard_normal(indices.size).astype(np.float32)
    w = pf.CSR(ctx, N, K, indptr.astype(np.int32), indices, values)
    for seed in (1, 2):
        X = np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)
        y = w(torch.from_numpy(X).cuda()).cpu().numpy()
        ctx.check()
        c = wl.CsrCase(N, K, indptr.astype(np.int32), indices, values, X)
        assert normwise_rel(y, oracle(c)) <= FP32_TOL
        np.testing.assert_array_equal(y[:, counts == 0], 0.0)


def _ragged_csr(rng, N, K, max_row, zero_every=7):
    counts = rng.integers(0, max_row, N)
    counts[::zero_every] = 0
    counts[1::11] = rng.integers(1, 4, counts[1::11].size)   # rows shorter than one 16-byte group
    counts[-3:] = 0
    indptr = np.zeros(N + 1, np.int64)
    indptr[1:] = np.cumsum(counts)
    indices = np.concatenate([np.sort(rng.choice(K, k, replace=False)) for k in counts]).astype(np.int32)
    values = rng.standard_normal(indices.size).astype(np.float32)
    return counts, indptr.astype(np.int32), indices, values


@pytest.mark.parametrize("K,x_offset", [(1001, 0), (1024, 1), (1024, 0)])
@pytest.mark.parametrize("bank_order", ["1", "0"])
def test_single_row_batch_kernel(ctx, K, x_offset, bank_order, monkeypatch):
    """M = 1 (the row kernel with X in shared memory): rows from empty to
    several load rounds long, X staged by 16-byte async copies (K % 4 == 0,
    X aligned) or element by element (odd K, or X at a 4-byte offset), and
    the CSR uploaded in bank order or in the caller's order."""
    monkeypatch.setenv("PFRT_CSR_BANK_ORDER", bank_order)
    rng = np.random.default_rng(K + x_offset)
    N = 2000
    counts, indptr, indices, values = _ragged_csr(rng, N, K, 1000)
    X = rng.standard_normal((1, K)).astype(np.float32)
    buf = torch.zeros(K + 4, dtype=torch.float32, device="cuda")
    buf[x_offset:x_offset + K] = torch.from_numpy(X[0]).cuda()
    x = buf[x_offset:x_offset + K].reshape(1, K)
    w = pf.CSR(ctx, N, K, indptr, indices, values)
    y = w(x).cpu().numpy()
    ctx.check()
    c = wl.CsrCase(N, K, indptr, indices, values, X)
    assert normwise_rel(y, oracle(c)) <= FP32_TOL
    np.testing.assert_array_equal(y[:, counts == 0], 0.0)


def test_bank_order_keeps_rows(ctx, monkeypatch):
    """Bank order only reorders entries inside rows: with every value a power
    of two and X integer-valued, each row sum is exact in any order, so the
    two uploads agree bit for bit (and with the oracle)."""
    rng = np.random.default_rng(3)
    N, K = 1500, 4096
    counts, indptr, indices, _ = _ragged_csr(rng, N, K, 900)
    values = (2.0 ** rng.integers(-4, 4, indices.size)).astype(np.float32)
    X = rng.integers(-8, 9, (1, K)).astype(np.float32)
    ys = []
    for flag in ("1", "0"):
        monkeypatch.setenv("PFRT_CSR_BANK_ORDER", flag)
        w = pf.CSR(ctx, N, K, indptr, indices, values)
        ys.append(w(torch.from_numpy(X).cuda()).cpu().numpy())
        ctx.check()
    np.testing.assert_array_equal(ys[0], ys[1])
    np.testing.assert_array_equal(ys[0], oracle(wl.CsrCase(N, K, indptr, indices, values, X)))


def test_raw_api_single_row_batch_bad_index(ctx):
    """Caller-owned CSR at M = 1 large enough for the shared-memory row
    kernel: an index >= K is skipped and reported, the other rows are exact
    against the oracle."""
    rng = np.random.default_rng(21)
    N, K = 3000, 512
    counts, indptr, indices, values = _ragged_csr(rng, N, K, 200)
    bad_row = int(np.argmax(counts))
    indices = indices.copy()
    indices[indptr[bad_row]] = K + 5
    X = rng.standard_normal((1, K)).astype(np.float32)
    y = ctx.spmm_csr_raw(1, N, K, indices.size, torch.from_numpy(indptr).cuda(), torch.from_numpy(indices).cuda(),
                         torch.from_numpy(values).cuda(), torch.from_numpy(X).cuda())
    with pytest.raises(pf.PfrtError) as ei:
        ctx.check()
    assert ei.value.status == 2
    keep = np.ones(indices.size, bool)
    keep[indptr[bad_row]] = False
    rows = np.repeat(np.arange(N), counts)
    W = np.zeros((N, K), np.float64)
    np.add.at(W, (rows[keep], indices[keep]), values[keep].astype(np.float64))
    ref = (X.astype(np.float64) @ W.T)
    assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("M,N,K", [(64, 256, 512), (200, 300, 1000), (16, 128, 128), (1024, 512, 1024),
                                   (130, 260, 1001), (64, 4096, 4096), (256, 4096, 4096)])
def test_structured_sparse_kernel(ctx, M, N, K, monkeypatch):
    """Weights with 2:4 structure along K on the structured-sparse tensor
    cores (tcgen05.mma.sp, bf16 x3 split, spmm_sp.cuh): normwise <= 1e-5
    against the reference's sparse_matmul, with N, K and M ragged (N not a
    multiple of 128, K not a multiple of 128 or of 4, M not a multiple of 64),
    groups holding two, one or no entries, and units shared between CTAs.
    Equal, within the same tolerance, to the other paths on the same weight."""
    c = wl.structured24_case(M, N, K, seed=M + N + K)
    monkeypatch.setenv("PFRT_SPMM_SP", "1")
    y = gpu(ctx, c)
    ref = oracle(c)
    assert normwise_rel(y, ref) <= FP32_TOL
    monkeypatch.setenv("PFRT_SPMM_SP", "0")
    assert normwise_rel(gpu(ctx, c), y) <= 2 * FP32_TOL


def test_structured_sparse_from_nm_pruning(ctx, monkeypatch):
    """The N:M pruning path end to end: a dense weight W [N, K] pruned 2:4 as
    NMSparsityPruning(2, 4).compute_mask does (groups of four consecutive
    weights of the row-major tensor; K % 4 == 0, so along K), kept as CSR,
    multiplied on the structured-sparse kernel, repeatedly and with M
    changing between calls."""
    rng = np.random.default_rng(11)
    N, K = 384, 768
    W = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.05)
    mask = po.nm_mask(W, 2, 4)
    indptr, indices, values = po.masked_csr(W, mask)
    monkeypatch.setenv("PFRT_SPMM_SP", "1")
    w = pf.CSR(ctx, N, K, indptr, indices, values)
    for M in (64, 33, 300, 64):
        X = rng.standard_normal((M, K), dtype=np.float32)
        y = w(torch.from_numpy(X).cuda()).cpu().numpy()
        ctx.check()
        assert normwise_rel(y, po.spmm_linear(indptr, indices, values, X, N)) <= FP32_TOL


@pytest.mark.parametrize("M,N,K,sparsity", [(96, 256, 512, 0.5), (64, 520, 1000, 0.9), (300, 4096, 4096, 0.9),
                                            (64, 8192, 8192, 0.95), (17, 130, 259, 0.7)])
def test_structured_sparse_with_remainder(ctx, M, N, K, sparsity, monkeypatch):
    """Unstructured weights on the structured-sparse kernel: W = W24 + R, the
    2:4 part on the tensor cores and the remainder R (entries past the second
    of their group of four) added in fp32 by its own kernel afterwards.
    Normwise <= 1e-5 against the reference."""
    monkeypatch.setenv("PFRT_SPMM_SP", "1")
    c = wl.spmm_case(M, N, K, sparsity=sparsity, seed=N + K)
    assert normwise_rel(gpu(ctx, c), oracle(c)) <= FP32_TOL


def test_structured_sparse_duplicate_columns(ctx, monkeypatch):
    """A column stored twice in a row is summed, as the reference's
    sparse_matmul sums it, also on the structured-sparse kernel."""
    monkeypatch.setenv("PFRT_SPMM_SP", "1")
    d = wl.structured24_case(96, 130, 256, seed=9)
    ip = d.indptr.astype(np.int64)
    idx = np.insert(d.indices, ip[0], d.indices[ip[0]])
    val = np.insert(d.values, ip[0], np.float32(0.5))
    ip = ip.copy()
    ip[1:] += 1
    dup = wl.CsrCase(d.N, d.K, ip.astype(np.int32), idx.astype(np.int32), val.astype(np.float32), d.X)
    assert normwise_rel(gpu(ctx, dup), oracle(dup)) <= FP32_TOL


@pytest.mark.parametrize("M,N,K,sparsity", [(64, 256, 512, None), (130, 260, 1001, None), (17, 130, 259, 0.7),
                                            (64, 520, 1000, 0.9), (300, 4096, 4096, 0.9), (64, 8192, 8192, 0.9),
                                            (1024, 512, 1024, 0.95), (33, 200, 640, 1.0)])
def test_structured_sparse_forms_agree(ctx, M, N, K, sparsity, monkeypatch):
    """The structured-sparse kernel reading W24 as prepared images and as the
    compressed form (per row metadata, slot mask and bf16 x3 values, expanded
    into shared memory and TMEM by the kernel's producer warps) gives the
    same bits: both put the same operands and metadata before the same MMAs.
    Cases: 2:4 weights (sparsity None, whose value runs overflow the
    kernel's slot, so the producers read global memory), unstructured ones
    with a remainder, ragged shapes, and a weight with no entries; the
    compressed result within 1e-5 normwise of the reference."""
    c = (wl.structured24_case(M, N, K, seed=M + N) if sparsity is None
         else wl.spmm_case(M, N, K, sparsity=sparsity, seed=N + K))
    monkeypatch.setenv("PFRT_SPMM_SP", "1")
    out = {}
    for form in ("image", "compressed"):
        monkeypatch.setenv("PFRT_SPMM_SP_FORM", form)
        out[form] = gpu(ctx, c)
    ref = oracle(c)
    if np.abs(ref).max() == 0:
        assert not out["compressed"].any() and not out["image"].any()
    else:
        assert normwise_rel(out["compressed"], ref) <= FP32_TOL
    assert np.array_equal(out["image"], out["compressed"])
