"""Magnitude pruning into a CSR weight on the GPU
(pfrt_csr_from_magnitude_pruning) vs the reference's
MagnitudePruning::compute_mask (src/pruning/magnitude_pruning.cpp:22-102) and
to_sparse(W*mask) (src/pruning/sparse_tensor.cpp:560-587), through the
oracle's restatement (itself pinned to the compiled reference on CPU).
The mask and the CSR must be identical."""
import numpy as np
import pytest
import torch

import pyflamert_b200 as pf
from oracle import pyoracle as po
from tests.helpers import FP32_TOL, normwise_rel

pytestmark = pytest.mark.gpu


def weights(kind, shape, seed):
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return rng.standard_normal(shape).astype(np.float32)
    if kind == "ties":
        return (rng.integers(-3, 4, shape) / 4).astype(np.float32)
    if kind == "zeros":
        return np.where(rng.random(shape) < 0.5, 0.0, rng.standard_normal(shape)).astype(np.float32)
    return np.full(shape, -0.5, np.float32)


def prune(ctx, w, sparsity):
    wd = torch.from_numpy(w).cuda()
    mask = torch.full(w.shape, 7.0, dtype=torch.float32, device="cuda")
    csr = pf.CSR.from_magnitude_pruning(ctx, wd, sparsity, mask=mask)
    ctx.check()
    return csr, mask.cpu().numpy()


def dense_of(ctx, csr):
    """The CSR's matrix, read back exactly: Y = I W^T has one product per
    output when the CSR kernels (fp32 FMAs) compute it, not the 3xTF32 path."""
    import os
    old = {k: os.environ.get(k) for k in ("PFRT_SPMM_DENSE", "PFRT_SPMM_TILED")}
    os.environ["PFRT_SPMM_DENSE"], os.environ["PFRT_SPMM_TILED"] = "0", "1"
    try:
        eye = torch.eye(csr.K, dtype=torch.float32, device="cuda")
        y = csr(eye).cpu().numpy()  # [K, N] = W^T
        ctx.check()
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return y.T


@pytest.mark.parametrize("kind", ["normal", "ties", "zeros", "equal"])
@pytest.mark.parametrize("sparsity", [-0.1, 0.0, 0.3, 0.9, 0.95, 0.999, 1.0])
def test_mask_and_csr_match_reference(ctx, kind, sparsity):
    w = weights(kind, (97, 131), hash((kind, sparsity)) % 2**32)
    csr, mask = prune(ctx, w, sparsity)
    ref_mask = po.magnitude_mask(w, sparsity)
    np.testing.assert_array_equal(mask, ref_mask)
    ip, ix, v = po.masked_csr(w, ref_mask)
    assert csr.nnz == ip[-1]
    np.testing.assert_array_equal(dense_of(ctx, csr), w * ref_mask)


@pytest.mark.parametrize("shape,sparsity", [((1024, 1024), 0.9), ((4096, 4097), 0.9), ((3000, 777), 0.5)])
def test_large_weights(ctx, shape, sparsity):
    """Sizes past 2^24 elements, where the reference's float product
    (size_t)(n * sparsity) differs from the exact count."""
    w = weights("normal", shape, shape[0])
    csr, mask = prune(ctx, w, sparsity)
    ref_mask = po.magnitude_mask(w, sparsity)
    np.testing.assert_array_equal(mask, ref_mask)
    ip, ix, v = po.masked_csr(w, ref_mask)
    assert csr.nnz == ip[-1]
    X = np.random.default_rng(1).standard_normal((8, shape[1])).astype(np.float32)
    y = csr(torch.from_numpy(X).cuda()).cpu().numpy()
    assert normwise_rel(y, po.spmm_linear(ip, ix, v, X, shape[0])) <= FP32_TOL


def test_rejects_nan_and_empty(ctx):
    w = np.ones((4, 4), np.float32)
    w[2, 3] = np.nan
    with pytest.raises(pf.PfrtError, match="NaN"):
        pf.CSR.from_magnitude_pruning(ctx, torch.from_numpy(w).cuda(), 0.5)
    with pytest.raises(pf.PfrtError, match="empty"):
        pf.CSR.from_magnitude_pruning(ctx, torch.zeros((0, 4), device="cuda"), 0.5)
    ctx.check()


@pytest.mark.parametrize("kind", ["normal", "ties", "zeros", "equal"])
@pytest.mark.parametrize("n,m", [(2, 4), (1, 2), (3, 4), (4, 8), (5, 16), (16, 32), (4, 4)])
@pytest.mark.parametrize("shape", [(64, 96), (37, 53)])
def test_nm_mask_and_csr_match_reference(ctx, kind, n, m, shape):
    """N:M pruning on the GPU (pfrt_csr_from_nm_pruning) vs the reference's
    NMSparsityPruning::compute_mask (nm_sparsity.cpp:45-126) through the
    oracle's restatement: identical mask (groups span rows at K = 53, and the
    last group is short), identical CSR of W * mask."""
    w = weights(kind, shape, hash((kind, n, m, shape)) % 2**32)
    wd = torch.from_numpy(w).cuda()
    mask = torch.full(w.shape, 7.0, dtype=torch.float32, device="cuda")
    csr = pf.CSR.from_nm_pruning(ctx, wd, n, m, mask=mask)
    ctx.check()
    ref_mask = po.nm_mask(w, n, m)
    np.testing.assert_array_equal(mask.cpu().numpy(), ref_mask)
    ip, ix, v = po.masked_csr(w, ref_mask)
    assert csr.nnz == ip[-1]
    np.testing.assert_array_equal(dense_of(ctx, csr), w * ref_mask)


def test_nm_rejects_bad_n_m(ctx):
    wd = torch.ones((4, 8), device="cuda")
    with pytest.raises(pf.PfrtError, match="N must be <= M"):
        pf.CSR.from_nm_pruning(ctx, wd, 5, 4)
    with pytest.raises(pf.PfrtError, match="N and M must be > 0"):
        pf.CSR.from_nm_pruning(ctx, wd, 0, 4)
    with pytest.raises(pf.PfrtError, match="above 32"):
        pf.CSR.from_nm_pruning(ctx, wd, 2, 64)
    ctx.check()
