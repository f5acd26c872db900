"""Pins the CPU oracle (oracle/oracle.c) to the PyFlameRT reference.

* the reference's own hot-path known-answer test (ExecutorTest.MatMul,
  tests/cpp/test_executor.cpp:162-208);
* the golden fixtures in tests/golden/golden_ref.npz, produced by the
  reference compiled from its own sources (tests/golden/make_golden.py);
* random cases run side by side through oracle/_ref when it is built.

All comparisons are bit-exact: the restatement follows the reference's
evaluation order, so fp32 results match to the last bit."""
import hashlib

import numpy as np
import pytest

from oracle import pyoracle as po
from pyflamert_b200 import workloads as wl
from tests.golden import cases as gcases

CASES = gcases.all_cases()


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            h.update(b"none")
        else:
            a = np.ascontiguousarray(a)
            h.update(str(a.dtype).encode() + str(a.shape).encode())
            h.update(a.tobytes())
    return h.hexdigest()


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint8) if a.dtype.itemsize == 1 else a.view(np.int32 if a.dtype.itemsize == 4 else np.int64)


def oracle_output(case):
    kind = case["kind"]
    if kind == "matmul":
        return po.matmul(case["A"], case["B"]), _sha(case["A"], case["B"])
    if kind == "gemm":
        g = case["case"]
        y = po.gemm(g.A, g.B, g.C, g.alpha, g.beta, g.trans_a, g.trans_b)
        return y[: case.get("rows", y.shape[0])], _sha(g.A, g.B, g.C)
    if kind in ("qmm_per_tensor", "qlinear_per_channel"):
        q = case["case"]
        rows = case.get("rows", q.a.shape[0])
        y = po.qlinear(q.a[:rows], q.a_scale, q.a_zp, q.w, q.w_scale, q.w_zp, bias=q.bias, relu=q.relu,
                       out=q.out, y_scale=q.y_scale, y_zp=q.y_zp)
        h = _sha(q.a, q.w, q.w_scale) if kind == "qmm_per_tensor" else _sha(q.a, q.w, q.w_scale, q.bias)
        return y, h
    if kind == "quantize":
        return po.quantize(case["x"], case["scale"], case["zp"], case["out"]), _sha(case["x"])
    if kind == "spmm":
        c = case["case"]
        rows = case.get("rows", c.X.shape[0])
        y = po.spmm_linear(c.indptr, c.indices, c.values, c.X[:rows], c.N)
        return y, _sha(c.indptr, c.indices, c.values, c.X)
    raise ValueError(kind)


def test_reference_known_answer_matmul():
    """ExecutorTest.MatMul: [[1,2,3],[4,5,6]] x [[1,2],[3,4],[5,6]] = [[22,28],[49,64]]."""
    case = CASES["kat_matmul"]
    y, _ = oracle_output(case)
    np.testing.assert_array_equal(y, np.array([[22, 28], [49, 64]], np.float32))


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_golden(name, golden):
    ys, shas = golden
    y, h = oracle_output(CASES[name])
    assert h == shas[name], f"{name}: input generator drifted from the fixture"
    ref = ys[name]
    assert y.shape == ref.shape and y.dtype == ref.dtype
    np.testing.assert_array_equal(_bits(y), _bits(ref))


needs_ref = pytest.mark.skipif(not po.ref_available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("seed", range(4))
def test_oracle_gemm_vs_reference_random(seed):
    rng = np.random.default_rng(100 + seed)
    M, N, K = rng.integers(1, 40, 3)
    ta, tb = int(rng.integers(0, 2)), int(rng.integers(0, 2))
    c_len = int(rng.choice([0, 1, N, M * N]))
    g = wl.gemm_case(M, N, K, seed=200 + seed, trans_a=ta, trans_b=tb, c_len=c_len,
                     alpha=float(rng.uniform(-2, 2)), beta=float(rng.uniform(-2, 2)))
    a = po.gemm(g.A, g.B, g.C, g.alpha, g.beta, ta, tb)
    b = po.ref_gemm(g.A, g.B, g.C, g.alpha, g.beta, ta, tb)
    np.testing.assert_array_equal(_bits(a), _bits(b))


@needs_ref
@pytest.mark.parametrize("out", ["f32", "int8", "uint8"])
@pytest.mark.parametrize("relu", [False, True])
def test_oracle_qlinear_per_channel_vs_reference(out, relu):
    q = wl.qlinear_case(10, 37, 75, seed=300, bias=True, relu=relu, out=out, y_scale=0.4, y_zp=5)
    a = po.qlinear(q.a, q.a_scale, q.a_zp, q.w, q.w_scale, bias=q.bias, relu=relu, out=out,
                   y_scale=q.y_scale, y_zp=q.y_zp)
    b = po.ref_qlinear_per_channel(q.a, q.a_scale, q.a_zp, q.w, q.w_scale, bias=q.bias, relu=relu,
                                   out=out, y_scale=q.y_scale, y_zp=q.y_zp)
    np.testing.assert_array_equal(_bits(a), _bits(b))


@needs_ref
def test_oracle_spmm_vs_reference_random():
    c = wl.spmm_case(11, 70, 130, sparsity=0.8, seed=400)
    a = po.spmm_linear(c.indptr, c.indices, c.values, c.X, c.N)
    b = po.ref_sparse_matmul(c.indptr, c.indices, c.values, np.ascontiguousarray(c.X.T)).T
    np.testing.assert_array_equal(_bits(a), _bits(np.ascontiguousarray(b)))


@needs_ref
def test_reference_graph_op_misreads_uint8():
    """The registered QuantizedMatMul op (quantized_ops.cpp:143-144) reads uint8
    as int8; the library quantized_matmul (the oracle) does not.  They agree
    for int8 x int8 and differ for uint8 activations >= 128."""
    q = wl.qlinear_case(6, 8, 32, seed=500, a_signed=True, out="f32")
    q.w_scale[:] = np.float32(0.01)
    op = po.ref_quantized_matmul_op(q.a, q.a_scale, 0, q.w, 0.01, 0)
    lib = po.ref_quantized_matmul(q.a, q.a_scale, 0, q.w, 0.01, 0, out="f32")
    np.testing.assert_array_equal(op, lib)
    q = wl.qlinear_case(6, 8, 32, seed=501, out="f32")
    op = po.ref_quantized_matmul_op(q.a, q.a_scale, 128, q.w, 0.01, 0)
    lib = po.ref_quantized_matmul(q.a, q.a_scale, 128, q.w, 0.01, 0, out="f32")
    assert not np.array_equal(op, lib)


def test_qmm_accumulators_exact_vs_float64_matmul():
    """The oracle's int64 accumulators equal an exact float64 product (all
    partial sums stay below 2**53)."""
    q = wl.qlinear_case(20, 30, 300, seed=600)
    acc = po.qmm_acc(q.a, q.w, q.a_zp)
    ref = (q.a.astype(np.float64) - q.a_zp) @ q.w.astype(np.float64)
    np.testing.assert_array_equal(acc, ref.astype(np.int64))


@pytest.mark.skipif(not po.ref_available(), reason="compiled reference not built")
@pytest.mark.parametrize("kind", ["normal", "ties", "zeros", "equal"])
@pytest.mark.parametrize("sparsity", [-0.1, 0.0, 0.3, 0.5, 0.9, 0.95, 0.999, 1.0])
def test_magnitude_mask_matches_reference(kind, sparsity):
    """The restated MagnitudePruning::compute_mask (threshold by sorted
    magnitude, ties restored in index order) and to_sparse(W*mask) equal the
    reference's own, compiled from src/pruning/{magnitude_pruning,sparse_tensor}.cpp."""
    rng = np.random.default_rng(abs(hash((kind, sparsity))) % 2**32)
    shape = (97, 131)
    if kind == "normal":
        w = rng.standard_normal(shape).astype(np.float32)
    elif kind == "ties":
        w = (rng.integers(-3, 4, shape) / 4).astype(np.float32)
    elif kind == "zeros":
        w = np.where(rng.random(shape) < 0.5, 0.0, rng.standard_normal(shape)).astype(np.float32)
    else:
        w = np.full(shape, -0.5, np.float32)
    m = po.magnitude_mask(w, sparsity)
    np.testing.assert_array_equal(m, po.ref_magnitude_mask(w, sparsity))
    ip, ix, v = po.masked_csr(w, m)
    rip, rix, rv = po.ref_to_sparse_csr(w * m)
    np.testing.assert_array_equal(ip, rip)
    np.testing.assert_array_equal(ix, rix)
    np.testing.assert_array_equal(v, rv)


@pytest.mark.skipif(not po.ref_available(), reason="compiled reference not built")
def test_magnitude_mask_empty_weight_raises():
    with pytest.raises(RuntimeError, match="empty"):
        po.magnitude_mask(np.zeros((0, 4), np.float32), 0.5)
    with pytest.raises(RuntimeError, match="empty"):
        po.ref_magnitude_mask(np.zeros((1, 0), np.float32), 0.5)


@pytest.mark.parametrize("n,m", [(1, 2), (2, 4), (3, 4), (2, 8), (4, 8), (5, 16), (16, 32), (3, 3)])
@pytest.mark.parametrize("kind", ["ties", "normal", "nan", "zeros"])
def test_nm_mask_matches_reference(n, m, kind):
    """The restated N:M selection (ties resolved as libstdc++'s heap-based
    std::partial_sort resolves them) equals NMSparsityPruning::compute_mask
    compiled from src/pruning/nm_sparsity.cpp, including a short last group."""
    rng = np.random.default_rng(n * 100 + m)
    for total in (m * 7, m * 7 + 1, m * 5 - 1, 1):
        if kind == "ties":
            w = rng.choice(np.array([0.0, -0.0, 1.0, -1.0, 2.0, -2.0, 0.5], np.float32), total)
        elif kind == "nan":
            w = rng.standard_normal(total).astype(np.float32)
            w[rng.random(total) < 0.2] = np.nan
        elif kind == "zeros":
            w = np.where(rng.random(total) < 0.6, 0.0, rng.standard_normal(total)).astype(np.float32)
        else:
            w = rng.standard_normal(total).astype(np.float32)
        np.testing.assert_array_equal(po.nm_mask(w, n, m), po.ref_nm_mask(w, n, m))
