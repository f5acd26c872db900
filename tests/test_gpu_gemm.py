"""fp32 Gemm / MatMul on the GPU (3xTF32 tcgen05) vs cpu_gemm
(src/backends/cpu/ops/math.cpp:377-438).

Summation order differs from the reference's k-sequential loop, so parity is
normwise: max|gpu - ref| / max|ref| <= 1e-5.  The GPU error against an fp64
restatement is also bounded, to show the tensor-core path is as accurate as
the CPU path."""
import numpy as np
import pytest
import torch

import pyflamert_b200 as pf
from oracle import pyoracle as po
from pyflamert_b200 import workloads as wl
from tests.golden import cases as gcases
from tests.helpers import FP32_TOL, normwise_rel

pytestmark = pytest.mark.gpu


def gpu_dense(ctx, g: wl.GemmCase):
    A = torch.from_numpy(g.A).cuda()
    B = torch.from_numpy(g.B).cuda()
    C = None if g.C is None else torch.from_numpy(g.C).cuda()
    y = ctx.gemm_f32_dense(A, B, C, g.alpha, g.beta, g.trans_a, g.trans_b)
    ctx.check()
    return y.cpu().numpy()


def gpu_weight(ctx, g: wl.GemmCase):
    w = pf.FWeight(ctx, g.B, g.trans_b)
    A = torch.from_numpy(g.A).cuda()
    C = None if g.C is None else torch.from_numpy(g.C).cuda()
    y = w(A, C, g.alpha, g.beta, g.trans_a)
    ctx.check()
    return y.cpu().numpy()


def oracle(g: wl.GemmCase):
    return po.gemm(g.A, g.B, g.C, g.alpha, g.beta, g.trans_a, g.trans_b)


@pytest.mark.parametrize("name", [n for n, c in gcases.all_cases().items() if c["kind"] in ("gemm", "matmul")])
@pytest.mark.parametrize("path", ["dense", "weight"])
def test_golden(ctx, golden, name, path):
    case = gcases.all_cases()[name]
    if case["kind"] == "matmul":
        g = wl.GemmCase(case["A"], case["B"], None, 1.0, 0.0)
    else:
        g = case["case"]
    y = (gpu_dense if path == "dense" else gpu_weight)(ctx, g)
    ref = golden[0][name]
    y = y[: ref.shape[0]]
    assert normwise_rel(y, ref) <= FP32_TOL


def test_reference_known_answer_exact(ctx):
    """ExecutorTest.MatMul (tests/cpp/test_executor.cpp:162-208): small
    integers are exact in tf32 splits, so the answer is exact."""
    g = wl.GemmCase(np.array([[1, 2, 3], [4, 5, 6]], np.float32),
                    np.array([[1, 2], [3, 4], [5, 6]], np.float32), None, 1.0, 0.0)
    np.testing.assert_array_equal(gpu_dense(ctx, g), np.array([[22, 28], [49, 64]], np.float32))


@pytest.mark.parametrize("path", ["dense", "weight"])
def test_config1_full(ctx, path):
    g = wl.gemm_case()
    y = (gpu_dense if path == "dense" else gpu_weight)(ctx, g)
    ref = oracle(g)
    f64 = po.gemm_f64(g.A, g.B, g.C, g.alpha, g.beta)
    assert normwise_rel(y, ref) <= FP32_TOL
    assert normwise_rel(y, f64) <= 2 * normwise_rel(ref, f64) + 1e-6


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (130, 70, 33), (257, 129, 300), (64, 512, 2048)])
def test_shapes_and_transposes(ctx, ta, tb, M, N, K):
    g = wl.gemm_case(M, N, K, seed=M * 7 + N * 3 + K + ta + 2 * tb, trans_a=ta, trans_b=tb,
                     alpha=0.75, beta=-1.5)
    y = gpu_dense(ctx, g)
    assert normwise_rel(y, oracle(g)) <= FP32_TOL
    y2 = gpu_weight(ctx, g)
    assert normwise_rel(y2, oracle(g)) <= FP32_TOL


@pytest.mark.parametrize("c_len", [0, 1, 7, "N", "MN"])
def test_bias_broadcasts(ctx, c_len):
    M, N = 40, 24
    cl = {"N": N, "MN": M * N}.get(c_len, c_len)
    g = wl.gemm_case(M, N, 64, seed=99, c_len=cl, beta=0.5)
    y = gpu_dense(ctx, g)
    assert normwise_rel(y, oracle(g)) <= FP32_TOL


def test_empty_k(ctx):
    """K = 0: the product is empty and Y = beta * C."""
    A = torch.zeros((3, 0), device="cuda")
    B = torch.zeros((0, 5), device="cuda")
    C = torch.arange(5, dtype=torch.float32, device="cuda")
    y = ctx.gemm_f32_dense(A, B, C, 1.0, 2.0)
    ctx.check()
    np.testing.assert_array_equal(y.cpu().numpy(), np.tile(2.0 * np.arange(5, dtype=np.float32), (3, 1)))


@pytest.mark.parametrize("splits", ["1", "4"])
def test_split_k(ctx, splits, monkeypatch):
    monkeypatch.setenv("PFRT_GEMM_SPLITS", splits)
    g = wl.gemm_case(256, 384, 1024, seed=5)
    assert normwise_rel(gpu_weight(ctx, g), oracle(g)) <= FP32_TOL


def test_large_values_accuracy(ctx):
    """Inputs with a wide exponent range: the 3xTF32 split keeps fp32-level accuracy."""
    rng = np.random.default_rng(77)
    A = (rng.standard_normal((128, 512)) * np.exp(rng.uniform(-8, 8, (128, 512)))).astype(np.float32)
    B = (rng.standard_normal((512, 96)) * np.exp(rng.uniform(-8, 8, (512, 96)))).astype(np.float32)
    g = wl.GemmCase(A, B, None, 1.0, 0.0)
    y = gpu_dense(ctx, g)
    f64 = po.gemm_f64(A, B)
    assert normwise_rel(y, f64) <= FP32_TOL


@pytest.mark.parametrize("splits", ["5", "8"])
@pytest.mark.parametrize("M,N,K,c_len", [(256, 1024, 1024, None), (130, 300, 1000, 7), (64, 100, 4096, "MN")])
def test_fresh_weights_with_split_k(ctx, splits, M, N, K, c_len, monkeypatch):
    """A new prepared weight per call, several calls in a row, with K split:
    each result within the fp32 bound.  (Weight preparation once read its
    staging copy before a pageable host-to-device copy had landed, which
    only showed on later weights.)"""
    c = {None: None, "MN": M * N}.get(c_len, c_len)
    g = wl.gemm_case(M, N, K, seed=M + N + K, c_len=c)
    monkeypatch.setenv("PFRT_GEMM_SPLITS", splits)
    ref = oracle(g)
    for _ in range(4):
        assert normwise_rel(gpu_weight(ctx, g), ref) <= FP32_TOL
