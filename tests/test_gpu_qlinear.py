"""int8 path on the GPU vs the reference arithmetic -- bit-exact.

The CUDA path (tcgen05 kind::i8 GEMM with the fused zero-point / dequant /
bias / ReLU / requant epilogue, through the C ABI) must reproduce
quantization::quantized_matmul + quantize_tensor
(src/quantization/quant_ops.cpp:387-506, 15-127) to the last bit, and its
int32 accumulators must be exact."""
import os

import numpy as np
import pytest
import torch

import pyflamert_b200 as pf
from oracle import pyoracle as po
from pyflamert_b200 import workloads as wl
from tests.golden import cases as gcases

pytestmark = pytest.mark.gpu


def exact_acc(a, a_zp, w, w_zp=0):
    """Exact sum_k (a-a_zp)(w-w_zp) via a float64 product (every partial sum < 2**53)."""
    return ((a.astype(np.float64) - a_zp) @ (w.astype(np.float64) - w_zp)).astype(np.int64)


def run(ctx, q: wl.QCase, rows=None, want_acc=True, lda_pad=0):
    w = pf.QWeight(ctx, q.w, q.w_scale, q.w_zp)
    a = q.a if rows is None else q.a[:rows]
    if lda_pad:
        buf = np.zeros((a.shape[0], a.shape[1] + lda_pad), a.dtype)
        buf[:, : a.shape[1]] = a
        a_dev = torch.from_numpy(buf).cuda()[:, : a.shape[1]]
        # pass the strided view through the raw ABI (row stride = K + pad)
        M, K = a.shape
        mode = pf.OUT_MODES[q.out]
        dt = {0: torch.float32, 1: torch.int8, 2: torch.uint8}[mode]
        y = torch.empty((M, w.N), dtype=dt, device="cuda")
        acc = torch.empty((M, w.N), dtype=torch.int32, device="cuda")
        bias = None if q.bias is None else torch.from_numpy(q.bias).cuda()
        import ctypes as C
        st = pf.lib().pfrt_qlinear(ctx.handle, w._h, M, a_dev.data_ptr(), K + lda_pad,
                                   int(a.dtype == np.uint8), q.a_scale, q.a_zp,
                                   None if bias is None else bias.data_ptr(), int(q.relu), mode,
                                   q.y_scale, q.y_zp, y.data_ptr(), w.N, acc.data_ptr(),
                                   pf._stream(None))
        pf._abi.check(st)
    else:
        a_dev = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        bias = None if q.bias is None else torch.from_numpy(q.bias).cuda()
        acc = torch.empty((a.shape[0], w.N), dtype=torch.int32, device="cuda") if want_acc else None
        y = w(a_dev, q.a_scale, q.a_zp, bias=bias, relu=q.relu, out=q.out, y_scale=q.y_scale,
              y_zp=q.y_zp, acc_out=acc)
    ctx.check()
    return y.cpu().numpy(), (None if acc is None else acc.cpu().numpy())


def oracle(q: wl.QCase, rows=None):
    a = q.a if rows is None else q.a[:rows]
    return po.qlinear(a, q.a_scale, q.a_zp, q.w, q.w_scale, q.w_zp, bias=q.bias, relu=q.relu,
                      out=q.out, y_scale=q.y_scale, y_zp=q.y_zp)


def bits(y):
    return y.view(np.uint8) if y.dtype.itemsize == 1 else y.view(np.int32)


@pytest.mark.parametrize("name", [n for n, c in gcases.all_cases().items()
                                  if c["kind"] in ("qmm_per_tensor", "qlinear_per_channel")])
def test_golden(ctx, golden, name):
    case = gcases.all_cases()[name]
    q = case["case"]
    y, _ = run(ctx, q, rows=case.get("rows"))
    ref = golden[0][name]
    np.testing.assert_array_equal(bits(y), bits(ref))


def test_config2_full(ctx):
    """Config 2 at full size (512 x 4096 x 4096, per-channel, int8 out)."""
    q = wl.qlinear_case()
    y, acc = run(ctx, q)
    ex = exact_acc(q.a, q.a_zp, q.w)
    np.testing.assert_array_equal(acc.astype(np.int64), ex)
    ref = po.qepilogue(ex, q.a_scale, q.w_scale, None, False, q.out, q.y_scale, q.y_zp)
    np.testing.assert_array_equal(y, ref)
    np.testing.assert_array_equal(y[:8], oracle(q, rows=8))


@pytest.mark.parametrize("out", ["f32", "int8", "uint8"])
@pytest.mark.parametrize("relu,bias", [(False, False), (True, True)])
def test_out_modes(ctx, out, relu, bias):
    q = wl.qlinear_case(200, 320, 384, seed=7, bias=bias, relu=relu, out=out, y_scale=0.5, y_zp=2)
    y, acc = run(ctx, q)
    np.testing.assert_array_equal(bits(y), bits(oracle(q)))
    np.testing.assert_array_equal(acc.astype(np.int64), exact_acc(q.a, q.a_zp, q.w))


@pytest.mark.parametrize("M,N,K", [(1, 16, 16), (1, 4096, 4096), (129, 40, 100), (7, 300, 33),
                                   (300, 257, 528), (64, 1000, 4000), (2, 8, 1)])
def test_ragged_shapes(ctx, M, N, K):
    q = wl.qlinear_case(M, N, K, seed=M + N + K, bias=True, relu=True, out="uint8", y_scale=0.7)
    y, acc = run(ctx, q)
    np.testing.assert_array_equal(y, oracle(q))
    np.testing.assert_array_equal(acc.astype(np.int64), exact_acc(q.a, q.a_zp, q.w))


def test_signed_activations_and_weight_zero_point(ctx):
    q = wl.qlinear_case(150, 96, 256, seed=8, a_signed=True, w_zp=-3, out="int8", y_scale=2.0, y_zp=-5)
    q.a_zp = 7
    y, acc = run(ctx, q)
    np.testing.assert_array_equal(y, oracle(q))
    np.testing.assert_array_equal(acc.astype(np.int64), exact_acc(q.a, q.a_zp, q.w, q.w_zp))


def test_strided_activations(ctx):
    """Row stride not a multiple of 16 bytes: the padded-copy path."""
    q = wl.qlinear_case(70, 64, 200, seed=9, out="f32")
    y, acc = run(ctx, q, lda_pad=3)
    np.testing.assert_array_equal(y.view(np.int32), oracle(q).view(np.int32))


@pytest.mark.parametrize("bn,splits", [("128", "1"), ("256", "1"), ("128", "3"), ("256", "2")])
def test_tile_and_split_variants(ctx, bn, splits, monkeypatch):
    monkeypatch.setenv("PFRT_QGEMM_BN", bn)
    monkeypatch.setenv("PFRT_QGEMM_SPLITS", splits)
    q = wl.qlinear_case(384, 512, 1024, seed=10, bias=True, relu=True, out="uint8", y_scale=1.0)
    y, acc = run(ctx, q)
    np.testing.assert_array_equal(y, oracle(q))
    np.testing.assert_array_equal(acc.astype(np.int64), exact_acc(q.a, q.a_zp, q.w))


def test_4096_cube(ctx):
    """The 4096^3 shape of the tensor-peak target; accumulators checked in full."""
    q = wl.qlinear_case(4096, 4096, 4096, seed=12)
    y, acc = run(ctx, q)
    rows = np.r_[0:4, 2047:2051, 4092:4096]
    ex = exact_acc(q.a[rows], q.a_zp, q.w)
    np.testing.assert_array_equal(acc[rows].astype(np.int64), ex)
    np.testing.assert_array_equal(y[rows], po.qepilogue(ex, q.a_scale, q.w_scale, out="int8",
                                                        y_scale=q.y_scale))
    # every accumulator: compare against the exact product on the GPU in fp64
    a = torch.from_numpy(q.a).cuda().double() - q.a_zp
    w = torch.from_numpy(q.w).cuda().double()
    full = (a @ w).round().to(torch.int64).cpu().numpy()
    np.testing.assert_array_equal(acc.astype(np.int64), full)


def test_invalid_arguments(ctx):
    with pytest.raises(pf.PfrtError, match="scale"):
        pf.QWeight(ctx, np.zeros((4, 4), np.int8), np.zeros(4, np.float32))
    with pytest.raises(pf.PfrtError, match="K > 65536"):
        pf.QWeight(ctx, np.zeros((70000, 1), np.int8), np.ones(1, np.float32))
    w = pf.QWeight(ctx, np.ones((16, 4), np.int8), np.ones(4, np.float32))
    a = torch.zeros((2, 16), dtype=torch.uint8, device="cuda")
    with pytest.raises(pf.PfrtError, match="invalid scale"):
        w(a, 0.02, 128, out="int8", y_scale=0.0)


@pytest.mark.parametrize("M,N,K,bn", [(1100, 4100, 1000, None), (512, 4096, 1024, "256"), (2048, 600, 777, "256"),
                                      (4096, 4096, 512, None)])
def test_narrow_tail_units(ctx, M, N, K, bn, monkeypatch):
    """Shapes whose 128x256 tiles leave the last wave at most half full run
    that wave as 128x128 half tiles.  Outputs and accumulators are bit-exact,
    with the tail half tiles past N (N = 4100: a half tile of 4 columns and
    one of none), and equal to the run without the narrow tail."""
    monkeypatch.setenv("PFRT_QGEMM_PAIR", "0")  # the one-CTA kernel is the one with the narrow tail
    if bn:
        monkeypatch.setenv("PFRT_QGEMM_BN", bn)
    q = wl.qlinear_case(M, N, K, seed=M + N + K, bias=True, relu=True, out="int8", y_scale=4.0)
    y, acc = run(ctx, q)
    ex = exact_acc(q.a, q.a_zp, q.w)
    np.testing.assert_array_equal(acc.astype(np.int64), ex)
    np.testing.assert_array_equal(y, po.qepilogue(ex, q.a_scale, q.w_scale, q.bias, True, "int8", 4.0, 0))
    np.testing.assert_array_equal(y[:3], oracle(q, rows=3))
    monkeypatch.setenv("PFRT_QGEMM_NARROW", "0")
    y0, acc0 = run(ctx, q)
    np.testing.assert_array_equal(y0, y)
    np.testing.assert_array_equal(acc0, acc)


@pytest.mark.parametrize("M,N,K,bn", [(512, 4096, 4096, "128"), (1024, 4096, 1024, "256"), (300, 1000, 777, "128"),
                                      (1, 384, 96, "128"), (700, 520, 4096, "256"), (4096, 4096, 4096, "256")])
def test_pair_kernel(ctx, M, N, K, bn, monkeypatch):
    """The CTA-pair kernel (tcgen05 cta_group::2, 256-row tiles split over two
    SMs, B halves in each SM): outputs and accumulators bit-exact, with M, N
    and K tails (M = 1 leaves the second CTA's rows all past M)."""
    monkeypatch.setenv("PFRT_QGEMM_PAIR", "1")
    monkeypatch.setenv("PFRT_QGEMM_BN", bn)
    q = wl.qlinear_case(M, N, K, seed=M + 3 * N + K, bias=True, relu=True, out="int8", y_scale=8.0)
    y, acc = run(ctx, q)
    ex = exact_acc(q.a, q.a_zp, q.w)
    np.testing.assert_array_equal(acc.astype(np.int64), ex)
    np.testing.assert_array_equal(y, po.qepilogue(ex, q.a_scale, q.w_scale, q.bias, True, "int8", 8.0, 0))


@pytest.mark.parametrize("M,N,K,out,relu,bias,y_zp", [
    (512, 4096, 4096, "int8", False, False, 0),     # config 2
    (512, 4096, 4096, "int8", True, True, 0),
    (100, 300, 256, "uint8", True, True, 3),         # two k-blocks, N and M tails
    (129, 520, 384, "f32", False, True, 0),          # odd k-block count: halves of 2 and 1
    (7, 256, 4000, "int8", True, False, -4),         # K tail inside the last k-block
    (256, 1000, 777, "uint8", False, False, 0),
])
def test_split_k_cluster_kernel(ctx, M, N, K, out, relu, bias, y_zp, monkeypatch):
    """K split over a cluster of two CTAs (umma_gemm_sk.cuh): each CTA
    accumulates about half of the k-blocks of a 128 x 256 tile and the
    partials meet through an L2-resident exchange buffer.  Outputs and
    accumulators bit-exact and equal to the one-CTA kernel's."""
    monkeypatch.setenv("PFRT_QGEMM_SK2", "1")
    q = wl.qlinear_case(M, N, K, seed=M + 5 * N + K, bias=bias, relu=relu, out=out, y_scale=6.0, y_zp=y_zp)
    y, acc = run(ctx, q)
    ex = exact_acc(q.a, q.a_zp, q.w)
    np.testing.assert_array_equal(acc.astype(np.int64), ex)
    np.testing.assert_array_equal(bits(y), bits(po.qepilogue(ex, q.a_scale, q.w_scale, q.bias, relu, out, 6.0,
                                                             y_zp)))
    np.testing.assert_array_equal(bits(y[:2]), bits(oracle(q, rows=2)))
    y1, _ = run(ctx, q, want_acc=False)  # the int8 fast epilogue (no accumulator copy)
    np.testing.assert_array_equal(bits(y1), bits(y))
    monkeypatch.setenv("PFRT_QGEMM_SK2", "0")
    y0, acc0 = run(ctx, q)
    np.testing.assert_array_equal(bits(y0), bits(y))
    np.testing.assert_array_equal(acc0, acc)


@pytest.mark.parametrize("M,N,K,tail", [
    (512, 4096, 4096, 1),       # config 2, odd tail: phase-1 ranges of 15 and 16 k-blocks
    (512, 4096, 4096, 30),      # the longest tail: one phase-1 k-block per CTA
    (512, 4096, 4096, 99),      # clipped to kb_total - 2
    (129, 520, 1152, 3),        # 9 k-blocks, N tail inside the own half of the last tile
    (7, 256, 4000, 7),          # K tail inside the last k-block
    (300, 1000, 777, 2),
])
def test_split_k_cluster_early_exchange(ctx, M, N, K, tail, monkeypatch):
    """The split-K cluster kernel's early exchange: each CTA's last `tail`
    k-blocks accumulate only its own half of the columns while the other half
    is exchanged.  Every tail gives the exact accumulators and bit-identical
    outputs."""
    monkeypatch.setenv("PFRT_QGEMM_SK2", "1")
    monkeypatch.setenv("PFRT_QGEMM_SK2_TAIL", str(tail))
    q = wl.qlinear_case(M, N, K, seed=7 * M + N + K + tail, bias=True, relu=True, out="int8", y_scale=6.0,
                        y_zp=1)
    y, acc = run(ctx, q)
    ex = exact_acc(q.a, q.a_zp, q.w)
    np.testing.assert_array_equal(acc.astype(np.int64), ex)
    np.testing.assert_array_equal(y, po.qepilogue(ex, q.a_scale, q.w_scale, q.bias, True, "int8", 6.0, 1))
    y1, _ = run(ctx, q, want_acc=False)
    np.testing.assert_array_equal(y1, y)


@pytest.mark.parametrize("out", ["int8", "uint8"])
@pytest.mark.parametrize("y_scale", [0.05, 1e-12, 1e-40])
@pytest.mark.parametrize("relu,bias", [(False, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (130, 300, 256)])
def test_zero_point_zero_requant_extremes(ctx, M, N, K, relu, bias, y_scale, out):
    """Output zero-point 0 takes a saturating 8-bit conversion in the fused
    epilogue.  A tiny y_scale drives y / y_scale past 2^31 (the reference's
    conversion gives INT32_MIN there, which clamps to the type's minimum), and
    y_scale = 1e-40 makes 1 / y_scale infinite, so zero accumulators give NaN
    and the others +-inf.  Rows of A equal to its zero-point give zero
    accumulators.  Bit-exact against the reference arithmetic."""
    q = wl.qlinear_case(M, N, K, seed=M + N + int(-np.log10(y_scale)), bias=bias, relu=relu, out=out,
                        y_scale=y_scale, y_zp=0)
    q.a[::7] = q.a_zp
    y, acc = run(ctx, q, want_acc=False)
    ex = exact_acc(q.a, q.a_zp, q.w)
    np.testing.assert_array_equal(y, po.qepilogue(ex, q.a_scale, q.w_scale, q.bias, relu, out, y_scale, 0))
    np.testing.assert_array_equal(y[:3], oracle(q, rows=3))


def test_split_k_cluster_weight_zero_point(ctx, monkeypatch):
    monkeypatch.setenv("PFRT_QGEMM_SK2", "1")
    q = wl.qlinear_case(150, 512, 640, seed=21, a_signed=True, w_zp=-3, out="int8", y_scale=2.0, y_zp=-5)
    q.a_zp = 7
    y, acc = run(ctx, q)
    np.testing.assert_array_equal(y, oracle(q))
    np.testing.assert_array_equal(acc.astype(np.int64), exact_acc(q.a, q.a_zp, q.w, q.w_zp))


@pytest.mark.parametrize("out", ["int8", "uint8", "f32"])
def test_host_buffer_call(ctx, out):
    """pfrt_qlinear_host: host activations in, host output back, async on a
    stream; equal to the device call, with padded host rows left untouched."""
    q = wl.qlinear_case(300, 520, 4096, seed=31, bias=True, relu=True, out=out, y_scale=4.0, y_zp=1)
    w = pf.QWeight(ctx, q.w, q.w_scale)
    bias = torch.from_numpy(q.bias).cuda()
    ref = w(torch.from_numpy(q.a).cuda(), q.a_scale, q.a_zp, bias=bias, relu=True, out=out, y_scale=4.0, y_zp=1)
    dt = {"int8": torch.int8, "uint8": torch.uint8, "f32": torch.float32}[out]
    a_pad = torch.zeros((300, 4096 + 32), dtype=torch.uint8).pin_memory()
    a_pad[:, :4096] = torch.from_numpy(q.a)
    y_pad = torch.full((300, 520 + 8), 7, dtype=dt).pin_memory()
    s = torch.cuda.Stream()
    w.host_call(a_pad[:, :4096], q.a_scale, q.a_zp, y_pad[:, :520], bias=bias, relu=True, out=out, y_scale=4.0,
                y_zp=1, stream=s)
    s.synchronize()
    ctx.check()
    assert torch.equal(y_pad[:, :520], ref.cpu())
    assert bool((y_pad[:, 520:] == 7).all())
    np.testing.assert_array_equal(bits(y_pad[:, :520].numpy()), bits(oracle(q)))
    w.close()
