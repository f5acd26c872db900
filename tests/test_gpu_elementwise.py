"""Standalone requantize / bias Add / Relu kernels vs the reference -- bit-exact."""
import numpy as np
import pytest
import torch

from oracle import pyoracle as po
from tests.golden import cases as gcases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["quant_s8", "quant_u8_zp"])
def test_quantize_golden(ctx, golden, name):
    case = gcases.all_cases()[name]
    x = torch.from_numpy(case["x"]).cuda()
    q = ctx.quantize(x, case["scale"], case["zp"], case["out"])
    ctx.check()
    np.testing.assert_array_equal(q.cpu().numpy(), golden[0][name])


def test_quantize_nan_and_overflow_like_reference(ctx):
    """(int32)std::round(x) of a value outside int32, or of NaN, is INT32_MIN on
    the reference's x86-64 target; the kernel reproduces it."""
    x = np.array([np.nan, np.inf, -np.inf, 3e9, -3e9, 1e30, 2.0], np.float32)
    q = ctx.quantize(torch.from_numpy(x).cuda(), 0.5, 10, "int8")
    ctx.check()
    np.testing.assert_array_equal(q.cpu().numpy(), po.quantize(x, 0.5, 10, "int8"))


def test_add_rowvec_and_relu(ctx):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((37, 53)).astype(np.float32)
    b = rng.standard_normal(53).astype(np.float32)
    y = ctx.add_rowvec(torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda())
    r = ctx.relu(y)
    ctx.check()
    np.testing.assert_array_equal(y.cpu().numpy(), x + b)
    np.testing.assert_array_equal(r.cpu().numpy(), np.maximum(np.float32(0), x + b))


@pytest.mark.parametrize("nbytes", [1, 1000, (256 << 10) - 1, 256 << 10, (256 << 10) + 1, (3 << 20) + 7,
                                    (9 << 20) + 4093])
def test_staged_copies_round_trip(ctx, nbytes):
    """pfrt_memcpy_h2d_staged / pfrt_memcpy_d2h_staged (pageable host memory
    through the context's pinned ring, host copies split over threads): every
    byte arrives, for sizes around the 256 KiB chunk and the 8-slot ring
    (9 MiB wraps the ring more than once), called twice in a row on the same
    ring."""
    import ctypes as C

    import pyflamert_b200 as pf
    rng = np.random.default_rng(nbytes)
    L = pf.lib()
    d = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        src = rng.integers(0, 256, nbytes, dtype=np.uint8)
        dst = np.zeros(nbytes, np.uint8)
        pf._abi.check(L.pfrt_memcpy_h2d_staged(ctx.handle, C.c_void_p(d.data_ptr()), src.ctypes.data, nbytes, None),
                      "pfrt_memcpy_h2d_staged")
        src_copy = src.copy()
        src[:] = 0  # the call returned: the host buffer may be reused at once
        pf._abi.check(L.pfrt_memcpy_d2h_staged(ctx.handle, dst.ctypes.data, C.c_void_p(d.data_ptr()), nbytes, None),
                      "pfrt_memcpy_d2h_staged")
        ctx.check(stream=None)
        np.testing.assert_array_equal(dst, src_copy)
