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
