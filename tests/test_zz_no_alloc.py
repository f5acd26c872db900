"""The allocation-free fp32 Gemm entry point, pfrt_gemm_f32_noalloc.

It exists for callers that cannot allocate device memory while they run --
for example a host program whose device memory is all handed out by its own
pool, or a latency-critical loop that must not pay for cudaMalloc's device
synchronization.  It keeps its per-call scratch (the hi/lo split of A) in a
fixed 16 MiB array built into the library, so it can only take calls with
M * Kpad <= 2**21 elements (Kpad = K rounded up to 32).

The test calls it twice in a row through the C ABI, on different shapes so
that contents left in the shared array by the first call would show up in
the second, and compares each result with the allocating entry point
pfrt_gemm_f32 and with the oracle (cpu_gemm's arithmetic, pinned to the
reference) within the fp32 tolerance the other tests use.  A call exactly at
the size limit must be accepted and match too.  This file is named so that
pytest collects it last."""
import ctypes as C

import numpy as np
import pytest
import torch

import pyflamert_b200 as pf
from pyflamert_b200 import workloads as wl
from tests.helpers import FP32_TOL, normwise_rel

pytestmark = pytest.mark.gpu


def _noalloc(ctx, w, a, c, alpha, beta, trans_a, M):
    y = torch.empty((M, w.N), dtype=torch.float32, device="cuda")
    st = pf.lib().pfrt_gemm_f32_noalloc(ctx.handle, M, int(trans_a), float(alpha), a.data_ptr(), w._h,
                                        float(beta), None if c is None else c.data_ptr(),
                                        0 if c is None else c.numel(), y.data_ptr(), pf._stream(None))
    pf._abi.check(st, "pfrt_gemm_f32_noalloc")
    return y


def _oracle(g):
    from oracle import pyoracle as po
    return po.gemm(g.A, g.B, g.C, g.alpha, g.beta, g.trans_a, g.trans_b)


def test_noalloc_matches_allocating_entry_point_twice(ctx):
    cases = [wl.gemm_case(256, 1024, 1024, seed=1),                         # config 1
             wl.gemm_case(70, 200, 333, seed=9, trans_a=1, alpha=0.5, beta=-2.0)]
    for g in cases:
        M = g.A.shape[1] if g.trans_a else g.A.shape[0]
        w = pf.FWeight(ctx, g.B, g.trans_b)
        a = torch.from_numpy(g.A).cuda()
        c = None if g.C is None else torch.from_numpy(g.C).cuda()
        ref = w(a, c, g.alpha, g.beta, g.trans_a)
        y = _noalloc(ctx, w, a, c, g.alpha, g.beta, g.trans_a, M)
        ctx.check()
        y = y.cpu().numpy()
        assert normwise_rel(y, ref.cpu().numpy()) <= FP32_TOL
        assert normwise_rel(y, _oracle(g)) <= FP32_TOL
        w.close()


def test_noalloc_accepts_the_limit(ctx):
    g = wl.gemm_case((1 << 21) // 64, 48, 64, seed=4)   # M * Kpad == 2**21 exactly
    w = pf.FWeight(ctx, g.B)
    a = torch.from_numpy(g.A).cuda()
    c = torch.from_numpy(g.C).cuda()
    y = _noalloc(ctx, w, a, c, g.alpha, g.beta, 0, g.A.shape[0])
    ctx.check()
    assert normwise_rel(y.cpu().numpy(), _oracle(g)) <= FP32_TOL
    w.close()


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    g = wl.gemm_case(8, 16, 64, seed=3)
    w = pf.FWeight(ctx, g.B)
    M = (1 << 21) // 64 + 1            # M * Kpad just above the limit
    a = torch.zeros((M, 64), dtype=torch.float32, device="cuda")
    y = torch.empty((M, 16), dtype=torch.float32, device="cuda")
    st = pf.lib().pfrt_gemm_f32_noalloc(ctx.handle, M, 0, 1.0, a.data_ptr(), w._h, 0.0, None, 0,
                                        y.data_ptr(), pf._stream(None))
    assert st == 5  # PFRT_ERR_UNSUPPORTED
    assert "fixed scratch limit" in pf._abi.last_error()
    w.close()
