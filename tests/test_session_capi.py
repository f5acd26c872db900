"""The drop-in through its C entry points (include/pfrt_session.h,
libpfrt_session.so: the reference's InferenceSession with the CUDA seam) and
the Python .pfm writer (pyflamert_b200/pfm.py).

CPU: a model written by pfm.save loads in the reference's own loader and runs
on device "cpu" (the reference's CPUExecutor) with the oracle's result, and a
bad device string is rejected by the session's own validation.
GPU: the same model on device "cuda", "cuda:0" and the two-slice batch split
"cuda:0,0" gives the oracle's int8 output bit for bit."""
import os

import numpy as np
import pytest

from pyflamert_b200 import pfm, workloads as wl


def _lib_or_skip():
    if not os.path.exists(pfm.session_lib_path()):
        from pyflamert_b200 import build
        if build.reference_include() is None:
            pytest.skip("needs the PyFlameRT sources to build libpfrt_session.so")
        build.build_cuda()
        build.build_backend()
        build.build_session_lib()


def _qlinear_model(path, q):
    """Config 2's layer as a graph: QuantizedMatMul (per-channel b_scales) ->
    Quantize int8."""
    M, K = q.a.shape
    N = q.w.shape[1]
    pfm.save(path, "qlinear", inputs=[("A", np.uint8, (M, K))], outputs=[("Y", np.int8, (M, N))],
             initializers={"W": q.w},
             nodes=[("qmm", "QuantizedMatMul", ["A", "W"], ["t0"],
                     {"a_scale": q.a_scale, "a_zero_point": q.a_zp, "b_scales": q.w_scale}),
                    ("quant", "Quantize", ["t0"], ["Y"], {"scale": q.y_scale, "dtype": "int8"})])


def _gemm_model(path, g):
    M, K = g.A.shape
    N = g.B.shape[1]
    pfm.save(path, "gemm", inputs=[("A", np.float32, (M, K))], outputs=[("Y", np.float32, (M, N))],
             initializers={"B": g.B, "C": g.C},
             nodes=[("gemm", "Gemm", ["A", "B", "C"], ["Y"], {"alpha": 1.0, "beta": 1.0})])


def test_pfm_writer_and_cpu_session(tmp_path):
    _lib_or_skip()
    from oracle import pyoracle as po
    g = wl.gemm_case(16, 24, 40, seed=3)
    path = str(tmp_path / "gemm.pfm")
    _gemm_model(path, g)
    s = pfm.Session(path, "cpu")
    try:
        y = s.run({"A": g.A})[0]
    finally:
        s.close()
    np.testing.assert_array_equal(y, po.gemm(g.A, g.B, g.C))   # the reference's cpu_gemm, bit for bit


def test_bad_device_string_rejected(tmp_path):
    _lib_or_skip()
    g = wl.gemm_case(4, 8, 8, seed=1)
    path = str(tmp_path / "g.pfm")
    _gemm_model(path, g)
    with pytest.raises(RuntimeError, match="Invalid device"):
        pfm.Session(path, "tpu")


@pytest.mark.gpu
@pytest.mark.parametrize("device", ["cuda", "cuda:0", "cuda:0,0"])
def test_cuda_session_matches_oracle(tmp_path, device, monkeypatch):
    _lib_or_skip()
    from oracle import pyoracle as po
    monkeypatch.setenv("PFRT_SPLIT_MIN_ROWS", "64")
    q = wl.qlinear_case(512, 1024, 768, seed=5)
    path = str(tmp_path / "q.pfm")
    _qlinear_model(path, q)
    ref = po.qlinear(q.a, q.a_scale, q.a_zp, q.w, q.w_scale, out="int8", y_scale=q.y_scale)
    s = pfm.Session(path, device)
    try:
        for _ in range(2):
            y = s.run({"A": q.a})[0]
            np.testing.assert_array_equal(y, ref)
    finally:
        s.close()
