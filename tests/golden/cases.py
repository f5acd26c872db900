"""Seeded cases behind the golden fixtures (tests/golden/golden_ref.npz).

Shared by make_golden.py (which runs the reference on them) and the tests
(which run the oracle restatement and the CUDA path on them)."""
from __future__ import annotations

import numpy as np

from pyflamert_b200 import workloads as wl


def all_cases():
    c = {}
    # The reference's only hot-path known-answer test:
    # ExecutorTest.MatMul (tests/cpp/test_executor.cpp:162-208).
    c["kat_matmul"] = dict(kind="matmul",
                           A=np.array([[1, 2, 3], [4, 5, 6]], np.float32),
                           B=np.array([[1, 2], [3, 4], [5, 6]], np.float32))
    # Gemm (cpu_gemm, math.cpp:377-438): transposes, alpha/beta, bias broadcasts.
    c["gemm_nn_bias_n"] = dict(kind="gemm", case=wl.gemm_case(33, 40, 70, seed=11))
    c["gemm_tn_alpha"] = dict(kind="gemm", case=wl.gemm_case(17, 24, 45, seed=12, trans_a=1,
                                                             alpha=0.5, beta=2.0))
    c["gemm_nt_scalar_c"] = dict(kind="gemm", case=wl.gemm_case(9, 31, 64, seed=13, trans_b=1, c_len=1))
    c["gemm_tt_full_c"] = dict(kind="gemm", case=wl.gemm_case(12, 20, 33, seed=14, trans_a=1, trans_b=1,
                                                              c_len=12 * 20, beta=-1.0))
    c["gemm_odd_c_len"] = dict(kind="gemm", case=wl.gemm_case(7, 10, 16, seed=15, c_len=7))
    c["gemm_no_c"] = dict(kind="gemm", case=wl.gemm_case(5, 6, 7, seed=16, c_len=0))
    c["cfg1_rows8"] = dict(kind="gemm", case=wl.gemm_case(seed=1), rows=8)
    # quantized_matmul + quantize_tensor (quant_ops.cpp:387-506, 15-127), per-tensor.
    for out in ("f32", "int8", "uint8"):
        q = wl.qlinear_case(16, 48, 96, seed=21, out=out, y_scale=0.05, y_zp=3 if out != "f32" else 0)
        q.w_scale[:] = np.float32(0.0125)
        c[f"qmm_u8s8_{out}"] = dict(kind="qmm_per_tensor", case=q)
    q = wl.qlinear_case(16, 40, 64, seed=22, a_signed=True, w_zp=3, out="int8", y_scale=0.5)
    q.w_scale[:] = np.float32(0.01)
    c["qmm_s8s8_wzp"] = dict(kind="qmm_per_tensor", case=q)
    # Per-output-channel chain QuantizedMatMul -> Add -> Relu -> Quantize.
    c["qlin_pc_bias_relu_u8"] = dict(kind="qlinear_per_channel",
                                     case=wl.qlinear_case(12, 64, 128, seed=23, bias=True, relu=True,
                                                          out="uint8", y_scale=0.3))
    c["qlin_pc_f32"] = dict(kind="qlinear_per_channel",
                            case=wl.qlinear_case(8, 33, 50, seed=24, bias=True, out="f32"))
    c["cfg2_rows4"] = dict(kind="qlinear_per_channel", case=wl.qlinear_case(seed=2), rows=4)
    # quantize_tensor with round-half-away ties and saturation.
    x = np.concatenate([np.array([0.025, -0.025, 0.075, -0.125, 6.4, -6.45, 1e9, -1e9, 0.0, -0.0],
                                 np.float32),
                        np.random.default_rng(31).standard_normal(200).astype(np.float32) * 4])
    c["quant_s8"] = dict(kind="quantize", x=x, scale=0.05, zp=0, out="int8")
    c["quant_u8_zp"] = dict(kind="quantize", x=x, scale=0.05, zp=100, out="uint8")
    # sparse_matmul (sparse_tensor.cpp:473-519).
    c["spmm_small"] = dict(kind="spmm", case=wl.spmm_case(8, 64, 96, sparsity=0.9, seed=41))
    c["spmm_dense_rows"] = dict(kind="spmm", case=wl.spmm_case(3, 16, 40, sparsity=0.0, seed=42))
    c["cfg3_rows4"] = dict(kind="spmm", case=wl.spmm_case(seed=3), rows=4)
    return c
