"""Comparison helpers shared by the tests."""
import numpy as np


def normwise_rel(y, ref) -> float:
    """max|y - ref| / max|ref| -- the fp32 parity measure (<= 1e-5)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.max(np.abs(ref)) if ref.size else 0.0
    if den == 0.0:
        return float(np.max(np.abs(y - ref))) if y.size else 0.0
    return float(np.max(np.abs(y - ref)) / den)


def elementwise_rel(y, ref) -> float:
    """max |y - ref| / (|ref| + 1e-3 * rms(ref)): elementwise error with a floor
    for outputs that cancel to ~0."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size == 0:
        return 0.0
    rms = float(np.sqrt(np.mean(ref * ref)))
    return float(np.max(np.abs(y - ref) / (np.abs(ref) + 1e-3 * rms + 1e-30)))


FP32_TOL = 1e-5  # north-star parity bound for fp32 Gemm and SpMM (normwise)
