"""Generates the golden fixtures in tests/golden/ from the PyFlameRT reference
itself: the reference's hot-path sources compiled by oracle/Makefile into
oracle/_ref/libpfrt_ref.so (Gemm and MatMul through its CPUExecutor,
quantization::quantized_matmul + quantize_tensor, pruning::sparse_matmul).

    make -C oracle && python tests/golden/make_golden.py

Inputs are not stored: they are regenerated from seeds by
pyflamert_b200.workloads (or written inline below), and each fixture keeps the
SHA-256 of its inputs so a change in the generators is caught.  Only outputs
(small cases, or a few rows of the full benchmark configurations) are stored.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import pyoracle as po  # noqa: E402
from tests.golden import cases  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            h.update(b"none")
        else:
            a = np.ascontiguousarray(a)
            h.update(str(a.dtype).encode() + str(a.shape).encode())
            h.update(a.tobytes())
    return h.hexdigest()


def main():
    if not po.ref_available():
        raise SystemExit("build the reference oracle first: make -C oracle")
    fixtures = {}
    for name, case in cases.all_cases().items():
        kind = case["kind"]
        if kind == "matmul":
            y = po.ref_matmul(case["A"], case["B"])
            fixtures[name] = dict(y=y, sha=sha(case["A"], case["B"]))
        elif kind == "gemm":
            g = case["case"]
            y = po.ref_gemm(g.A, g.B, g.C, g.alpha, g.beta, g.trans_a, g.trans_b)
            fixtures[name] = dict(y=y[: case.get("rows", y.shape[0])], sha=sha(g.A, g.B, g.C))
        elif kind == "qmm_per_tensor":
            q = case["case"]
            y = po.ref_quantized_matmul(q.a, q.a_scale, q.a_zp, q.w, float(q.w_scale[0]), q.w_zp,
                                        out=q.out, y_scale=q.y_scale, y_zp=q.y_zp)
            fixtures[name] = dict(y=y, sha=sha(q.a, q.w, q.w_scale))
        elif kind == "qlinear_per_channel":
            q = case["case"]
            rows = case.get("rows", q.a.shape[0])
            y = po.ref_qlinear_per_channel(q.a[:rows], q.a_scale, q.a_zp, q.w, q.w_scale, q.w_zp,
                                           bias=q.bias, relu=q.relu, out=q.out, y_scale=q.y_scale,
                                           y_zp=q.y_zp)
            fixtures[name] = dict(y=y, sha=sha(q.a, q.w, q.w_scale, q.bias))
        elif kind == "quantize":
            y = po.ref_quantize(case["x"], case["scale"], case["zp"], case["out"])
            fixtures[name] = dict(y=y, sha=sha(case["x"]))
        elif kind == "spmm":
            c = case["case"]
            rows = case.get("rows", c.X.shape[0])
            X = c.X[:rows]
            yt = po.ref_sparse_matmul(c.indptr, c.indices, c.values, np.ascontiguousarray(X.T))
            fixtures[name] = dict(y=np.ascontiguousarray(yt.T), sha=sha(c.indptr, c.indices, c.values, c.X))
        else:
            raise ValueError(kind)
        print(f"{name:28s} {fixtures[name]['y'].shape} {fixtures[name]['y'].dtype}")
    flat = {}
    for name, d in fixtures.items():
        flat[f"{name}__y"] = d["y"]
        flat[f"{name}__sha"] = np.frombuffer(d["sha"].encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(OUT, "golden_ref.npz"), **flat)
    print("wrote", os.path.join(OUT, "golden_ref.npz"))


if __name__ == "__main__":
    main()
