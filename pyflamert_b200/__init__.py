"""B200 (sm_100a) backend for PyFlameRT's MatMul / Gemm / QuantizedMatMul /
sparse-weight MatMul hot path.

The product is the C ABI in ``include/pfrt_cuda.h`` (``lib/libpfrt_cuda.so``)
and the PyFlameRT ``Backend`` plugin built on it (``backend/``).  This module
binds the C ABI with ctypes for Python callers, tests and the benchmark.
Device buffers are torch CUDA tensors (PyTorch is used for device memory and
streams only); host buffers are numpy arrays.

There is no CPU fallback: importing works anywhere, but every compute call
goes through ``libpfrt_cuda.so`` and fails loudly when the library is missing
or no sm_100 GPU is present.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _abi
from ._abi import (PFRT_OUT_F32, PFRT_OUT_S8, PFRT_OUT_U8, PfrtError, lib,  # noqa: F401
                   lib_path)

__all__ = [
    "Context", "QWeight", "FWeight", "CSR", "PfrtError", "lib", "lib_path",
    "PFRT_OUT_F32", "PFRT_OUT_S8", "PFRT_OUT_U8", "OUT_MODES",
]

OUT_MODES = {"f32": PFRT_OUT_F32, "int8": PFRT_OUT_S8, "uint8": PFRT_OUT_U8}


def _check(st: int, what: str = "") -> None:
    _abi.check(st, what)


def _dptr(t) -> int:
    """Device address of a torch CUDA tensor (or None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy: the device's legacy default stream


def _stream(stream) -> int:
    """The CUDA stream handle to pass to the C ABI.  torch's default stream has
    handle 0, which the C ABI reads as "the context's own stream"; it is
    passed as cudaStreamLegacy instead so that work stays ordered with torch."""
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    h = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    return h if h else CUDA_STREAM_LEGACY


class Context:
    """One pfrt context per device (pfrt_ctx_create)."""

    def __init__(self, device: int = 0):
        self.device = device
        self._h = C.c_void_p()
        _check(lib().pfrt_ctx_create(device, C.byref(self._h)), "pfrt_ctx_create")

    @property
    def handle(self):
        return self._h

    def num_sms(self) -> int:
        n = C.c_int()
        _check(lib().pfrt_ctx_num_sms(self._h, C.byref(n)))
        return n.value

    def check(self, stream=None) -> None:
        """Synchronize `stream` and raise on a recorded device-side failure."""
        _check(lib().pfrt_ctx_check(self._h, _stream(stream)), "pfrt_ctx_check")

    def close(self) -> None:
        if self._h:
            lib().pfrt_ctx_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- ops
    def gemm_f32_dense(self, a, b, c=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0, y=None,
                       stream=None):
        """Gemm with device A, B (and C); mirrors cpu_gemm's argument meaning."""
        import torch
        M = a.shape[1] if trans_a else a.shape[0]
        K = a.shape[0] if trans_a else a.shape[1]
        N = b.shape[0] if trans_b else b.shape[1]
        kb = b.shape[1] if trans_b else b.shape[0]
        if kb != K:
            raise PfrtError(1, f"Gemm: incompatible dimensions - A has K={K}, B has K={kb}")
        if y is None:
            y = torch.empty((M, N), dtype=torch.float32, device=a.device)
        c_len = 0 if c is None else c.numel()
        _check(lib().pfrt_gemm_f32_dense(self._h, M, N, K, int(trans_a), int(trans_b), alpha,
                                         _dptr(a), _dptr(b), beta, _dptr(c), c_len, _dptr(y),
                                         _stream(stream)), "pfrt_gemm_f32_dense")
        return y

    def quantize(self, x, scale, zp, out="int8", q=None, stream=None):
        import torch
        if q is None:
            q = torch.empty(x.shape, dtype=torch.uint8 if out == "uint8" else torch.int8, device=x.device)
        _check(lib().pfrt_quantize_f32(self._h, x.numel(), _dptr(x), scale, zp, int(out == "uint8"),
                                       _dptr(q), _stream(stream)), "pfrt_quantize_f32")
        return q

    def add_rowvec(self, x, b, y=None, stream=None):
        import torch
        if y is None:
            y = torch.empty_like(x)
        _check(lib().pfrt_add_rowvec_f32(self._h, x.shape[0], x.shape[1], _dptr(x), _dptr(b), _dptr(y),
                                         _stream(stream)), "pfrt_add_rowvec_f32")
        return y

    def relu(self, x, y=None, stream=None):
        import torch
        if y is None:
            y = torch.empty_like(x)
        _check(lib().pfrt_relu_f32(self._h, x.numel(), _dptr(x), _dptr(y), _stream(stream)),
               "pfrt_relu_f32")
        return y

    def spmm_csr_raw(self, M, N, K, nnz, indptr, indices, values, x, y=None, stream=None):
        """Y[M,N] = X W^T on a caller-owned device CSR (int32)."""
        import torch
        if y is None:
            y = torch.empty((M, N), dtype=torch.float32, device=x.device)
        _check(lib().pfrt_spmm_csr_f32(self._h, M, N, K, nnz, _dptr(indptr), _dptr(indices),
                                       _dptr(values), _dptr(x), K, _dptr(y), N, _stream(stream)),
               "pfrt_spmm_csr_f32")
        return y


class QWeight:
    """int8 weight [K,N] (reference B layout) prepared once (pfrt_qweight_create)."""

    def __init__(self, ctx: Context, w: np.ndarray, w_scale, w_zp: int = 0):
        w = np.ascontiguousarray(w, dtype=np.int8)
        ws = np.ascontiguousarray(np.atleast_1d(np.asarray(w_scale, dtype=np.float32)))
        self.ctx, self.K, self.N = ctx, int(w.shape[0]), int(w.shape[1])
        self._h = C.c_void_p()
        _check(lib().pfrt_qweight_create(ctx.handle, self.K, self.N, w.ctypes.data_as(C.c_void_p),
                                         int(w_zp), ws.ctypes.data_as(C.c_void_p), ws.size,
                                         C.byref(self._h)), "pfrt_qweight_create")

    def __call__(self, a, a_scale, a_zp, bias=None, relu=False, out="int8", y_scale=1.0, y_zp=0,
                 y=None, acc_out=None, stream=None):
        import torch
        M = a.shape[0]
        mode = OUT_MODES[out]
        if y is None:
            dt = {PFRT_OUT_F32: torch.float32, PFRT_OUT_S8: torch.int8, PFRT_OUT_U8: torch.uint8}[mode]
            y = torch.empty((M, self.N), dtype=dt, device=a.device)
        _check(lib().pfrt_qlinear(self.ctx.handle, self._h, M, _dptr(a), a.shape[1],
                                  int(a.dtype == torch.uint8), float(a_scale), int(a_zp), _dptr(bias),
                                  int(bool(relu)), mode, float(y_scale), int(y_zp), _dptr(y),
                                  y.shape[1], _dptr(acc_out), _stream(stream)), "pfrt_qlinear")
        return y

    def host_call(self, a_host, a_scale, a_zp, y_host, bias=None, relu=False, out="int8", y_scale=1.0, y_zp=0,
                  stream=None):
        """The layer on HOST buffers (pfrt_qlinear_host): a_host [M, K] and
        y_host [M, N] are CPU tensors (pinned for asynchronous copies); the
        copy in, the layer and the copy out are enqueued on `stream`, and
        y_host holds the result once that stream is synchronized."""
        import torch
        M = a_host.shape[0]
        _check(lib().pfrt_qlinear_host(self.ctx.handle, self._h, M, a_host.data_ptr(), a_host.stride(0),
                                       int(a_host.dtype == torch.uint8), float(a_scale), int(a_zp), _dptr(bias),
                                       int(bool(relu)), OUT_MODES[out], float(y_scale), int(y_zp),
                                       y_host.data_ptr(), y_host.stride(0), _stream(stream)), "pfrt_qlinear_host")
        return y_host

    def close(self):
        if self._h:
            lib().pfrt_qweight_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class FWeight:
    """fp32 B operand prepared once (pfrt_fweight_create): [K,N], or [N,K] if trans_b."""

    def __init__(self, ctx: Context, b: np.ndarray, trans_b: int = 0):
        b = np.ascontiguousarray(b, dtype=np.float32)
        self.ctx = ctx
        self.K, self.N = (b.shape[1], b.shape[0]) if trans_b else (b.shape[0], b.shape[1])
        self._h = C.c_void_p()
        _check(lib().pfrt_fweight_create(ctx.handle, self.K, self.N, int(trans_b),
                                         b.ctypes.data_as(C.c_void_p), C.byref(self._h)),
               "pfrt_fweight_create")

    def __call__(self, a, c=None, alpha=1.0, beta=1.0, trans_a=0, y=None, stream=None):
        import torch
        M = a.shape[1] if trans_a else a.shape[0]
        K = a.shape[0] if trans_a else a.shape[1]
        if K != self.K:
            raise PfrtError(1, f"Gemm: incompatible dimensions - A has K={K}, B has K={self.K}")
        if y is None:
            y = torch.empty((M, self.N), dtype=torch.float32, device=a.device)
        c_len = 0 if c is None else c.numel()
        _check(lib().pfrt_gemm_f32(self.ctx.handle, M, int(trans_a), float(alpha), _dptr(a), self._h,
                                   float(beta), _dptr(c), c_len, _dptr(y), _stream(stream)),
               "pfrt_gemm_f32")
        return y

    def close(self):
        if self._h:
            lib().pfrt_fweight_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CSR:
    """Sparse weight W [N,K] in CSR, validated and uploaded once (pfrt_csr_create)."""

    def __init__(self, ctx: Context, N: int, K: int, indptr, indices, values):
        ip = np.ascontiguousarray(indptr)
        ix = np.ascontiguousarray(indices)
        if ip.dtype not in (np.int32, np.int64) or ix.dtype != ip.dtype:
            ip, ix = ip.astype(np.int64), ix.astype(np.int64)
        v = np.ascontiguousarray(values, dtype=np.float32)
        self.ctx, self.N, self.K, self.nnz = ctx, int(N), int(K), int(v.size)
        self._h = C.c_void_p()
        _check(lib().pfrt_csr_create(ctx.handle, self.N, self.K, self.nnz, ip.ctypes.data_as(C.c_void_p),
                                     ix.ctypes.data_as(C.c_void_p), 32 if ip.dtype == np.int32 else 64,
                                     v.ctypes.data_as(C.c_void_p), C.byref(self._h)), "pfrt_csr_create")

    @classmethod
    def from_magnitude_pruning(cls, ctx: Context, w, sparsity: float, mask=None):
        """Magnitude-prune the device weight W [N, K] (a CUDA fp32 tensor) to
        `sparsity` as MagnitudePruning::compute_mask does and keep the result
        as a CSR weight (pfrt_csr_from_magnitude_pruning).  `mask` (optional,
        a CUDA fp32 tensor of W's size) receives the 0/1 mask."""
        N, K = int(w.shape[0]), int(w.shape[1])
        self = cls.__new__(cls)
        self.ctx, self.N, self.K = ctx, N, K
        self._h = C.c_void_p()
        _check(lib().pfrt_csr_from_magnitude_pruning(ctx.handle, N, K, _dptr(w), float(sparsity), _dptr(mask),
                                                     C.byref(self._h)), "pfrt_csr_from_magnitude_pruning")
        nnz = C.c_int64()
        _check(lib().pfrt_csr_info(self._h, None, None, C.byref(nnz)), "pfrt_csr_info")
        self.nnz = int(nnz.value)
        return self

    @classmethod
    def from_nm_pruning(cls, ctx: Context, w, n: int = 2, m: int = 4, mask=None):
        """N:M-prune the device weight W [N, K] (a CUDA fp32 tensor) as
        NMSparsityPruning(n, m).compute_mask does (groups of m consecutive
        weights in row-major order keep their n largest |w|) and keep the
        result as a CSR weight (pfrt_csr_from_nm_pruning).  `mask` (optional,
        a CUDA fp32 tensor of W's size) receives the 0/1 mask."""
        N, K = int(w.shape[0]), int(w.shape[1])
        self = cls.__new__(cls)
        self.ctx, self.N, self.K = ctx, N, K
        self._h = C.c_void_p()
        _check(lib().pfrt_csr_from_nm_pruning(ctx.handle, N, K, _dptr(w), int(n), int(m), _dptr(mask),
                                              C.byref(self._h)), "pfrt_csr_from_nm_pruning")
        nnz = C.c_int64()
        _check(lib().pfrt_csr_info(self._h, None, None, C.byref(nnz)), "pfrt_csr_info")
        self.nnz = int(nnz.value)
        return self

    def __call__(self, x, y=None, stream=None):
        import torch
        M = x.shape[0]
        if x.shape[1] != self.K:
            raise PfrtError(1, "Dimension mismatch in sparse matmul")
        if y is None:
            y = torch.empty((M, self.N), dtype=torch.float32, device=x.device)
        _check(lib().pfrt_spmm(self.ctx.handle, self._h, M, _dptr(x), x.shape[1], _dptr(y), y.shape[1],
                               _stream(stream)), "pfrt_spmm")
        return y

    def close(self):
        if self._h:
            lib().pfrt_csr_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def native_library_path() -> str:
    return lib_path()


def is_built() -> bool:
    return os.path.exists(lib_path())
