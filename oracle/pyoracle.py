"""ctypes bindings for the test oracle.  TEST INFRASTRUCTURE ONLY.

Two libraries are bound here:

* ``oracle/_build/liboracle.so`` -- the C restatement (``oracle.c``) of the
  reference hot path.  Always built (``make -C oracle oracle``).
* ``oracle/_ref/libpfrt_ref.so`` -- the PyFlameRT reference's own hot-path
  sources compiled by ``oracle/Makefile`` plus ``ref_shim.cpp``.  Built when
  the reference sources are present; the built file travels with the repo
  snapshot, so it is also usable where the sources are absent.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline
may import this module.  The product never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libpfrt_ref.so")

_i64, _i32, _f32, _f64, _p, _int = C.c_int64, C.c_int32, C.c_float, C.c_double, C.c_void_p, C.c_int

_lib = None
_ref = None


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"oracle not built: {ORACLE_SO} (run make -C oracle)")
        L = C.CDLL(ORACLE_SO)
        L.oracle_gemm_f32.argtypes = [_i64, _i64, _i64, _int, _int, _f32, _f32, _p, _p, _p, _i64, _p]
        L.oracle_matmul_f32.argtypes = [_i64, _i64, _i64, _p, _p, _p]
        L.oracle_qmm_acc.argtypes = [_i64, _i64, _i64, _p, _int, _i32, _p, _i32, _p]
        L.oracle_qlinear.argtypes = [_i64, _i64, _i64, _p, _int, _f32, _i32, _p, _i32, _p, _p,
                                     _int, _int, _f32, _i32, _p, _p, _p]
        L.oracle_qepilogue.argtypes = [_i64, _i64, _p, _f32, _p, _p, _int, _int, _f32, _i32, _p, _p]
        L.oracle_quantize.argtypes = [_i64, _p, _f32, _i32, _int, _p]
        L.oracle_csr_spmm.argtypes = [_i64, _i64, _p, _p, _p, _p, _p]
        L.oracle_spmm_linear.argtypes = [_i64, _i64, _i64, _p, _p, _p, _p, _p]
        L.oracle_spmm_linear_f64.argtypes = [_i64, _i64, _i64, _p, _p, _p, _p, _p]
        L.oracle_gemm_f64.argtypes = [_i64, _i64, _i64, _int, _int, _f64, _f64, _p, _p, _p, _i64, _p]
        L.oracle_magnitude_mask.argtypes = [_i64, _p, _f32, _p]
        L.oracle_nm_mask.argtypes = [_i64, _p, _int, _int, _p]
        L.oracle_masked_csr.argtypes = [_i64, _i64, _p, _p, _p, _p, _p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"reference oracle not built: {REF_SO}")
        L = C.CDLL(REF_SO)
        L.pfref_last_error.restype = C.c_char_p
        L.pfref_gemm.argtypes = [_i64, _i64, _i64, _int, _int, _f32, _f32, _p, _p, _p, _i64, _p, _int]
        L.pfref_matmul.argtypes = [_i64, _i64, _i64, _p, _p, _p, _int]
        L.pfref_quantized_matmul.argtypes = [_i64, _i64, _i64, _p, _int, _f32, _i32, _p, _int, _f32,
                                             _i32, _int, _f32, _i32, _p, _int]
        L.pfref_qlinear_per_channel.argtypes = [_i64, _i64, _i64, _p, _int, _f32, _i32, _p, _i32, _p,
                                                _p, _int, _int, _f32, _i32, _p]
        L.pfref_quantized_matmul_op.argtypes = [_i64, _i64, _i64, _p, _int, _f32, _i32, _p, _f32, _i32, _p]
        L.pfref_quantize.argtypes = [_i64, _p, _f32, _i32, _int, _p]
        L.pfref_sparse_matmul.argtypes = [_i64, _i64, _i64, _p, _p, _p, _i64, _p, _p, _int]
        L.pfref_magnitude_mask.argtypes = [_i64, _i64, _p, _f32, _p]
        L.pfref_nm_mask.argtypes = [_i64, _p, _i64, _i64, _p]
        L.pfref_to_sparse_csr.argtypes = [_i64, _i64, _p, _f32, _i64, _p, _p, _p, _p]
        _ref = L
    return _ref


def _check_ref(rc):
    if rc != 0:
        raise RuntimeError("reference raised: " + ref().pfref_last_error().decode())


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ---------------------------------------------------------------- restatement
def gemm(A, B, C=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0):
    A, B = _c(A, np.float32), _c(B, np.float32)
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    Cc = None if C is None else _c(C, np.float32).ravel()
    Y = np.empty((M, N), np.float32)
    lib().oracle_gemm_f32(M, N, K, trans_a, trans_b, alpha, beta, _ptr(A), _ptr(B), _ptr(Cc),
                          0 if Cc is None else Cc.size, _ptr(Y))
    return Y


def gemm_f64(A, B, C=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0):
    A, B = _c(A, np.float32), _c(B, np.float32)
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    Cc = None if C is None else _c(C, np.float32).ravel()
    Y = np.empty((M, N), np.float64)
    lib().oracle_gemm_f64(M, N, K, trans_a, trans_b, alpha, beta, _ptr(A), _ptr(B), _ptr(Cc),
                          0 if Cc is None else Cc.size, _ptr(Y))
    return Y


def matmul(A, B):
    A, B = _c(A, np.float32), _c(B, np.float32)
    Y = np.empty((A.shape[0], B.shape[1]), np.float32)
    lib().oracle_matmul_f32(A.shape[0], B.shape[1], A.shape[1], _ptr(A), _ptr(B), _ptr(Y))
    return Y


def qmm_acc(a, w, a_zp, w_zp=0):
    """int64 accumulators sum_k (a-a_zp)(w-w_zp); a u8/s8 [M,K], w s8 [K,N]."""
    a_is_u8 = a.dtype == np.uint8
    a, w = np.ascontiguousarray(a), _c(w, np.int8)
    acc = np.empty((a.shape[0], w.shape[1]), np.int64)
    lib().oracle_qmm_acc(a.shape[0], w.shape[1], a.shape[1], _ptr(a), int(a_is_u8), a_zp, _ptr(w),
                         w_zp, _ptr(acc))
    return acc


def qlinear(a, a_scale, a_zp, w, w_scale, w_zp=0, bias=None, relu=False, out="int8",
            y_scale=1.0, y_zp=0, want_acc=False):
    """Per-output-channel quantized linear layer.  w is int8 [K,N] (the
    reference's B layout); out in {"f32", "int8", "uint8"}."""
    a_is_u8 = a.dtype == np.uint8
    a, w = np.ascontiguousarray(a), _c(w, np.int8)
    M, K = a.shape
    N = w.shape[1]
    ws = _c(w_scale, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    mode = {"f32": 0, "int8": 1, "uint8": 2}[out]
    yf = np.empty((M, N), np.float32) if mode == 0 else None
    yq = np.empty((M, N), np.int8 if mode == 1 else np.uint8) if mode else None
    acc = np.empty((M, N), np.int32) if want_acc else None
    lib().oracle_qlinear(M, N, K, _ptr(a), int(a_is_u8), a_scale, a_zp, _ptr(w), w_zp, _ptr(ws),
                         _ptr(b), int(relu), mode, y_scale, y_zp, _ptr(yf), _ptr(yq), _ptr(acc))
    y = yf if mode == 0 else yq
    return (y, acc) if want_acc else y


def qepilogue(acc, a_scale, w_scale, bias=None, relu=False, out="int8", y_scale=1.0, y_zp=0):
    """Dequant / bias / ReLU / requant tail applied to exact accumulators."""
    acc = _c(acc, np.int64)
    M, N = acc.shape
    ws = _c(w_scale, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    mode = {"f32": 0, "int8": 1, "uint8": 2}[out]
    yf = np.empty((M, N), np.float32) if mode == 0 else None
    yq = np.empty((M, N), np.int8 if mode == 1 else np.uint8) if mode else None
    lib().oracle_qepilogue(M, N, _ptr(acc), a_scale, _ptr(ws), _ptr(b), int(relu), mode, y_scale,
                           y_zp, _ptr(yf), _ptr(yq))
    return yf if mode == 0 else yq


def quantize(x, scale, zp, out="int8"):
    x = _c(x, np.float32)
    u8 = out == "uint8"
    q = np.empty(x.shape, np.uint8 if u8 else np.int8)
    lib().oracle_quantize(x.size, _ptr(x), scale, zp, int(u8), _ptr(q))
    return q


def spmm_linear(indptr, indices, values, X, N):
    """Y[M,N] = X[M,K] W^T, W [N,K] CSR with int32 indptr/indices."""
    X = _c(X, np.float32)
    ip, ix, v = _c(indptr, np.int32), _c(indices, np.int32), _c(values, np.float32)
    M, K = X.shape
    Y = np.empty((M, N), np.float32)
    lib().oracle_spmm_linear(M, N, K, _ptr(ip), _ptr(ix), _ptr(v), _ptr(X), _ptr(Y))
    return Y


def spmm_linear_f64(indptr, indices, values, X, N):
    X = _c(X, np.float32)
    ip, ix, v = _c(indptr, np.int32), _c(indices, np.int32), _c(values, np.float32)
    M, K = X.shape
    Y = np.empty((M, N), np.float64)
    lib().oracle_spmm_linear_f64(M, N, K, _ptr(ip), _ptr(ix), _ptr(v), _ptr(X), _ptr(Y))
    return Y


def csr_spmm(indptr, indices, values, B):
    """Yt[R,C] = W[R,Kw] B[Kw,C] (reference orientation)."""
    B = _c(B, np.float32)
    ip, ix, v = _c(indptr, np.int32), _c(indices, np.int32), _c(values, np.float32)
    R = ip.size - 1
    Yt = np.empty((R, B.shape[1]), np.float32)
    lib().oracle_csr_spmm(R, B.shape[1], _ptr(ip), _ptr(ix), _ptr(v), _ptr(B), _ptr(Yt))
    return Yt


# ------------------------------------------------------ reference (compiled)
def ref_gemm(A, B, C=None, alpha=1.0, beta=1.0, trans_a=0, trans_b=0, nthreads=1):
    A, B = _c(A, np.float32), _c(B, np.float32)
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    Cc = None if C is None else _c(C, np.float32).ravel()
    Y = np.empty((M, N), np.float32)
    _check_ref(ref().pfref_gemm(M, N, K, trans_a, trans_b, alpha, beta, _ptr(A), _ptr(B), _ptr(Cc),
                                0 if Cc is None else Cc.size, _ptr(Y), nthreads))
    return Y


def ref_matmul(A, B, nthreads=1):
    A, B = _c(A, np.float32), _c(B, np.float32)
    Y = np.empty((A.shape[0], B.shape[1]), np.float32)
    _check_ref(ref().pfref_matmul(A.shape[0], B.shape[1], A.shape[1], _ptr(A), _ptr(B), _ptr(Y),
                                  nthreads))
    return Y


def ref_quantized_matmul(a, a_scale, a_zp, b, b_scale, b_zp, out="f32", y_scale=1.0, y_zp=0,
                         nthreads=1):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    M, K = a.shape
    N = b.shape[1]
    mode = {"f32": 0, "int8": 1, "uint8": 2}[out]
    y = np.empty((M, N), {0: np.float32, 1: np.int8, 2: np.uint8}[mode])
    _check_ref(ref().pfref_quantized_matmul(M, N, K, _ptr(a), int(a.dtype == np.uint8), a_scale,
                                            a_zp, _ptr(b), int(b.dtype == np.uint8), b_scale,
                                            b_zp, mode, y_scale, y_zp, _ptr(y), nthreads))
    return y


def ref_qlinear_per_channel(a, a_scale, a_zp, w, w_scale, w_zp=0, bias=None, relu=False,
                            out="int8", y_scale=1.0, y_zp=0):
    a, w = np.ascontiguousarray(a), _c(w, np.int8)
    M, K = a.shape
    N = w.shape[1]
    mode = {"f32": 0, "int8": 1, "uint8": 2}[out]
    y = np.empty((M, N), {0: np.float32, 1: np.int8, 2: np.uint8}[mode])
    ws = _c(w_scale, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    _check_ref(ref().pfref_qlinear_per_channel(M, N, K, _ptr(a), int(a.dtype == np.uint8), a_scale,
                                               a_zp, _ptr(w), w_zp, _ptr(ws), _ptr(b), int(relu),
                                               mode, y_scale, y_zp, _ptr(y)))
    return y


def ref_quantized_matmul_op(a, a_scale, a_zp, b, b_scale, b_zp):
    a, b = np.ascontiguousarray(a), _c(b, np.int8)
    M, K = a.shape
    N = b.shape[1]
    y = np.empty((M, N), np.float32)
    _check_ref(ref().pfref_quantized_matmul_op(M, N, K, _ptr(a), int(a.dtype == np.uint8), a_scale,
                                               a_zp, _ptr(b), b_scale, b_zp, _ptr(y)))
    return y


def ref_quantize(x, scale, zp, out="int8"):
    x = _c(x, np.float32)
    u8 = out == "uint8"
    q = np.empty(x.shape, np.uint8 if u8 else np.int8)
    _check_ref(ref().pfref_quantize(x.size, _ptr(x), scale, zp, int(u8), _ptr(q)))
    return q


def ref_sparse_matmul(indptr, indices, values, B, nthreads=1):
    """Reference sparse_matmul: W [R,Kw] CSR (int64 copies) times dense B [Kw,C]."""
    B = _c(B, np.float32)
    ip, ix, v = _c(indptr, np.int64), _c(indices, np.int64), _c(values, np.float32)
    R = ip.size - 1
    out = np.empty((R, B.shape[1]), np.float32)
    _check_ref(ref().pfref_sparse_matmul(R, B.shape[0], B.shape[1], _ptr(ip), _ptr(ix), _ptr(v),
                                         v.size, _ptr(B), _ptr(out), nthreads))
    return out


def magnitude_mask(w, sparsity):
    """Restated MagnitudePruning::compute_mask on W (any shape): 0/1 float mask."""
    w = _c(w, np.float32)
    mask = np.empty(w.shape, np.float32)
    rc = lib().oracle_magnitude_mask(w.size, _ptr(w), float(sparsity), _ptr(mask))
    if rc != 0:
        raise RuntimeError("Cannot prune empty weight tensor")
    return mask


def masked_csr(w, mask):
    """to_sparse(W * mask, 0, CSR) of W [rows, cols]: (indptr, indices, values) int32/int32/fp32."""
    w, mask = _c(w, np.float32), _c(mask, np.float32)
    rows, cols = w.shape
    nnz_max = int(np.count_nonzero(mask))
    ip = np.empty(rows + 1, np.int32)
    ix = np.empty(max(nnz_max, 1), np.int32)
    v = np.empty(max(nnz_max, 1), np.float32)
    lib().oracle_masked_csr(rows, cols, _ptr(w), _ptr(mask), _ptr(ip), _ptr(ix), _ptr(v))
    return ip, ix[: ip[-1]], v[: ip[-1]]


def ref_magnitude_mask(w, sparsity):
    w = _c(w, np.float32)
    rows, cols = (w.shape if w.ndim == 2 else (1, w.size))
    mask = np.empty(w.shape, np.float32)
    _check_ref(ref().pfref_magnitude_mask(rows, cols, _ptr(w), float(sparsity), _ptr(mask)))
    return mask


def nm_mask(w, n, m):
    """Restated NMSparsityPruning(n, m).compute_mask on W (flat order): 0/1 float mask."""
    w = _c(w, np.float32)
    mask = np.empty(w.shape, np.float32)
    if lib().oracle_nm_mask(w.size, _ptr(w), int(n), int(m), _ptr(mask)) != 0:
        raise ValueError("N:M pruning needs 0 < n <= m <= 64")
    return mask


def ref_nm_mask(w, n, m):
    w = _c(w, np.float32)
    mask = np.empty(w.shape, np.float32)
    _check_ref(ref().pfref_nm_mask(w.size, _ptr(w), int(n), int(m), _ptr(mask)))
    return mask


def ref_to_sparse_csr(d, threshold=0.0):
    d = _c(d, np.float32)
    rows, cols = d.shape
    cap = int(np.count_nonzero(np.abs(d) > threshold))
    ip = np.empty(rows + 1, np.int64)
    ix = np.empty(max(cap, 1), np.int64)
    v = np.empty(max(cap, 1), np.float32)
    nnz = np.zeros(1, np.int64)
    _check_ref(ref().pfref_to_sparse_csr(rows, cols, _ptr(d), float(threshold), cap, _ptr(ip), _ptr(ix), _ptr(v),
                                         _ptr(nnz)))
    return ip, ix[: nnz[0]], v[: nnz[0]]
