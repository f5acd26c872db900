"""Writing PyFlameRT .pfm model files from Python, and running them through
the reference's InferenceSession with the CUDA backend (libpfrt_session.so,
include/pfrt_session.h).

The writer produces the reference's on-disk layout
(src/io/pyflame_format.cpp:253-390, PyFlameFormat::save): magic "PFM\\0",
u32 version 1, the graph name, the inputs and outputs (name, u32 dtype,
u64 ndim, i64 dims), the initializers (name, u32 dtype, u64 ndim, i64 dims,
u64 byte count, bytes), then the nodes (name, op type, inputs, outputs,
attributes tagged 0 int64 / 1 float / 2 string / 3 int64 vector / 4 float
vector), little-endian throughout.
"""
from __future__ import annotations

import ctypes as C
import os
import struct

import numpy as np

# pyflame_rt::DType values (include/pyflame_rt/types.hpp)
DTYPES = {np.dtype(np.float32): 0, np.dtype(np.float64): 3, np.dtype(np.int64): 4, np.dtype(np.int32): 5,
          np.dtype(np.int16): 6, np.dtype(np.int8): 7, np.dtype(np.uint8): 8, np.dtype(np.bool_): 9}
NP_OF = {v: k for k, v in DTYPES.items()}


def _s(b: bytearray, text: str) -> None:
    raw = text.encode()
    b += struct.pack("<Q", len(raw)) + raw


def _info(b: bytearray, name: str, dtype, shape) -> None:
    _s(b, name)
    b += struct.pack("<IQ", DTYPES[np.dtype(dtype)], len(shape))
    for d in shape:
        b += struct.pack("<q", -1 if d is None else int(d))


def _attr(b: bytearray, name: str, v) -> None:
    _s(b, name)
    if isinstance(v, (bool, int, np.integer)):
        b += struct.pack("<Iq", 0, int(v))
    elif isinstance(v, (float, np.floating)):
        b += struct.pack("<If", 1, float(v))
    elif isinstance(v, str):
        b += struct.pack("<I", 2)
        _s(b, v)
    else:
        arr = np.asarray(v)
        if arr.dtype.kind in "iu":
            b += struct.pack("<IQ", 3, arr.size) + arr.astype("<i8").tobytes()
        else:
            b += struct.pack("<IQ", 4, arr.size) + arr.astype("<f4").tobytes()


def save(path: str, name: str, inputs, outputs, initializers: dict, nodes) -> None:
    """inputs/outputs: [(name, dtype, shape)]; initializers: {name: ndarray};
    nodes: [(name, op_type, [inputs], [outputs], {attr: value})]."""
    b = bytearray(b"PFM\0") + struct.pack("<I", 1)
    _s(b, name)
    for group in (inputs, outputs):
        b += struct.pack("<Q", len(group))
        for n, dt, shape in group:
            _info(b, n, dt, shape)
    b += struct.pack("<Q", len(initializers))
    for n, arr in initializers.items():
        arr = np.ascontiguousarray(arr)
        _info(b, n, arr.dtype, arr.shape)
        raw = arr.tobytes()
        b += struct.pack("<Q", len(raw)) + raw
    b += struct.pack("<Q", len(nodes))
    for n, op, ins, outs, attrs in nodes:
        _s(b, n)
        _s(b, op)
        for group in (ins, outs):
            b += struct.pack("<Q", len(group))
            for x in group:
                _s(b, x)
        b += struct.pack("<Q", len(attrs))
        for k, v in attrs.items():
            _attr(b, k, v)
    with open(path, "wb") as f:
        f.write(b)


def session_lib_path() -> str:
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libpfrt_session.so")


_SLIB = None


def _slib():
    global _SLIB
    if _SLIB is None:
        p = session_lib_path()
        if not os.path.exists(p):
            raise RuntimeError(f"{p} is not built (it needs the PyFlameRT sources: python -m pyflamert_b200.build)")
        L = C.CDLL(p)
        L.pfrt_session_open.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]
        L.pfrt_session_run.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_void_p),
                                       C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int64), C.c_int,
                                       C.POINTER(C.c_char_p), C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]
        L.pfrt_session_close.argtypes = [C.c_void_p]
        L.pfrt_session_close.restype = None
        L.pfrt_outputs_count.argtypes = [C.c_void_p]
        L.pfrt_outputs_get.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t),
                                       C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_int64)]
        L.pfrt_outputs_free.argtypes = [C.c_void_p]
        L.pfrt_outputs_free.restype = None
        _SLIB = L
    return _SLIB


class Session:
    """InferenceSession(pfm_path, device) through include/pfrt_session.h;
    run() takes and returns host numpy arrays, as session.run does."""

    def __init__(self, pfm_path: str, device: str = "cuda"):
        self._h = C.c_void_p()
        self._last = None
        err = C.create_string_buffer(4096)
        if _slib().pfrt_session_open(pfm_path.encode(), device.encode(), C.byref(self._h), err, 4096):
            raise RuntimeError(err.value.decode())

    def run(self, feeds: dict, output_names=(), copy=True):
        """feeds: {name: ndarray}.  Returns the outputs as numpy arrays (copies
        unless copy=False, which returns views of the session's output
        Tensors, valid until the next run() or close())."""
        self._release()
        names = list(feeds)
        arrs = [np.ascontiguousarray(feeds[n]) for n in names]
        n_in = len(names)
        c_names = (C.c_char_p * max(1, n_in))(*[n.encode() for n in names])
        c_data = (C.c_void_p * max(1, n_in))(*[a.ctypes.data for a in arrs])
        c_dt = (C.c_int32 * max(1, n_in))(*[DTYPES[a.dtype] for a in arrs])
        c_nd = (C.c_int32 * max(1, n_in))(*[a.ndim for a in arrs])
        dims = [d for a in arrs for d in a.shape]
        c_dims = (C.c_int64 * max(1, len(dims)))(*dims)
        outs = list(output_names)
        c_out = (C.c_char_p * max(1, len(outs)))(*[o.encode() for o in outs])
        res = C.c_void_p()
        err = C.create_string_buffer(4096)
        L = _slib()
        if L.pfrt_session_run(self._h, n_in, c_names, c_data, c_dt, c_nd, c_dims, len(outs), c_out,
                              C.byref(res), err, 4096):
            raise RuntimeError(err.value.decode())
        try:
            result = []
            for i in range(L.pfrt_outputs_count(res)):
                p, nb, dt, nd = C.c_void_p(), C.c_size_t(), C.c_int32(), C.c_int32()
                d8 = (C.c_int64 * 8)()
                L.pfrt_outputs_get(res, i, C.byref(p), C.byref(nb), C.byref(dt), C.byref(nd), d8)
                shape = tuple(d8[k] for k in range(nd.value))
                dtype = NP_OF[dt.value]
                if nb.value:
                    buf = (C.c_char * nb.value).from_address(p.value)
                    a = np.frombuffer(buf, dtype=dtype).reshape(shape)
                else:
                    a = np.zeros(shape, dtype)
                result.append(a.copy() if copy else a)
        finally:
            if copy:
                L.pfrt_outputs_free(res)
            else:
                self._last = res
        return result

    def _release(self):
        if self._last is not None:
            _slib().pfrt_outputs_free(self._last)
            self._last = None

    def close(self):
        self._release()
        if self._h:
            _slib().pfrt_session_close(self._h)
            self._h = C.c_void_p()
