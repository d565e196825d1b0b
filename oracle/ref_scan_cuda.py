"""ctypes binding of oracle/_ref/libref_scan_cuda.so: the reference's own CUDA
FP32 selective scan (cuda/selective_scan.cu) built for sm_100a
(TEST INFRASTRUCTURE ONLY).

Needs a CUDA driver to load, so only GPU tests use it; `load()` returns None
where it is absent or cannot load.
"""
from __future__ import annotations

import ctypes
import os

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_scan_cuda.so")
_lib = None


class Shape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_uint64), ("length", ctypes.c_uint64), ("channels", ctypes.c_uint64),
                ("state", ctypes.c_uint64), ("a_rows", ctypes.c_uint64), ("c_width", ctypes.c_uint64),
                ("has_d", ctypes.c_int32)]


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(PATH):
        return None
    try:
        L = ctypes.CDLL(PATH)
    except OSError:
        return None
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    L.ref_scan_cuda_load.argtypes = [ctypes.c_char_p, sz]
    L.ref_scan_cuda.argtypes = [ctypes.POINTER(Shape)] + [vp] * 9 + [ctypes.c_char_p, sz]
    _lib = L
    msg = ctypes.create_string_buffer(4096)
    if L.ref_scan_cuda_load(msg, 4096) != 0:
        raise RuntimeError(msg.value.decode())
    return _lib


def scan(shape: Shape, u, delta, a, b, c, d, y, status, stream) -> None:
    """saccade::selective_scan_cuda of the reference on device pointers (ints) and a stream handle."""
    msg = ctypes.create_string_buffer(1024)
    if load().ref_scan_cuda(ctypes.byref(shape), u, delta, a, b, c, d, y, status, stream, msg, 1024) != 0:
        raise RuntimeError(msg.value.decode())
