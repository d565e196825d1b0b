"""ctypes binding of oracle/_ref/libref_frame.so: the reference's own frame
protocol and model-producer kernels (TEST INFRASTRUCTURE ONLY).

The library is built by oracle/Makefile from the reference sources
(cuda/scan_frame.cu, cuda/model_producer.cu, src/postprocess.cpp) and needs a
CUDA driver to load, so only the GPU tests use it; `load()` returns None where
it is absent or cannot load.
"""
from __future__ import annotations

import ctypes
import os

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_frame.so")
_lib = None


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
    vp, sz, i, i64, u64 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64
    for name, args in (("ref_frame_load", []),
                       ("ref_frame_initialize", [vp, u64, vp, vp]),
                       ("ref_frame_begin", [vp, u64, i64, vp]),
                       ("ref_frame_gate", [vp, ctypes.POINTER(vp), ctypes.c_uint, vp, i64, vp]),
                       ("ref_frame_publish", [vp, vp, sz, vp, vp, vp, i64, vp]),
                       ("ref_frame_commit", [vp, vp]),
                       ("ref_frame_packet", [vp, vp, vp]),
                       ("ref_frame_check_finite", [vp, sz, vp, ctypes.c_uint32, vp]),
                       ("ref_model_producer", [vp, sz, ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(sz),
                                               ctypes.POINTER(sz), ctypes.POINTER(vp), vp, vp, sz, vp, i])):
        getattr(L, name).argtypes = args
        getattr(L, name).restype = i
    L.ref_frame_error.restype = ctypes.c_char_p
    L.ref_frame_digest.argtypes = [vp, sz]
    L.ref_frame_digest.restype = u64
    for name in ("ref_frame_control_bytes", "ref_frame_record_bytes", "ref_producer_workspace_bytes"):
        getattr(L, name).restype = sz
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(_lib.ref_frame_error().decode())


def ptrs(values) -> ctypes.Array:
    return (ctypes.c_void_p * max(len(values), 1))(*values)


def sizes(values) -> ctypes.Array:
    return (ctypes.c_size_t * len(values))(*values)
