"""ctypes access to the reference's own binary64 head (TEST INFRASTRUCTURE ONLY).

oracle/_ref/libref_head.so is src/head_reference.cpp and its dependencies from
the reference checkout, compiled by oracle/Makefile with ref_head_shim.cpp;
it exists where the checkout was present at build time.  Used by the CPU
tests that pin oracle/mamba_oracle.py and by tests/golden/make_head_golden.py.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_head.so")
_lib = None
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)
_MSG = 1024

HEAD_LEVELS = ("p3", "p4", "p5")
PROFILES = {"t01": 0, "hr": 1}


def available() -> bool:
    return os.path.exists(_PATH)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(_PATH)
        i64, sz, cp = ctypes.c_int64, ctypes.c_size_t, ctypes.c_char_p
        L.sacc_ref_head_run.argtypes = [ctypes.c_uint64, cp, ctypes.c_uint64, ctypes.c_int, cp, sz]
        L.sacc_ref_head_tensor.argtypes = [cp, _i64p, ctypes.POINTER(ctypes.c_int), _f64p, _f64p, cp, sz]
        L.sacc_ref_head_weight.argtypes = [cp, _i64p, ctypes.POINTER(ctypes.c_int), _f32p, cp, sz]
        L.sacc_ref_head_linear.argtypes = [_f64p, i64, i64, _f32p, i64, _f32p, _f64p, _f64p, cp, sz]
        L.sacc_ref_head_causal_conv1d.argtypes = [_f64p, i64, i64, i64, _f32p, i64, _f32p, _f64p, cp, sz]
        L.sacc_ref_head_silu.argtypes = [_f64p, i64, _f64p, cp, sz]
        L.sacc_ref_head_multiply.argtypes = [_f64p, _f64p, i64, _f64p, cp, sz]
        L.sacc_ref_head_add.argtypes = [_f64p, _f64p, i64, _f64p, cp, sz]
        L.sacc_ref_head_selective_scan.argtypes = [_f64p] * 5 + [_f32p, i64, i64, i64, i64, _f64p, _f64p, cp, sz]
        L.sacc_ref_head_softplus.restype = ctypes.c_double
        L.sacc_ref_head_softplus.argtypes = [ctypes.c_double]
        _lib = L
    return _lib


def _d(a):
    a = np.ascontiguousarray(a, np.float64)
    return a, a.ctypes.data_as(_f64p)


def _f(a):
    if a is None:
        return None, ctypes.cast(None, _f32p)
    a = np.ascontiguousarray(a, np.float32)
    return a, a.ctypes.data_as(_f32p)


def _call(fn, *args):
    msg = ctypes.create_string_buffer(_MSG)
    rc = fn(*args, msg, _MSG)
    if rc != 0:
        raise RuntimeError(msg.value.decode())


def run_head(weight_seed: int, kind: str, feature_seed: int, profile: str) -> None:
    """head_reference on synthetic_head_weights(weight_seed) and head_test_features(kind, feature_seed, profile),
    intermediates kept for tensor() / weight()."""
    _call(lib().sacc_ref_head_run, weight_seed, kind.encode(), feature_seed, PROFILES[profile])


def tensor(name: str, want_sigma: bool = False):
    """Intermediate `name` of the last run_head ("p5.tokens", ...): binary64 values (and scales)."""
    shape = (ctypes.c_int64 * 4)()
    rank = ctypes.c_int(0)
    _call(lib().sacc_ref_head_tensor, name.encode(), shape, ctypes.byref(rank), None, None)
    dims = tuple(shape[i] for i in range(rank.value))
    v = np.zeros(dims, np.float64)
    s = np.zeros(dims, np.float64)
    _call(lib().sacc_ref_head_tensor, name.encode(), shape, ctypes.byref(rank), v.ctypes.data_as(_f64p), s.ctypes.data_as(_f64p))
    return (v, s) if want_sigma else v


def weight(name: str) -> np.ndarray:
    """FP32 parameter `name` of the last run_head's weights ("p5.mamba.in_proj.weight", ...)."""
    shape = (ctypes.c_int64 * 4)()
    rank = ctypes.c_int(0)
    _call(lib().sacc_ref_head_weight, name.encode(), shape, ctypes.byref(rank), None)
    dims = tuple(shape[i] for i in range(rank.value))
    v = np.zeros(dims, np.float32)
    _call(lib().sacc_ref_head_weight, name.encode(), shape, ctypes.byref(rank), v.ctypes.data_as(_f32p))
    return v


def block_params(level: str) -> dict:
    """The Mamba block parameters of `level` in the block oracle's naming (A as A_log, rank-1 C, no RMSNorm)."""
    m = level + ".mamba."
    return {"w_in": weight(m + "in_proj.weight"), "conv_w": weight(m + "conv1d.weight")[:, 0, :],
            "conv_b": weight(m + "conv1d.bias"), "w_x": weight(m + "x_proj.weight"), "w_dt": weight(m + "dt_proj.weight"),
            "dt_bias": weight(m + "dt_proj.bias"), "A_log": weight(m + "A_log"), "D": weight(m + "D"),
            "w_out": weight(m + "out_proj.weight")}


def linear(x, w, bias=None) -> np.ndarray:
    x, xp = _d(x)
    w, wp = _f(w)
    b, bp = _f(bias)
    y = np.zeros(x.shape[:-1] + (w.shape[0],), np.float64)
    _call(lib().sacc_ref_head_linear, xp, x.size // x.shape[-1], x.shape[-1], wp, w.shape[0], bp, y.ctypes.data_as(_f64p),
          ctypes.cast(None, _f64p))
    return y


def causal_conv1d(x, w, bias) -> np.ndarray:
    """x (B, L, C), w (C, K), bias (C)."""
    x, xp = _d(x)
    w, wp = _f(w)
    b, bp = _f(bias)
    y = np.zeros_like(x)
    _call(lib().sacc_ref_head_causal_conv1d, xp, x.shape[0], x.shape[1], x.shape[2], wp, w.shape[-1], bp, y.ctypes.data_as(_f64p))
    return y


def silu(x) -> np.ndarray:
    x, xp = _d(x)
    y = np.zeros_like(x)
    _call(lib().sacc_ref_head_silu, xp, x.size, y.ctypes.data_as(_f64p))
    return y


def multiply(a, b) -> np.ndarray:
    a, ap = _d(a)
    b, bp = _d(b)
    y = np.zeros_like(a)
    _call(lib().sacc_ref_head_multiply, ap, bp, a.size, y.ctypes.data_as(_f64p))
    return y


def add(a, b) -> np.ndarray:
    a, ap = _d(a)
    b, bp = _d(b)
    y = np.zeros_like(a)
    _call(lib().sacc_ref_head_add, ap, bp, a.size, y.ctypes.data_as(_f64p))
    return y


def selective_scan(u, delta, a, b, c, d=None, want_sigma: bool = False):
    """u, delta (B, L, Dc); a (N,) shared; b (B, L, N); c (B, L, 1); d (Dc) or None; delta already holds the bias."""
    u, up = _d(u)
    dl, dp = _d(delta)
    a, ap = _d(np.reshape(a, -1))
    b, bp = _d(b)
    c, cp = _d(c)
    dd, ddp = _f(d)
    y = np.zeros_like(u)
    s = np.zeros_like(u)
    _call(lib().sacc_ref_head_selective_scan, up, dp, ap, bp, cp, ddp, u.shape[0], u.shape[1], u.shape[2], a.size,
          y.ctypes.data_as(_f64p), s.ctypes.data_as(_f64p))
    return (y, s) if want_sigma else y


def softplus(x: float) -> float:
    return lib().sacc_ref_head_softplus(x)
