"""ctypes front end of the CPU oracle (oracle/scan_oracle.c) and of the
reference's own CPU scan built into oracle/_ref/libref_scan.so.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm may import this module; the product path in
saccade_v1_b200/ never does.

Case generators restate the reference's test fixtures:
  filled / varied / gen   tests/selective_scan_tests.cpp:99-106, 222-233
  Random / random_case    tests/scan_cuda_suite.hpp:145-165 (xorshift64)
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field, replace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(HERE, "liboracle.so")
_REF = os.path.join(HERE, "_ref", "libref_scan.so")

OK, INVALID, RANGE = 0, 1, 2


class _Shape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_uint64), ("length", ctypes.c_uint64), ("channels", ctypes.c_uint64),
                ("state", ctypes.c_uint64), ("a_rows", ctypes.c_uint64), ("c_width", ctypes.c_uint64),
                ("has_d", ctypes.c_int32)]


class _ExShape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_uint64), ("length", ctypes.c_uint64), ("channels", ctypes.c_uint64),
                ("state", ctypes.c_uint64), ("groups", ctypes.c_uint64), ("c_width", ctypes.c_uint64),
                ("a_rows", ctypes.c_uint64), ("layout", ctypes.c_int32), ("has_d", ctypes.c_int32),
                ("has_z", ctypes.c_int32), ("has_bias", ctypes.c_int32), ("apply_softplus", ctypes.c_int32),
                ("has_h0", ctypes.c_int32), ("want_final", ctypes.c_int32), ("nseq", ctypes.c_int32)]


_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int32)
_lib = None
_ref = None


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference checkout is present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build()
        L = ctypes.CDLL(_LIB)
        L.sacc_oracle_softplus.restype = ctypes.c_double
        L.sacc_oracle_softplus.argtypes = [ctypes.c_double]
        L.sacc_oracle_scan_ref.restype = ctypes.c_int
        L.sacc_oracle_scan_ref.argtypes = [ctypes.POINTER(_Shape)] + [_f32p, ctypes.c_size_t] * 6 + [
            _f64p, ctypes.c_char_p, ctypes.c_size_t]
        L.sacc_oracle_scan_bound.restype = None
        L.sacc_oracle_scan_bound.argtypes = [ctypes.POINTER(_Shape)] + [_f32p] * 6 + [_f64p]
        L.sacc_oracle_scan_ex.restype = None
        L.sacc_oracle_scan_ex.argtypes = [ctypes.POINTER(_ExShape)] + [_f32p] * 9 + [_i32p, _f64p, _f64p, _f64p]
        L.sacc_oracle_silu.argtypes = [_f64p, ctypes.c_size_t, _f64p]
        L.sacc_oracle_neg_exp.argtypes = [_f32p, ctypes.c_size_t, _f64p]
        L.sacc_oracle_scan_ex_f64.argtypes = [ctypes.POINTER(_ExShape)] + [_f64p] * 5 + [_f32p, _f64p] + [_f32p] * 2 + [
            _i32p, _f64p, _f64p, _f64p]
        L.sacc_oracle_cross_scan_source.restype = ctypes.c_size_t
        L.sacc_oracle_cross_scan_source.argtypes = [ctypes.c_size_t] * 4
        L.sacc_oracle_cross_scan_expand.restype = None
        L.sacc_oracle_cross_scan_expand.argtypes = [_f32p] + [ctypes.c_size_t] * 4 + [_f32p]
        L.sacc_oracle_cross_scan_merge.restype = None
        L.sacc_oracle_cross_scan_merge.argtypes = [_f64p] + [ctypes.c_size_t] * 4 + [_f64p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF)


def ref_lib():
    """The reference's own selective_scan_reference (oracle/_ref), or None."""
    global _ref
    if _ref is None and ref_available():
        R = ctypes.CDLL(_REF)
        R.sacc_ref_selective_scan.restype = ctypes.c_int
        R.sacc_ref_selective_scan.argtypes = [ctypes.POINTER(_Shape)] + [_f32p, ctypes.c_size_t] * 6 + [
            _f64p, ctypes.c_char_p, ctypes.c_size_t]
        R.sacc_ref_selective_scan_threads.restype = ctypes.c_int
        R.sacc_ref_selective_scan_threads.argtypes = [ctypes.POINTER(_Shape)] + [_f32p] * 6 + [_f64p, ctypes.c_int]
        R.sacc_ref_softplus.restype = ctypes.c_double
        R.sacc_ref_softplus.argtypes = [ctypes.c_double]
        _ref = R
    return _ref


def _fp(a):
    if a is None or a.size == 0:
        return ctypes.cast(None, _f32p)
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _dp(a):
    if a is None or a.size == 0:
        return ctypes.cast(None, _f64p)
    assert a.dtype == np.float64 and a.flags.c_contiguous
    return a.ctypes.data_as(_f64p)


# ----------------------------------------------------------------- cases

@dataclass
class Shape:
    """(batch, length, channels, state, a_rows, c_width, has_d), include/saccade/selective_scan.hpp:19-27."""
    batch: int
    length: int
    channels: int
    state: int
    a_rows: int = 1
    c_width: int = 1
    has_d: bool = True

    def c(self) -> _Shape:
        return _Shape(self.batch, self.length, self.channels, self.state, self.a_rows, self.c_width, int(self.has_d))


def _f32(v):
    return np.ascontiguousarray(np.asarray(v, dtype=np.float32).reshape(-1))


@dataclass
class Case:
    shape: Shape
    u: np.ndarray
    delta: np.ndarray
    a: np.ndarray
    b: np.ndarray
    c: np.ndarray
    d: np.ndarray = field(default_factory=lambda: np.zeros(0, np.float32))

    def __post_init__(self):
        for k in ("u", "delta", "a", "b", "c", "d"):
            setattr(self, k, _f32(getattr(self, k)))

    def copy(self) -> "Case":
        return Case(replace(self.shape), self.u.copy(), self.delta.copy(), self.a.copy(), self.b.copy(),
                    self.c.copy(), self.d.copy())

    def inputs(self):
        return self.u, self.delta, self.a, self.b, self.c, self.d


def filled(s: Shape, u: float, delta: float, b: float, c: float) -> Case:
    """tests/selective_scan_tests.cpp:99-104 (A defaults to -1, D to 0)."""
    tokens = s.batch * s.length
    return Case(s, np.full(tokens * s.channels, u, np.float32), np.full(tokens * s.channels, delta, np.float32),
                np.full(s.a_rows * s.state, -1.0, np.float32), np.full(tokens * s.state, b, np.float32),
                np.full(tokens * s.c_width, c, np.float32),
                np.zeros(s.channels if s.has_d else 0, np.float32))


def gen(a: int, m: int, offset: int, scale: float) -> np.float32:
    """tests/selective_scan_tests.cpp:106 (C++ % on non-negative a)."""
    return np.float32(np.float32(a % m - offset) / np.float32(scale))


def _gen_vec(idx, m, offset, scale):
    idx = np.asarray(idx, dtype=np.int64)
    return ((idx % m - offset).astype(np.float32) / np.float32(scale)).astype(np.float32)


def varied(s: Shape) -> Case:
    """tests/selective_scan_tests.cpp:222-233."""
    k = filled(s, 0, 0, 0, 0)
    i = np.arange(k.u.size)
    k.u = _gen_vec(5 * i + 1, 11, 5, 4)
    k.delta = _gen_vec(3 * i + 2, 13, 6, 2)
    k.b = _gen_vec(7 * np.arange(k.b.size) + 3, 9, 4, 4)
    k.c = _gen_vec(3 * np.arange(k.c.size) + 1, 7, 3, 2)
    ia = np.arange(k.a.size)
    k.a = (-((ia % s.state) + 1).astype(np.float32) / np.float32(4)).astype(np.float32)
    k.d = _gen_vec(np.arange(k.d.size), 3, 1, 2)
    return k


class Random:
    """Deterministic xorshift64, tests/scan_cuda_suite.hpp:147-153."""
    M = (1 << 64) - 1

    def __init__(self, seed: int):
        self.state = seed & self.M

    def next_raw(self) -> int:
        s = self.state
        s ^= (s << 13) & self.M
        s ^= s >> 7
        s ^= (s << 17) & self.M
        self.state = s
        return s

    def uniform_array(self, n: int, lo: float, hi: float) -> np.ndarray:
        # lo + (hi - lo) * float(double(state >> 40) * 2^-24), all in FP32 as the C++ does.
        raw = np.fromiter((self.next_raw() >> 40 for _ in range(n)), dtype=np.float64, count=n)
        frac = (raw * 2.0 ** -24).astype(np.float32)
        return (np.float32(lo) + np.float32(np.float32(hi) - np.float32(lo)) * frac).astype(np.float32)


@dataclass
class Ranges:
    """tests/scan_cuda_suite.hpp:154."""
    u: float = 2
    delta_lo: float = -6
    delta_hi: float = 3
    a_lo: float = -4
    a_hi: float = -0.05
    bc: float = 1.5
    d: float = 1


def random_case(s: Shape, seed: int, r: Ranges | None = None) -> Case:
    """tests/scan_cuda_suite.hpp:155-165: u, delta, a, b, c, d drawn in that order."""
    r = r or Ranges()
    g = Random(seed)
    k = filled(s, 0, 0, 0, 0)
    k.u = g.uniform_array(k.u.size, -r.u, r.u)
    k.delta = g.uniform_array(k.delta.size, r.delta_lo, r.delta_hi)
    k.a = g.uniform_array(k.a.size, r.a_lo, r.a_hi)
    k.b = g.uniform_array(k.b.size, -r.bc, r.bc)
    k.c = g.uniform_array(k.c.size, -r.bc, r.bc)
    k.d = g.uniform_array(k.d.size, -r.d, r.d)
    return k


# ------------------------------------------------------------- wrappers

def softplus(x: float) -> float:
    return lib().sacc_oracle_softplus(float(x))


def _out_count(s: Shape) -> int:
    n = s.batch * s.length * s.channels
    return n if n < 2 ** 31 else 0  # over capacity: rejected before any write


def scan_ref(k: Case):
    """Oracle restatement of selective_scan_reference: (status, y float64, message)."""
    s = k.shape
    y = np.zeros(_out_count(s), np.float64)
    msg = ctypes.create_string_buffer(512)
    args = []
    for t in k.inputs():
        args += [_fp(t), t.size]
    st = lib().sacc_oracle_scan_ref(ctypes.byref(s.c()), *args, _dp(y), msg, 512)
    return st, y, msg.value.decode()


def scan_reference_impl(k: Case):
    """The reference's own selective_scan_reference (oracle/_ref): (status, y, message)."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("oracle/_ref/libref_scan.so is not built")
    s = k.shape
    y = np.zeros(_out_count(s), np.float64)
    msg = ctypes.create_string_buffer(512)
    args = []
    for t in k.inputs():
        args += [_fp(t), t.size]
    st = R.sacc_ref_selective_scan(ctypes.byref(s.c()), *args, _dp(y), msg, 512)
    return st, y, msg.value.decode()


def run(k: Case) -> np.ndarray:
    st, y, msg = scan_ref(k)
    if st != OK:
        raise ValueError(msg)
    return y


def scan_bound(k: Case) -> np.ndarray:
    s = k.shape
    out = np.zeros(s.batch * s.length * s.channels, np.float64)
    lib().sacc_oracle_scan_bound(ctypes.byref(s.c()), *[_fp(t) for t in k.inputs()], _dp(out))
    return out


def scan_ex(u, delta, a, b, c, *, layout: str = "BLD", d=None, z=None, delta_bias=None, softplus: bool = True,
            h0=None, want_final: bool = False, cu_seqlens=None, groups: int = 1, c_width: int | None = None,
            want_scale: bool = False, exact: bool = False):
    """Extended scan in binary64 (see scan_oracle.c sacc_oracle_scan_ex).

    Shapes, layout "BLD": u/delta/z (B, L, D); b (B, L, G, N); c (B, L, G, CW).
    Layout "BDL": u/delta/z (B, D, L); b (B, G, N, L); c (B, G, CW, L).
    a (D or 1, N); d, delta_bias (D,); h0 (nseq, D, N).
    Returns (y float64 with u's shape, h_final float64 (nseq, D, N) or None),
    plus the per-element term magnitude sum_n |C h| + |D u| (times |silu(z)|)
    when want_scale.  exact: u, delta, a, b, c and z are taken as binary64
    values (sacc_oracle_scan_ex_f64) instead of being rounded to FP32 first.
    """
    act = np.float64 if exact else np.float32
    u = np.ascontiguousarray(u, act)
    if layout == "BLD":
        B, L, D = u.shape
        N = b.shape[-1]
        CW = c.shape[-1] if c_width is None else c_width
    else:
        B, D, L = u.shape
        N = b.shape[-2]
        CW = c.shape[-2] if c_width is None else c_width
    a = np.ascontiguousarray(a, act).reshape(-1, N)
    nseq = (len(cu_seqlens) - 1) if cu_seqlens is not None else B
    sh = _ExShape(B, L, D, N, groups, CW, a.shape[0], 0 if layout == "BLD" else 1, int(d is not None),
                  int(z is not None), int(delta_bias is not None), int(softplus), int(h0 is not None),
                  int(want_final), nseq)
    y = np.zeros(u.shape, np.float64)
    sc = np.zeros(u.shape, np.float64) if want_scale else None
    hf = np.zeros((nseq, D, N), np.float64) if want_final else None
    conv = lambda t: None if t is None else np.ascontiguousarray(t, np.float32)
    cu = None if cu_seqlens is None else np.ascontiguousarray(cu_seqlens, np.int32)
    if exact:
        convd = lambda t: None if t is None else np.ascontiguousarray(t, np.float64)
        fn = lib().sacc_oracle_scan_ex_f64
        ptrs = [_dp(u), _dp(convd(delta)), _dp(a), _dp(convd(b)), _dp(convd(c)), _fp(conv(d)), _dp(convd(z)),
                _fp(conv(delta_bias)), _fp(conv(h0))]
    else:
        fn = lib().sacc_oracle_scan_ex
        tensors = [u, conv(delta), a, conv(b), conv(c), conv(d), conv(z), conv(delta_bias), conv(h0)]
        ptrs = [_fp(t) for t in tensors]
    fn(ctypes.byref(sh), *ptrs,
                              ctypes.cast(None, _i32p) if cu is None else cu.ctypes.data_as(_i32p),
                              _dp(y), _dp(hf) if hf is not None else ctypes.cast(None, _f64p),
                              _dp(sc) if sc is not None else ctypes.cast(None, _f64p))
    return (y, hf, sc) if want_scale else (y, hf)


def silu(x) -> np.ndarray:
    """x sigmoid(x) in binary64, the reference head's form (src/head_reference.cpp:54-58, :221-232)."""
    x = np.ascontiguousarray(x, np.float64)
    y = np.empty_like(x)
    lib().sacc_oracle_silu(_dp(x), x.size, _dp(y))
    return y


def neg_exp(a_log) -> np.ndarray:
    """A = -exp(A_log) in binary64 from FP32 A_log (src/head_reference.cpp:347-354)."""
    a_log = np.ascontiguousarray(a_log, np.float32)
    a = np.empty(a_log.shape, np.float64)
    lib().sacc_oracle_neg_exp(_fp(a_log), a_log.size, _dp(a))
    return a


def cross_scan_source(direction: int, token: int, height: int, width: int) -> int:
    r = lib().sacc_oracle_cross_scan_source(direction, token, height, width)
    if r == (1 << 64) - 1:
        raise ValueError("cross_scan: token or direction out of range")
    return r


def cross_scan_expand(x, batch, channels, height, width) -> np.ndarray:
    x = _f32(x)
    out = np.zeros(4 * x.size, np.float32)
    lib().sacc_oracle_cross_scan_expand(_fp(x), batch, channels, height, width, _fp(out))
    return out


def cross_scan_merge(y, batch, channels, height, width) -> np.ndarray:
    y = np.ascontiguousarray(y, np.float64).reshape(-1)
    out = np.zeros(y.size // 4, np.float64)
    lib().sacc_oracle_cross_scan_merge(_dp(y), batch, channels, height, width, _dp(out))
    return out
