"""Binary64 oracle of one Mamba block forward (TEST INFRASTRUCTURE ONLY).

Restates the reference's binary64 head block (src/head_reference.cpp:471-495:
linear :158-188, causal_conv1d :190-216, silu :221-232, selective_scan
:363-430, multiply :235, add :248) plus BASELINE's RMSNorm prologue (not in
the reference).

Two modes, by the `dt` argument:
  "f64"          the reference's arithmetic bit for bit: every linear summed
                 over its inputs in index order, the conv taps in order before
                 the bias, silu as x sigmoid(x) with the C library's exp, the
                 scan on binary64 activations (oracle/scan_oracle.c), A as
                 -exp(A_log) when the parameters carry "A_log".  Pinned to the
                 reference's own build (oracle/_ref/libref_head.so) by
                 tests/test_block_oracle_ref.py, stage by stage and for the
                 whole block and head level.
  "bf16" / "f16" the comparator of the device pipeline: the same stages
                 (linears as one BLAS product: a reordering of the same sum,
                 within a few ulp of the sequential one), rounding to the
                 activation dtype exactly where the device stores an
                 activation (x_in, z, u, dt, B, C, delta, y, out), so that the
                 comparison measures arithmetic, not storage choices.
                 (For dt_rank 8 or 16 the device forms delta inside the scan in
                 FP32 and does not store it, except in its fused chunk-parallel
                 mode; the oracle still rounds delta there, a perturbation below
                 half an FP16 / BF16 ulp of delta that the tests'
                 1e-3 + 1e-2 |ref| tolerance covers.)
The scan itself is the C oracle (oracle/scan_oracle.c), pinned to the
reference build.
"""
from __future__ import annotations

import numpy as np
import torch

from . import oracle

_TORCH = {"bf16": torch.bfloat16, "f16": torch.float16}


def rnd(a: np.ndarray, dt: str) -> np.ndarray:
    """Round to the activation dtype and back (what the device stores); "f64" keeps binary64."""
    if dt == "f64":
        return np.asarray(a, np.float64)
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(_TORCH[dt]).double().numpy()


def linear(x, w, exact: bool = False) -> np.ndarray:
    """y[..., o] = sum_i w[o, i] x[..., i] in binary64 (no bias).  exact: the
    terms added in index order as head_ref::linear (src/head_reference.cpp:158-188),
    bit for bit; otherwise one BLAS product."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    if not exact:
        return x @ w.T
    acc = np.zeros(x.shape[:-1] + (w.shape[0],), np.float64)
    for i in range(w.shape[1]):
        acc += x[..., i:i + 1] * w[:, i]
    return acc


def causal_conv1d(x, w, b) -> np.ndarray:
    """x (B, L, C) along L, w (C, K), b (C) or None: y[t] = sum_k w[k] x[t + k - (K - 1)] + b, zero for
    t + k - (K - 1) < 0; the taps added in k order before the bias (src/head_reference.cpp:190-216)."""
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64)
    L, K = x.shape[1], w.shape[-1]
    acc = np.zeros_like(x)
    for k in range(K):
        shift = K - 1 - k
        acc[:, shift:, :] += w[:, k] * x[:, : L - shift, :]
    return acc + (np.asarray(b, np.float64) if b is not None else 0.0)


def silu(x) -> np.ndarray:
    """x sigmoid(x) (src/head_reference.cpp:221-232), the C library's exp."""
    return oracle.silu(x)


def a_matrix(p) -> np.ndarray:
    """A (rows, N): -exp(A_log) in binary64 when the parameters carry "A_log"
    (src/head_reference.cpp:347-354), else the given A."""
    if p.get("A_log") is not None:
        return oracle.neg_exp(p["A_log"])
    return np.asarray(p["A"], np.float32)


def block_forward(x, p, dt: str, eps: float = 1e-5, residual: bool = True, stages: dict | None = None) -> np.ndarray:
    """x (B, L, d_model) float (already dtype-rounded in the 16-bit modes); p: dict of float arrays
    ("A" or "A_log", "norm_w" optional).  stages, when given, receives each intermediate."""
    exact = dt == "f64"
    x = np.asarray(x, np.float64)
    B, L, dm = x.shape
    D = p["w_in"].shape[0] // 2
    N = (p["A_log"] if p.get("A_log") is not None else p["A"]).shape[1]
    R = p["w_dt"].shape[1]
    keep = (lambda k, v: stages.__setitem__(k, v)) if stages is not None else (lambda k, v: None)
    xn = x
    if p.get("norm_w") is not None:
        r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
        xn = x * r * np.asarray(p["norm_w"], np.float64)
    xz = linear(xn, p["w_in"], exact)                                        # in_proj (no bias)
    keep("in_proj", xz)
    xin, z = rnd(xz[..., :D], dt), rnd(xz[..., D:], dt)
    conv = causal_conv1d(xin, p["conv_w"], p.get("conv_b"))
    keep("conv1d", conv)
    u = rnd(silu(conv), dt)
    keep("u", u)
    cw = p["w_x"].shape[0] - R - N                                           # C width: N, or 1 (one C per token, the reference head)
    dbc = linear(u, p["w_x"], exact)                                         # x_proj
    keep("x_proj", dbc)
    dtl, bm, cm = rnd(dbc[..., :R], dt), rnd(dbc[..., R:R + N], dt), rnd(dbc[..., R + N:R + N + cw], dt)
    delta = rnd(linear(dtl, p["w_dt"], exact), dt)                           # dt_proj (bias added in the scan)
    keep("delta", delta + (np.asarray(p["dt_bias"], np.float64) if p.get("dt_bias") is not None else 0.0))
    act = np.float64 if exact else np.float32
    y, _ = oracle.scan_ex(u.astype(act), delta.astype(act), a_matrix(p), bm[:, :, None, :].astype(act),
                          cm[:, :, None, :].astype(act), layout="BLD", d=np.asarray(p["D"], np.float32),
                          z=z.astype(act), delta_bias=None if p.get("dt_bias") is None else np.asarray(p["dt_bias"], np.float32),
                          c_width=cw, exact=exact)
    keep("gate", y)
    y = rnd(y, dt)
    out = linear(y, p["w_out"], exact)                                       # out_proj (no bias)
    keep("out_proj", out)
    if residual:
        out = out + x
    return out


def random_block(seed: int, d_model: int, d_inner: int, d_state: int, dt_rank: int, d_conv: int, dt: str,
                 norm: bool = True, c_width: int | None = None):
    """Synthetic block weights: uniform +-1/sqrt(fan_in) (as the reference's synthetic head weights,
    include/saccade/head_reference.hpp:125-127), A = -(1..N), D = 1, dt_bias = softplus^-1(logU[1e-3, 1e-1])."""
    r = np.random.default_rng(seed)
    u = lambda shape, fan: r.uniform(-1, 1, shape) / np.sqrt(fan)
    p = {
        "w_in": rnd(u((2 * d_inner, d_model), d_model), dt),
        "conv_w": u((d_inner, d_conv), d_conv).astype(np.float32),
        "conv_b": u((d_inner,), d_conv).astype(np.float32),
        "w_x": rnd(u((dt_rank + d_state + (d_state if c_width is None else c_width), d_inner), d_inner), dt),
        "w_dt": rnd(u((d_inner, dt_rank), dt_rank), dt),
        "dt_bias": np.log(np.expm1(np.exp(r.uniform(np.log(1e-3), np.log(1e-1), d_inner)))).astype(np.float32),
        "A": -np.tile(np.arange(1, d_state + 1, dtype=np.float32), (d_inner, 1)),
        "D": np.ones(d_inner, np.float32),
        "w_out": rnd(u((d_model, d_inner), d_inner), dt),
    }
    if norm:
        p["norm_w"] = (1.0 + 0.1 * r.standard_normal(d_model)).astype(np.float32)
    return p


def cross_expand(x) -> np.ndarray:
    """(B, C, H, W) -> (4 B, H W, C), direction-major (row k B + b): direction k of image b reads the k-flipped
    map in row-major order (0 identity, 1 flip H and W, 2 flip W, 3 flip H; src/head_reference.cpp:306-318,
    src/selective_scan.cpp:111 cross_scan_source), any float dtype."""
    x = np.asarray(x)
    B, C, H, W = x.shape
    flips = [x, x[:, :, ::-1, ::-1], x[:, :, :, ::-1], x[:, :, ::-1, :]]
    t = np.stack([f.reshape(B, C, H * W).transpose(0, 2, 1) for f in flips], axis=0)  # (4, B, L, C)
    return np.ascontiguousarray(t.reshape(4 * B, H * W, C))


def cross_merge(y, B, C, H, W) -> np.ndarray:
    """(4 B, H W, C) -> (B, C, H, W): each direction mapped back, (((y0 + y1) + y2) + y3) / 4
    (src/head_reference.cpp:322-345), binary64."""
    y = np.asarray(y, np.float64).reshape(4, B, H, W, C)
    back = [y[0], y[1, :, ::-1, ::-1], y[2, :, :, ::-1], y[3, :, ::-1, :]]
    s = ((back[0] + back[1]) + back[2]) + back[3]
    return np.ascontiguousarray((s / 4).transpose(0, 3, 1, 2))


def cross_block_forward(x, p, dt: str, eps: float = 1e-5, residual: bool = True) -> np.ndarray:
    """One Cross-Scan head level in binary64, in the reference's order
    (src/head_trt_network.cpp:200-232, steps 3-5; src/head_reference.cpp:469-495):
    tokens = expand(x), r_k = block(tokens_k) (+ tokens_k), out = merge(r).
    x (B, C, H, W); returns (B, C, H, W) float64.  In the 16-bit modes x is
    FP32, the block sees the tokens rounded to the activation dtype (what the
    device's in_proj reads) and the residual adds the FP32 tokens; the device
    reorders this by linearity (in_proj once per position, the merge before
    out_proj), so it agrees to rounding, not bit for bit.  In "f64" x may be
    any binary64 map (the reference's downsample output) and the level is the
    reference's own arithmetic."""
    x = np.asarray(x, np.float64 if dt == "f64" else np.float32)
    B, C, H, W = x.shape
    tokens = cross_expand(x).astype(np.float64)
    out = block_forward(rnd(tokens, dt), p, dt, eps, residual=False)
    if residual:
        out = out + tokens
    return cross_merge(out, B, C, H, W)
