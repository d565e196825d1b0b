"""Binary64 oracle of one Mamba block forward (TEST INFRASTRUCTURE ONLY).

Restates the reference's binary64 head block (src/head_reference.cpp:471-495:
linear :158-188, causal_conv1d :190-216, silu :221, selective_scan :363-430,
multiply :235, add :248) plus BASELINE's RMSNorm prologue (not in the
reference), computing in float64 and rounding to the activation dtype exactly
where the device pipeline stores an activation (x_in, z, u, dt, B, C, delta,
y, out), so that the comparison measures arithmetic, not storage choices.
(For dt_rank 8 or 16 the device forms delta inside the scan in FP32 and does
not store it, except in its fused chunk-parallel mode; the oracle still rounds
delta there, a perturbation below half an FP16 / BF16 ulp of delta that the
tests' 1e-3 + 1e-2 |ref| tolerance covers.)
The scan itself is the C oracle (oracle/scan_oracle.c), pinned to the
reference build.
"""
from __future__ import annotations

import numpy as np
import torch

from . import oracle

_TORCH = {"bf16": torch.bfloat16, "f16": torch.float16}


def rnd(a: np.ndarray, dt: str) -> np.ndarray:
    """Round to the activation dtype and back (what the device stores)."""
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(_TORCH[dt]).double().numpy()


def block_forward(x, p, dt: str, eps: float = 1e-5, residual: bool = True) -> np.ndarray:
    """x (B, L, d_model) float (already dtype-rounded); p: dict of float arrays."""
    x = np.asarray(x, np.float64)
    B, L, dm = x.shape
    D = p["w_in"].shape[0] // 2
    N = p["A"].shape[1]
    R = p["w_dt"].shape[1]
    f = lambda k: np.asarray(p[k], np.float64)
    xn = x
    if p.get("norm_w") is not None:
        r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
        xn = x * r * f("norm_w")
    xz = xn @ f("w_in").T                                   # in_proj (no bias)
    xin, z = rnd(xz[..., :D], dt), rnd(xz[..., D:], dt)
    w, K = f("conv_w"), p["conv_w"].shape[-1]
    conv = np.zeros_like(xin) + (f("conv_b") if p.get("conv_b") is not None else 0.0)
    for k in range(K):                                      # s = t + k - (K - 1), zero outside
        shift = K - 1 - k
        conv[:, shift:, :] += w[:, k] * xin[:, : L - shift, :]
    u = rnd(conv / (1.0 + np.exp(-conv)), dt)
    cw = p["w_x"].shape[0] - R - N                          # C width: N, or 1 (one C per token, the reference head)
    dbc = u @ f("w_x").T                                    # x_proj
    dtl, bm, cm = rnd(dbc[..., :R], dt), rnd(dbc[..., R:R + N], dt), rnd(dbc[..., R + N:R + N + cw], dt)
    delta = rnd(dtl @ f("w_dt").T, dt)                      # dt_proj (bias added in the scan)
    y, _ = oracle.scan_ex(u.astype(np.float32), delta.astype(np.float32), np.asarray(p["A"], np.float32),
                          bm[:, :, None, :].astype(np.float32), cm[:, :, None, :].astype(np.float32), layout="BLD",
                          d=np.asarray(p["D"], np.float32), z=z.astype(np.float32),
                          delta_bias=np.asarray(p["dt_bias"], np.float32), c_width=cw)
    y = rnd(y, dt)
    out = y @ f("w_out").T
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


def cross_block_forward(x, p, dt: str, eps: float = 1e-5, residual: bool = True) -> np.ndarray:
    """One Cross-Scan head level in binary64, in the reference's order
    (src/head_trt_network.cpp:200-232, steps 3-5): tokens = expand(x)
    (cuda/selective_scan.cu:157-175; exact in FP32), r_k = block(tokens_k)
    (+ tokens_k), out = merge(r) (:177-192).  x (B, C, H, W) float32; returns
    (B, C, H, W) float64.  The block sees the tokens rounded to the activation
    dtype (what the device's in_proj reads); the residual adds the FP32 tokens.
    The device reorders this by linearity (in_proj once per position, the
    merge before out_proj), so it agrees to rounding, not bit for bit."""
    x = np.ascontiguousarray(x, np.float32)
    B, C, H, W = x.shape
    L = H * W
    tokens = oracle.cross_scan_expand(x, B, C, H, W).reshape(4 * B, L, C).astype(np.float64)
    out = block_forward(rnd(tokens, dt), p, dt, eps, residual=False)
    if residual:
        out = out + tokens
    return oracle.cross_scan_merge(out, B, C, H, W).reshape(B, C, H, W)
