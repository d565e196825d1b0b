"""CPU checks of the Mamba block oracle (oracle/mamba_oracle.py).

Its scan stage is the C oracle, bit-exact to the reference build
(tests/test_oracle.py).  Here its remaining stages are checked against a
loop-level restatement of the reference's binary64 primitives
(src/head_reference.cpp: linear :158-188, causal_conv1d :190-216, silu :221,
multiply :235, add :248), and the RMSNorm prologue against its definition.
"""
import numpy as np

from oracle import mamba_oracle as mo
from oracle import oracle


def loop_conv(x, w, b):
    B, L, C = x.shape
    K = w.shape[1]
    y = np.zeros_like(x)
    for bb in range(B):
        for t in range(L):
            for c in range(C):
                acc = 0.0
                for k in range(K):
                    s = t + k - (K - 1)
                    if 0 <= s < L:
                        acc += w[c, k] * x[bb, s, c]
                y[bb, t, c] = acc + b[c]
    return y


def test_block_oracle_matches_loop_restatement():
    dt = "f16"
    p = mo.random_block(3, 16, 16, 4, 8, 4, dt)
    p["A"] = p["A"][:, :4]
    x = mo.rnd(np.random.default_rng(1).standard_normal((2, 8, 16)) * 0.1, dt)
    got = mo.block_forward(x, p, dt)

    f = {k: np.asarray(v, np.float64) for k, v in p.items()}
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-5)
    xn = x * r * f["norm_w"]
    xz = np.einsum("blk,nk->bln", xn, f["w_in"])
    xin, z = mo.rnd(xz[..., :16], dt), mo.rnd(xz[..., 16:], dt)
    conv = loop_conv(xin, f["conv_w"], f["conv_b"])
    u = mo.rnd(conv * (1.0 / (1.0 + np.exp(-conv))), dt)
    dbc = np.einsum("bld,nd->bln", u, f["w_x"])
    dtl, bm, cm = mo.rnd(dbc[..., :8], dt), mo.rnd(dbc[..., 8:12], dt), mo.rnd(dbc[..., 12:16], dt)
    delta = mo.rnd(np.einsum("blr,dr->bld", dtl, f["w_dt"]), dt)
    y = np.zeros_like(u)
    for bb in range(2):
        for d in range(16):
            h = np.zeros(4)
            for t in range(8):
                dv = oracle.softplus(float(delta[bb, t, d]) + float(np.float32(p["dt_bias"][d])))
                h = np.exp(dv * f["A"][d]) * h + dv * bm[bb, t] * u[bb, t, d]
                acc = float(np.dot(cm[bb, t], h)) + f["D"][d] * u[bb, t, d]
                y[bb, t, d] = acc * z[bb, t, d] / (1 + np.exp(-z[bb, t, d]))
    want = np.einsum("bld,nd->bln", mo.rnd(y, dt), f["w_out"]) + x
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-12)


def test_cross_level_oracle_on_a_single_position():
    """On a 1 x 1 map the four Cross-Scan directions are the same one token, so
    the level oracle (expand -> block -> + tokens -> merge) must equal the block
    on that token plus x there."""
    p = mo.random_block(91, 128, 256, 16, 16, 4, "bf16", norm=False, c_width=1)
    x = (np.random.default_rng(92).standard_normal((2, 128, 1, 1)) * 0.5).astype(np.float32)
    got = mo.cross_block_forward(x, p, "bf16")
    tok = x.reshape(2, 1, 128).astype(np.float64)
    want = (mo.block_forward(mo.rnd(tok, "bf16"), p, "bf16", residual=False) + tok).reshape(2, 128, 1, 1)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_cross_level_oracle_direction_symmetry():
    """On a 1 x W map directions 0 and 3 (identity, flip H) see the row in map
    order and directions 1 and 2 (flip H and W, flip W) the reversed row: the
    level is the merge of the block over the row and over the reversed row,
    read back in map order."""
    p = mo.random_block(93, 128, 256, 16, 16, 4, "bf16", norm=False, c_width=1)
    W = 6
    x = (np.random.default_rng(94).standard_normal((1, 128, 1, W)) * 0.5).astype(np.float32)
    got = mo.cross_block_forward(x, p, "bf16")
    tok = np.transpose(x[0, :, 0, :]).astype(np.float64)[None]                # (1, W, 128) in map order
    fwd = mo.block_forward(mo.rnd(tok, "bf16"), p, "bf16", residual=False) + tok
    rev = mo.block_forward(mo.rnd(tok[:, ::-1].copy(), "bf16"), p, "bf16", residual=False) + tok[:, ::-1]
    want = (((fwd[0] + rev[0, ::-1]) + rev[0, ::-1]) + fwd[0]) * 0.25       # merge order: k = 0, 1, 2, 3
    np.testing.assert_allclose(got[0, :, 0, :], np.transpose(want), rtol=1e-12, atol=1e-12)
