"""The block oracle (oracle/mamba_oracle.py) pinned to the reference's own binary64 head.

oracle/_ref/libref_head.so is the reference's src/head_reference.cpp (with
head_weights, torch_checkpoint, sha256, file_io) compiled from the reference
checkout by oracle/Makefile.  In its "f64" mode the block oracle must equal it
BIT FOR BIT:
  * stage by stage on random inputs: linear (:158-188), causal_conv1d
    (:190-216), silu (:221-232), the gate multiply(y, silu(z)) (:235, :490),
    the selective scan (:363-430) and A = -exp(A_log) (:347-354);
  * on the reference's complete head (head_reference :434-441 on
    synthetic_head_weights and head_test_features, the T01 and HR profiles):
    every kept intermediate of each level's Mamba block (in_proj, conv1d, u,
    x_proj, delta, gate, out_proj), the block output with the residual and the
    Cross-Scan level's merged map;
  * at BASELINE config 1's dimensions (dt_rank 8; d_model 128, d_inner 256,
    N 16, L 32), against the reference's primitives composed in the order of
    src/head_reference.cpp:471-494 (rank-1 C and a shared A, as that scan
    takes them).
The BLAS linear of the 16-bit modes is held to the reordered-summation bound of
the sequential one, and the 16-bit comparator (rounding where the device
stores) to the device tolerance 1e-3 + 1e-2 |ref| of the reference.
tests/golden/head_ref_p5.npz (tests/golden/make_head_golden.py) repeats the
head check without the reference build.
"""
import os

import numpy as np
import pytest

from oracle import mamba_oracle as mo
from oracle import oracle
from oracle import ref_head as rh

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "head_ref_p5.npz")
STAGES = ("in_proj", "conv1d", "u", "x_proj", "delta", "gate", "out_proj")

needs_ref = pytest.mark.skipif(not rh.available(), reason="oracle/_ref/libref_head.so not built (no reference checkout)")


def same(name, got, want):
    got = np.asarray(got, np.float64).reshape(np.shape(want))
    assert np.array_equal(got, want), f"{name}: {int(np.sum(got != want))} of {got.size} differ, max |d| {np.max(np.abs(got - want)):.3g}"


@needs_ref
def test_stages_bitwise_on_random_inputs():
    r = np.random.default_rng(7)
    x = r.standard_normal((3, 29, 40))
    w = (r.uniform(-1, 1, (24, 40)) / np.sqrt(40)).astype(np.float32)
    b = r.uniform(-0.5, 0.5, 24).astype(np.float32)
    same("linear", mo.linear(x, w, exact=True), rh.linear(x, w))
    same("linear+bias", mo.linear(x, w, exact=True) + b.astype(np.float64), rh.linear(x, w, b))
    # The BLAS product reorders the same sum: within the reordered-summation bound I eps sum |w x|.
    mag = np.abs(x) @ np.abs(w.astype(np.float64)).T
    assert np.all(np.abs(mo.linear(x, w) - rh.linear(x, w)) <= 40 * 2.0 ** -53 * mag * 2)
    cw = (r.uniform(-1, 1, (40, 4)) / 2).astype(np.float32)
    cb = r.uniform(-0.5, 0.5, 40).astype(np.float32)
    same("causal_conv1d", mo.causal_conv1d(x, cw, cb), rh.causal_conv1d(x, cw, cb))
    v = np.concatenate([r.standard_normal(2000) * 6, [0.0, -0.0, 745.0, -745.0, 30.0, -30.0, 1e-300]])
    same("silu", mo.silu(v), rh.silu(v))
    a_log = np.log(np.arange(1, 17, dtype=np.float64)).astype(np.float32)[None, :]
    a = mo.a_matrix({"A_log": a_log})
    assert np.array_equal(a, -np.exp(a_log.astype(np.float64)))  # one exp per value, no rounding in between


@needs_ref
@pytest.mark.parametrize("L,D", [(1, 8), (37, 16), (200, 24)])
def test_scan_and_gate_bitwise(L, D):
    """Rank-1 C, A shared by all channels, D skip: head_ref::selective_scan on binary64 activations, then
    multiply(y, silu(z)), against the C oracle's binary64 scan with the gate fused."""
    r = np.random.default_rng(L)
    B, N = 2, 16
    u, z = r.standard_normal((B, L, D)), r.standard_normal((B, L, D)) * 3
    delta = r.standard_normal((B, L, D)) - 3
    bm, cm = r.standard_normal((B, L, N)), r.standard_normal((B, L, 1))
    a = -np.exp(r.uniform(-1, 1.5, N))
    dsk = r.standard_normal(D).astype(np.float32)
    y_ref = rh.multiply(rh.selective_scan(u, delta, a, bm, cm, dsk), rh.silu(z))
    y, _ = oracle.scan_ex(u, delta, a[None, :], bm[:, :, None, :], cm[:, :, None, :], layout="BLD", d=dsk, z=z,
                          c_width=1, exact=True)
    same("scan+gate", y, y_ref)
    y_plain, _ = oracle.scan_ex(u, delta, a[None, :], bm[:, :, None, :], cm[:, :, None, :], layout="BLD", d=dsk, c_width=1,
                                exact=True)
    same("scan", y_plain, rh.selective_scan(u, delta, a, bm, cm, dsk))


def check_level(level, stages_too=True):
    p = rh.block_params(level)
    st = {}
    out = mo.block_forward(rh.tensor(level + ".tokens"), p, "f64", stages=st)
    if stages_too:
        for k in STAGES:
            same(f"{level}.{k}", st[k], rh.tensor(f"{level}.{k}"))
    same(f"{level}.residual", out, rh.tensor(level + ".residual"))
    same(f"{level}.merge", mo.cross_block_forward(rh.tensor(level + ".downsample"), p, "f64"), rh.tensor(level + ".merge"))
    return p


@needs_ref
def test_reference_head_t01_levels_bitwise():
    """T01 640x640: P3 (4 x 400 tokens), P4 (4 x 100), P5 (4 x 25)."""
    rh.run_head(3, "random", 1, "t01")
    for level in rh.HEAD_LEVELS:
        check_level(level)


@needs_ref
def test_reference_head_hr_levels_bitwise():
    """HR 1280x768, the deployed shapes: P3 (4 x 960 tokens), P4 (4 x 240), P5 (4 x 60); other weights and
    features."""
    rh.run_head(5, "asymmetric", 2, "hr")
    for level in rh.HEAD_LEVELS:
        check_level(level, stages_too=level == "p5")


def reference_block(x, p):
    """The reference's block from its own primitives, in the order of src/head_reference.cpp:471-494."""
    D = p["w_in"].shape[0] // 2
    R = p["w_dt"].shape[1]
    N = p["A_log"].shape[1]
    xz = rh.linear(x, p["w_in"])
    xs, z = xz[..., :D], xz[..., D:]
    u = rh.silu(rh.causal_conv1d(xs, p["conv_w"], p["conv_b"]))
    dbc = rh.linear(u, p["w_x"])
    dt, bm, cm = dbc[..., :R], dbc[..., R:R + N], dbc[..., R + N:R + N + 1]
    delta = rh.linear(dt, p["w_dt"], p["dt_bias"])
    a = -np.exp(p["A_log"].astype(np.float64)).reshape(-1)
    y = rh.selective_scan(u, delta, a, bm, cm, p["D"])
    o = rh.linear(rh.multiply(y, rh.silu(z)), p["w_out"])
    return rh.add(o, x)


@needs_ref
def test_config1_dimensions_bitwise():
    """BASELINE config 1's block dimensions (d_model 128, d_inner 256, N 16, dt_rank 8, L 32) on 6 tracks, with
    the reference scan's rank-1 C and shared A."""
    r = np.random.default_rng(11)
    dm, D, N, R = 128, 256, 16, 8
    p = mo.random_block(12, dm, D, N, R, 4, "f16", norm=False, c_width=1)
    p = {k: np.asarray(v, np.float32) for k, v in p.items()}
    p.pop("A")
    p["A_log"] = np.log(np.arange(1, N + 1, dtype=np.float64)).astype(np.float32)[None, :]
    x = r.standard_normal((6, 32, dm)) * 0.1
    same("config1_block", mo.block_forward(x, p, "f64"), reference_block(x, p))


@needs_ref
def test_16bit_comparator_within_device_tolerance_of_reference():
    """The 16-bit comparator (fp16 weights and activations rounded where the device stores them) against the
    reference's binary64 block: within the device tolerance 1e-3 + 1e-2 |ref| used by the GPU tests."""
    rh.run_head(3, "random", 1, "t01")
    p = rh.block_params("p4")
    tok = rh.tensor("p4.tokens")
    ref = rh.tensor("p4.residual")
    p16 = dict(p)
    for k in ("w_in", "w_x", "w_dt", "w_out"):
        p16[k] = mo.rnd(p[k], "f16")
    got = mo.block_forward(mo.rnd(tok, "f16"), p16, "f16", residual=False) + tok
    err = np.abs(got - ref)
    assert np.all(err <= 1e-3 + 1e-2 * np.abs(ref)), float(np.max(err / (1e-3 + 1e-2 * np.abs(ref))))


def test_golden_head_level_bitwise():
    """tests/golden/head_ref_p5.npz (the reference's own head, T01 P5 level): the binary64 block oracle on the
    recorded tokens and downsampled map reproduces the recorded block output and merged map bit for bit."""
    g = np.load(GOLDEN)
    p = {k[2:]: g[k] for k in g.files if k.startswith("w.")}
    same("golden.residual", mo.block_forward(g["tokens"], p, "f64"), g["residual"])
    same("golden.merge", mo.cross_block_forward(g["downsample"], p, "f64"), g["merge"])
