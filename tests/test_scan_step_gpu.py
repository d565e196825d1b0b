"""GPU parity of the per-frame step (sacc_selective_scan_step).

The step is the reference recurrence (src/selective_scan.cpp:88-107) applied
to one token from carried state.  It is pinned by:
  - the oracle's extended scan with L = 1, initial and final state;
  - T consecutive steps == one T-token scan from the same initial state;
  - a slot map: each sequence updates only its own state row, a negative slot
    skips the sequence (y = 0) and leaves every row untouched.
Tolerances: 16-bit outputs 1e-3 + 1e-2 |ref|; FP32 state rtol 1e-4 / atol 1e-5
(state is computed from the same 16-bit-rounded inputs); FP32 activations use
the library exp (rtol 1e-5).
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import saccade_v1_b200 as sb  # noqa: E402

TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def rounded(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(TORCH[dt]).float().numpy()


def make(seed, nseq, D, N, dt, G=1, c_full=True):
    r = np.random.default_rng(seed)
    f = lambda *s: r.standard_normal(s).astype(np.float32)
    t = dict(u=f(nseq, D), delta=f(nseq, D), z=f(nseq, D), b=f(nseq, G, N), c=f(nseq, G, N if c_full else 1))
    for k in list(t):
        t[k] = rounded(t[k], dt)
    t["bias"] = np.log(np.expm1(np.exp(r.uniform(np.log(1e-3), np.log(1e-1), D)))).astype(np.float32)
    t["A"] = -np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1))
    t["D"] = np.ones(D, np.float32)
    t["h0"] = (r.standard_normal((nseq, D, N)) * 0.5).astype(np.float32)
    return t


def gpu_step(t, dt, state, slot=None, s=None):
    s = s or torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = lambda k: torch.from_numpy(np.ascontiguousarray(t[k])).to(device="cuda", dtype=TORCH[dt])
        f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
        y = sb.selective_scan_step(g("u"), g("delta"), f(t["A"]), g("b"), g("c"), state, D=f(t["D"]), z=g("z"),
                                   delta_bias=f(t["bias"]), slot=slot, stream=s)
    s.synchronize()
    return y.float().cpu().numpy()


def oracle_step(t, h0):
    # one token per sequence: (nseq, 1, D) in BLD with B/C (nseq, 1, G, N)
    u = t["u"][:, None, :]
    y, hf = oracle.scan_ex(u, t["delta"][:, None, :], t["A"], t["b"][:, None], t["c"][:, None], layout="BLD",
                           d=t["D"], z=t["z"][:, None, :], delta_bias=t["bias"], h0=h0, want_final=True,
                           groups=t["b"].shape[1])
    return y[:, 0, :], hf


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("N", [16, 8, 32, 4])
def test_step_matches_oracle(dt, N):
    t = make(N, 48, 256, N, dt)
    state = torch.from_numpy(t["h0"].copy()).cuda()
    y = gpu_step(t, dt, state)
    ry, rh = oracle_step(t, t["h0"])
    if dt == "f32":
        np.testing.assert_allclose(y, ry, rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(state.cpu().numpy(), rh, rtol=1e-5, atol=1e-6)
    else:
        assert np.all(np.abs(y - ry) <= 1e-3 + 1e-2 * np.abs(ry))
        np.testing.assert_allclose(state.cpu().numpy(), rh, rtol=1e-4, atol=1e-5)


def test_steps_chain_into_a_scan():
    """T single-token steps from h0 == one T-token scan from h0 (carried state)."""
    T, nseq, D, N = 6, 16, 128, 16
    ts = [make(100 + k, nseq, D, N, "f16") for k in range(T)]
    for t in ts[1:]:  # per-channel parameters are fixed across frames
        t["bias"] = ts[0]["bias"]
    h0 = ts[0]["h0"]
    state = torch.from_numpy(h0.copy()).cuda()
    ys = [gpu_step(t, "f16", state) for t in ts]
    stack = lambda k: np.stack([t[k] for t in ts], axis=1)
    ry, rh = oracle.scan_ex(stack("u"), stack("delta"), ts[0]["A"], stack("b"), stack("c"), layout="BLD",
                            d=ts[0]["D"], z=stack("z"), delta_bias=ts[0]["bias"], h0=h0, want_final=True)
    got = np.stack(ys, axis=1)
    assert np.all(np.abs(got - ry) <= 1e-3 + 1e-2 * np.abs(ry))
    np.testing.assert_allclose(state.cpu().numpy(), rh, rtol=1e-4, atol=1e-5)


def test_slot_map_updates_only_named_rows():
    nseq, slots, D, N = 12, 20, 128, 16
    t = make(7, nseq, D, N, "f16")
    rng = np.random.default_rng(8)
    rows = rng.permutation(slots)[:nseq].astype(np.int32)
    rows[3] = -1  # skipped sequence
    table = (rng.standard_normal((slots, D, N)) * 0.5).astype(np.float32)
    state = torch.from_numpy(table.copy()).cuda()
    y = gpu_step(t, "f16", state, slot=torch.from_numpy(rows).cuda())
    ry, rh = oracle_step(t, table[np.maximum(rows, 0)])
    got = state.cpu().numpy()
    for i, r in enumerate(rows):
        if r < 0:
            assert np.all(y[i] == 0)
            continue
        assert np.all(np.abs(y[i] - ry[i]) <= 1e-3 + 1e-2 * np.abs(ry[i]))
        np.testing.assert_allclose(got[r], rh[i], rtol=1e-4, atol=1e-5)
    untouched = sorted(set(range(slots)) - set(int(r) for r in rows if r >= 0))
    assert np.array_equal(got[untouched], table[untouched])


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_step16_rank1_c_groups_shared_a_ragged(dt):
    """The 16-bit N = 16 path with rank-1 C, 3 groups, one shared A row and a
    lane count that fills no whole grid."""
    nseq, D, N, G = 37, 384, 16, 3
    t = make(41, nseq, D, N, dt, G=G, c_full=False)
    t["A"] = t["A"][:1].copy() * 0.37
    state = torch.from_numpy(t["h0"].copy()).cuda()
    y = gpu_step(t, dt, state)
    u = t["u"][:, None, :]
    ry, rh = oracle.scan_ex(u, t["delta"][:, None, :], t["A"], t["b"][:, None], t["c"][:, None], layout="BLD", d=t["D"],
                            z=t["z"][:, None, :], delta_bias=t["bias"], h0=t["h0"], want_final=True, groups=G,
                            c_width=1)
    assert np.all(np.abs(y - ry[:, 0, :]) <= 1e-3 + 1e-2 * np.abs(ry[:, 0, :]))
    np.testing.assert_allclose(state.cpu().numpy(), rh, rtol=1e-4, atol=1e-5)


def offset_view(t):
    """The same values at an address 2 bytes past a 16-byte boundary."""
    wide = torch.zeros(t.numel() + 1, dtype=t.dtype, device=t.device)
    wide[1:] = t.reshape(-1)
    return wide[1:].view(t.shape)


def step_variants(t, dt, table, slot, G=1):
    """The same step through the three kernels: TMA-pipelined (all operands
    16-byte aligned), one-thread-per-lane (z 2 bytes off a 16-byte boundary,
    which the pipelined kernel's bulk copies cannot take) and the generic
    four-threads-per-lane kernel (B 2 bytes off, which rules out both)."""
    s = torch.cuda.Stream()
    outs = []
    with torch.cuda.stream(s):
        g = lambda k: torch.from_numpy(np.ascontiguousarray(t[k])).to(device="cuda", dtype=TORCH[dt])
        f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
        slot = None if slot is None else torch.from_numpy(slot).cuda()
        b, z = g("b"), g("z")
        for bb, zz in ((b, z), (b, offset_view(z)), (offset_view(b), z)):
            st = torch.from_numpy(table.copy()).cuda()
            y = sb.selective_scan_step(g("u"), g("delta"), f(t["A"]), bb, g("c"), st, D=f(t["D"]), z=zz,
                                       delta_bias=f(t["bias"]), slot=slot, stream=s)
            outs.append((y, st))
    s.synchronize()
    return outs


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_step_kernels_agree_bitwise(dt):
    """All three step kernels apply the same operations in the same order, so
    outputs and states agree bit for bit.  Slot map with an arbitrary negative
    entry and an out-of-table one (both skipped, y = 0)."""
    nseq, D, N, slots = 300, 256, 16, 310
    t = make(43, nseq, D, N, dt)
    rng = np.random.default_rng(44)
    rows = rng.permutation(slots)[:nseq].astype(np.int32)
    rows[5], rows[9] = -7, slots + 3
    table = (rng.standard_normal((slots, D, N)) * 0.5).astype(np.float32)
    outs = step_variants(t, dt, table, rows)
    y0, s0 = outs[0]
    for y1, s1 in outs[1:]:
        assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))
        assert torch.equal(s0.view(torch.int32), s1.view(torch.int32))
    assert bool((y0[5] == 0).all()) and bool((y0[9] == 0).all())
    untouched = sorted(set(range(slots)) - set(int(r) for r in rows if 0 <= r < slots))
    assert np.array_equal(s0.cpu().numpy()[untouched], table[untouched])
    ry, rh = oracle_step(t, table[np.clip(rows, 0, slots - 1)])
    live = [i for i, r in enumerate(rows) if 0 <= r < slots]
    yv = y0.float().cpu().numpy()
    assert np.all(np.abs(yv[live] - ry[live]) <= 1e-3 + 1e-2 * np.abs(ry[live]))
    np.testing.assert_allclose(s0.cpu().numpy()[rows[live]], rh[live], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_step_pipe_partial_channel_block_and_groups(dt):
    """384 channels = one full and one half 256-channel tile (rows past the
    table's channels are zero-filled on load and not stored), 3 groups."""
    nseq, D, N, G = 260, 384, 16, 3
    t = make(47, nseq, D, N, dt, G=G)
    outs = step_variants(t, dt, t["h0"], None, G)
    y0, s0 = outs[0]
    for y1, s1 in outs[1:]:
        assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))
        assert torch.equal(s0.view(torch.int32), s1.view(torch.int32))
    u = t["u"][:, None, :]
    ry, rh = oracle.scan_ex(u, t["delta"][:, None, :], t["A"], t["b"][:, None], t["c"][:, None], layout="BLD", d=t["D"],
                            z=t["z"][:, None, :], delta_bias=t["bias"], h0=t["h0"], want_final=True, groups=G)
    yv = y0.float().cpu().numpy()
    assert np.all(np.abs(yv - ry[:, 0, :]) <= 1e-3 + 1e-2 * np.abs(ry[:, 0, :]))
    np.testing.assert_allclose(s0.cpu().numpy(), rh, rtol=1e-4, atol=1e-5)
    assert sb.scan_fault() == 0


def test_config3_scale_property():
    """Config 3 size (4096 tracks x 256 x 16, fp16): sampled tracks against the oracle."""
    nseq, D, N = 4096, 256, 16
    t = make(3, nseq, D, N, "f16")
    state = torch.from_numpy(t["h0"].copy()).cuda()
    y = gpu_step(t, "f16", state)
    pick = np.random.default_rng(4).integers(0, nseq, 24)
    sub = {k: (v[pick] if k in ("u", "delta", "z", "b", "c", "h0") else v) for k, v in t.items()}
    ry, rh = oracle_step(sub, sub["h0"])
    assert np.all(np.abs(y[pick] - ry) <= 1e-3 + 1e-2 * np.abs(ry))
    np.testing.assert_allclose(state.cpu().numpy()[pick], rh, rtol=1e-4, atol=1e-5)


def test_step_rejections():
    s = torch.cuda.Stream()
    u = torch.zeros(4, 128, dtype=torch.float16, device="cuda")
    A = torch.zeros(128, 16, device="cuda")
    B = torch.zeros(4, 16, dtype=torch.float16, device="cuda")
    state = torch.zeros(4, 128, 16, device="cuda")
    with pytest.raises(sb.ScanInvalidArgument, match="non-default stream"):
        sb.selective_scan_step(u, u, A, B, B, state, stream=0)
    alias = state.view(torch.float16).reshape(-1)[:512].view(4, 128)
    with pytest.raises(sb.ScanInvalidArgument, match="state overlaps y"):
        sb.selective_scan_step(u, u, A, B, B, state, out=alias, stream=s)
    with pytest.raises(sb.ScanInvalidArgument, match="power of two"):
        sb.selective_scan_step(u, u, torch.zeros(128, 3, device="cuda"), B[:, :3].contiguous(), B[:, :3].contiguous(),
                               torch.zeros(4, 128, 3, device="cuda"), stream=s)
