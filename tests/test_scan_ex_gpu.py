"""GPU parity of the extended scan (sacc_selective_scan_ex) against the oracle.

Tolerances (fixed before the first GPU run):
  fp32 activations: |gpu - ref| <= max(2 E, 1e-5 S) + 1e-5 |ref|, where E is
      the reference's running error bound (oracle scan_bound) when the case is
      expressible in the reference ABI and S the term magnitude
      sum_n |C h| + |D u| (times |silu(z)|), i.e. rtol 1e-5 with an absolute
      floor on the scale rounding errors grow with;
  bf16 / fp16 activations: |gpu - ref| <= 1e-3 + 1e-2 |ref| against the
      binary64 oracle on the same 16-bit-rounded inputs (FP32 state).
Extensions are pinned by contract equalities derived from the reference
recurrence: state chaining across a split, packed varlen == separate calls,
L = 1 step == last row of a rescan, BDL == transposed BLD.
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
    """FP32 value of x after rounding to dtype dt (what the device reads)."""
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(TORCH[dt]).float().numpy()


def make(seed, B, L, D, N, G=1, layout="BDL", dt="bf16", c_full=True, a_rows=None, spread=1.0):
    """BASELINE config-0 distributions: u, z, B, C, dt_pre ~ N(0,1); dt_bias = softplus^-1(logU[1e-3, 1e-1]);
    A[d, n] = -(n + 1); D = 1."""
    r = np.random.default_rng(seed)
    f = lambda *s: (r.standard_normal(s) * spread).astype(np.float32)
    if layout == "BDL":
        u, delta, z = f(B, D, L), f(B, D, L), f(B, D, L)
        b, c = f(B, G, N, L), f(B, G, N if c_full else 1, L)
    else:
        u, delta, z = f(B, L, D), f(B, L, D), f(B, L, D)
        b, c = f(B, L, G, N), f(B, L, G, N if c_full else 1)
    dtb = np.exp(r.uniform(np.log(1e-3), np.log(1e-1), D))
    bias = np.log(np.expm1(dtb)).astype(np.float32)
    A = -np.tile(np.arange(1, N + 1, dtype=np.float32), (D if a_rows is None else a_rows, 1))
    Dv = np.ones(D, np.float32)
    t = dict(u=u, delta=delta, z=z, b=b, c=c, bias=bias, A=A, D=Dv)
    for k in ("u", "delta", "z", "b", "c"):
        t[k] = rounded(t[k], dt)
    return t


def gpu_run(t, dt, layout, use=("D", "z", "bias"), h0=None, want_final=False, cu=None, stream=None):
    s = stream or torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = lambda k: torch.from_numpy(np.ascontiguousarray(t[k])).to(device="cuda", dtype=TORCH[dt])
        f32 = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
        nseq = t["u"].shape[0] if cu is None else len(cu) - 1
        N = t["A"].shape[1]
        hf = torch.full((nseq, t["D"].size, N), np.nan, device="cuda") if want_final else None
        y = sb.selective_scan_ex(g("u"), g("delta"), f32(t["A"]), g("b"), g("c"),
                                 D=f32(t["D"]) if "D" in use else None, z=g("z") if "z" in use else None,
                                 delta_bias=f32(t["bias"]) if "bias" in use else None, h0=f32(h0), h_final=hf,
                                 cu_seqlens=None if cu is None else torch.tensor(cu, dtype=torch.int32, device="cuda"),
                                 layout=layout, stream=s)
    s.synchronize()
    return y.float().cpu().numpy(), (hf.cpu().numpy() if hf is not None else None)


def oracle_run(t, layout, use=("D", "z", "bias"), h0=None, want_final=False, cu=None, groups=1):
    return oracle.scan_ex(t["u"], t["delta"], t["A"], t["b"], t["c"], layout=layout,
                          d=t["D"] if "D" in use else None, z=t["z"] if "z" in use else None,
                          delta_bias=t["bias"] if "bias" in use else None, h0=h0, want_final=want_final,
                          cu_seqlens=cu, groups=groups, want_scale=True)


def check_16bit(name, gpu, ref):
    err = np.abs(gpu.astype(np.float64) - ref)
    tol = 1e-3 + 1e-2 * np.abs(ref)
    bad = ~(err <= tol)
    assert not bad.any(), f"{name}: {int(bad.sum())}/{gpu.size} beyond 1e-3 + 1e-2|ref|; max err {err.max():.3g}"


def check_f32(name, gpu, ref, scale, bound=None):
    floor = 1e-5 * scale if bound is None else np.maximum(2 * bound, 1e-5 * scale)
    err = np.abs(gpu.astype(np.float64) - ref)
    tol = floor + 1e-5 * np.abs(ref)
    bad = ~(err <= tol)
    assert not bad.any(), f"{name}: {int(bad.sum())}/{gpu.size} beyond tolerance; max err {err.max():.3g}"


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("layout", ["BDL", "BLD"])
def test_16bit_matches_oracle(dt, layout):
    for seed, (B, L, D, N, G) in enumerate([(1, 16, 64, 16, 1), (2, 37, 48, 16, 2), (3, 129, 32, 8, 1),
                                            (2, 64, 64, 32, 1), (1, 10, 24, 4, 1)]):
        t = make(seed, B, L, D, N, G, layout, dt)
        y, _ = gpu_run(t, dt, layout)
        ref, _, _ = oracle_run(t, layout, groups=G)
        check_16bit(f"{dt}_{layout}_{B}x{L}x{D}x{N}", y, ref)


def test_config0_fp32_with_final_state():
    """B=1, D=64, L=16, N=16, fp32, y (B,D,L) and final state (B,D,N)."""
    t = make(0, 1, 16, 64, 16, 1, "BDL", "f32")
    y, hf = gpu_run(t, "f32", "BDL", want_final=True)
    ref, hr, scale = oracle_run(t, "BDL", want_final=True)
    check_f32("config0_y", y, ref, scale)
    np.testing.assert_allclose(hf, hr, rtol=1e-5, atol=1e-6)


def test_fp32_reduces_to_reference_abi():
    """No bias / gate / state: the extended scan is the reference operator."""
    k = oracle.random_case(oracle.Shape(2, 37, 5, 16, 5, 16, True), 0x5eed0701)
    s = k.shape
    t = dict(u=k.u.reshape(2, 37, 5), delta=k.delta.reshape(2, 37, 5), b=k.b.reshape(2, 37, 1, 16),
             c=k.c.reshape(2, 37, 1, 16), A=k.a.reshape(5, 16), D=k.d, z=None, bias=None)
    y, _ = gpu_run(t, "f32", "BLD", use=("D",))
    check_f32("ref_abi", y.reshape(-1), oracle.run(k), np.abs(oracle.run(k)), oracle.scan_bound(k))


@pytest.mark.parametrize("layout", ["BDL", "BLD"])
def test_state_chains_across_split(layout):
    t = make(5, 2, 50, 32, 16, 1, layout, "f32")
    h0 = np.random.default_rng(1).standard_normal((2, 32, 16)).astype(np.float32) * 0.5
    y, hf = gpu_run(t, "f32", layout, h0=h0, want_final=True)
    ref, hr, scale = oracle_run(t, layout, h0=h0, want_final=True)
    check_f32("full", y, ref, scale)
    cut = 21
    ax = 2 if layout == "BDL" else 1
    sl = lambda a, lo, hi: np.ascontiguousarray(np.take(a, np.arange(lo, hi), axis=ax))
    part = lambda lo, hi: dict(t, u=sl(t["u"], lo, hi), delta=sl(t["delta"], lo, hi), z=sl(t["z"], lo, hi),
                               b=sl(t["b"], lo, hi) if layout == "BLD" else np.ascontiguousarray(t["b"][..., lo:hi]),
                               c=sl(t["c"], lo, hi) if layout == "BLD" else np.ascontiguousarray(t["c"][..., lo:hi]))
    y1, h1 = gpu_run(part(0, cut), "f32", layout, h0=h0, want_final=True)
    y2, h2 = gpu_run(part(cut, 50), "f32", layout, h0=h1, want_final=True)
    np.testing.assert_allclose(np.concatenate([y1, y2], axis=ax), y, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(h2, hf, rtol=1e-5, atol=1e-5)


def test_varlen_equals_separate_calls():
    t = make(7, 1, 60, 32, 16, 1, "BLD", "f32")
    cu = [0, 7, 8, 33, 60]
    h0 = np.random.default_rng(2).standard_normal((4, 32, 16)).astype(np.float32)
    y, hf = gpu_run(t, "f32", "BLD", h0=h0, want_final=True, cu=cu)
    ref, hr, scale = oracle_run(t, "BLD", h0=h0, want_final=True, cu=np.array(cu, np.int32))
    check_f32("varlen", y, ref, scale)
    np.testing.assert_allclose(hf, hr, rtol=1e-5, atol=1e-5)


def test_step_equals_last_row_of_rescan():
    """A per-frame L = 1 update of carried state equals the last token of a full rescan."""
    t = make(9, 8, 12, 32, 16, 1, "BLD", "f32")
    y, hf = gpu_run(t, "f32", "BLD", want_final=True)
    head = dict(t, u=t["u"][:, :11].copy(), delta=t["delta"][:, :11].copy(), z=t["z"][:, :11].copy(),
                b=t["b"][:, :11].copy(), c=t["c"][:, :11].copy())
    _, h11 = gpu_run(head, "f32", "BLD", want_final=True)
    last = dict(t, u=t["u"][:, 11:].copy(), delta=t["delta"][:, 11:].copy(), z=t["z"][:, 11:].copy(),
                b=t["b"][:, 11:].copy(), c=t["c"][:, 11:].copy())
    y1, h12 = gpu_run(last, "f32", "BLD", h0=h11, want_final=True)
    np.testing.assert_allclose(y1[:, 0], y[:, 11], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(h12, hf, rtol=1e-6, atol=1e-6)


def test_layouts_agree():
    t = make(11, 2, 40, 48, 16, 2, "BLD", "bf16")
    y1, _ = gpu_run(t, "bf16", "BLD")
    tr = lambda a: np.ascontiguousarray(np.moveaxis(a, 1, -1))
    t2 = dict(t, u=tr(t["u"]), delta=tr(t["delta"]), z=tr(t["z"]), b=tr(t["b"]), c=tr(t["c"]))
    y2, _ = gpu_run(t2, "bf16", "BDL")
    ref, _, _ = oracle_run(t, "BLD", groups=2)
    check_16bit("bld", y1, ref)
    check_16bit("bdl", np.moveaxis(y2, -1, 1), ref)


def test_rejections():
    t = make(0, 1, 16, 64, 16)
    u = torch.zeros(1, 64, 16, dtype=torch.bfloat16, device="cuda")
    A = torch.zeros(64, 16, device="cuda")
    B = torch.zeros(1, 1, 16, 16, dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.Stream()
    with pytest.raises(sb.ScanInvalidArgument, match="non-default stream"):
        sb.selective_scan_ex(u, u, A, B, B, stream=0)
    with pytest.raises(sb.ScanInvalidArgument, match="power of two"):
        sb.selective_scan_ex(u, u, torch.zeros(64, 3, device="cuda"),
                             torch.zeros(1, 1, 3, 16, dtype=torch.bfloat16, device="cuda"),
                             torch.zeros(1, 1, 3, 16, dtype=torch.bfloat16, device="cuda"), stream=s)
    with pytest.raises(sb.ScanInvalidArgument, match="y overlaps u"):
        sb.selective_scan_ex(u, u.clone(), A, B, B, out=u, stream=s)
    del t


# ---------------------------------------------------------------- bulk path
# Shapes inside the bulk kernel's domain: 16-bit (B, D, L), N = 16,
# D a multiple of 128 (per group); (B, D, L) needs L a multiple of 8, (B, L, D) any L.

@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("layout", ["BDL", "BLD"])
@pytest.mark.parametrize("case", [
    dict(B=2, L=96, D=256, G=1, c_full=True, use=("D", "z", "bias")),
    dict(B=2, L=200, D=128, G=1, c_full=True, use=("D", "bias")),        # partial last chunk
    dict(B=2, L=64, D=256, G=2, c_full=False, use=("D", "z", "bias")),   # groups, rank-1 C
    dict(B=3, L=40, D=384, G=1, c_full=True, use=()),                    # no bias / D / gate
    dict(B=2, L=37, D=256, G=1, c_full=True, use=("D", "z", "bias")),   # (B, L, D): any length
])
def test_bulk_path_matches_oracle(dt, layout, case):
    t = make(21, case["B"], case["L"], case["D"], 16, case["G"], layout, dt, c_full=case["c_full"])
    y, _ = gpu_run(t, dt, layout, use=case["use"])
    ref, _, _ = oracle_run(t, layout, use=case["use"], groups=case["G"])
    check_16bit(f"bulk_{dt}_{layout}_{case}", y, ref)


@pytest.mark.parametrize("layout", ["BDL", "BLD"])
def test_bulk_path_state_in_out(layout):
    t = make(22, 2, 72, 256, 16, 1, layout, "bf16")
    h0 = (np.random.default_rng(3).standard_normal((2, 256, 16)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, "bf16", layout, h0=h0, want_final=True)
    ref, hr, _ = oracle_run(t, layout, h0=h0, want_final=True)
    check_16bit("bulk_state_y", y, ref)
    np.testing.assert_allclose(hf, hr, rtol=1e-3, atol=1e-3)


def test_bulk_config2_full_size_sampled_lanes():
    """BASELINE config 2 at full size (64 x 1536 x 2048, N = 16, bf16): 48 sampled
    lanes against the oracle run on exactly those lanes."""
    B, D, L, N = 64, 1536, 2048, 16
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    with torch.cuda.stream(s):
        u = torch.randn(B, D, L, device="cuda", generator=g).to(torch.bfloat16)
        dl = torch.randn(B, D, L, device="cuda", generator=g).to(torch.bfloat16)
        bm = torch.randn(B, 1, N, L, device="cuda", generator=g).to(torch.bfloat16)
        cm = torch.randn(B, 1, N, L, device="cuda", generator=g).to(torch.bfloat16)
        rng = np.random.default_rng(5)
        bias = np.log(np.expm1(np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D)))).astype(np.float32)
        A = -np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1))
        y = sb.selective_scan_ex(u, dl, torch.from_numpy(A).cuda(), bm, cm, D=torch.ones(D, device="cuda"),
                                 delta_bias=torch.from_numpy(bias).cuda(), layout="BDL", stream=s)
    s.synchronize()
    picks = [(int(b), int(d)) for b, d in zip(rng.integers(0, B, 48), rng.integers(0, D, 48))]
    for b, d in picks:
        f = lambda x: x.float().cpu().numpy()
        ref, _ = oracle.scan_ex(f(u[b:b + 1, d:d + 1]), f(dl[b:b + 1, d:d + 1]), A[d:d + 1], f(bm[b:b + 1]),
                                f(cm[b:b + 1]), layout="BDL", d=np.ones(1, np.float32), delta_bias=bias[d:d + 1])
        check_16bit(f"c2_lane_{b}_{d}", f(y[b:b + 1, d:d + 1]), ref)
    fault = ctypes_fault()
    assert fault == 0


def ctypes_fault():
    import ctypes
    from saccade_v1_b200 import _lib
    v = ctypes.c_uint32(0)
    assert _lib.load().sacc_scan_fault(ctypes.byref(v), 0) == 0
    return v.value


# ---------------------------------------------------------------- bulk varlen
# Packed sequences ((1, total, D) with cu_seqlens, 16-bit, N = 16, D a multiple
# of 128): the bulk kernel with one CTA per (sequence, 128 channels).

def packed(seed, lens, D, dt, G=1):
    t = make(seed, 1, int(sum(lens)), D, 16, G, "BLD", dt)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return t, cu


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_bulk_varlen_matches_oracle(dt):
    lens = [1, 7, 8, 9, 31, 32, 33, 64, 65, 100, 3, 17, 40, 2, 56, 71]
    D = 256
    t, cu = packed(31, lens, D, dt)
    h0 = (np.random.default_rng(32).standard_normal((len(lens), D, 16)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, dt, "BLD", h0=h0, want_final=True, cu=list(cu))
    ref, hr, _ = oracle_run(t, "BLD", h0=h0, want_final=True, cu=cu)
    check_16bit(f"bulk_varlen_{dt}", y, ref)
    np.testing.assert_allclose(hf, hr, rtol=1e-3, atol=1e-3)
    assert ctypes_fault() == 0


def test_bulk_varlen_bitwise_equals_separate_calls():
    """Sequences of multiple-of-8 lengths through one packed call and through
    one unpacked bulk call each: the same kernel arithmetic, the same bits."""
    lens, D = [8, 16, 40, 64, 72], 384
    t, cu = packed(33, lens, D, "bf16", G=3)
    h0 = (np.random.default_rng(34).standard_normal((len(lens), D, 16)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, "bf16", "BLD", h0=h0, want_final=True, cu=list(cu))
    for k, (a, b) in enumerate(zip(cu[:-1], cu[1:])):
        part = dict(t, u=t["u"][:, a:b].copy(), delta=t["delta"][:, a:b].copy(), z=t["z"][:, a:b].copy(),
                    b=t["b"][:, a:b].copy(), c=t["c"][:, a:b].copy())
        y1, h1 = gpu_run(part, "bf16", "BLD", h0=h0[k:k + 1], want_final=True)
        assert np.array_equal(y[:, a:b].view(np.uint32), y1.view(np.uint32)), k
        assert np.array_equal(hf[k:k + 1].view(np.uint32), h1.view(np.uint32)), k


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_varlen_entries_are_clamped(dt):
    """cu_seqlens past the end or below zero are clamped to [0, length]; a
    sequence whose end precedes its start is empty (its final state is h0).
    f32 takes the general kernel, bf16 with D = 256 the bulk kernel."""
    D, L = 256, 100
    t = make(35, 1, L, D, 16, 1, "BLD", dt)
    h0 = (np.random.default_rng(36).standard_normal((4, D, 16)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, dt, "BLD", h0=h0, want_final=True, cu=[0, 30, 30, 500, -5])
    ref, hr, scale = oracle_run(t, "BLD", h0=h0, want_final=True, cu=np.array([0, 30, 30, 100, 100], np.int32))
    if dt == "f32":
        check_f32("clamped", y, ref, scale)
        np.testing.assert_allclose(hf, hr, rtol=1e-5, atol=1e-5)
    else:
        check_16bit("clamped", y, ref)
        np.testing.assert_allclose(hf, hr, rtol=1e-3, atol=1e-3)
    np.testing.assert_array_equal(hf[1], h0[1])
    np.testing.assert_array_equal(hf[3], h0[3])
    assert ctypes_fault() == 0


@pytest.mark.parametrize("layout", ["BDL", "BLD"])
def test_bulk_split_launch_bitwise_equals_unsplit(layout):
    """A batch large enough that the units exceed one wave of CTAs is split
    along L (each unit's parts hand their state over through the output,
    part-major items on a multi-wave grid); the same rows run as 32-row slices
    are split into a different number of parts, or not at all.  The hand-off
    moves exact FP32 states, so outputs and final states agree bit for bit.
    Gate, h0 and h_final included."""
    B, L, D, N = 64, 1024, 1536, 16  # 768 units of 128 channels: more than one wave in either layout
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(61)
    bf = torch.bfloat16
    with torch.cuda.stream(s):
        if layout == "BDL":
            mk = lambda: torch.randn(B, D, L, device="cuda", generator=g).to(bf)
            mkbc = lambda: torch.randn(B, 1, N, L, device="cuda", generator=g).to(bf)
        else:
            mk = lambda: torch.randn(B, L, D, device="cuda", generator=g).to(bf)
            mkbc = lambda: torch.randn(B, L, 1, N, device="cuda", generator=g).to(bf)
        u, dl, z, bm, cm = mk(), mk(), mk(), mkbc(), mkbc()
        A = -(torch.rand(D, N, device="cuda", generator=g) * 4 + 0.1)
        Dv = torch.randn(D, device="cuda", generator=g)
        bias = torch.full((D,), -3.0, device="cuda")
        h0 = torch.randn(B, D, N, device="cuda", generator=g) * 0.5
        hf = torch.empty(B, D, N, device="cuda")
        y = sb.selective_scan_ex(u, dl, A, bm, cm, D=Dv, z=z, delta_bias=bias, h0=h0, h_final=hf, layout=layout, stream=s)
        ys, hs = [], []
        rows = 32  # 384 units: the one-thread-per-lane kernel (the four-thread kernel takes <= 296 units)
        for b0 in range(0, B, rows):
            sl = slice(b0, b0 + rows)
            hfi = torch.empty(rows, D, N, device="cuda")
            ys.append(sb.selective_scan_ex(u[sl].contiguous(), dl[sl].contiguous(), A, bm[sl].contiguous(), cm[sl].contiguous(),
                                           D=Dv, z=z[sl].contiguous(), delta_bias=bias, h0=h0[sl].contiguous(), h_final=hfi,
                                           layout=layout, stream=s))
            hs.append(hfi)
    s.synchronize()
    assert torch.equal(y.view(torch.int16), torch.cat(ys).view(torch.int16))
    assert torch.equal(hf.view(torch.int32), torch.cat(hs).view(torch.int32))
    assert ctypes_fault() == 0


def test_bulk_split_launch_in_cuda_graph():
    """The split launch (parts handing states over through the outputs) captured in a CUDA graph and
    replayed twice gives the eager launch's bits."""
    B, L, D, N = 64, 512, 1536, 16
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(71)
    bf = torch.bfloat16
    with torch.cuda.stream(s):
        u = torch.randn(B, D, L, device="cuda", generator=g).to(bf)
        dl = torch.randn(B, D, L, device="cuda", generator=g).to(bf)
        bm = torch.randn(B, 1, N, L, device="cuda", generator=g).to(bf)
        cm = torch.randn(B, 1, N, L, device="cuda", generator=g).to(bf)
        A = -(torch.rand(D, N, device="cuda", generator=g) * 4 + 0.1)
        Dv = torch.randn(D, device="cuda", generator=g)
        bias = torch.full((D,), -3.0, device="cuda")
        ref = sb.selective_scan_ex(u, dl, A, bm, cm, D=Dv, delta_bias=bias, layout="BDL", stream=s)
        out = torch.zeros_like(ref)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        sb.selective_scan_ex(u, dl, A, bm, cm, D=Dv, delta_bias=bias, layout="BDL", out=out, stream=s)
    for _ in range(2):
        out.zero_()
        with torch.cuda.stream(s):
            graph.replay()
        s.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert ctypes_fault() == 0


@pytest.mark.parametrize("layout,B,L", [("BDL", 62, 1000), ("BLD", 62, 1000), ("BDL", 100, 520), ("BLD", 100, 520)])
def test_bulk_split_parts_bitwise_equals_unsplit(layout, B, L):
    """Units just over one wave of CTAs (62 rows x 12 tiles = 744) and about
    two waves (1200), with L a multiple of 8 but not of 32 (a ragged last
    chunk, so the last part is shorter): the launch splits each unit into
    parts handed over through the outputs (part-major items on a multi-wave
    grid); the same rows as slices of 25-31 rows split into other part counts
    or not at all.  Exact FP32 hand-offs: outputs and final states agree bit
    for bit, h0 and a gate included."""
    D, N = 1536, 16
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(67 + B + L)
    bf = torch.bfloat16
    with torch.cuda.stream(s):
        shp = (B, D, L) if layout == "BDL" else (B, L, D)
        bshp = (B, 1, N, L) if layout == "BDL" else (B, L, 1, N)
        u, dl, z = (torch.randn(shp, device="cuda", generator=g).to(bf) for _ in range(3))
        bm, cm = (torch.randn(bshp, device="cuda", generator=g).to(bf) for _ in range(2))
        A = -(torch.rand(D, N, device="cuda", generator=g) * 2 + 0.01)
        Dv = torch.randn(D, device="cuda", generator=g)
        bias = torch.full((D,), -4.0, device="cuda")
        h0 = torch.randn(B, D, N, device="cuda", generator=g) * 0.5
        hf = torch.empty(B, D, N, device="cuda")
        y = sb.selective_scan_ex(u, dl, A, bm, cm, D=Dv, z=z, delta_bias=bias, h0=h0, h_final=hf, layout=layout, stream=s)
        ys, hs = [], []
        # Slices of 25..31 rows (300..372 units): the one-thread-per-lane kernel (above the four-thread kernel's
        # 296 units), split differently from the whole batch or not at all.
        rows = 31 if B == 62 else 25
        for b0 in range(0, B, rows):
            sl = slice(b0, b0 + rows)
            hfi = torch.empty(rows, D, N, device="cuda")
            ys.append(sb.selective_scan_ex(u[sl].contiguous(), dl[sl].contiguous(), A, bm[sl].contiguous(), cm[sl].contiguous(),
                                           D=Dv, z=z[sl].contiguous(), delta_bias=bias, h0=h0[sl].contiguous(), h_final=hfi,
                                           layout=layout, stream=s))
            hs.append(hfi)
    s.synchronize()
    assert torch.equal(y.view(torch.int16), torch.cat(ys).view(torch.int16))
    assert torch.equal(hf.view(torch.int32), torch.cat(hs).view(torch.int32))
    assert ctypes_fault() == 0


def long_memory(t, N=16):
    """Small Delta (softplus(x - 5) ~ 0.007) and A in [-2, -0.01]: states that
    carry across hundreds of tokens, so a wrong hand-off shows in the output."""
    t = dict(t)
    t["bias"] = np.full_like(t["bias"], -5.0)
    t["A"] = -np.tile(np.geomspace(0.01, 2.0, N).astype(np.float32), (t["A"].shape[0], 1))
    return t


@pytest.mark.parametrize("layout,dt,B,L,c_full", [("BLD", "f16", 4, 960, True), ("BDL", "bf16", 2, 1024, False),
                                                  ("BLD", "bf16", 4, 240, True), ("BDL", "f16", 1, 200, True)])
def test_bulk_chunk_parallel_matches_oracle(layout, dt, B, L, c_full):
    """Few units of 128 channels over a long sequence (4 to 8 units here, far
    fewer than the SMs) run chunk-parallel: a local pass over up to 32 parts
    of the sequence, parts after the first from a zero state; a combine that
    chains the parts' end states through exp(A * sum of Delta); a final pass
    over parts 1.. from the combined states.  Gate, h0 and h_final included."""
    D = 256 if B > 1 else 128
    t = long_memory(make(81, B, L, D, 16, 1, layout, dt, c_full=c_full))
    h0 = (np.random.default_rng(82).standard_normal((B, D, 16)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, dt, layout, h0=h0, want_final=True)
    ref, hr, _ = oracle_run(t, layout, h0=h0, want_final=True)
    check_16bit(f"chunked_{layout}_{dt}_L{L}", y, ref)
    np.testing.assert_allclose(hf, hr, rtol=1e-3, atol=1e-3)
    assert ctypes_fault() == 0


@pytest.mark.parametrize("layout", ["BDL", "BLD"])
def test_bulk_chunk_parallel_close_to_one_pass(layout):
    """The same rows through the chunk-parallel passes (4 rows: 8 units) and
    through one sequential pass (the rows repeated ten times: 80 units, too
    many for the chunk-parallel mode) agree to FP32 rounding in the states and
    to one 16-bit rounding step in the outputs."""
    B, L, D, N = 4, 960, 256, 16
    t = long_memory(make(83, B, L, D, N, 1, layout, "bf16"))
    h0 = (np.random.default_rng(84).standard_normal((B, D, N)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, "bf16", layout, h0=h0, want_final=True)
    rep = dict(t)
    for k in ("u", "delta", "z", "b", "c"):
        rep[k] = np.concatenate([t[k]] * 10)
    y10, hf10 = gpu_run(rep, "bf16", layout, h0=np.concatenate([h0] * 10), want_final=True)
    np.testing.assert_allclose(hf, hf10[:B], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(y, y10[:B], rtol=8e-3, atol=1e-4)
    assert ctypes_fault() == 0


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_four_thread_kernel_close_to_one_thread(dt):
    """Few units run four threads per lane (state quarters, shuffled Delta and
    partial sums); the same rows inside a batch large enough for the
    one-thread-per-lane kernel agree to FP32 rounding in the states and to one
    16-bit rounding step in the outputs.  (B, L, D), gate, h0 / h_final, a
    ragged last chunk."""
    B, L, D, N = 4, 200, 256, 16
    t = long_memory(make(91, B, L, D, N, 1, "BLD", dt))
    h0 = (np.random.default_rng(92).standard_normal((B, D, N)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, dt, "BLD", h0=h0, want_final=True)
    rep = dict(t)
    for k in ("u", "delta", "z", "b", "c"):
        rep[k] = np.concatenate([t[k]] * 80)  # 640 units of 128 channels
    y80, hf80 = gpu_run(rep, dt, "BLD", h0=np.concatenate([h0] * 80), want_final=True)
    np.testing.assert_allclose(hf, hf80[:B], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(y, y80[:B], rtol=8e-3, atol=1e-4)
    ref, hr, _ = oracle_run(t, "BLD", h0=h0, want_final=True)
    check_16bit(f"quad_{dt}", y, ref)
    assert ctypes_fault() == 0


def test_bounded_waits_report_a_fault_and_leave_the_context_usable():
    """A wait that runs out (a flag nothing sets, an mbarrier nothing arrives
    at, polled with the scan kernels' helpers) sets the fault word instead of
    hanging; the next scan runs normally on the same context."""
    import ctypes

    from saccade_v1_b200 import _lib
    L = _lib.load()
    v = ctypes.c_uint32(0)
    assert L.sacc_scan_fault(ctypes.byref(v), 1) == 0  # clear
    s = torch.cuda.Stream()
    assert L.sacc_scan_wait_probe(1000, s.cuda_stream) == 0, _lib.last_error()
    s.synchronize()
    assert L.sacc_scan_fault(ctypes.byref(v), 1) == 0 and v.value & 1
    assert L.sacc_scan_wait_probe(0, s.cuda_stream) == _lib.SACC_EINVAL
    t = make(95, 2, 96, 256, 16, 1, "BLD", "bf16")
    y, _ = gpu_run(t, "bf16", "BLD")
    ref, _, _ = oracle_run(t, "BLD")
    check_16bit("after_probe", y, ref)
    assert ctypes_fault() == 0


def ulp_off(A):
    """A with its last state's value moved by one FP32 ulp in every row: no row is S4D-real any more, so the
    scan takes the exp-per-state path."""
    A = np.array(A, np.float32)
    A[:, -1] = np.nextafter(A[:, -1], np.float32(0))
    return A


@pytest.mark.parametrize("layout,B,L,D,dt,c_full", [
    ("BDL", 2, 96, 256, "bf16", True),     # one item per CTA
    ("BDL", 2, 64, 256, "f16", False),     # rank-1 C
    ("BLD", 2, 200, 256, "bf16", True),    # (B, L, D), ragged last chunk, four threads per lane
    ("BLD", 4, 960, 256, "f16", True),     # chunk-parallel passes
    ("BDL", 2, 1024, 128, "bf16", True),   # chunk-parallel passes, (B, D, L)
])
def test_power_form_decays_match_oracle_and_exp_path(layout, B, L, D, dt, c_full):
    """S4D-real A (A[d, n] = -(n + 1)) takes the power-form decays (one exponential per token, the 16 decays as
    powers of it); the same inputs with A moved by one ulp in the last state take the exp-per-state path.
    Both are held to the oracle on their own A, and to each other to one 16-bit rounding step."""
    t = make(101, B, L, D, 16, 1, layout, dt, c_full=c_full)
    h0 = (np.random.default_rng(102).standard_normal((B, D, 16)) * 0.5).astype(np.float32)
    y, hf = gpu_run(t, dt, layout, h0=h0, want_final=True)
    ref, hr, _ = oracle_run(t, layout, h0=h0, want_final=True)
    check_16bit(f"pow_{layout}_{dt}_L{L}", y, ref)
    np.testing.assert_allclose(hf, hr, rtol=1e-3, atol=1e-3)
    t2 = dict(t, A=ulp_off(t["A"]))
    y2, hf2 = gpu_run(t2, dt, layout, h0=h0, want_final=True)
    ref2, _, _ = oracle_run(t2, layout, h0=h0, want_final=True)
    check_16bit(f"exp_{layout}_{dt}_L{L}", y2, ref2)
    np.testing.assert_allclose(y, y2, rtol=8e-3, atol=1e-3)
    np.testing.assert_allclose(hf, hf2, rtol=1e-4, atol=1e-5)
    assert ctypes_fault() == 0


def test_power_form_per_lane_rows_and_scales():
    """Per-channel A rows: S4D-real rows scaled by exact and inexact per-channel factors (the condition is
    A[n] == (n + 1) A[0] in FP32 arithmetic), rows of zeros, and one non-S4D row in the second 128-channel
    tile, which sends that tile's CTAs to the exp-per-state path while the other tiles take the power form."""
    B, L, D, N = 2, 160, 384, 16
    t = make(103, B, L, D, N, 1, "BDL", "bf16")
    r = np.random.default_rng(104)
    scale = np.where(np.arange(D) % 3 == 0, 0.5, r.uniform(0.2, 3.0, D)).astype(np.float32)
    A = (-np.arange(1, N + 1, dtype=np.float32)[None, :] * scale[:, None]).astype(np.float32)
    A[7] = 0.0
    A[200] = -np.geomspace(0.05, 4.0, N).astype(np.float32)
    t["A"] = A
    y, hf = gpu_run(t, "bf16", "BDL", want_final=True)
    ref, hr, _ = oracle_run(t, "BDL", want_final=True)
    check_16bit("pow_rows", y, ref)
    np.testing.assert_allclose(hf, hr, rtol=1e-3, atol=1e-3)
    assert ctypes_fault() == 0


@pytest.mark.parametrize("layout", ["BLD", "BDL"])
@pytest.mark.parametrize("B", [32, 64])
def test_bulk_gated_matches_oracle_lanes(B, layout):
    """A gate and a full C in the one-thread-per-lane kernel, whose gate comes in two 16-token halves of a TMA
    tile: 32 rows x 12 tiles = 384 units (a split launch at four CTAs per SM), 64 rows = 768 units (split into
    more parts).  L = 520: a last chunk of 8 tokens, whose gate's second half arrives unread.  h0 in, h_final
    out; sampled lanes against the binary64 oracle on the same 16-bit inputs, in both layouts."""
    L, D, N = 520, 1536, 16
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(90 + B + (7 if layout == "BDL" else 0))
    bf = torch.bfloat16
    shp = (B, L, D) if layout == "BLD" else (B, D, L)
    bshp = (B, L, 1, N) if layout == "BLD" else (B, 1, N, L)
    with torch.cuda.stream(s):
        u, dl, z = (torch.randn(shp, device="cuda", generator=g).to(bf) for _ in range(3))
        bm, cm = (torch.randn(bshp, device="cuda", generator=g).to(bf) for _ in range(2))
        A = -(torch.rand(D, N, device="cuda", generator=g) * 2 + 0.01)
        Dv = torch.randn(D, device="cuda", generator=g)
        bias = torch.full((D,), -3.0, device="cuda")
        h0 = torch.randn(B, D, N, device="cuda", generator=g) * 0.5
        hf = torch.empty(B, D, N, device="cuda")
        y = sb.selective_scan_ex(u, dl, A, bm, cm, D=Dv, z=z, delta_bias=bias, h0=h0, h_final=hf, layout=layout, stream=s)
    s.synchronize()
    f = lambda x: x.float().cpu().numpy()
    An, Dn, hn = f(A), f(Dv), f(h0)
    lane = (lambda t, b, d: t[b:b + 1, :, d:d + 1]) if layout == "BLD" else (lambda t, b, d: t[b:b + 1, d:d + 1])
    rng = np.random.default_rng(91 + B)
    for b, d in zip(rng.integers(0, B, 10), rng.integers(0, D, 10)):
        b, d = int(b), int(d)
        ref, href = oracle.scan_ex(f(lane(u, b, d)), f(lane(dl, b, d)), An[d:d + 1], f(bm[b:b + 1]), f(cm[b:b + 1]),
                                   layout=layout, d=Dn[d:d + 1], z=f(lane(z, b, d)), delta_bias=np.full(1, -3.0, np.float32),
                                   h0=hn[b:b + 1, d:d + 1], want_final=True)
        check_16bit(f"gated_{layout}_{B}_{b}_{d}", f(lane(y, b, d)), ref)
        np.testing.assert_allclose(f(hf[b:b + 1, d:d + 1]), href, rtol=1e-3, atol=1e-3)
    assert ctypes_fault() == 0


@pytest.mark.parametrize("layout", ["BDL", "BLD"])
def test_power_form_split_launch_matches_oracle_lanes(layout):
    """The split launch (units beyond one wave, parts handing states over through the outputs) with S4D-real A:
    sampled lanes against the oracle, and the whole output bit-identical to the same rows run unsplit."""
    B, L, D, N = 64, 1024, 1536, 16
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(105)
    bf = torch.bfloat16
    with torch.cuda.stream(s):
        shp = (B, D, L) if layout == "BDL" else (B, L, D)
        bshp = (B, 1, N, L) if layout == "BDL" else (B, L, 1, N)
        u, dl = (torch.randn(shp, device="cuda", generator=g).to(bf) for _ in range(2))
        bm, cm = (torch.randn(bshp, device="cuda", generator=g).to(bf) for _ in range(2))
        A = -torch.arange(1, N + 1, dtype=torch.float32, device="cuda").repeat(D, 1)
        bias = torch.full((D,), -3.0, device="cuda")
        hf = torch.empty(B, D, N, device="cuda")
        y = sb.selective_scan_ex(u, dl, A, bm, cm, D=torch.ones(D, device="cuda"), delta_bias=bias, h_final=hf,
                                 layout=layout, stream=s)
        ys, hs = [], []
        for b0 in range(0, B, 32):
            sl = slice(b0, b0 + 32)
            hfi = torch.empty(32, D, N, device="cuda")
            ys.append(sb.selective_scan_ex(u[sl].contiguous(), dl[sl].contiguous(), A, bm[sl].contiguous(), cm[sl].contiguous(),
                                           D=torch.ones(D, device="cuda"), delta_bias=bias, h_final=hfi, layout=layout,
                                           stream=s))
            hs.append(hfi)
    s.synchronize()
    assert torch.equal(y.view(torch.int16), torch.cat(ys).view(torch.int16))
    assert torch.equal(hf.view(torch.int32), torch.cat(hs).view(torch.int32))
    rng = np.random.default_rng(106)
    f = lambda x: x.float().cpu().numpy()
    An = f(A)
    for b, d in zip(rng.integers(0, B, 12), rng.integers(0, D, 12)):
        b, d = int(b), int(d)
        if layout == "BDL":
            ref, _ = oracle.scan_ex(f(u[b:b + 1, d:d + 1]), f(dl[b:b + 1, d:d + 1]), An[d:d + 1], f(bm[b:b + 1]), f(cm[b:b + 1]),
                                    layout="BDL", d=np.ones(1, np.float32), delta_bias=np.full(1, -3.0, np.float32))
            got = f(y[b:b + 1, d:d + 1])
        else:
            ref, _ = oracle.scan_ex(f(u[b:b + 1, :, d:d + 1]), f(dl[b:b + 1, :, d:d + 1]), An[d:d + 1], f(bm[b:b + 1]),
                                    f(cm[b:b + 1]), layout="BLD", d=np.ones(1, np.float32),
                                    delta_bias=np.full(1, -3.0, np.float32))
            got = f(y[b:b + 1, :, d:d + 1])
        check_16bit(f"pow_split_{layout}_{b}_{d}", got, ref)
    assert ctypes_fault() == 0
