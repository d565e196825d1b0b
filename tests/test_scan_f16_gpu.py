"""The FP16-activation scan (sacc_selective_scan_f16, plugin SelectiveScan v3)
on the GPU: for inputs already in FP16 it equals the FP32 reference-ABI scan on
the same values widened to FP32, rounded to nearest FP16, bit for bit, with
the same status words; a failure poisons y with the FP16 quiet NaN 0x7E00; an
output FP16 cannot hold (|y| >= 65520) is an output range failure."""
import numpy as np
import pytest
import torch

from oracle.oracle import Shape, filled, random_case

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as gu  # noqa: E402
import saccade_v1_b200 as sb  # noqa: E402
import scan_cases as sc  # noqa: E402

OUTPUT_RANGE = 1 << 13
F16_QNAN = 0x7E00


@pytest.fixture(scope="module", autouse=True)
def loaded():
    assert "scan_f16io_n16" in sb.load_kernels()


def widened(k):
    """k with u, delta, B and C rounded to FP16 and widened back (exact)."""
    k = k.copy()
    with np.errstate(over="ignore"):  # values beyond FP16 become infinities, as on the device
        for name in ("u", "delta", "b", "c"):
            setattr(k, name, getattr(k, name).astype(np.float16).astype(np.float32))
    return k


def run_f16(k, s=None):
    s = s or gu.stream()
    sh = k.shape
    shape = sb.SelectiveScanShape(sh.batch, sh.length, sh.channels, sh.state, sh.a_rows, sh.c_width, sh.has_d)
    with torch.cuda.stream(s):
        h = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda().half()
        f = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        y = torch.full((k.u.size,), -0.0, dtype=torch.float16, device="cuda")
        y.view(torch.int16).fill_(0x5A5A)
        st = gu.new_status()
        sb.selective_scan_f16(shape, h(k.u), h(k.delta), f(k.a), h(k.b), h(k.c), f(k.d) if sh.has_d else None, y, st,
                              stream=s)
    s.synchronize()
    return y.cpu().numpy().view(np.uint16).copy(), gu.status_words(st)


def prefix(k, length):
    """A one-lane case cut to its first `length` tokens."""
    sh = k.shape
    out = k.copy()
    out.shape = Shape(1, length, 1, sh.state, sh.a_rows, sh.c_width, sh.has_d)
    out.u, out.delta = k.u[:length].copy(), k.delta[:length].copy()
    out.b, out.c = k.b[:length * sh.state].copy(), k.c[:length * sh.c_width].copy()
    return out


def fails_by(k, length):
    """(failed, overflowed) of the FP32 path over the first `length` tokens."""
    y, (flags, _) = gu.run_f32(prefix(k, length))
    return flags != 0, flags == 0 and bool(np.any(np.abs(y) >= 65520.0))


def expect_f16(k):
    """Expected (y bits, status) from the FP32 path on the widened inputs.  A
    lane stops at its first failure in token order, and with FP16 outputs an
    output of 65520 or more is one: where the FP32 path fails, a one-lane case
    whose output crosses 65520 before the FP32 failure token fails with
    OUTPUT_RANGE instead (the multi-lane failure cases have no such lane)."""
    y32, (flags, done) = gu.run_f32(k)
    if flags == 0 and y32.size and np.any(np.abs(y32) >= 65520.0):
        flags = OUTPUT_RANGE
    elif flags and k.shape.batch * k.shape.channels == 1:
        lo, hi = 0, k.shape.length  # smallest prefix that fails or overflows
        while lo + 1 < hi:
            mid = (lo + hi) // 2
            if any(fails_by(k, mid)):
                hi = mid
            else:
                lo = mid
        failed, overflowed = fails_by(k, hi)
        if overflowed and not failed:
            flags = OUTPUT_RANGE
    if flags:
        return np.full(y32.size, F16_QNAN, np.uint16), (flags, done)
    return y32.astype(np.float16).view(np.uint16), (flags, done)


def check(name, k):
    k = widened(k)
    got_y, got_st = run_f16(k)
    want_y, want_st = expect_f16(k)
    assert got_st == want_st, f"{name}: status {got_st} != {want_st}"
    assert np.array_equal(got_y, want_y), f"{name}: {int(np.sum(got_y != want_y))} of {got_y.size} outputs differ"


@pytest.mark.parametrize("name", sorted(sc.coverage_cases(include_large=True)))
def test_f16_is_the_rounded_f32_scan(name):
    check(name, sc.coverage_cases(include_large=True)[name])


@pytest.mark.parametrize("length", [60, 240, 960])
def test_f16_hr_deploy_shapes(length):
    check(f"hr_L{length}", random_case(Shape(4, length, 256, 16, 1, 1, True), 0x5eed0900 + length))


def test_f16_empty_sequence():
    check("empty", sc.empty_case())


@pytest.mark.parametrize("case", sc.failure_cases(), ids=lambda c: c[0])
def test_f16_failures_match_f32(case):
    name, k, _, _, _ = case
    check(name, k)


@pytest.mark.parametrize("d,flag", [(65504.0, 0), (65519.99, 0), (65520.0, OUTPUT_RANGE), (-65520.0, OUTPUT_RANGE),
                                    (1e6, OUTPUT_RANGE)])
def test_f16_output_range_boundary(d, flag):
    """y = D u with B = 0 (so C h = 0): 65519.99 still rounds to 65504, 65520
    rounds to infinity and fails the call."""
    k = filled(Shape(1, 3, 8, 16, 1, 1, True), 1.0, 0.5, 0.0, 1.0)
    k.d = np.full(8, d, np.float32)
    got_y, (flags, done) = run_f16(k)
    assert (flags, done) == (flag, sb.SCAN_DONE)
    if flag:
        assert np.all(got_y == F16_QNAN)
    else:
        assert np.array_equal(got_y, np.full(k.u.size, d, np.float32).astype(np.float16).view(np.uint16))


def test_f16_nonfinite_half_inputs():
    """FP16 NaN / infinity in each activation sets that tensor's input bit."""
    base = random_case(Shape(2, 9, 24, 16, 1, 16, True), 0x5eed0950)
    for field, bit in (("u", 1 << 0), ("delta", 1 << 1), ("b", 1 << 3), ("c", 1 << 4)):
        for bad in (np.nan, np.inf, -np.inf):
            k = widened(base)
            getattr(k, field)[getattr(k, field).size - 1] = bad
            got_y, (flags, done) = run_f16(k)
            assert flags & bit and done == sb.SCAN_DONE, (field, bad, hex(flags))
            assert np.all(got_y == F16_QNAN)
