"""GPU parity of the reference-ABI FP32 scan (sacc_selective_scan_f32).

Restates the reference's GPU acceptance groups (tests/scan_cuda_suite.hpp):
s01_values :364, coverage :461, softplus :510, intermediate_range :560,
failures :580, plus reset / determinism / graph capture
(tests/selective_scan_cuda_tests.cpp:18-59) and the host rejections.
Every output element must lie within twice the running error bound of the
reference's FP32 algorithm (computed by the oracle) around the binary64
reference result; failures must set the exact status bits, poison the whole
output with the quiet NaN and still complete the status.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from oracle.oracle import Shape, filled, random_case, varied
import scan_cases as sc

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as gu  # noqa: E402
import saccade_v1_b200 as sb  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def loaded():
    report = sb.load_kernels()
    assert "scan_f32_n16" in report
    # The loader also fills the residency figures the chunk split uses (>= 1 CTA per SM).
    resident = dict(line.split("=") for line in report.splitlines() if line.startswith("scan_f32_resident_ctas_per_sm_n"))
    assert len(resident) == 6 and all(int(v) >= 1 for v in resident.values()), resident
    return report


def scan_case(name, k):
    ref = oracle.run(k)
    bound = oracle.scan_bound(k)
    y, (flags, done) = gu.run_f32(k)
    assert flags == 0 and done == sb.SCAN_DONE, f"{name}: status {flags:#x} {done:#x}"
    return gu.compare_bound(name, y, ref, bound)


def test_s01_values():
    for name, (k, _) in sc.contract_cases().items():
        scan_case("s01_" + name, k)
    for length in (25, 100, 400):
        scan_case(f"s01_m_head_abi_L{length}", sc.m_head_case(length))
    k = filled(Shape(1, 2, 1, 1, 1, 1, False), sc.DENORM_MIN, 0, 1, 1)
    y, _ = gu.run_f32(k)
    assert y[0] == np.float32(sc.DENORM_MIN), "subnormal results are not flushed to zero"


def test_coverage():
    for name, k in sc.coverage_cases().items():
        scan_case(name, k)
    k = sc.empty_case()
    y, (flags, done) = gu.run_f32(k)
    assert flags == 0 and done == sb.SCAN_DONE and y.size == 0


def test_softplus_sweep_and_discrimination():
    cases = sc.softplus_cases(oracle.softplus)
    k = cases["softplus_minus18"]
    ref, bound = oracle.run(k), oracle.scan_bound(k)
    scan_case("softplus_minus18", k)
    legacy = sc.legacy_softplus(-18.0) * 1e8
    assert abs(legacy - ref[0]) > 2 * bound[0], "the bound rejects the legacy softplus at x = -18"
    k = cases["softplus_sweep"]
    ref, bound = oracle.run(k), oracle.scan_bound(k)
    scan_case("softplus_sweep", k)
    rejected = sum(abs(sc.legacy_softplus(x) * 2.0 ** 100 * float(k.u[i]) - ref[i]) > 2 * bound[i]
                   for i, x in enumerate(k.delta))
    assert rejected >= 10


def test_intermediate_range():
    for name, k in sc.intermediate_cases().items():
        scan_case(name, k)


def test_failures_set_exact_bits_and_poison():
    for name, k, bit, exact, diag in sc.failure_cases():
        st, _, msg = oracle.scan_ref(k)
        assert st != oracle.OK and diag in msg
        y, (flags, done) = gu.run_f32(k)
        assert done == sb.SCAN_DONE, name
        if bit & sc.INPUT_FAILURES:
            assert flags & sc.INPUT_FAILURES == bit, (name, hex(flags))
        elif exact:
            assert flags == bit, (name, hex(flags))
        else:
            assert flags & bit == bit and flags & ~sc.RANGE_FAILURES == 0, (name, hex(flags))
        assert np.all(y.view(np.uint32) == gu.POISON), name


def test_reset_between_calls_and_determinism():
    """A -> B -> A on the same buffers: nothing survives a call (selective_scan_cuda_tests.cpp:18-59)."""
    good = random_case(Shape(2, 64, 40, 16, 1, 1, True), 0x5eed0200)
    bad = good.copy()
    bad.u[7] = np.nan
    s = gu.stream()
    shape = sb.SelectiveScanShape(2, 64, 40, 16, 1, 1, True)
    with torch.cuda.stream(s):
        bufs = [gu.dev(x) for x in good.inputs()]
        y = torch.empty(good.u.size, device="cuda")
        st = gu.new_status()
        outs = []
        for case in (good, bad, good):
            for dst, src in zip(bufs, case.inputs()):
                dst.copy_(torch.from_numpy(src))
            sb.selective_scan_cuda(shape, *bufs, y, st, stream=s)
            s.synchronize()
            outs.append((y.cpu().numpy().copy(), gu.status_words(st)))
    assert outs[0][1] == (0, sb.SCAN_DONE) and outs[2][1] == (0, sb.SCAN_DONE)
    # Input bits are exact; range bits carry no meaning when an input bit is set
    # (include/saccade/selective_scan_cuda.hpp:27-29 of the reference).
    assert outs[1][1][0] & sc.INPUT_FAILURES == sc.NONFINITE_U and outs[1][1][1] == sb.SCAN_DONE
    assert np.all(outs[1][0].view(np.uint32) == gu.POISON)
    assert np.array_equal(outs[0][0].view(np.uint32), outs[2][0].view(np.uint32)), "bitwise deterministic"


def test_graph_capture_replays_with_new_inputs():
    k1 = random_case(Shape(4, 120, 256, 16, 1, 1, True), 0x5eed0300)
    k2 = random_case(Shape(4, 120, 256, 16, 1, 1, True), 0x5eed0301)
    shape = sb.SelectiveScanShape(4, 120, 256, 16, 1, 1, True)
    s = gu.stream()
    with torch.cuda.stream(s):
        bufs = [gu.dev(x) for x in k1.inputs()]
        y = torch.empty(k1.u.size, device="cuda")
        st = gu.new_status()
        sb.selective_scan_cuda(shape, *bufs, y, st, stream=s)  # warm (kernels loaded)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        sb.selective_scan_cuda(shape, *bufs, y, st, stream=s)
    for k in (k2, k1):
        with torch.cuda.stream(s):
            for dst, src in zip(bufs, k.inputs()):
                dst.copy_(torch.from_numpy(src))
            st.copy_(gu.new_status())
            g.replay()
        s.synchronize()
        assert gu.status_words(st) == (0, sb.SCAN_DONE)
        gu.compare_bound("graph", y.cpu().numpy(), oracle.run(k), oracle.scan_bound(k))


def test_host_rejections_leave_status_untouched():
    k = varied(Shape(1, 4, 4, 16, 1, 1, True))
    s = gu.stream()
    with torch.cuda.stream(s):
        bufs = [gu.dev(x) for x in k.inputs()]
        y = torch.empty(k.u.size, device="cuda")
        st = gu.new_status()
    s.synchronize()
    good = sb.SelectiveScanShape(1, 4, 4, 16, 1, 1, True)
    cases = [
        (sb.SelectiveScanShape(1, 4, 4, 3, 1, 1, True), bufs, y, st, s, "must be a power of two in [1, 32]"),
        (sb.SelectiveScanShape(1, 4, 4, 16, 2, 1, True), bufs, y, st, s, "A rows must be 1 or channels"),
        (sb.SelectiveScanShape(0, 4, 4, 16, 1, 1, True), bufs, y, st, s, "batch and channels must be positive"),
        (sb.SelectiveScanShape(1, 65536, 65536, 1, 1, 1, False), bufs, y, st, s, "exceeds int32 capacity"),
        (good, bufs, y, st, 0, "an explicit non-default stream is required"),
        (good, bufs, bufs[0], st, s, "y overlaps u"),
        (good, bufs, y, y, s, "status overlaps y"),
    ]
    for shape, ins, out, status, stream, diag in cases:
        with pytest.raises(sb.ScanInvalidArgument, match=diag.replace("[", r"\[").replace("]", r"\]")):
            sb.selective_scan_cuda(shape, *ins, out, status, stream=stream)
    with pytest.raises(sb.ScanInvalidArgument, match="is null"):
        sb.selective_scan_cuda(good, bufs[0], None, *bufs[2:], y, st, stream=s)
    assert gu.status_words(st) == gu.STATUS_SENTINEL


def test_deploy_shapes_random():
    """HR and T01 deploy shapes (4, L, 256, 16), shared A, rank-1 C, D."""
    for length in (960, 240, 60, 25):
        k = random_case(Shape(4, length, 256, 16, 1, 1, True), 456 + length)
        scan_case(f"deploy_L{length}", k)


def test_four_threads_per_lane_equal_one_thread(monkeypatch):
    """N >= 8 runs four threads per lane (states q, q + 4, ... each, the reference's butterfly sum finished by
    two xor shuffles); with the one-thread kernel (SACC_F32_KERNEL=one_thread) splitting the lanes into the
    same chunks, outputs and status bits are identical: at the deploy shapes (rank-1 C), with a full C, for
    N = 8 and 32, and on the failure cases."""
    cases = {f"deploy_L{L}": random_case(Shape(4, L, 256, 16, 1, 1, True), 900 + L) for L in (960, 240, 60, 7)}
    cases["full_c_per_channel_a"] = random_case(Shape(3, 200, 64, 16, 64, 16, True), 77)
    # N = 8 and 32 on 40,960 lanes, where both kernels run one chunk per lane.
    for n in (8, 32):
        cases[f"n{n}_full_c"] = random_case(Shape(5, 16, 8192, n, 1, n, True), 80 + n)
        cases[f"n{n}_rank1_c"] = random_case(Shape(5, 16, 8192, n, 8192, 1, False), 90 + n)
    cases.update({name: k for name, k, _, _, _ in sc.failure_cases() if k.shape.state >= 8})
    for name, k in cases.items():
        monkeypatch.setenv("SACC_F32_KERNEL", "one_thread")
        want = gu.run_f32(k)
        monkeypatch.delenv("SACC_F32_KERNEL")
        got = gu.run_f32(k)
        assert got[1] == want[1], (name, got[1], want[1])
        assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32)), name
