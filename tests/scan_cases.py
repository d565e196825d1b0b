"""Selective-scan test cases, restated from the reference's own test suites.

Each builder returns oracle.Case objects whose FP32 bytes are fed both to the
CPU oracle and to the CUDA path.  Sources (reference paths):
  contract_cases      tests/selective_scan_tests.cpp:108-219 (S01 values)
  coverage_cases      tests/scan_cuda_suite.hpp:461-501
  softplus_cases      tests/scan_cuda_suite.hpp:503-557
  intermediate_cases  tests/scan_cuda_suite.hpp:559-578
  failure_cases       tests/scan_cuda_suite.hpp:580-616
  rejection_cases     tests/selective_scan_tests.cpp:279-317
"""
from __future__ import annotations

import math

import numpy as np

from oracle.oracle import Case, Ranges, Shape, filled, gen, random_case, varied

FLT_MAX = float(np.finfo(np.float32).max)
DENORM_MIN = float(np.float32(2.0 ** -149))

# ScanFailure bits, include/saccade/selective_scan_cuda.hpp:30-44
NONFINITE_U, NONFINITE_DELTA, NONFINITE_A, NONFINITE_B, NONFINITE_C, NONFINITE_D = (1 << i for i in range(6))
DECAY_RANGE, DRIVE_RANGE, STATE_RANGE, TERM_RANGE, SKIP_RANGE, OUTPUT_RANGE = (1 << i for i in range(8, 14))
INPUT_FAILURES, RANGE_FAILURES = 0x3F, 0x3F00


def pow2(e: int) -> float:
    return float(np.float32(math.ldexp(1.0, e)))


def m_head_case(length: int) -> Case:
    """The m head's scan node, (4, L, 256, 16), shared A, rank-1 C, D (selective_scan_tests.cpp:166-188)."""
    k = filled(Shape(4, length, 256, 16, 1, 1, True), 0, 0, 0, 0)
    k.a = -np.arange(1, 17, dtype=np.float32)
    k.d = np.array([gen(7 * d, 5, 2, 4) for d in range(256)], np.float32)
    b_row = np.array([(n % 4 + 1) / 4 for n in range(16)], np.float32)
    for b in range(4):
        for t in range(length):
            token = b * length + t
            k.c[token] = np.float32((b + 1) / 2)
            k.b[token * 16:(token + 1) * 16] = b_row
            k.u[token * 256:(token + 1) * 256] = [gen(37 * b + 11 * d, 17, 8, 8) for d in range(256)]
    return k


def contract_cases() -> dict[str, tuple[Case, str]]:
    """S01 numeric fixtures: name -> (case, tolerance kind 'unit'|'relative')."""
    out = {}
    out["single_token"] = (Case(Shape(1, 1, 2, 2, 1, 2, True), [2, -4], [0, 21], [-1, -2], [0.5, 0.75], [1, 2],
                                [0.5, -1]), "unit")
    k = filled(Shape(1, 3, 1, 1, 1, 1, False), 0, 0, 1, 1)
    k.u = np.array([1, 2, 3], np.float32)
    out["three_token_decay"] = (k, "unit")
    k = filled(Shape(1, 1, 6, 1, 1, 1, False), 1, 0, 1, 1)
    k.delta = np.array([-30, -20, -1, 0, 20, 20.5], np.float32)
    out["softplus_branches"] = (k, "relative")
    k = filled(Shape(1, 400, 4, 16, 1, 1, True), 0, 0, 1, 1)
    k.u = np.tile(np.array([(d + 1) / 4 for d in range(4)], np.float32), 400)
    k.a = -np.arange(1, 17, dtype=np.float32)
    k.d = np.full(4, 0.5, np.float32)
    out["geometric_p3_length"] = (k, "unit")
    k = filled(Shape(1, 25, 3, 2, 3, 2, True), 0, 0, 0, 0)
    k.a = np.array([-1, -2, -0.5, -4, 0, -1], np.float32)
    k.d = np.array([0, 0.25, -1], np.float32)
    k.u = np.tile(np.array([1, -2, 0.5], np.float32), 25)
    k.b = np.tile(np.array([1, -0.5], np.float32), 25)
    k.c = np.tile(np.array([2, 1], np.float32), 25)
    out["per_channel_a"] = (k, "unit")
    k = filled(Shape(1, 100, 2, 32, 1, 1, False), 1, 0, 1, 0.5)
    k.a = (-np.arange(1, 33, dtype=np.float32) / np.float32(8)).astype(np.float32)
    k.u[1::2] = -1
    out["state_32_p4_length"] = (k, "unit")
    k = filled(Shape(2, 7, 3, 4, 1, 4, True), 0, 0, 0, 0)
    k.a = np.array([-0.5, -1, -2, -3], np.float32)
    k.d = np.array([-0.5, 0, 0.5], np.float32)
    for b in range(2):
        for t in range(7):
            token = b * 7 + t
            for d in range(3):
                k.delta[token * 3 + d] = gen(7 * b + 3 * t + 5 * d, 13, 6, 2)
                k.u[token * 3 + d] = gen(5 * b + 7 * t + 3 * d, 11, 5, 4)
            for n in range(4):
                k.b[token * 4 + n] = gen(3 * b + 5 * t + 7 * n, 9, 4, 4)
                k.c[token * 4 + n] = gen(7 * b + 3 * t + 5 * n, 7, 3, 2)
    out["varying_direct_sum"] = (k, "unit")
    big, small, top = pow2(100), pow2(-100), pow2(127)
    k = filled(Shape(1, 3, 1, 1, 1, 1, False), 0, big, small, 1)
    k.u = np.array([3, -5, 7], np.float32)
    out["extreme_large_delta_memoryless"] = (k, "relative")
    k = filled(Shape(1, 2, 1, 1, 1, 1, True), 0, -big, 1, 1)
    k.u = np.array([big, -big], np.float32)
    k.d = np.array([small], np.float32)
    out["extreme_negative_delta"] = (k, "relative")
    out["extreme_fp32_max_input"] = (filled(Shape(1, 1, 1, 1, 1, 1, False), top, -100, 1, 1), "relative")
    out["extreme_near_fp32_limit_output"] = (filled(Shape(1, 1, 1, 1, 1, 1, False), top, 21, pow2(-5), 1), "relative")
    out["extreme_subnormal_input"] = (filled(Shape(1, 2, 1, 1, 1, 1, False), DENORM_MIN, 0, 1, 1), "relative")
    k = filled(Shape(1, 3, 1, 1, 1, 1, False), 0, 0, 1, 1)
    k.u = np.array([1, 2, 3], np.float32)
    k.a = np.array([-FLT_MAX], np.float32)
    out["extreme_most_negative_a"] = (k, "unit")
    return out


def m_head_expected(length: int, k_table: np.ndarray, k: Case) -> np.ndarray:
    """Expected y of m_head_abi_L<length>: C_b u K_t + D_d u (selective_scan_tests.cpp:174-186)."""
    u = k.u.astype(np.float64).reshape(4, length, 256)
    c = k.c.astype(np.float64).reshape(4, length, 1)
    kt = np.asarray(k_table[:length], np.float64).reshape(1, length, 1)
    d = k.d.astype(np.float64).reshape(1, 1, 256)
    return (c * u * kt + d * u).reshape(-1)


def coverage_cases(include_large: bool = True) -> dict[str, Case]:
    """tests/scan_cuda_suite.hpp:461-501 (same shapes, seeds and ranges)."""
    out = {}
    seed = 0x5eed0001
    for n in (1, 2, 4, 8, 16, 32):
        tag = f"_N{n}"
        seed += 1
        out["shared_a_rank1_c_d" + tag] = random_case(Shape(2, 37, 5, n, 1, 1, True), seed)
        seed += 1
        out["per_channel_a_full_c_no_d" + tag] = random_case(Shape(3, 11, 7, n, 7, n, False), seed)
        seed += 1
        out["single_token_per_channel_a" + tag] = random_case(Shape(1, 1, 3, n, 3, 1, True), seed)
    seed += 1
    out["tail_1x1x1_N1"] = random_case(Shape(1, 1, 1, 1, 1, 1, False), seed)
    seed += 1
    out["tail_Dc13_N2"] = random_case(Shape(5, 3, 13, 2, 13, 2, True), seed)
    seed += 1
    out["tail_Dc257_N4"] = random_case(Shape(2, 4, 257, 4, 1, 4, True), seed)
    seed += 1
    out["tail_Dc33_N32"] = random_case(Shape(1, 3, 33, 32, 33, 32, True), seed)
    seed += 1  # empty_sequence consumes a seed (scan_cuda_suite.hpp:475)
    seed += 1
    out["long_slow_decay_L2000"] = random_case(Shape(1, 2000, 4, 16, 1, 1, True), seed,
                                               Ranges(1, -4, -2, -0.01, -0.001, 1, 1))
    for length in (25, 100, 400):
        seed += 1
        k = random_case(Shape(4, length, 256, 16, 1, 1, True), seed, Ranges(3, -5, 2, -1, -1, 2, 1))
        k.a = -np.arange(1, 17, dtype=np.float32)
        if include_large or length < 400:
            out[f"m_head_random_L{length}"] = k
    seed += 1
    k = random_case(Shape(1, 50, 3, 2, 1, 2, False), seed)
    k.a = np.array([-1.0, -1.0001], np.float32)
    for t in range(50):
        k.b[t * 2 + 1] = k.b[t * 2]
        k.c[t * 2] = 1
        k.c[t * 2 + 1] = -1
    out["cancellation_two_states"] = k
    return out


def empty_case() -> Case:
    return random_case(Shape(2, 0, 3, 4, 1, 1, True), 0x5eed0001 + 23)


def legacy_softplus(x: float) -> float:
    """The legacy kernel softplus emulated in FP32 (scan_cuda_suite.hpp:504-508)."""
    x = np.float32(x)
    if x > 20:
        return float(x)
    if x < -20:
        return float(np.exp(x))
    return float(np.log(np.float32(1) + np.exp(x)))


SOFTPLUS_SWEEP = [-1100, -1024, -1000, -300, -160, -150, -120, -110, -103.5, -100, -95, -90, -87.5, -85, -80.5,
                  float(np.nextafter(np.float32(-80), np.float32(-1000))), -80,
                  float(np.nextafter(np.float32(-80), np.float32(0))), -79.5, -60, -50, -30, -25, -20.5, -20, -19.5,
                  -18, -17, -15, -12, -10, -9, -8, -6, -4, -2, -1, -0.5, 0, 0.5, 1, 2, 5, 10, 15, 19.5, 20,
                  float(np.nextafter(np.float32(20), np.float32(100))), 20.5, 25, 100, 1000]


def softplus_cases(softplus) -> dict[str, Case]:
    """scan_cuda_suite.hpp:510-557; `softplus` is the binary64 reference softplus."""
    out = {"softplus_minus18": filled(Shape(1, 1, 1, 1, 1, 1, True), 1, -18, 1e8, 1)}
    xs = np.array(SOFTPLUS_SWEEP, np.float32)
    k = filled(Shape(1, 1, xs.size, 1, 1, 1, False), 1, 0, pow2(100), 1)
    k.delta = xs.copy()
    for i, x in enumerate(xs):
        delta = softplus(float(x)) * 2.0 ** 100
        e = int(math.floor(math.log2(delta))) if delta > 0 else -127
        k.u[i] = np.float32(math.ldexp(1.0, min(max(-e, -126), 127)))
    out["softplus_sweep"] = k
    return out


def intermediate_cases() -> dict[str, Case]:
    """scan_cuda_suite.hpp:560-578: reference-finite cases whose plain FP32 intermediates leave range."""
    p = 1
    out = {
        "drive_intermediate_overflow": filled(Shape(1, 2, 1, 1, 1, 1, False), pow2(-100), pow2(100), pow2(100), p),
        "drive_delta_underflow_minus100": filled(Shape(1, 1, 1, 1, 1, 1, False), pow2(27), -100, pow2(100), p),
        "drive_delta_underflow_minus150": filled(Shape(1, 1, 1, 1, 1, 1, False), pow2(127), -150, pow2(127), p),
        "drive_subnormal_b": filled(Shape(1, 1, 1, 1, 1, 1, False), pow2(127), 0.5413248, pow2(-140), p),
    }
    k = filled(Shape(1, 1, 1, 4, 1, 1, True), 1, 21, 0, 1.75)
    k.b = np.array([pow2(122), -pow2(122), pow2(122), -pow2(122)], np.float32)
    k.d = np.array([1], np.float32)
    out["butterfly_partial_sum_overflow"] = k
    k = filled(Shape(1, 1, 1, 2, 1, 1, True), 1, 21, pow2(122), 1.75)
    k.d = np.array([-pow2(127)], np.float32)
    out["partial_sum_overflow_restored_by_skip"] = k
    return out


def failure_cases() -> list[tuple[str, Case, int, bool, str]]:
    """scan_cuda_suite.hpp:580-616: (name, case, expected bits, exact, reference diagnostic)."""
    ok = varied(Shape(1, 4, 4, 16, 1, 1, True))
    nan, inf = float("nan"), float("inf")
    out = []

    def mod(name, field, idx, value, bit, diag, base=None):
        k = (base or ok).copy()
        getattr(k, field)[idx] = value
        out.append((name, k, bit, True, diag))

    mod("nonfinite_u", "u", 5, nan, NONFINITE_U, "u[5] is not finite")
    mod("nonfinite_delta", "delta", 0, inf, NONFINITE_DELTA, "delta[0] is not finite")
    mod("nonfinite_a", "a", 3, -inf, NONFINITE_A, "A[3] is not finite")
    mod("nonfinite_b", "b", 63, nan, NONFINITE_B, "B[63] is not finite")
    mod("nonfinite_c", "c", 2, inf, NONFINITE_C, "C[2] is not finite")
    mod("nonfinite_d", "d", 1, nan, NONFINITE_D, "D[1] is not finite")
    mod("empty_nonfinite_a", "a", 2, nan, NONFINITE_A, "A[2] is not finite", varied(Shape(2, 0, 3, 4, 1, 1, True)))
    mod("empty_nonfinite_d", "d", 2, -inf, NONFINITE_D, "D[2] is not finite", varied(Shape(2, 0, 3, 4, 3, 1, True)))
    top = pow2(127)
    out.append(("range_drive", filled(Shape(1, 1, 1, 1, 1, 1, False), top, 21, 4, 1), DRIVE_RANGE, True,
                "drive leaves FP32 range at batch 0, token 0"))
    k = filled(Shape(1, 1, 1, 1, 1, 1, False), 1, 21, 1, 1)
    k.a = np.array([100], np.float32)
    out.append(("range_decay", k, DECAY_RANGE, True, "decay leaves FP32 range"))
    k = filled(Shape(1, 200, 1, 1, 1, 1, False), 1, 0, 1, 1)
    k.a = np.array([1], np.float32)
    out.append(("range_state", k, STATE_RANGE, True, "state leaves FP32 range"))
    out.append(("range_c_state", filled(Shape(1, 2, 1, 1, 1, 1, False), 1, 21, pow2(120), top), TERM_RANGE, True,
                "C*state leaves FP32 range"))
    k = filled(Shape(1, 1, 1, 1, 1, 1, True), top, -100, 1, 1)
    k.d = np.array([4], np.float32)
    out.append(("range_d_u", k, SKIP_RANGE, True, "D*u leaves FP32 range"))
    out.append(("range_output", filled(Shape(1, 1, 1, 4, 1, 1, False), top, 21, pow2(-5), 1), OUTPUT_RANGE, True,
                "output leaves FP32 range"))
    k = random_case(Shape(2, 5, 6, 4, 1, 4, True), 0x5eed0100)
    at = (1 * 5 + 3) * 6 + 2
    k.u[at] = top
    k.delta[at] = 21
    k.b[(1 * 5 + 3) * 4:(1 * 5 + 3) * 4 + 4] = 1
    out.append(("range_one_lane_of_twelve", k, DRIVE_RANGE, False,
                "drive leaves FP32 range at batch 1, token 3, channel 2"))
    return out


def rejection_cases() -> list[tuple[str, Case, str]]:
    """selective_scan_tests.cpp:279-301 (shape, size and capacity rejections)."""
    ok = varied(Shape(1, 4, 4, 16, 1, 1, True))
    out = []
    for n in (0, 3, 64):
        k = ok.copy()
        k.shape.state = n
        out.append((f"state_{n}", k, "must be a power of two in [1, 32]"))
    k = ok.copy(); k.shape.a_rows = 2; k.a = np.zeros(32, np.float32)
    out.append(("a_rows", k, "A rows must be 1 or channels"))
    k = ok.copy(); k.shape.c_width = 4; k.c = np.zeros(16, np.float32)
    out.append(("c_width", k, "C width must be 1 or state"))
    k = ok.copy(); k.shape.batch = 0
    out.append(("batch_zero", k, "batch and channels must be positive"))
    k = ok.copy(); k.shape.channels = 0
    out.append(("channels_zero", k, "batch and channels must be positive"))
    return out


def capacity_shapes() -> list[tuple[Shape, str]]:
    """selective_scan_tests.cpp:299-301: rejected from the declared shape alone."""
    return [(Shape(1, 65536, 65536, 1, 1, 1, False), "u/delta/y element count exceeds int32 capacity"),
            (Shape(1, 1 << 27, 1, 32, 1, 1, False), "B element count exceeds int32 capacity"),
            (Shape(2, (1 << 64) // 2 - 1, 1, 1, 1, 1, False), "exceeds int32 capacity")]
