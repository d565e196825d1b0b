"""The four-threads-per-lane reference-ABI scan keeps the reference's summation tree.

The reference sums a token's N terms C_n h_n with an xor butterfly over N lanes, offset N/2 first
(cuda/selective_scan.cu:63-66).  scan_f32_quad_kernel (saccade_v1_b200/csrc/scan_f32.cu) gives thread q of a
lane the states q, q + 4, ..., q + N - 4, sums its own N/4 terms with the same butterfly (offset N/8 first
over its values: the reference's levels of offset 4 and more), then adds the partner's partial at xor 2 and
at xor 1.  This test replays both in binary32 arithmetic and requires the same bits on all four threads.
"""
import numpy as np
import pytest


def butterfly(v):
    """Reference order: v[i] = v[i] + v[i + w] for w = N/2, N/4, ..., 1, in binary32."""
    v = np.array(v, dtype=np.float32)
    w = len(v) // 2
    while w > 0:
        v[:w] = v[:w] + v[w:2 * w]
        w //= 2
    return v[0]


def quad(v):
    """The four threads' partials, then the xor-2 and xor-1 exchanges; returns every thread's result."""
    v = np.asarray(v, dtype=np.float32)
    part = [butterfly(v[q::4]) for q in range(4)]
    part = [np.float32(part[q] + part[q ^ 2]) for q in range(4)]
    return [np.float32(part[q] + part[q ^ 1]) for q in range(4)]


@pytest.mark.parametrize("n", [8, 16, 32])
def test_four_thread_sum_is_the_reference_butterfly(n):
    rng = np.random.default_rng(n)
    for trial in range(2000):
        scale = 10.0 ** rng.integers(-30, 30, size=n)
        v = (rng.standard_normal(n) * scale).astype(np.float32)
        if trial % 3 == 0:
            v[rng.integers(0, n)] = -v.sum(dtype=np.float32)  # cancellation
        want = butterfly(v)
        for got in quad(v):
            assert np.float32(got).view(np.uint32) == np.float32(want).view(np.uint32), (n, trial)


def test_a_different_split_would_change_bits():
    """States in contiguous blocks of N/4 per thread give another association; the test above is not vacuous."""
    rng = np.random.default_rng(7)
    differ = 0
    for _ in range(2000):
        v = (rng.standard_normal(16) * 10.0 ** rng.integers(-8, 8, size=16)).astype(np.float32)
        blocks = [butterfly(v[4 * q:4 * q + 4]) for q in range(4)]
        other = np.float32(np.float32(blocks[0] + blocks[1]) + np.float32(blocks[2] + blocks[3]))
        differ += other.view(np.uint32) != butterfly(v).view(np.uint32)
    assert differ > 0
