"""GPU parity of Cross-Scan expand / merge and the expand -> scan -> merge
pipeline (reference tests/scan_cuda_suite.hpp:627-721): expand bit-identical
to the reference permutation, merge within 2 (gamma_4 sum|y_k| / 4 + eta),
the pipeline within the propagated scan bound, non-finite inputs flagged with
the whole output poisoned."""
import numpy as np
import pytest
import torch

from oracle import oracle
from oracle.oracle import Random, Shape, filled, random_case

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as gu  # noqa: E402
import saccade_v1_b200 as sb  # noqa: E402

U = 2.0 ** -24
G4 = 4 * U / (1 - 4 * U)
ETA = 2.0 ** -150


def rand_floats(n, seed, rng):
    return Random(seed).uniform_array(n, -rng, rng)


def expand(shape, x):
    s = gu.stream()
    with torch.cuda.stream(s):
        dx = gu.dev(x)
        t = torch.empty(4 * x.size, device="cuda")
        st = gu.new_status()
        sb.cross_scan_expand_cuda(sb.CrossScanShape(*shape), dx, t, st, stream=s)
    s.synchronize()
    return t.cpu().numpy(), gu.status_words(st)


def merge(shape, y):
    s = gu.stream()
    with torch.cuda.stream(s):
        dy = gu.dev(y)
        o = torch.empty(y.size // 4, device="cuda")
        st = gu.new_status()
        sb.cross_scan_merge_cuda(sb.CrossScanShape(*shape), dy, o, st, stream=s)
    s.synchronize()
    return o.cpu().numpy(), gu.status_words(st)


def merge_bound(shape, y):
    b, c, h, w = shape
    L = h * w
    out = np.zeros(b * c * L)
    for i in range(b):
        for ch in range(c):
            for p in range(L):
                s = sum(abs(float(y[((k * b + i) * L + oracle.cross_scan_source(k, p, h, w)) * c + ch])) for k in range(4))
                out[(i * c + ch) * L + p] = G4 * s / 4 + ETA
    return out


SHAPES = [(1, 2, 2, 3), (2, 3, 3, 5), (1, 4, 1, 4), (1, 4, 4, 1), (1, 1, 1, 1), (2, 5, 7, 3), (1, 128, 20, 20),
          (1, 128, 10, 10), (1, 128, 5, 5)]


def test_expand_bitwise_and_merge_within_bound():
    seed = 0x5eed0400
    for shape in SHAPES:
        n = int(np.prod(shape))
        seed += 1
        x = rand_floats(n, seed, 4)
        if shape == (1, 2, 2, 3):
            x = np.array([100 * c + 10 * h + w for c in range(2) for h in range(2) for w in range(3)], np.float32)
        t, st = expand(shape, x)
        assert st == (0, sb.SCAN_DONE)
        assert np.array_equal(t.view(np.uint32), oracle.cross_scan_expand(x, *shape).view(np.uint32)), shape
        seed += 1
        y = rand_floats(4 * n, seed, 8)
        m, st = merge(shape, y)
        assert st == (0, sb.SCAN_DONE)
        ref = oracle.cross_scan_merge(y.astype(np.float64), *shape)
        if n <= 2000:
            gu.compare_bound(f"merge_{shape}", m, ref, merge_bound(shape, y))
        else:
            assert np.all(np.abs(m - ref) <= 2 * (G4 * np.abs(ref) * 4 + 1e-30) + 1e-6), shape


def test_merge_partial_sum_overflow_and_nonfinite():
    shape = (1, 2, 1, 2)
    y = np.full(16, 0.75 * np.finfo(np.float32).max, np.float32)
    y[8:] = -y[8:] / 3
    m, st = merge(shape, y)
    assert st == (0, sb.SCAN_DONE)
    gu.compare_bound("merge_overflow", m, oracle.cross_scan_merge(y.astype(np.float64), *shape), merge_bound(shape, y))
    x = np.ones(12, np.float32)
    x[7] = np.inf
    t, st = expand((1, 2, 2, 3), x)
    assert st == (1 << 16, sb.SCAN_DONE) and np.all(t.view(np.uint32) == gu.POISON)
    y = np.ones(48, np.float32)
    y[30] = np.nan
    m, st = merge((1, 2, 2, 3), y)
    assert st == (1 << 16, sb.SCAN_DONE) and np.all(m.view(np.uint32) == gu.POISON)


def test_expand_scan_merge_pipeline():
    seed = 0x5eed0500
    for shape in [(1, 1, 2, 3), (1, 8, 5, 5)]:
        _, C, H, W = shape
        L = H * W
        hand = C == 1
        seed += 1
        x = np.arange(1, 7, dtype=np.float32) if hand else rand_floats(C * L, seed, 2)
        seed += 1
        k = filled(Shape(4, L, 1, 1, 1, 1, False), 0, 0, 1, 1) if hand else random_case(Shape(4, L, C, 4, 1, 1, True), seed)
        if hand:
            k.a = np.zeros(1, np.float32)
        k.u = oracle.cross_scan_expand(x, 1, C, H, W)
        ref_y = oracle.run(k)
        scan_e = oracle.scan_bound(k)
        ref = oracle.cross_scan_merge(ref_y, 1, C, H, W)
        bound = np.zeros(ref.size)
        for ch in range(C):
            for p in range(L):
                at = [(d * L + oracle.cross_scan_source(d, p, H, W)) * C + ch for d in range(4)]
                bound[ch * L + p] = (1 + G4) * sum(scan_e[a] for a in at) / 4 + G4 * sum(abs(ref_y[a]) for a in at) / 4 + ETA
        t, st = expand(shape, x)
        assert st == (0, sb.SCAN_DONE)
        k2 = k.copy()
        k2.u = t
        y, st = gu.run_f32(k2)
        assert st == (0, sb.SCAN_DONE)
        m, st = merge(shape, y)
        assert st == (0, sb.SCAN_DONE)
        gu.compare_bound(f"pipeline_{shape}", m, ref, bound)
