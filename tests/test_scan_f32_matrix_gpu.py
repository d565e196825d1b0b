"""The reference's verification matrix for its FP32 operator
(tools/scan_benchmark.cpp:184-234), run through sacc_selective_scan_f32.

Same shapes, case kinds and failure constructions, seeded inputs:
  * 144 matrix cases: N in {1..32} x shared / per-channel A x rank-1 / full C
    x with / without D x L in {0, 1, 19}, on (2, L, 17);
  * 18 deploy cases: (4, L, 256, 16), shared A, rank-1 C, D, L in
    {960, 240, 60, 400, 100, 25}, three seeds each;
  * per N: softplus at its branch thresholds, a drive whose plain FP32
    product Delta * B overflows while the scaled one is finite, a Delta
    underflowing below FP32's normal range, a NaN / infinity in each of the
    six tensors, and the six range failures.
Valid cases: every output within 2x the reference's running error bound of
the binary64 oracle, status (0, SACC_SCAN_DONE), and the same bits from a
repeated call and from a CUDA-graph replay.  Failures: the exact input bit,
or the range bit of the quantity the oracle reports first (single-lane
cases), y poisoned, done written.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from oracle.oracle import Shape, filled, random_case

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as gu  # noqa: E402
import saccade_v1_b200 as sb  # noqa: E402
import scan_cases as sc  # noqa: E402

RANGE_BIT = {"decay": 1 << 8, "drive": 1 << 9, "state": 1 << 10, "C*state": 1 << 11, "D*u": 1 << 12, "output": 1 << 13}
INPUT_BIT = [1 << i for i in range(6)]  # u, delta, A, B, C, D
THRESHOLDS = [-1100, -1024, np.nextafter(np.float32(-1024), np.float32(0)), -150, -100,
              np.nextafter(np.float32(-80), np.float32(-100)), -80, np.nextafter(np.float32(-80), np.float32(0)), -18,
              -0.0, 0, np.nextafter(np.float32(20), np.float32(0)), 20, np.nextafter(np.float32(20), np.float32(100)), 100,
              1000]


def matrix_cases():
    out, seed = [], 123
    for n in (1, 2, 4, 8, 16, 32):
        for shared in (True, False):
            for rank1 in (True, False):
                for has_d in (True, False):
                    for length in (0, 1, 19):
                        seed += 1
                        sh = Shape(2, length, 17, n, 1 if shared else 17, 1 if rank1 else n, has_d)
                        out.append((f"matrix-{seed}", random_case(sh, seed)))
    deploy = []
    for length in (960, 240, 60, 400, 100, 25):
        for _ in range(3):
            seed += 1
            deploy.append((f"deploy-L{length}-seed{seed}", random_case(Shape(4, length, 256, 16, 1, 1, True), seed)))
    return out, deploy, seed


def graph_bits(k):
    """y bits of one call captured in a CUDA graph and replayed."""
    sh = k.shape
    shape = sb.SelectiveScanShape(sh.batch, sh.length, sh.channels, sh.state, sh.a_rows, sh.c_width, sh.has_d)
    s = gu.stream()
    with torch.cuda.stream(s):
        bufs = [gu.dev(x) for x in k.inputs()]
        y = torch.empty(k.u.size, device="cuda")
        st = gu.new_status()
        sb.selective_scan_cuda(shape, *bufs, y, st, stream=s)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        sb.selective_scan_cuda(shape, *bufs, y, st, stream=s)
    y.zero_()
    with torch.cuda.stream(s):
        g.replay()
    s.synchronize()
    assert gu.status_words(st) == (0, sb.SCAN_DONE)
    return y.cpu().numpy().view(np.uint32).copy()


def check_valid(name, k, graph=False):
    y, st = gu.run_f32(k)
    assert st == (0, sb.SCAN_DONE), f"{name}: status {st}"
    if k.u.size == 0:
        return
    gu.compare_bound(name, y, oracle.run(k), oracle.scan_bound(k))
    y2, st2 = gu.run_f32(k)
    assert st2 == st and np.array_equal(y.view(np.uint32), y2.view(np.uint32)), f"{name}: repeat differs"
    if graph:
        assert np.array_equal(y.view(np.uint32), graph_bits(k)), f"{name}: graph replay differs"


def test_matrix_and_deploy_cases():
    matrix, deploy, _ = matrix_cases()
    assert len(matrix) == 144 and len(deploy) == 18
    for name, k in matrix:
        check_valid(name, k)
    for name, k in deploy:
        check_valid(name, k, graph=True)


@pytest.mark.parametrize("n", [1, 2, 4, 8, 16, 32])
def test_per_state_count_cases(n):
    _, _, seed = matrix_cases()
    seed += 6 * (n.bit_length() - 1)  # distinct seeds per N for the invalid-tensor cases
    k = filled(Shape(1, len(THRESHOLDS), 3, n, 1, 1, True), 1, 0, 1, 1)
    k.delta = np.repeat(np.array(THRESHOLDS, np.float32), 3)
    check_valid(f"softplus-N{n}", k)
    k = filled(Shape(1, 3, 3, n, 1, n, True), 2.0 ** -100, 2.0 ** 100, 2.0 ** 100, 2.0 ** -100)
    check_valid(f"scaled-drive-N{n}", k)
    k = filled(Shape(1, 3, 3, n, 1, 1, True), 2.0 ** 100, -150, 2.0 ** 100, 2.0 ** -100)
    check_valid(f"scaled-delta-N{n}", k)
    for tensor in range(6):
        seed += 1
        k = random_case(Shape(1, 5, 3, n, 1, 1, True), seed)
        field = ("u", "delta", "a", "b", "c", "d")[tensor]
        getattr(k, field)[0] = np.nan if tensor % 2 else np.inf
        y, (flags, done) = gu.run_f32(k)
        assert flags & sc.INPUT_FAILURES == INPUT_BIT[tensor] and done == sb.SCAN_DONE, (n, tensor, hex(flags))
        assert np.all(y.view(np.uint32) == gu.POISON), (n, tensor)
    for kind in range(6):
        k = filled(Shape(1, 3, 1, n, 1, 1, True), 1, 0, 1, 1)
        if kind == 0:
            k.a[:], k.delta[:] = 1000, 1
        elif kind == 1:
            k.u[:], k.b[:] = 2.0 ** 100, 2.0 ** 100
        elif kind == 2:
            k.a[:], k.delta[:], k.u[:] = 1, 40, 2.0 ** 60
        elif kind == 3:
            k.u[:], k.c[:] = 2.0 ** 90, 2.0 ** 90
        elif kind == 4:
            k.u[:], k.d[:] = 2.0 ** 100, 2.0 ** 100
        else:
            k.a[:], k.u[:], k.b[:] = -100, 2.0 ** 126, 4
        status, _, msg = oracle.scan_ref(k)
        y, (flags, done) = gu.run_f32(k)
        assert done == sb.SCAN_DONE, (n, kind)
        if status == oracle.OK:
            assert flags == 0, (n, kind, hex(flags))
            continue
        quantity = msg.split("selective_scan: ")[1].split(" leaves")[0]
        assert flags == RANGE_BIT[quantity], (n, kind, quantity, hex(flags))
        assert np.all(y.view(np.uint32) == gu.POISON), (n, kind)
