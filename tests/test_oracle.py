"""Pins the CPU oracle before anything is checked against it.

The C restatement (oracle/scan_oracle.c) must
  - reproduce the bc-derived closed forms of the reference's
    fixtures/selective-scan/expected.tsv within the reference's own
    tolerances (tests/selective_scan_tests.cpp:43-47),
  - reproduce the outputs and diagnostics of the reference's own
    selective_scan_reference (recorded in tests/golden/scan_ref_outputs.npz)
    bit for bit,
  - satisfy the reference's contract equalities (selective_scan_tests.cpp:235-277).
The extended entry (state in/out, varlen, bias, gate, layouts) reduces to the
reference recurrence exactly and is pinned by contract equalities derived
from it.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle
from oracle.oracle import Shape, filled, varied
import scan_cases as sc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
UNIT = (1e-10, 1e-10)
RELATIVE = (0.0, 1e-10)


@pytest.fixture(scope="module")
def expected():
    with open(os.path.join(GOLDEN, "scan_expected.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def ref_out():
    z = np.load(os.path.join(GOLDEN, "scan_ref_outputs.npz"))
    meta = json.loads(bytes(z["meta"]).decode())
    return z, meta


def within(actual, want, tol):
    atol, rtol = tol
    want = np.asarray(want, np.float64)
    return np.all(np.abs(np.asarray(actual) - want) <= atol + rtol * np.abs(want))


def test_softplus_threshold_and_reference_values(ref_out):
    z, _ = ref_out
    assert abs(oracle.softplus(20.0) - 20.0000000020611536203) < 1e-13
    assert oracle.softplus(20.25) == 20.25
    got = np.array([oracle.softplus(x) for x in z["softplus_points"]])
    assert np.array_equal(got, z["softplus_values"])


def test_contract_values_match_bc_closed_forms(expected):
    for name, (k, kind) in sc.contract_cases().items():
        y = oracle.run(k)
        assert within(y, expected[name], UNIT if kind == "unit" else RELATIVE), name
    table = np.array(expected["m_head_k"])
    for length in (25, 100, 400):
        k = sc.m_head_case(length)
        assert within(oracle.run(k), sc.m_head_expected(length, table, k), UNIT), length


def _check_against_reference(name, k, z, meta):
    st, y, msg = oracle.scan_ref(k)
    m = meta[name]
    assert st == m["status"], (name, msg, m["message"])
    assert msg == m["message"], name
    if st != 0:
        return
    if name in z.files:
        assert np.array_equal(y, z[name]), name
    else:
        idx = z[name + ".idx"]
        assert np.array_equal(y[idx], z[name + ".val"]), name
        assert float(np.sum(y)) == m["sum"] and float(np.sum(np.abs(y))) == m["abs_sum"], name


def test_oracle_is_bit_identical_to_reference_implementation(ref_out):
    z, meta = ref_out
    for name, (k, _) in sc.contract_cases().items():
        _check_against_reference("contract." + name, k, z, meta)
    for length in (25, 100, 400):
        _check_against_reference(f"contract.m_head_abi_L{length}", sc.m_head_case(length), z, meta)
    for name, k in sc.coverage_cases().items():
        _check_against_reference("coverage." + name, k, z, meta)
    for name, k in sc.softplus_cases(oracle.softplus).items():
        _check_against_reference("softplus." + name, k, z, meta)
    for name, k in sc.intermediate_cases().items():
        _check_against_reference("intermediate." + name, k, z, meta)


def test_failures_and_rejections_carry_reference_diagnostics(ref_out):
    z, meta = ref_out
    for name, k, bit, exact, diag in sc.failure_cases():
        _check_against_reference("failure." + name, k, z, meta)
        st, _, msg = oracle.scan_ref(k)
        assert st == (oracle.INVALID if bit & sc.INPUT_FAILURES else oracle.RANGE)
        assert diag in msg
    for name, k, diag in sc.rejection_cases():
        _check_against_reference("rejection." + name, k, z, meta)
        assert diag in oracle.scan_ref(k)[2]


def test_size_and_capacity_rejections():
    ok = varied(Shape(1, 4, 4, 16, 1, 1, True))
    cases = [("u", -1, "u has 15 values, shape needs 16"), ("delta", +1, "delta has 17 values"),
             ("a", -1, "A has 15 values"), ("b", -1, "B has 63 values"), ("c", +1, "C has 5 values"),
             ("d", -1, "D has 3 values")]
    for field, delta, diag in cases:
        k = ok.copy()
        arr = getattr(k, field)
        setattr(k, field, arr[:-1].copy() if delta < 0 else np.append(arr, np.float32(0)))
        st, _, msg = oracle.scan_ref(k)
        assert st == oracle.INVALID and diag in msg, (field, msg)
    k = ok.copy()
    k.shape.has_d = False
    assert "D has 4 values, shape needs 0" in oracle.scan_ref(k)[2]
    for shape, diag in sc.capacity_shapes():
        empty = oracle.Case(shape, [], [], [], [], [], [])
        st, _, msg = oracle.scan_ref(empty)
        assert st == oracle.INVALID and diag in msg, msg


def test_contract_equalities():
    """selective_scan_tests.cpp:235-277."""
    base = Shape(2, 9, 3, 8, 1, 1, True)
    rank1 = varied(base)
    full = rank1.copy()
    full.shape.c_width = 8
    full.c = np.repeat(rank1.c, 8)
    assert np.array_equal(oracle.run(rank1), oracle.run(full))
    rows = rank1.copy()
    rows.shape.a_rows = 3
    rows.a = np.tile(rank1.a, 3)
    assert np.array_equal(oracle.run(rank1), oracle.run(rows))
    single = varied(Shape(1, 9, 3, 8, 1, 1, True))
    pair = single.copy()
    pair.shape.batch = 2
    pair.u = np.concatenate([np.full(27, 100, np.float32), pair.u])
    pair.delta = np.concatenate([np.full(27, 5, np.float32), pair.delta])
    pair.b = np.concatenate([np.ones(72, np.float32), pair.b])
    pair.c = np.concatenate([np.ones(9, np.float32), pair.c])
    pair.a = np.full(8, -0.001, np.float32)
    single.a = pair.a.copy()
    assert np.array_equal(oracle.run(pair)[27:], oracle.run(single))
    no_d = rank1.copy()
    no_d.shape.has_d = False
    no_d.d = np.zeros(0, np.float32)
    zero_d = rank1.copy()
    zero_d.d = np.zeros(3, np.float32)
    assert np.array_equal(oracle.run(no_d), oracle.run(zero_d))
    empty = varied(Shape(2, 0, 3, 4, 1, 1, True))
    assert empty.u.size == 0 and oracle.run(empty).size == 0


def _ex_from_case(k):
    s = k.shape
    u = k.u.reshape(s.batch, s.length, s.channels)
    delta = k.delta.reshape(u.shape)
    b = k.b.reshape(s.batch, s.length, 1, s.state)
    c = k.c.reshape(s.batch, s.length, 1, s.c_width)
    return u, delta, k.a.reshape(s.a_rows, s.state), b, c, (k.d if s.has_d else None)


def test_extended_scan_reduces_to_reference_exactly():
    for name, k in sc.coverage_cases(include_large=False).items():
        u, delta, a, b, c, d = _ex_from_case(k)
        y, _ = oracle.scan_ex(u, delta, a, b, c, layout="BLD", d=d)
        assert np.array_equal(y.reshape(-1), oracle.run(k)), name


def _rand_ex(seed, B=2, L=23, D=6, N=4, G=1):
    r = np.random.default_rng(seed)
    f = lambda *s: r.standard_normal(s).astype(np.float32)
    return dict(u=f(B, L, D), delta=(f(B, L, D) - 1).astype(np.float32), a=-np.abs(f(D, N)) - 0.1,
                b=f(B, L, G, N), c=f(B, L, G, N), d=f(D), z=f(B, L, D), bias=(0.3 * f(D)).astype(np.float32),
                h0=f(B, D, N))


def test_extended_layouts_agree():
    t = _rand_ex(1, G=2)
    y1, h1 = oracle.scan_ex(t["u"], t["delta"], t["a"], t["b"], t["c"], layout="BLD", d=t["d"], z=t["z"],
                            delta_bias=t["bias"], h0=t["h0"], want_final=True, groups=2)
    tr = lambda x: np.ascontiguousarray(np.moveaxis(x, 1, -1))
    y2, h2 = oracle.scan_ex(tr(t["u"]), tr(t["delta"]), t["a"], tr(t["b"]), tr(t["c"]), layout="BDL", d=t["d"],
                            z=tr(t["z"]), delta_bias=t["bias"], h0=t["h0"], want_final=True, groups=2)
    assert np.array_equal(y1, np.moveaxis(y2, -1, 1)) and np.array_equal(h1, h2)


def test_extended_split_sequence_chains_through_state():
    t = _rand_ex(2)
    kw = dict(layout="BLD", d=t["d"], z=t["z"], delta_bias=t["bias"], want_final=True)
    y, h = oracle.scan_ex(t["u"], t["delta"], t["a"], t["b"], t["c"], h0=t["h0"], **kw)
    cut = 9
    sl = lambda x, a, b: np.ascontiguousarray(x[:, a:b])
    y1, h1 = oracle.scan_ex(*(sl(t[k], 0, cut) for k in ("u", "delta")), t["a"],
                            *(sl(t[k], 0, cut) for k in ("b", "c")), h0=t["h0"], **{**kw, "z": sl(t["z"], 0, cut)})
    y2, h2 = oracle.scan_ex(*(sl(t[k], cut, None) for k in ("u", "delta")), t["a"],
                            *(sl(t[k], cut, None) for k in ("b", "c")), h0=h1.astype(np.float32),
                            **{**kw, "z": sl(t["z"], cut, None)})
    # State crosses the cut rounded to FP32 (the state dtype of the device path).
    np.testing.assert_allclose(np.concatenate([y1, y2], axis=1), y, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(h2, h, rtol=1e-6, atol=1e-6)
    assert np.array_equal(y1, y[:, :cut])


def test_extended_varlen_equals_separate_calls():
    t = _rand_ex(3, B=1, L=30)
    cu = np.array([0, 7, 8, 21, 30], np.int32)
    h0 = np.random.default_rng(9).standard_normal((4, 6, 4)).astype(np.float32)
    y, hf = oracle.scan_ex(t["u"], t["delta"], t["a"], t["b"], t["c"], d=t["d"], z=t["z"], delta_bias=t["bias"],
                           h0=h0, want_final=True, cu_seqlens=cu)
    for s in range(4):
        a, b = cu[s], cu[s + 1]
        sl = lambda x: np.ascontiguousarray(x[:, a:b])
        ys, hs = oracle.scan_ex(sl(t["u"]), sl(t["delta"]), t["a"], sl(t["b"]), sl(t["c"]), d=t["d"], z=sl(t["z"]),
                                delta_bias=t["bias"], h0=h0[s:s + 1], want_final=True)
        assert np.array_equal(ys, y[:, a:b]) and np.array_equal(hs[0], hf[s])


def test_extended_bias_and_gate_match_pre_add_and_multiply():
    t = _rand_ex(4)
    y, _ = oracle.scan_ex(t["u"], t["delta"], t["a"], t["b"], t["c"], d=t["d"], z=t["z"], delta_bias=t["bias"])
    pre = (t["delta"].astype(np.float64) + t["bias"].astype(np.float64))
    y0, _ = oracle.scan_ex(t["u"], pre.astype(np.float32), t["a"], t["b"], t["c"], d=t["d"])
    z = t["z"].astype(np.float64)
    np.testing.assert_allclose(y, y0 * z / (1 + np.exp(-z)), rtol=1e-5, atol=1e-6)


def test_cross_scan_orders():
    """selective_scan_tests.cpp:319-350 (hand-listed orders, batching, merge inverts expand)."""
    x = np.zeros(12, np.float32)
    for c in range(2):
        for h in range(2):
            for w in range(3):
                x[(c * 2 + h) * 3 + w] = 100 * c + 10 * h + w
    order = [[0, 1, 2, 10, 11, 12], [12, 11, 10, 2, 1, 0], [2, 1, 0, 12, 11, 10], [10, 11, 12, 0, 1, 2]]
    tokens = oracle.cross_scan_expand(x, 1, 2, 2, 3)
    for k in range(4):
        for t in range(6):
            for c in range(2):
                assert tokens[(k * 6 + t) * 2 + c] == 100 * c + order[k][t]
    row = [[0, 1, 2, 3], [3, 2, 1, 0], [3, 2, 1, 0], [0, 1, 2, 3]]
    column = [[0, 1, 2], [2, 1, 0], [0, 1, 2], [2, 1, 0]]
    for k in range(4):
        assert [oracle.cross_scan_source(k, t, 1, 4) for t in range(4)] == row[k]
        assert [oracle.cross_scan_source(k, t, 3, 1) for t in range(3)] == column[k]
    two = np.concatenate([x, x + 1000])
    batched = oracle.cross_scan_expand(two, 2, 2, 2, 3)
    merged = oracle.cross_scan_merge(batched.astype(np.float64), 2, 2, 2, 3)
    assert np.array_equal(merged, two.astype(np.float64))
    with pytest.raises(ValueError):
        oracle.cross_scan_source(4, 0, 2, 3)


def test_cross_scan_prefix_merge_matches_bc(expected):
    k = filled(Shape(4, 6, 1, 1, 1, 1, False), 0, 0, 1, 1)
    k.u = oracle.cross_scan_expand(np.arange(1, 7, dtype=np.float32), 1, 1, 2, 3)
    k.a = np.zeros(1, np.float32)
    got = oracle.cross_scan_merge(oracle.run(k), 1, 1, 2, 3)
    assert within(got, expected["cross_scan_prefix_merge"], UNIT)
