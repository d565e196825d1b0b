"""Generates the golden fixtures under tests/golden/ from the reference.

Run from the repository root, naming the reference checkout on the command
line or in SACC_REFERENCE_ROOT:
    make -C oracle REF=<reference checkout>   # builds oracle/_ref/libref_scan.so from it
    python tests/golden/make_golden.py <reference checkout>

Writes
  scan_expected.json  the bc-derived closed-form values of the reference's
                      fixtures/selective-scan/expected.tsv (value * 2^exp2),
                      read as text and re-encoded as float64 per case
  scan_ref_outputs.npz outputs and diagnostics of the reference's own
                      selective_scan_reference (oracle/_ref) on the case
                      inputs of tests/scan_cases.py: full outputs for small
                      cases, a digest (sum, sum |y|, 257 sampled elements) for
                      the large deploy-shape cases.
The tests read only these files; they never open the reference checkout.
"""
from __future__ import annotations

import json
import os
import sys
from decimal import Decimal, getcontext

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle import oracle  # noqa: E402
import scan_cases as sc  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
FULL_LIMIT = 10000


def digest_indices(n: int) -> np.ndarray:
    return np.unique(np.linspace(0, n - 1, 257).astype(np.int64)) if n else np.zeros(0, np.int64)


def expected_table(ref_root: str) -> dict[str, list[float]]:
    getcontext().prec = 60
    table: dict[str, list[float]] = {}
    with open(os.path.join(ref_root, "fixtures", "selective-scan", "expected.tsv")) as f:
        for line in f:
            name, index, value, exp2 = line.rstrip("\n").split("\t")
            col = table.setdefault(name, [])
            assert int(index) == len(col), line
            col.append(float(Decimal(value) * (Decimal(2) ** int(exp2))))
    return table


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SACC_REFERENCE_ROOT", "")
    if not ref_root or not os.path.isdir(ref_root):
        sys.exit("usage: make_golden.py <reference checkout> (or set SACC_REFERENCE_ROOT)")
    with open(os.path.join(OUT, "scan_expected.json"), "w") as f:
        json.dump(expected_table(ref_root), f, indent=0)

    assert oracle.ref_available(), "build oracle/_ref first: make -C oracle"
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {}

    def record(name: str, k: oracle.Case) -> None:
        st, y, msg = oracle.scan_reference_impl(k)
        meta[name] = {"status": st, "message": msg, "count": int(y.size)}
        if st == 0:
            if y.size <= FULL_LIMIT:
                arrays[name] = y
            else:
                idx = digest_indices(y.size)
                arrays[name + ".idx"] = idx
                arrays[name + ".val"] = y[idx]
                meta[name]["sum"] = float(np.sum(y))
                meta[name]["abs_sum"] = float(np.sum(np.abs(y)))

    for name, (k, _) in sc.contract_cases().items():
        record("contract." + name, k)
    for length in (25, 100, 400):
        record(f"contract.m_head_abi_L{length}", sc.m_head_case(length))
    for name, k in sc.coverage_cases().items():
        record("coverage." + name, k)
    for name, k in sc.softplus_cases(oracle.ref_lib().sacc_ref_softplus).items():
        record("softplus." + name, k)
    for name, k in sc.intermediate_cases().items():
        record("intermediate." + name, k)
    for name, k, _, _, _ in sc.failure_cases():
        record("failure." + name, k)
    for name, k, _ in sc.rejection_cases():
        record("rejection." + name, k)
    xs = np.array(sc.SOFTPLUS_SWEEP + [20.25, -18.0, 0.0], np.float64)
    arrays["softplus_points"] = xs
    arrays["softplus_values"] = np.array([oracle.ref_lib().sacc_ref_softplus(float(x)) for x in xs])
    arrays["meta"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(OUT, "scan_ref_outputs.npz"), **arrays)
    print(f"wrote {len(meta)} reference cases")


if __name__ == "__main__":
    main()
