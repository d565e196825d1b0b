"""Helpers for the GPU parity tests: run oracle cases through the C ABI.

Mirrors the reference's DirectBackend (tests/scan_cuda_suite.hpp:242-316):
fresh device buffers per case, y pre-filled with 0xA5 bytes and the status
with the sentinel {0xFFFFFFFF, 0x12345678}, so that every call must clear and
complete both.
"""
from __future__ import annotations

import numpy as np
import torch

import saccade_v1_b200 as sb
from oracle import oracle

STATUS_SENTINEL = (0xFFFFFFFF, 0x12345678)
POISON = 0x7FC00000


def stream():
    return torch.cuda.Stream()


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def new_status():
    return torch.tensor(np.array(STATUS_SENTINEL, np.uint32).view(np.int32), device="cuda")


def status_words(t) -> tuple[int, int]:
    w = t.cpu().numpy().view(np.uint32)
    return int(w[0]), int(w[1])


def run_f32(k: oracle.Case, s=None):
    """Runs a reference-ABI case on the GPU; returns (y float32 numpy, (flags, done))."""
    s = s or stream()
    shape = sb.SelectiveScanShape(k.shape.batch, k.shape.length, k.shape.channels, k.shape.state,
                                  k.shape.a_rows, k.shape.c_width, k.shape.has_d)
    with torch.cuda.stream(s):
        t = [dev(x) for x in k.inputs()]
        y = torch.empty(k.u.size, dtype=torch.int32, device="cuda")
        y.fill_(np.int32(np.uint32(0xA5A5A5A5).view(np.int32)))
        st = new_status()
        sb.selective_scan_cuda(shape, *t, y, st, stream=s)
    s.synchronize()
    return y.cpu().numpy().view(np.float32).copy(), status_words(st)


def compare_bound(name, gpu, ref, bound):
    """|gpu - ref| <= 2 * bound elementwise (tests/scan_cuda_suite.hpp:208-238)."""
    gpu = np.asarray(gpu, np.float64)
    err = np.abs(gpu - ref)
    tol = 2 * bound
    bad = ~(err <= tol)
    if bad.any():
        i = int(np.argmax(np.where(bad, err / np.maximum(tol, 1e-300), -1)))
        raise AssertionError(f"{name}: {int(bad.sum())} of {gpu.size} elements beyond 2x bound; worst index {i}: "
                             f"gpu {gpu[i]!r} ref {ref[i]!r} tol {tol[i]!r}")
    ratio = float(np.max(np.where(tol > 0, err / np.where(tol > 0, tol, 1), 0))) if gpu.size else 0.0
    return ratio
