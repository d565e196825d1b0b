"""The device's Mamba block and Cross-Scan head level against the reference's own binary64 head.

tests/golden/head_ref_p5.npz holds what the reference's head_reference
(src/head_reference.cpp:434-441) computed on synthetic_head_weights(3) and
head_test_features("random", 1) at the T01 profile, P5 level: the block's FP32
parameters, its 4 x 25 input tokens, the block output with the residual, the
downsampled map and the merged level output (generator:
tests/golden/make_head_golden.py).  The device runs with FP16 weights and
activations, as the reference's FP16 engine does; tolerance (BASELINE, 16-bit
activations against an FP32-or-better reference): |gpu - ref| <= 1e-3 + 1e-2 |ref|.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import saccade_v1_b200 as sb  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "head_ref_p5.npz")


def device_params(g, dtype):
    p = {k[2:]: np.asarray(g[k], np.float32) for k in g.files if k.startswith("w.")}
    D = p["w_in"].shape[0] // 2
    a = (-np.exp(p.pop("A_log").astype(np.float64))).astype(np.float32)
    p["A"] = np.tile(a.reshape(1, -1), (D, 1))
    out = {}
    for k, v in p.items():
        t = torch.from_numpy(np.ascontiguousarray(v)).cuda()
        out[k] = t.to(dtype) if k in ("w_in", "w_x", "w_dt", "w_out") else t
    return out


def check(name, got, ref):
    err = np.abs(got.astype(np.float64) - ref)
    bad = ~(err <= 1e-3 + 1e-2 * np.abs(ref))
    assert not bad.any(), f"{name}: {int(bad.sum())}/{got.size} beyond 1e-3 + 1e-2|ref|, max err {err.max():.3g}"


def test_block_matches_reference_head_block():
    g = np.load(GOLDEN)
    p = device_params(g, torch.float16)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x = torch.from_numpy(g["tokens"].astype(np.float32)).cuda().to(torch.float16)
        y = sb.mamba_block_forward(x, p, stream=s)
    s.synchronize()
    check("p5.residual", y.float().cpu().numpy(), g["residual"])
    assert sb.scan_fault() == 0


def test_head_level_matches_reference_merge():
    g = np.load(GOLDEN)
    p = device_params(g, torch.float16)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x = torch.from_numpy(np.ascontiguousarray(g["downsample"], np.float32)).cuda()
        out = sb.cross_scan_block_forward(x, p, dtype=torch.float16, stream=s)
    s.synchronize()
    check("p5.merge", out.cpu().numpy(), g["merge"])
    assert sb.scan_fault() == 0
