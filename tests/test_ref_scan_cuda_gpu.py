"""The reference's own CUDA scan on the same B200, beside this library's reference-ABI kernel.

oracle/_ref/libref_scan_cuda.so is the reference's cuda/selective_scan.cu
(kernels :78-155, host :270-311) built for sm_100a with its own scan flags by
oracle/Makefile.  On the reference's deploy shapes (HR 1280x768: 4 directions
x L = 960 / 240 / 60 tokens; T01 640x640: L = 400 / 100 / 25; 256 channels,
N = 16, shared A, rank-1 C, D) both implementations run on the same inputs:
  * both within twice the reference's running error bound of the binary64
    oracle (the reference's acceptance rule, tests/scan_cuda_suite.hpp), with
    status done and no flags;
  * each call's device time (CUDA events, eager, mean of 50 after warm-up, and
    the three levels replayed from one CUDA graph), written to
    gpurun_out/ref_scan_cuda_times.json when that folder exists; this
    library's three-level total must be below the reference's.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from oracle import ref_scan_cuda as rsc

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)
if rsc.load() is None:
    pytest.skip("oracle/_ref/libref_scan_cuda.so not built", allow_module_level=True)

import saccade_v1_b200 as sb  # noqa: E402
from gpu_util import compare_bound  # noqa: E402

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PROFILES = {"HR": (960, 240, 60), "T01": (400, 100, 25)}


def level_case(L, seed):
    k = oracle.random_case(oracle.Shape(4, L, 256, 16, 1, 1, True), seed)
    k.a[:] = -np.arange(1, 17, dtype=np.float32)
    return k


def device_inputs(k):
    return [torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in k.inputs()]


def time_us(stream, fn, iters=50, warmup=5):
    for _ in range(warmup):
        fn()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) * 1e3 / iters


def graph_us(stream, fns, iters=100):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for f in fns:
            f()

    def replay():
        with torch.cuda.stream(stream):
            g.replay()

    us = time_us(stream, replay, iters)
    del g
    return us


@pytest.mark.parametrize("profile", ["HR", "T01"])
def test_reference_cuda_kernel_against_oracle_and_timing(profile):
    s = torch.cuda.Stream()
    ours, refs, times = [], [], {}
    for i, L in enumerate(PROFILES[profile]):
        k = level_case(L, 900 + i)
        shape = sb.SelectiveScanShape(4, L, 256, 16, 1, 1, True)
        rshape = rsc.Shape(4, L, 256, 16, 1, 1, 1)
        with torch.cuda.stream(s):
            u, dl, a, b, c, d = device_inputs(k)
            y_ours, y_ref = torch.empty_like(u), torch.empty_like(u)
            st_ours = torch.zeros(2, dtype=torch.int32, device="cuda")
            st_ref = torch.zeros(2, dtype=torch.int32, device="cuda")
        call_ours = (lambda sh=shape, t=(u, dl, a, b, c, d, y_ours, st_ours): sb.selective_scan_cuda(sh, *t[:7], t[7], stream=s))
        call_ref = (lambda sh=rshape, t=(u, dl, a, b, c, d, y_ref, st_ref):
                    rsc.scan(sh, *[x.data_ptr() for x in t], s.cuda_stream))
        call_ours()
        call_ref()
        s.synchronize()
        ref, bound = oracle.run(k), oracle.scan_bound(k)
        for name, y, st in (("ours", y_ours, st_ours), ("reference_cuda", y_ref, st_ref)):
            words = st.cpu().numpy().view(np.uint32)
            assert words[0] == 0 and words[1] == sb.SCAN_DONE, (name, words)
            compare_bound(f"{profile}_L{L}_{name}", y.cpu().numpy(), ref, bound)
        times[f"L{L}"] = {"ours_us": round(time_us(s, call_ours), 2), "reference_cuda_us": round(time_us(s, call_ref), 2)}
        ours.append(call_ours)
        refs.append(call_ref)
    times["total"] = {"ours_us": round(sum(v["ours_us"] for v in times.values()), 2),
                      "reference_cuda_us": round(sum(v["reference_cuda_us"] for k_, v in times.items() if k_ != "total"), 2)}
    times["total_graph"] = {"ours_us": round(graph_us(s, ours), 2), "reference_cuda_us": round(graph_us(s, refs), 2)}
    out = os.path.join(ROOT, "gpurun_out")
    if os.path.isdir(out):
        path = os.path.join(out, "ref_scan_cuda_times.json")
        data = json.load(open(path)) if os.path.exists(path) else {}
        data[profile] = times
        json.dump(data, open(path, "w"), indent=1)
    print(profile, json.dumps(times))
    assert times["total"]["ours_us"] < times["total"]["reference_cuda_us"], times
