"""The reference's own GPU acceptance suite run against this library, unmodified.

oracle/_ref/selective_scan_cuda_tests is the reference's
tests/selective_scan_cuda_tests.cpp with tests/scan_cuda_suite.hpp (and its
src/selective_scan.cpp, src/file_io.cpp) compiled by oracle/Makefile against
include/saccade/selective_scan_cuda.hpp of this repository, the drop-in for
the reference's header, and linked to saccade_v1_b200/libsacc_scan.so.  It is
run the two ways the reference registers it (CMakeLists.txt:208-213): the
whole suite, and the "streams" group (held caller stream, graph capture with
its node count, concurrent streams) under CUDA_MODULE_LOADING=LAZY.  A
process-level timeout bounds each run.
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
SUITE = os.path.join(ROOT, "oracle", "_ref", "selective_scan_cuda_tests")

if not os.path.exists(SUITE):
    pytest.skip("oracle/_ref/selective_scan_cuda_tests not built (make -C oracle REF=<reference checkout>)",
                allow_module_level=True)


def run(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.update(env_extra or {})
    r = subprocess.run([SUITE, *args], capture_output=True, text=True, timeout=timeout, env=env)
    tail = (r.stdout + r.stderr)[-3000:]
    assert r.returncode == 0, f"suite failed (rc {r.returncode}):\n{tail}"
    return r.stdout


def test_reference_suite_passes():
    out = run([])
    last = out.strip().splitlines()[-1]
    assert last.startswith("selective_scan_cuda_tests:") and "checks passed" in last, last
    assert "identity\tbuild_flags=" in out or "identity\t" in out


def test_reference_streams_group_under_lazy_loading():
    out = run(["--group", "streams"], {"CUDA_MODULE_LOADING": "LAZY"}, timeout=120)
    assert "graph\tnodes=memset:1,kernel:3,other:0\tPASS" in out
    assert "checks passed" in out.strip().splitlines()[-1]
