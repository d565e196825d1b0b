"""C and C++ callers of the boundary, compiled and linked here (no GPU).

tests/callers/c_caller.c uses the C ABI of include/sacc_scan.h (C11, -Wall
-Wextra -Werror); tests/callers/cxx_caller.cpp uses the reference's C++
interface through include/saccade/selective_scan_cuda.hpp (C++17 and C++20,
-Wpedantic -Werror) with no reference header on the include path.  Both link
saccade_v1_b200/libsacc_scan.so and run: the C++ one checks a host rejection
(std::invalid_argument with the reference's diagnostic), both print the build
identity.  The reference's own GPU suite compiled against the same header is
tests/test_reference_suite_gpu.py.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
LIBDIR = os.path.join(ROOT, "saccade_v1_b200")
CUDA_INC = "/usr/local/cuda/include"

needs_lib = pytest.mark.skipif(not os.path.exists(os.path.join(LIBDIR, "libsacc_scan.so")),
                               reason="libsacc_scan.so not built")


def build_and_run(cmd, exe):
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    out = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stdout + out.stderr
    return out.stdout


def link_args():
    return ["-L" + LIBDIR, "-lsacc_scan", "-Wl,-rpath," + LIBDIR]


@needs_lib
def test_c_caller_compiles_links_and_runs(tmp_path):
    exe = str(tmp_path / "c_caller")
    out = build_and_run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I" + os.path.join(ROOT, "include"),
                         "-I" + CUDA_INC, os.path.join(ROOT, "tests", "callers", "c_caller.c"), "-o", exe, *link_args()], exe)
    assert "build_flags=" in out or len(out) > 0


@needs_lib
@pytest.mark.parametrize("std", ["c++17", "c++20"])
def test_cxx_caller_compiles_links_and_runs(tmp_path, std):
    exe = str(tmp_path / "cxx_caller")
    out = build_and_run(["g++", f"-std={std}", "-Wall", "-Wextra", "-Wpedantic", "-Werror",
                         "-I" + os.path.join(ROOT, "include"), "-I" + CUDA_INC,
                         os.path.join(ROOT, "tests", "callers", "cxx_caller.cpp"), "-o", exe, *link_args()], exe)
    assert len(out) > 0
