"""Builds libsacc_scan.so in-tree for sm_100a with nvcc.

    python -m saccade_v1_b200.build            # incremental
    python -m saccade_v1_b200.build --clean

Objects go to saccade_v1_b200/_build/, the library to
saccade_v1_b200/libsacc_scan.so (git-ignored, shipped with the tree).
The FP32 flags are the reference's scan flags (no fast-math, IEEE division
and square root, subnormals kept), so library math keeps its documented
error bounds; the CUDA runtime is linked statically so the library shares
the driver context with whatever runtime the host process already loaded.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsacc_scan.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FP_FLAGS = ["--ftz=false", "--prec-div=true", "--prec-sqrt=true", "--fmad=true"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-I" + os.path.join(ROOT, "include")]
SOURCES = ["scan_f32.cu", "scan_ex.cu", "scan_bulk.cu", "scan_step.cu", "cross_scan.cu", "gemm_tcgen05.cu", "block_kernels.cu", "cross_block.cu", "mamba_block.cpp", "block_noalloc.cu", "scan_frame.cu", "model_producer.cu", "scan_plugin.cpp", "capi.cpp"]


def _flags_string() -> str:
    return " ".join(ARCH + FP_FLAGS + ["-O3", "-lineinfo"])


def _deps(src: str) -> list[str]:
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return [src] + headers + [os.path.join(ROOT, "include", "sacc_scan.h"), os.path.join(ROOT, "include", "sacc_scan_plugin.h"),
                              os.path.join(ROOT, "include", "sacc_frame.h"),
                              os.path.abspath(__file__)]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src_name: str, verbose: bool) -> str:
    src = os.path.join(CSRC, src_name)
    obj = os.path.join(BUILD, src_name + ".o")
    if not _stale(obj, _deps(src)):
        return obj
    cmd = [NVCC, *ARCH, *FP_FLAGS, *COMMON, f'-DSACC_BUILD_FLAGS="{_flags_string()}"', "-Xptxas", "-v",
           "-c", src, "-o", obj]
    if src_name.endswith(".cpp"):
        cmd[cmd.index("-c"):cmd.index("-c")] = ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    with open(obj + ".log", "w") as f:
        f.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed on {src_name}")
    if verbose:
        sys.stdout.write(r.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = [s for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    if _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC", "-o", LIB, *objs, "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libsacc_scan.so failed")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    if args.clean:
        shutil.rmtree(BUILD, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    print(build(args.verbose))


if __name__ == "__main__":
    main()
