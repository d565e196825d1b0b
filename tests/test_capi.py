"""CPU checks of the C-ABI boundary: the library loads, exports every symbol
that include/*.h declares, and rejects bad calls on the host before touching
the GPU (no compute call is made here)."""
import ctypes
import glob
import os
import re

import pytest

import saccade_v1_b200 as sb
from saccade_v1_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(sacc_\w+)\s*\(", text, re.M))
    return names


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    names = declared_symbols()
    assert {"sacc_selective_scan_f32", "sacc_scan_load_kernels", "sacc_selective_scan_ex"} <= names
    for n in names:
        assert hasattr(L, n), n
    assert set(_lib.EXPORTS) <= names


def test_identity_names_the_target():
    ident = sb.identity()
    assert "arch=sm_100a" in ident and "--ftz=false" in ident


FAKE_STREAM = 0x5EED  # never dereferenced: every case below is rejected before any CUDA call


@pytest.mark.parametrize("shape,diag", [
    (sb.SelectiveScanShape(1, 4, 4, 3, 1, 1, True), "state 3 must be a power of two in [1, 32]"),
    (sb.SelectiveScanShape(1, 4, 4, 64, 1, 1, True), "state 64 must be a power of two in [1, 32]"),
    (sb.SelectiveScanShape(1, 4, 4, 16, 2, 1, True), "A rows must be 1 or channels"),
    (sb.SelectiveScanShape(1, 4, 4, 16, 1, 4, True), "C width must be 1 or state"),
    (sb.SelectiveScanShape(0, 4, 4, 16, 1, 1, True), "batch and channels must be positive"),
    (sb.SelectiveScanShape(1, 65536, 65536, 1, 1, 1, False), "u/delta/y element count exceeds int32 capacity"),
    (sb.SelectiveScanShape(1, 1 << 27, 1, 32, 1, 1, False), "B element count exceeds int32 capacity"),
])
def test_host_rejections_without_gpu(shape, diag):
    L = _lib.load()
    ins = _lib.ScanInputs(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000)
    rc = L.sacc_selective_scan_f32(ctypes.byref(shape.c()), ctypes.byref(ins), 0x7000, 0x8000, FAKE_STREAM)
    assert rc == _lib.SACC_EINVAL
    msg = _lib.last_error()
    assert msg.startswith("selective_scan_cuda: ") and diag in msg


def test_default_streams_are_rejected():
    L = _lib.load()
    shape = sb.SelectiveScanShape(1, 4, 4, 16, 1, 1, True)
    ins = _lib.ScanInputs(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000)
    for stream in (0, 1, 2):  # 0, cudaStreamLegacy, cudaStreamPerThread
        rc = L.sacc_selective_scan_f32(ctypes.byref(shape.c()), ctypes.byref(ins), 0x7000, 0x8000, stream)
        assert rc == _lib.SACC_EINVAL and "explicit non-default stream" in _lib.last_error()


def test_pointer_rules_without_gpu():
    L = _lib.load()
    shape = sb.SelectiveScanShape(1, 4, 4, 16, 1, 1, True)
    cases = [
        (_lib.ScanInputs(0, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000), 0x7000, 0x8000, "u is null"),
        (_lib.ScanInputs(0x1002, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000), 0x7000, 0x8000, "u is not 4-byte aligned"),
        (_lib.ScanInputs(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000), 0x1010, 0x8000, "y overlaps u"),
        (_lib.ScanInputs(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000), 0x7000, 0x2008, "status overlaps delta"),
        (_lib.ScanInputs(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000), 0x7000, 0x7004, "status overlaps y"),
    ]
    for ins, y, status, diag in cases:
        rc = L.sacc_selective_scan_f32(ctypes.byref(shape.c()), ctypes.byref(ins), y, status, FAKE_STREAM)
        assert rc == _lib.SACC_EINVAL and diag in _lib.last_error(), _lib.last_error()


def _level_args(batch=1, height=6, width=10, length=None, d_model=128, x=0x100000, out=0x200000):
    """A Cross-Scan head level's arguments with fake (never dereferenced) device addresses."""
    blk = _lib.MambaBlockArgs(batch, height * width if length is None else length, d_model, 256, 16, 4, 16,
                              _lib.DTYPE_BF16, 1, 1e-5, None, None, 0x300000, 0x400000, 0x410000, 0x420000, 0x430000,
                              0x440000, 0x450000, 0x460000, 0x470000, None, 1)
    return _lib.CrossScanBlockArgs(blk, height, width, x, out)


@pytest.mark.parametrize("kw,diag", [
    ({"length": 59}, "block.length must be height * width"),
    ({"batch": 0}, "batch (images) must be in [1, 65535]"),
    ({"d_model": 64}, "d_inner and d_model must be positive multiples of 128"),
    ({"out": 0x100000 + 4096}, "out overlaps x"),
    ({"x": 0x100004}, "x is not 16-byte aligned"),
])
def test_cross_scan_level_rejections_without_gpu(kw, diag):
    """sacc_cross_scan_block_forward rejects bad shapes and buffers on the host, before any CUDA call."""
    L = _lib.load()
    args = _level_args(**kw)
    rc = L.sacc_cross_scan_block_forward(ctypes.byref(args), 0x900000, 1 << 30, FAKE_STREAM)
    assert rc == _lib.SACC_EINVAL and diag in _lib.last_error(), _lib.last_error()
    assert _lib.last_error().startswith("cross_scan_block: ")
    rc = L.sacc_cross_scan_block_forward(ctypes.byref(_level_args()), 0x900000, 1 << 30, 0)
    assert rc == _lib.SACC_EINVAL and "explicit non-default stream" in _lib.last_error()


def test_cpp_adapter_compiles_and_links(tmp_path):
    """include/sacc_scan.hpp gives reference-signature C++ (selective_scan_cuda etc.) over the C ABI."""
    import shutil
    import subprocess
    src = tmp_path / "adapter.cpp"
    src.write_text(
        '#include "sacc_scan.hpp"\n'
        "int main() {\n"
        "  saccade::SelectiveScanShape s{4, 960, 256, 16, 1, 1, true};\n"
        "  saccade::SelectiveScanDeviceInputs in{};\n"
        "  try { saccade::selective_scan_cuda(s, in, nullptr, nullptr, nullptr); }\n"
        "  catch (const std::invalid_argument& e) {\n"
        "    return std::string(e.what()).find(\"explicit non-default stream\") == std::string::npos; }\n"
        "  return 2;\n"
        "}\n")
    exe = tmp_path / "adapter"
    cuda_inc = "/usr/local/cuda/include"
    cxx = shutil.which("g++")
    assert cxx
    lib_dir = os.path.join(ROOT, "saccade_v1_b200")
    subprocess.run([cxx, "-std=c++17", "-I", os.path.join(ROOT, "include"), "-I", cuda_inc, str(src), "-o", str(exe),
                    "-L", lib_dir, "-lsacc_scan", "-Wl,-rpath," + lib_dir], check=True)
    # Host rejection of the default stream happens before any CUDA call: runs without a GPU.
    assert subprocess.run([str(exe)]).returncode == 0
