"""Host-side front end of the selective-scan library for torch device buffers.

Mirrors the reference's C++ API (include/saccade/selective_scan_cuda.hpp):
  load_kernels()          selective_scan_cuda_load_kernels   (:57-62)
  selective_scan_cuda()   selective_scan_cuda                (:64-71)
  cross_scan_expand_cuda / cross_scan_merge_cuda             (:73-83)
with the same argument meaning and error behaviour: a host rejection raises
ScanInvalidArgument (the reference's std::invalid_argument) before anything is
enqueued; a failed CUDA call raises ScanCudaError (std::runtime_error).
Numeric failures are reported through the device status words, never raised.

selective_scan_ex() is the extended Mamba-layout entry (bf16/fp16/fp32
activations, FP32 state, fused bias/softplus/gate, state in/out, varlen).

Everything goes through libsacc_scan.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

SCAN_DONE = _lib.SCAN_DONE


class ScanInvalidArgument(ValueError):
    """Host rejection (shape, capacity, pointer, overlap or stream); nothing was enqueued."""


class ScanCudaError(RuntimeError):
    """A CUDA API call failed; the status never reaches done."""


def _check(rc: int) -> None:
    if rc == _lib.SACC_OK:
        return
    msg = _lib.last_error()
    if rc == _lib.SACC_EINVAL:
        raise ScanInvalidArgument(msg)
    raise ScanCudaError(msg)


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr() if t.numel() else None


def _stream_handle(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _stream_scratch(nbytes: int, device, stream):
    """A uint8 device buffer from torch's caching allocator for use on `stream`:
    allocated while that stream is current (so the allocator does not hand it
    to another stream's work while the call's kernels may still run), or, for
    a raw stream handle, marked as used by it."""
    if isinstance(stream, torch.cuda.Stream):
        with torch.cuda.stream(stream):
            return torch.empty(nbytes, dtype=torch.uint8, device=device)
    buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
    if isinstance(stream, int) and stream not in (0,):
        buf.record_stream(torch.cuda.ExternalStream(stream, device=device))
    return buf


def load_kernels() -> str:
    """Loads every kernel in the current CUDA context; returns the resource report."""
    L = _lib.load()
    buf = ctypes.create_string_buffer(1 << 16)
    _check(L.sacc_scan_load_kernels(buf, len(buf)))
    return buf.value.decode()


def identity() -> str:
    return _lib.load().sacc_scan_identity().decode()


@dataclass
class SelectiveScanShape:
    """include/saccade/selective_scan.hpp:19-27."""
    batch: int = 0
    length: int = 0
    channels: int = 0
    state: int = 0
    a_rows: int = 1
    c_width: int = 1
    has_d: bool = True

    def c(self) -> _lib.ScanShape:
        return _lib.ScanShape(self.batch, self.length, self.channels, self.state, self.a_rows, self.c_width,
                              int(self.has_d))


def selective_scan_cuda(shape: SelectiveScanShape, u, delta, a, b, c, d, y, status, stream=None) -> None:
    """Reference-ABI FP32 scan on device buffers (dense row-major float32 tensors).

    status is a device tensor of two 32-bit words {flags, done}.  Enqueues on
    `stream` (default: torch's current stream, which must not be the default
    stream) and returns without synchronising.
    """
    L = _lib.load()
    ins = _lib.ScanInputs(_ptr(u), _ptr(delta), _ptr(a), _ptr(b), _ptr(c), _ptr(d))
    _check(L.sacc_selective_scan_f32(ctypes.byref(shape.c()), ctypes.byref(ins), _ptr(y), _ptr(status),
                                     _stream_handle(stream)))


def selective_scan_f16(shape: SelectiveScanShape, u, delta, a, b, c, d, y, status, stream=None) -> None:
    """The same operator with FP16 activations (plugin SelectiveScan v3): u,
    delta, b, c and y float16 tensors, a and d float32.  y is the FP32 path's
    output on the widened inputs rounded to nearest FP16; an output FP16
    cannot hold sets SACC_SCAN_OUTPUT_RANGE."""
    L = _lib.load()
    ins = _lib.ScanInputsF16(_ptr(u), _ptr(delta), _ptr(a), _ptr(b), _ptr(c), _ptr(d))
    _check(L.sacc_selective_scan_f16(ctypes.byref(shape.c()), ctypes.byref(ins), _ptr(y), _ptr(status),
                                     _stream_handle(stream)))


@dataclass
class CrossScanShape:
    batch: int = 0
    channels: int = 0
    height: int = 0
    width: int = 0

    def c(self) -> _lib.CrossScanShape:
        return _lib.CrossScanShape(self.batch, self.channels, self.height, self.width)


def cross_scan_expand_cuda(shape: CrossScanShape, x, tokens, status, stream=None) -> None:
    _check(_lib.load().sacc_cross_scan_expand_f32(ctypes.byref(shape.c()), _ptr(x), _ptr(tokens), _ptr(status),
                                                  _stream_handle(stream)))


def cross_scan_merge_cuda(shape: CrossScanShape, y, out, status, stream=None) -> None:
    _check(_lib.load().sacc_cross_scan_merge_f32(ctypes.byref(shape.c()), _ptr(y), _ptr(out), _ptr(status),
                                                 _stream_handle(stream)))


_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def selective_scan_ex(u, delta, A, B, C, D=None, z=None, delta_bias=None, *, delta_softplus: bool = True,
                      h0=None, h_final=None, cu_seqlens=None, layout: str = "BDL", out=None, stream=None):
    """Extended selective scan (Mamba's selective_scan forward), returns y.

    layout "BDL": u, delta, z (batch, D, L); B, C (batch, groups, N|1, L).
    layout "BLD": u, delta, z (batch, L, D); B, C (batch, L, groups, N|1).
    B and C may also be given without the groups axis (groups = 1).
    A (D, N) or (1, N) float32; D, delta_bias (D,) float32.
    h0, h_final: (nseq, D, N) float32 device tensors (h_final is written).
    cu_seqlens: int32 (nseq + 1) with batch 1, packing sequences along L.
    """
    if layout not in ("BDL", "BLD"):
        raise ScanInvalidArgument("selective_scan_ex: layout must be BLD or BDL")
    if u.dtype not in _DTYPES:
        raise ScanInvalidArgument("selective_scan_ex: dtype must be f32, bf16 or f16")
    for name, t in (("delta", delta), ("B", B), ("C", C), ("z", z)):
        if t is not None and t.dtype != u.dtype:
            raise ScanInvalidArgument(f"selective_scan_ex: {name} dtype differs from u")
    if layout == "BDL":
        batch, dim, length = u.shape
        if B.dim() == 3:
            B, C = B.unsqueeze(1), C.unsqueeze(1)
        groups, state = B.shape[1], B.shape[2]
        c_width = C.shape[2]
    else:
        batch, length, dim = u.shape
        if B.dim() == 3:
            B, C = B.unsqueeze(2), C.unsqueeze(2)
        groups, state = B.shape[2], B.shape[3]
        c_width = C.shape[3]
    for name, t in (("u", u), ("delta", delta), ("B", B), ("C", C), ("z", z), ("A", A), ("D", D),
                    ("delta_bias", delta_bias), ("h0", h0), ("h_final", h_final), ("cu_seqlens", cu_seqlens)):
        if t is not None and not t.is_contiguous():
            raise ScanInvalidArgument(f"selective_scan_ex: {name} must be contiguous")
    if out is None:
        out = torch.empty_like(u)
    nseq = (cu_seqlens.numel() - 1) if cu_seqlens is not None else batch
    args = _lib.ScanExArgs(batch, length, dim, state, groups, A.shape[0] if A.dim() == 2 else 1, c_width,
                           _lib.LAYOUT_BDL if layout == "BDL" else _lib.LAYOUT_BLD, _DTYPES[u.dtype],
                           int(delta_softplus), nseq,
                           _ptr(u), _ptr(delta), _ptr(B), _ptr(C), _ptr(z), _ptr(A), _ptr(D), _ptr(delta_bias),
                           _ptr(h0), _ptr(h_final), _ptr(cu_seqlens), _ptr(out))
    _check(_lib.load().sacc_selective_scan_ex(ctypes.byref(args), _stream_handle(stream)))
    return out


def selective_scan_step(u, delta, A, B, C, state, D=None, z=None, delta_bias=None, *, slot=None,
                        delta_softplus: bool = True, out=None, stream=None):
    """One L = 1 update of carried state, in place; returns y.

    u, delta, z: (nseq, D); B, C: (nseq, N|1) or (nseq, groups, N|1) in u's dtype;
    state: (slots, D, N) float32, updated in place; slot: optional int32 (nseq)
    mapping each sequence to its state row (negative = skip, y = 0).
    """
    if u.dtype not in _DTYPES:
        raise ScanInvalidArgument("selective_scan_step: dtype must be f32, bf16 or f16")
    nseq, dim = u.shape
    if B.dim() == 2:
        B, C = B.unsqueeze(1), C.unsqueeze(1)
    groups, nstate, c_width = B.shape[1], B.shape[2], C.shape[2]
    for name, t in (("u", u), ("delta", delta), ("B", B), ("C", C), ("z", z), ("state", state), ("slot", slot)):
        if t is not None and not t.is_contiguous():
            raise ScanInvalidArgument(f"selective_scan_step: {name} must be contiguous")
    if out is None:
        out = torch.empty_like(u)
    args = _lib.ScanStepArgs(nseq, dim, nstate, groups, A.shape[0] if A.dim() == 2 else 1, c_width,
                             state.shape[0], _DTYPES[u.dtype], int(delta_softplus),
                             _ptr(u), _ptr(delta), _ptr(z), _ptr(B), _ptr(C), _ptr(A), _ptr(D), _ptr(delta_bias),
                             _ptr(state), _ptr(slot), _ptr(out))
    _check(_lib.load().sacc_selective_scan_step(ctypes.byref(args), _stream_handle(stream)))
    return out


def gemm(a, b, *, out=None, bias=None, residual=None, row_scale=None, out_dtype=None, stream=None):
    """C = diag(row_scale) a @ b.T (+ bias) (+ residual) on the tensor cores; a (m, k), b (n, k) bf16/fp16."""
    if a.dtype not in (torch.bfloat16, torch.float16) or b.dtype != a.dtype:
        raise ScanInvalidArgument("gemm: a and b must both be bf16 or both fp16")
    m, k = a.shape
    n = b.shape[0]
    if b.shape[1] != k:
        raise ScanInvalidArgument("gemm: a and b disagree on k")
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype or a.dtype, device=a.device)
    for name, t in (("a", a), ("b", b), ("out", out), ("residual", residual)):
        if t is not None and t.stride(-1) != 1:
            raise ScanInvalidArgument(f"gemm: {name} must have unit inner stride")
    args = _lib.GemmArgs(m, n, k, a.stride(0), b.stride(0), out.stride(0), residual.stride(0) if residual is not None else 0,
                         _DTYPES[a.dtype], _DTYPES[out.dtype], _ptr(a), _ptr(b), _ptr(out), _ptr(bias), _ptr(residual),
                         _ptr(row_scale))
    _check(_lib.load().sacc_gemm(ctypes.byref(args), _stream_handle(stream)))
    return out


def scan_fault(clear: bool = False) -> int:
    """The library's device fault word (0 = no kernel ever gave up a bounded wait); synchronous."""
    v = ctypes.c_uint32(0)
    _check(_lib.load().sacc_scan_fault(ctypes.byref(v), int(clear)))
    return v.value


BLOCK_KEYS = ("norm_w", "w_in", "conv_w", "conv_b", "w_x", "w_dt", "dt_bias", "A", "D", "w_out")


def _block_args(x, p, eps, residual, out):
    batch, length, d_model = x.shape
    d_inner = p["w_in"].shape[0] // 2
    d_conv = p["conv_w"].shape[-1]
    dt_rank = p["w_dt"].shape[1]
    d_state = p["A"].shape[1]
    for k in BLOCK_KEYS:
        t = p.get(k)
        if t is not None and not t.is_contiguous():
            raise ScanInvalidArgument(f"mamba_block: {k} must be contiguous")
    c_width = p["w_x"].shape[0] - dt_rank - d_state  # d_state, or 1 (rank-1 C)
    return _lib.MambaBlockArgs(batch, length, d_model, d_inner, d_state, d_conv, dt_rank, _DTYPES[x.dtype], int(residual),
                               float(eps), _ptr(x), _ptr(p.get("norm_w")), _ptr(p["w_in"]), _ptr(p["conv_w"]),
                               _ptr(p.get("conv_b")), _ptr(p["w_x"]), _ptr(p["w_dt"]), _ptr(p.get("dt_bias")),
                               _ptr(p["A"]), _ptr(p.get("D")), _ptr(p["w_out"]), _ptr(out), c_width)


def mamba_block_workspace(x, params, eps=1e-5, residual=True) -> int:
    n = ctypes.c_size_t(0)
    _check(_lib.load().sacc_mamba_block_workspace(ctypes.byref(_block_args(x, params, eps, residual, None)), ctypes.byref(n)))
    return n.value


def mamba_block_forward(x, params, *, eps=1e-5, residual=True, out=None, workspace=None, stream=None):
    """One Mamba block forward (RMSNorm when params["norm_w"] is given, in_proj, conv1d + SiLU,
    x_proj, dt_proj, selective scan with D skip and SiLU(z) gate, out_proj, + x).

    x (batch, length, d_model) bf16/fp16; weights as in include/sacc_scan.h
    (SaccMambaBlockArgs).  workspace: optional uint8 device tensor of at least
    mamba_block_workspace(...) bytes (allocated here when omitted).
    """
    if out is None:
        out = torch.empty_like(x)
    args = _block_args(x, params, eps, residual, out)
    need = mamba_block_workspace(x, params, eps, residual)
    if workspace is None:
        workspace = _stream_scratch(need + 256, x.device, stream)
    base = workspace.data_ptr()
    off = (-base) % 256
    _check(_lib.load().sacc_mamba_block_forward(ctypes.byref(args), base + off, workspace.numel() - off,
                                                _stream_handle(stream)))
    return out


def _cross_args(x, params, eps, residual, out, dtype):
    if x.dim() != 4 or x.dtype != torch.float32 or not x.is_contiguous():
        raise ScanInvalidArgument("cross_scan_block: x must be a contiguous (batch, d_model, height, width) float32 tensor")
    batch, d_model, height, width = x.shape
    # The block's shape fields from a stand-in of its (batch, length, d_model)
    # input; the level reads x and writes out as maps, so block.x stays null.
    blk = _block_args(torch.empty((), dtype=dtype).expand(batch, height * width, d_model), params, eps, residual, None)
    blk.x = None
    return _lib.CrossScanBlockArgs(blk, height, width, _ptr(x), _ptr(out))


def cross_scan_block_workspace(x, params, eps=1e-5, residual=True, dtype=torch.bfloat16) -> int:
    n = ctypes.c_size_t(0)
    args = _cross_args(x, params, eps, residual, None, dtype)
    _check(_lib.load().sacc_cross_scan_block_workspace(ctypes.byref(args), ctypes.byref(n)))
    return n.value


def cross_scan_block_forward(x, params, *, eps=1e-5, residual=True, dtype=torch.bfloat16, out=None, workspace=None,
                             stream=None):
    """One Cross-Scan head level: expand x into four scan directions, the Mamba
    block on each (with the residual on the tokens when `residual`), and the
    merge back to the map, in one call without the expanded tokens
    (reference src/head_trt_network.cpp:200-232).

    x (batch, d_model, height, width) float32; params as for
    mamba_block_forward, weights in `dtype` (bf16 / fp16, the block's
    activation type); returns out like x (float32).
    """
    if out is None:
        out = torch.empty_like(x)
    args = _cross_args(x, params, eps, residual, out, dtype)
    need = cross_scan_block_workspace(x, params, eps, residual, dtype)
    if workspace is None:
        workspace = _stream_scratch(need + 256, x.device, stream)
    base = workspace.data_ptr()
    off = (-base) % 256
    _check(_lib.load().sacc_cross_scan_block_forward(ctypes.byref(args), base + off, workspace.numel() - off,
                                                     _stream_handle(stream)))
    return out


def mamba_block_forward_noalloc(x, params, *, eps=1e-5, residual=True, out=None, stream=None):
    """mamba_block_forward with the intermediates in the library's static
    device scratch (SACC_NOALLOC_SCRATCH_BYTES per device) instead of a
    workspace: the call allocates nothing on the device when `out` is given.
    All calls on a device share that scratch, so calls that overlap on the
    GPU race; order them on one stream.  The first call on a device does the
    scratch set-up and should come before any stream capture."""
    if out is None:
        out = torch.empty_like(x)
    args = _block_args(x, params, eps, residual, out)
    _check(_lib.load().sacc_mamba_block_forward_noalloc(ctypes.byref(args), _stream_handle(stream)))
    return out
