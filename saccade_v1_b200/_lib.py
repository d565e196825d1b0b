"""ctypes binding of libsacc_scan.so (the C ABI declared in include/sacc_scan.h,
include/sacc_frame.h and include/sacc_shard.h).

The library is built in-tree (saccade_v1_b200/libsacc_scan.so).  There is no
fallback: if the library is missing or does not load, every entry point
raises, so a GPU caller can never silently run something else.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsacc_scan.so")

SACC_OK, SACC_EINVAL, SACC_ECUDA = 0, 1, 2
SCAN_DONE = 0x4E414353
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
LAYOUT_BLD, LAYOUT_BDL = 0, 1

# Exported symbols, in the order include/sacc_scan.h declares them.
EXPORTS = (
    "sacc_scan_load_kernels",
    "sacc_selective_scan_f32",
    "sacc_cross_scan_expand_f32",
    "sacc_cross_scan_merge_f32",
    "sacc_last_error",
    "sacc_scan_identity",
    "sacc_selective_scan_ex",
    "sacc_scan_fault",
    "sacc_scan_wait_probe",
    "sacc_selective_scan_step",
    "sacc_gemm",
    "sacc_mamba_block_workspace",
    "sacc_mamba_block_forward",
    "sacc_mamba_block_forward_noalloc",
    "sacc_cross_scan_block_workspace",
    "sacc_cross_scan_block_forward",
    "sacc_selective_scan_f16",
    # include/sacc_frame.h
    "sacc_scan_frame_load_kernels",
    "sacc_scan_frame_initialize",
    "sacc_scan_frame_begin",
    "sacc_scan_frame_gate",
    "sacc_scan_frame_publish",
    "sacc_scan_frame_commit",
    "sacc_scan_frame_packet",
    "sacc_scan_frame_step",
    "sacc_scan_frame_check_finite",
    "sacc_scan_frame_delay",
    "sacc_scan_frame_digest",
    "sacc_model_producer_workspace_bytes",
    "sacc_model_producer_load_kernels",
    "sacc_model_producer_cuda",
    # include/sacc_shard.h
    "sacc_shard_rows",
    "sacc_shard_group_create",
    "sacc_shard_group_destroy",
    "sacc_scan_sharded_forward",
)

FRAME_MAX_STATUSES = 16
MODEL_PRODUCER_PLUGINS = 9


class ScanShape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_uint64), ("length", ctypes.c_uint64), ("channels", ctypes.c_uint64),
                ("state", ctypes.c_uint64), ("a_rows", ctypes.c_uint64), ("c_width", ctypes.c_uint64),
                ("has_d", ctypes.c_int32)]


class ScanInputs(ctypes.Structure):
    _fields_ = [(k, ctypes.c_void_p) for k in ("u", "delta", "a", "b", "c", "d")]


class ScanInputsF16(ctypes.Structure):
    _fields_ = [(k, ctypes.c_void_p) for k in ("u", "delta", "a", "b", "c", "d")]


class CrossScanShape(ctypes.Structure):
    _fields_ = [(k, ctypes.c_uint64) for k in ("batch", "channels", "height", "width")]


class ScanExArgs(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_uint64), ("length", ctypes.c_uint64), ("channels", ctypes.c_uint64),
                ("state", ctypes.c_uint64), ("groups", ctypes.c_uint64), ("a_rows", ctypes.c_uint64),
                ("c_width", ctypes.c_uint64), ("layout", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("delta_softplus", ctypes.c_int32), ("nseq", ctypes.c_int32),
                ("u", ctypes.c_void_p), ("delta", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p),
                ("z", ctypes.c_void_p), ("a", ctypes.c_void_p), ("d", ctypes.c_void_p),
                ("delta_bias", ctypes.c_void_p), ("h0", ctypes.c_void_p), ("h_final", ctypes.c_void_p),
                ("cu_seqlens", ctypes.c_void_p), ("y", ctypes.c_void_p)]


class ScanStepArgs(ctypes.Structure):
    _fields_ = [("nseq", ctypes.c_uint64), ("channels", ctypes.c_uint64), ("state", ctypes.c_uint64),
                ("groups", ctypes.c_uint64), ("a_rows", ctypes.c_uint64), ("c_width", ctypes.c_uint64),
                ("slots", ctypes.c_uint64), ("dtype", ctypes.c_int32), ("delta_softplus", ctypes.c_int32),
                ("u", ctypes.c_void_p), ("delta", ctypes.c_void_p), ("z", ctypes.c_void_p), ("b", ctypes.c_void_p),
                ("c", ctypes.c_void_p), ("a", ctypes.c_void_p), ("d", ctypes.c_void_p), ("delta_bias", ctypes.c_void_p),
                ("state_io", ctypes.c_void_p), ("slot", ctypes.c_void_p), ("y", ctypes.c_void_p)]


class GemmArgs(ctypes.Structure):
    _fields_ = [("m", ctypes.c_uint64), ("n", ctypes.c_uint64), ("k", ctypes.c_uint64), ("lda", ctypes.c_uint64),
                ("ldb", ctypes.c_uint64), ("ldc", ctypes.c_uint64), ("ldr", ctypes.c_uint64),
                ("in_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32), ("a", ctypes.c_void_p),
                ("b", ctypes.c_void_p), ("c", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("residual", ctypes.c_void_p),
                ("row_scale", ctypes.c_void_p)]


class MambaBlockArgs(ctypes.Structure):
    _fields_ = [(k, ctypes.c_uint64) for k in ("batch", "length", "d_model", "d_inner", "d_state", "d_conv", "dt_rank")] + [
        ("dtype", ctypes.c_int32), ("residual", ctypes.c_int32), ("eps", ctypes.c_float)] + [
        (k, ctypes.c_void_p) for k in ("x", "norm_w", "w_in", "conv_w", "conv_b", "w_x", "w_dt", "dt_bias", "a", "d",
                                       "w_out", "out")] + [("c_width", ctypes.c_int32)]


class CrossScanBlockArgs(ctypes.Structure):
    _fields_ = [("block", MambaBlockArgs), ("height", ctypes.c_uint64), ("width", ctypes.c_uint64),
                ("x", ctypes.c_void_p), ("out", ctypes.c_void_p)]


class FrameControl(ctypes.Structure):
    _fields_ = [("epoch", ctypes.c_uint64), ("current", ctypes.c_int64), ("committed", ctypes.c_int64),
                ("fail_frame", ctypes.c_int64)] + [
        (k, ctypes.c_uint32) for k in ("committed_slot", "working_slot", "frame_status", "fail_code", "run_stage",
                                       "published", "scan_flags", "arrivals")] + [("digest_sum", ctypes.c_uint64)]


class FrameRecord(ctypes.Structure):
    _fields_ = [("flags", ctypes.c_uint32 * FRAME_MAX_STATUSES), ("done", ctypes.c_uint32 * FRAME_MAX_STATUSES),
                ("frame_status", ctypes.c_uint32), ("published", ctypes.c_uint32), ("digest", ctypes.c_uint64)]


class StatusList(ctypes.Structure):
    _fields_ = [("status", ctypes.c_void_p * FRAME_MAX_STATUSES), ("count", ctypes.c_uint)]


class RawView(ctypes.Structure):
    _fields_ = [("cls", ctypes.c_void_p * 3), ("reg", ctypes.c_void_p * 3), ("cls_elements", ctypes.c_size_t * 3),
                ("reg_elements", ctypes.c_size_t * 3)]


_lib = None


def load() -> ctypes.CDLL:
    """Loads libsacc_scan.so; raises if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built; run `python -m saccade_v1_b200.build` "
                          "(the selective-scan library has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    vp, sz, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    L.sacc_scan_load_kernels.argtypes = [ctypes.c_char_p, sz]
    L.sacc_scan_load_kernels.restype = i
    L.sacc_selective_scan_f32.argtypes = [ctypes.POINTER(ScanShape), ctypes.POINTER(ScanInputs), vp, vp, vp]
    L.sacc_selective_scan_f32.restype = i
    L.sacc_selective_scan_f16.argtypes = [ctypes.POINTER(ScanShape), ctypes.POINTER(ScanInputsF16), vp, vp, vp]
    L.sacc_selective_scan_f16.restype = i
    L.sacc_cross_scan_expand_f32.argtypes = [ctypes.POINTER(CrossScanShape), vp, vp, vp, vp]
    L.sacc_cross_scan_expand_f32.restype = i
    L.sacc_cross_scan_merge_f32.argtypes = [ctypes.POINTER(CrossScanShape), vp, vp, vp, vp]
    L.sacc_cross_scan_merge_f32.restype = i
    L.sacc_last_error.argtypes = []
    L.sacc_last_error.restype = ctypes.c_char_p
    L.sacc_scan_identity.argtypes = []
    L.sacc_scan_identity.restype = ctypes.c_char_p
    L.sacc_selective_scan_ex.argtypes = [ctypes.POINTER(ScanExArgs), vp]
    L.sacc_selective_scan_ex.restype = i
    L.sacc_scan_fault.argtypes = [ctypes.POINTER(ctypes.c_uint32), i]
    L.sacc_scan_fault.restype = i
    L.sacc_scan_wait_probe.argtypes = [ctypes.c_uint32, vp]
    L.sacc_scan_wait_probe.restype = i
    L.sacc_selective_scan_step.argtypes = [ctypes.POINTER(ScanStepArgs), vp]
    L.sacc_selective_scan_step.restype = i
    L.sacc_gemm.argtypes = [ctypes.POINTER(GemmArgs), vp]
    L.sacc_gemm.restype = i
    L.sacc_mamba_block_workspace.argtypes = [ctypes.POINTER(MambaBlockArgs), ctypes.POINTER(ctypes.c_size_t)]
    L.sacc_mamba_block_workspace.restype = i
    L.sacc_mamba_block_forward.argtypes = [ctypes.POINTER(MambaBlockArgs), vp, sz, vp]
    L.sacc_mamba_block_forward.restype = i
    L.sacc_mamba_block_forward_noalloc.argtypes = [ctypes.POINTER(MambaBlockArgs), vp]
    L.sacc_mamba_block_forward_noalloc.restype = i
    L.sacc_cross_scan_block_workspace.argtypes = [ctypes.POINTER(CrossScanBlockArgs), ctypes.POINTER(ctypes.c_size_t)]
    L.sacc_cross_scan_block_workspace.restype = i
    L.sacc_cross_scan_block_forward.argtypes = [ctypes.POINTER(CrossScanBlockArgs), vp, sz, vp]
    L.sacc_cross_scan_block_forward.restype = i
    L.sacc_shard_rows.argtypes = [ctypes.c_uint64, i, i, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
    L.sacc_shard_rows.restype = i
    L.sacc_shard_group_create.argtypes = [i, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(vp)]
    L.sacc_shard_group_create.restype = i
    L.sacc_shard_group_destroy.argtypes = [vp]
    L.sacc_shard_group_destroy.restype = i
    L.sacc_scan_sharded_forward.argtypes = [vp, ctypes.POINTER(ScanExArgs), ctypes.POINTER(vp), ctypes.POINTER(vp), sz]
    L.sacc_scan_sharded_forward.restype = i
    i64, u64 = ctypes.c_int64, ctypes.c_uint64
    for name, args in (
            ("sacc_scan_frame_load_kernels", [ctypes.c_char_p, sz]),
            ("sacc_scan_frame_initialize", [vp, u64, vp, vp]),
            ("sacc_scan_frame_begin", [vp, u64, i64, vp]),
            ("sacc_scan_frame_gate", [vp, ctypes.POINTER(StatusList), vp, i64, vp]),
            ("sacc_scan_frame_publish", [vp, vp, sz, vp, vp, vp, i64, vp]),
            ("sacc_scan_frame_commit", [vp, vp]),
            ("sacc_scan_frame_packet", [vp, vp, vp]),
            ("sacc_scan_frame_step", [vp, u64, i64, ctypes.POINTER(StatusList), vp, sz, vp, vp, vp, i64, vp, vp]),
            ("sacc_scan_frame_check_finite", [vp, sz, vp, ctypes.c_uint32, vp]),
            ("sacc_scan_frame_delay", [ctypes.c_uint, vp]),
            ("sacc_model_producer_load_kernels", [ctypes.c_char_p, sz]),
            ("sacc_model_producer_cuda", [vp, sz, ctypes.POINTER(RawView), ctypes.c_void_p * MODEL_PRODUCER_PLUGINS, vp,
                                          vp, sz, vp, i])):
        getattr(L, name).argtypes = args
        getattr(L, name).restype = i
    L.sacc_scan_frame_digest.argtypes = [vp, sz]
    L.sacc_scan_frame_digest.restype = u64
    L.sacc_model_producer_workspace_bytes.argtypes = []
    L.sacc_model_producer_workspace_bytes.restype = sz
    _lib = L
    return L


def last_error() -> str:
    return load().sacc_last_error().decode()
