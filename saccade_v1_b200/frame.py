"""Consumers of the scan status words over torch device buffers: the frame-end
protocol (reference cuda/scan_frame.cu, include/saccade/scan_frame_kernels.hpp)
and the model producer's status aggregate (cuda/model_producer.cu,
include/saccade/model_producer_cuda.hpp).

Same names and argument meaning as the reference; a host rejection raises
ScanInvalidArgument (std::invalid_argument) before anything is enqueued, a
failed CUDA call ScanCudaError (std::runtime_error).  Device buffers:

* control: ``new_control()`` (uint8, CONTROL_BYTES), set by scan_frame_initialize;
* statuses: an int32 tensor of shape (n, 2) whose rows are {flags, done}
  status words (any row of it can be passed as one status);
* records: ``new_records(capacity)`` (uint8, capacity x RECORD_BYTES);
* results: float32 of 2 x count (two result versions), result_frames int64 of 2;
* packet: uint8 of PACKET_BYTES.
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np
import torch

from . import _lib
from .scan import ScanInvalidArgument, _check, _stream_handle

CONTROL_BYTES = ctypes.sizeof(_lib.FrameControl)
RECORD_BYTES = ctypes.sizeof(_lib.FrameRecord)
MAX_STATUSES = _lib.FRAME_MAX_STATUSES
PACKET_BYTES = 80 + 256 * 48
ERROR_PROTOCOL, ERROR_NUMERIC = 1 << 0, 1 << 3
FRAME_NONFINITE_INPUT, FRAME_NONFINITE_OUTPUT = 1 << 20, 1 << 21
MODEL_PRODUCER_PLUGINS = _lib.MODEL_PRODUCER_PLUGINS
PRODUCER_DONE = 0x34525046
POSTPROCESS_NUMERIC, POSTPROCESS_UPSTREAM, POSTPROCESS_PROTOCOL = 1, 2, 4
PROFILES = {"t01-640x640": (0, 640, 640), "hr-1280x768": (1, 1280, 768)}


def _status_ptrs(statuses) -> list[int]:
    """Device addresses of status words: an (n, 2) int32 tensor (every row),
    or a list of 1-row views / addresses."""
    if isinstance(statuses, torch.Tensor):
        if statuses.dtype not in (torch.int32, torch.uint32) or statuses.dim() != 2 or statuses.shape[1] != 2 or \
                not statuses.is_contiguous():
            raise ScanInvalidArgument("statuses must be a contiguous (n, 2) int32 tensor")
        return [statuses.data_ptr() + 8 * i for i in range(statuses.shape[0])]
    return [s if isinstance(s, int) else s.data_ptr() for s in statuses]


def _status_list(statuses) -> _lib.StatusList:
    ptrs = _status_ptrs(statuses)
    lst = _lib.StatusList()
    lst.count = len(ptrs)
    for i, p in enumerate(ptrs[:MAX_STATUSES]):
        lst.status[i] = p
    return lst


def _addr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _need(name, t, dtype=None, numel=None, optional=False):
    """Host check of a device buffer's type, layout and size (the C ABI sees only pointers)."""
    if t is None:
        if optional:
            return
        raise ScanInvalidArgument(f"{name} is required")
    if not t.is_cuda or not t.is_contiguous():
        raise ScanInvalidArgument(f"{name} must be a contiguous CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ScanInvalidArgument(f"{name} must be {dtype}")
    if numel is not None and t.numel() * t.element_size() < numel:
        raise ScanInvalidArgument(f"{name} holds {t.numel() * t.element_size()} bytes, needs {numel}")


def _zeros(nbytes: int, device, stream) -> torch.Tensor:
    if isinstance(stream, torch.cuda.Stream):
        with torch.cuda.stream(stream):
            return torch.zeros(nbytes, dtype=torch.uint8, device=device)
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def new_control(device="cuda", stream=None) -> torch.Tensor:
    """A zeroed frame control block.  The zero fill runs on `stream` (default:
    the current stream): pass the stream the frame calls will use, or order
    the two streams, so that the fill lands before scan_frame_initialize."""
    return _zeros(CONTROL_BYTES, device, stream)


def new_records(capacity: int, device="cuda", stream=None) -> torch.Tensor:
    """`capacity` zeroed frame records; the zero fill runs on `stream` as in new_control."""
    return _zeros(max(capacity, 1) * RECORD_BYTES, device, stream)


def _need_payload(control, payload, results, result_frames, records, capacity):
    _need("control", control, numel=CONTROL_BYTES)
    _need("payload", payload, torch.float32)
    _need("results", results, torch.float32, 2 * payload.numel() * 4)
    _need("result_frames", result_frames, torch.int64, 16)
    _need("records", records, numel=max(capacity, 0) * RECORD_BYTES, optional=True)


def scan_frame_load_kernels() -> str:
    buf = ctypes.create_string_buffer(4096)
    _check(_lib.load().sacc_scan_frame_load_kernels(buf, len(buf)))
    return buf.value.decode()


def scan_frame_initialize(control, epoch: int, result_frames, stream=None) -> None:
    _need("control", control, numel=CONTROL_BYTES)
    _need("result_frames", result_frames, torch.int64, 16)
    _check(_lib.load().sacc_scan_frame_initialize(_addr(control), epoch, _addr(result_frames), _stream_handle(stream)))


def scan_frame_begin(control, epoch: int, frame: int, stream=None) -> None:
    _need("control", control, numel=CONTROL_BYTES)
    _check(_lib.load().sacc_scan_frame_begin(_addr(control), epoch, frame, _stream_handle(stream)))


def scan_frame_gate(control, statuses, records=None, capacity: int = 0, stream=None) -> None:
    _need("control", control, numel=CONTROL_BYTES)
    _need("records", records, numel=max(capacity, 0) * RECORD_BYTES, optional=True)
    lst = _status_list(statuses)
    _check(_lib.load().sacc_scan_frame_gate(_addr(control), ctypes.byref(lst), _addr(records), capacity, _stream_handle(stream)))


def scan_frame_publish(control, payload, results, result_frames, records=None, capacity: int = 0, stream=None) -> None:
    _need_payload(control, payload, results, result_frames, records, capacity)
    _check(_lib.load().sacc_scan_frame_publish(_addr(control), _addr(payload), payload.numel(), _addr(results),
                                               _addr(result_frames), _addr(records), capacity, _stream_handle(stream)))


def scan_frame_commit(control, stream=None) -> None:
    _need("control", control, numel=CONTROL_BYTES)
    _check(_lib.load().sacc_scan_frame_commit(_addr(control), _stream_handle(stream)))


def scan_frame_packet(control, packet, stream=None) -> None:
    _need("control", control, numel=CONTROL_BYTES)
    _need("packet", packet, numel=PACKET_BYTES)
    _check(_lib.load().sacc_scan_frame_packet(_addr(control), _addr(packet), _stream_handle(stream)))


def scan_frame_step(control, epoch: int, frame: int, statuses, payload, results, result_frames, records=None,
                    capacity: int = 0, packet=None, stream=None) -> None:
    """begin + gate + publish + commit (+ packet) of one frame as one launch."""
    _need_payload(control, payload, results, result_frames, records, capacity)
    _need("packet", packet, numel=PACKET_BYTES, optional=True)
    lst = _status_list(statuses)
    _check(_lib.load().sacc_scan_frame_step(_addr(control), epoch, frame, ctypes.byref(lst), _addr(payload), payload.numel(),
                                            _addr(results), _addr(result_frames), _addr(records), capacity, _addr(packet),
                                            _stream_handle(stream)))


def scan_frame_check_finite(data, status, flag: int, stream=None) -> None:
    _need("data", data, torch.float32)
    _need("status", status, numel=8)
    _check(_lib.load().sacc_scan_frame_check_finite(_addr(data), data.numel(), _addr(status), flag, _stream_handle(stream)))


def scan_frame_delay(cycles: int, stream=None) -> None:
    _check(_lib.load().sacc_scan_frame_delay(cycles, _stream_handle(stream)))


def scan_frame_digest(payload: np.ndarray) -> int:
    """Host twin of the publish digest (float32 payload)."""
    a = np.ascontiguousarray(payload, np.float32)
    return int(_lib.load().sacc_scan_frame_digest(a.ctypes.data if a.size else None, a.size))


def model_producer_workspace_bytes() -> int:
    return int(_lib.load().sacc_model_producer_workspace_bytes())


def model_producer_load_kernels() -> str:
    buf = ctypes.create_string_buffer(1024)
    _check(_lib.load().sacc_model_producer_load_kernels(buf, len(buf)))
    return buf.value.decode()


def model_producer_cuda(images, cls, reg, plugins, producer, workspace, stream=None, profile: str = "t01-640x640") -> None:
    """images (1, 3, H, W) float32; cls / reg: three float32 tensors each; plugins:
    nine status words ((9, 2) int32 tensor or nine rows); producer: int32 of 2."""
    if profile not in PROFILES:
        raise ScanInvalidArgument("unknown model profile (expected t01-640x640 or hr-1280x768)")
    for name, t in [("images", images)] + [(f"cls[{i}]", c) for i, c in enumerate(cls)] + \
            [(f"reg[{i}]", r) for i, r in enumerate(reg)]:
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ScanInvalidArgument(f"{name} must be a contiguous float32 tensor")
    raw = _lib.RawView()
    for level in range(3):
        raw.cls[level] = _addr(cls[level])
        raw.reg[level] = _addr(reg[level])
        raw.cls_elements[level] = cls[level].numel()
        raw.reg_elements[level] = reg[level].numel()
    ptrs = _status_ptrs(plugins)
    if len(ptrs) != MODEL_PRODUCER_PLUGINS:
        raise ScanInvalidArgument("model producer takes exactly nine plugin statuses")
    arr = (ctypes.c_void_p * MODEL_PRODUCER_PLUGINS)(*ptrs)
    _check(_lib.load().sacc_model_producer_cuda(_addr(images), images.numel(), ctypes.byref(raw), arr, _addr(producer),
                                                _addr(workspace), workspace.numel() * workspace.element_size(),
                                                _stream_handle(stream), PROFILES[profile][0]))


# ------------------------------------------------------------ host readers

def read_control(raw: bytes | np.ndarray) -> dict:
    c = _lib.FrameControl.from_buffer_copy(bytes(np.asarray(raw, np.uint8).tobytes())[:CONTROL_BYTES])
    return {k: getattr(c, k) for k, _ in _lib.FrameControl._fields_}


def read_record(raw: bytes | np.ndarray, index: int = 0) -> dict:
    b = bytes(np.asarray(raw, np.uint8).tobytes())[index * RECORD_BYTES:(index + 1) * RECORD_BYTES]
    r = _lib.FrameRecord.from_buffer_copy(b)
    return {"flags": list(r.flags), "done": list(r.done), "frame_status": r.frame_status, "published": r.published,
            "digest": r.digest}


def parse_packet(raw: bytes | np.ndarray) -> dict:
    """ResultPacket v1 header fields (little endian)."""
    b = bytes(np.asarray(raw, np.uint8).tobytes())
    magic, version, header, total, cap = struct.unpack_from("<4sHHII", b, 0)
    epoch, current, committed, fail_frame = struct.unpack_from("<Qqqq", b, 16)
    status, frame_error, fail_code = struct.unpack_from("<I4xII", b, 48)
    return {"magic": magic, "version": version, "header_bytes": header, "packet_bytes": total, "capacity": cap,
            "epoch": epoch, "frame": current, "committed": committed, "fail_frame": fail_frame, "status": status,
            "frame_error": frame_error, "fail_code": fail_code}
