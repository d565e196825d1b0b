"""Host model of the frame-end protocol and the model producer's aggregate
(TEST INFRASTRUCTURE ONLY).

Restates, as plain Python over integers, the state changes of the reference's
frame kernels (cuda/scan_frame.cu: initialize :29-36, begin :38-46, gate
:48-68, publish :70-89, commit :91-104, packet :112-127, digest :201-209) and
of the producer aggregate (cuda/model_producer.cu:51-71).  The GPU tests also
run the reference's own kernels (oracle/_ref/libref_frame.so, built by
oracle/Makefile from the reference sources) beside the library's on the same
inputs; this model pins the known answers of the reference's tests on the CPU
(tests/scan_trt_tests.cpp:704-776, tests/model_producer_cuda_tests.cpp:144-200).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

SCAN_DONE = 0x4E414353
PROTOCOL, NUMERIC = 1 << 0, 1 << 3
SCAN_INPUT_FAILURES, SCAN_RANGE_FAILURES = 0x3F, 0x3F00
CROSS_SCAN_NONFINITE_INPUT = 1 << 16
FRAME_NONFINITE_INPUT, FRAME_NONFINITE_OUTPUT = 1 << 20, 1 << 21
KNOWN_FLAGS = SCAN_INPUT_FAILURES | SCAN_RANGE_FAILURES | CROSS_SCAN_NONFINITE_INPUT | FRAME_NONFINITE_INPUT | \
    FRAME_NONFINITE_OUTPUT
MAX_STATUSES = 16
PACKET_CAPACITY, PACKET_HEADER_BYTES, PACKET_ROW_BYTES = 256, 80, 48
PACKET_BYTES = PACKET_HEADER_BYTES + PACKET_CAPACITY * PACKET_ROW_BYTES
M64 = (1 << 64) - 1

PRODUCER_DONE = 0x34525046
POST_NUMERIC, POST_PROTOCOL = 1 << 0, 1 << 2
PRODUCER_PLUGINS = 9


def mix64(x: int) -> int:
    """splitmix64's output function (Steele, Lea and Flood 2014)."""
    x = ((x ^ (x >> 30)) * 0xbf58476d1ce4e5b9) & M64
    x = ((x ^ (x >> 27)) * 0x94d049bb133111eb) & M64
    return x ^ (x >> 31)


def digest(payload: np.ndarray) -> int:
    """Sum mod 2^64 of mix64(index << 32 | float bits) (reference :201-209)."""
    bits = np.ascontiguousarray(payload, np.float32).view(np.uint32).astype(np.uint64)
    x = (np.arange(bits.size, dtype=np.uint64) << np.uint64(32)) | bits
    with np.errstate(over="ignore"):
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xbf58476d1ce4e5b9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94d049bb133111eb)
        x = x ^ (x >> np.uint64(31))
    return int(x.sum(dtype=np.uint64))


@dataclass
class Record:
    flags: list = field(default_factory=lambda: [0] * MAX_STATUSES)
    done: list = field(default_factory=lambda: [0] * MAX_STATUSES)
    frame_status: int = 0
    published: int = 0
    digest: int = 0


@dataclass
class Control:
    epoch: int = 0
    current: int = -1
    committed: int = -1
    fail_frame: int = -1
    committed_slot: int = 1
    working_slot: int = 0
    frame_status: int = 0
    fail_code: int = 0
    run_stage: int = 0
    published: int = 0
    scan_flags: int = 0


class FrameModel:
    """One frame stream: control block, two result versions, records."""

    def __init__(self, epoch: int, count: int, capacity: int):
        self.c = Control(epoch=epoch)
        self.results = np.zeros((2, count), np.float32)
        self.result_frames = [-1, -1]
        self.capacity = capacity
        self.records = [Record() for _ in range(max(capacity, 0))]

    def initialize(self, epoch: int) -> None:
        """reference :29-36: the control block and result_frames reset; the
        result versions and records keep their contents."""
        self.c = Control(epoch=epoch)
        self.result_frames = [-1, -1]

    def _record(self):
        c = self.c
        return self.records[c.current] if 0 <= c.current < self.capacity else None

    def begin(self, epoch: int, frame: int) -> None:
        c = self.c
        c.current = frame
        c.working_slot = 1 - c.committed_slot
        c.frame_status = 0
        c.run_stage = 0
        c.published = 0
        if epoch != c.epoch or (not c.fail_code and frame != c.committed + 1):
            c.frame_status |= PROTOCOL

    def gate(self, statuses: list[list[int]]) -> None:
        """statuses: [flags, done] pairs, retired in place to [0, 0]."""
        c = self.c
        rec = self._record()
        if rec is not None:
            self.records[c.current] = rec = Record()
        for i, s in enumerate(statuses):
            flags, done = s
            if done != SCAN_DONE:
                c.frame_status |= PROTOCOL
            if flags:
                c.frame_status |= NUMERIC
            if flags & ~KNOWN_FLAGS:
                c.frame_status |= PROTOCOL
            c.scan_flags |= flags
            s[0] = s[1] = 0
            if rec is not None:
                rec.flags[i], rec.done[i] = flags, done
        if not statuses:
            c.frame_status |= PROTOCOL
        if rec is not None:
            rec.frame_status = c.frame_status
        c.run_stage = int(not c.fail_code and not c.frame_status)

    def publish(self, payload: np.ndarray) -> None:
        c = self.c
        if not c.run_stage:
            return
        self.results[c.working_slot, :] = payload
        rec = self._record()
        if rec is not None:
            rec.digest = (rec.digest + digest(payload)) & M64
        self.result_frames[c.working_slot] = c.current
        c.published = 1
        if rec is not None:
            rec.published = 1

    def commit(self) -> None:
        c = self.c
        if not c.fail_code:
            if not c.frame_status and not c.published:
                c.frame_status |= PROTOCOL
            if c.frame_status:
                c.fail_frame = c.current
                c.fail_code = c.frame_status
            else:
                c.committed = c.current
                c.committed_slot = c.working_slot
        c.run_stage = 0

    def packet(self) -> bytes:
        c = self.c
        out = bytearray(PACKET_BYTES)
        status = 0 if not c.fail_code else (1 if c.current == c.fail_frame else 2)
        struct.pack_into("<4sHHII", out, 0, b"SCRP", 1, PACKET_HEADER_BYTES, PACKET_BYTES, PACKET_CAPACITY)
        struct.pack_into("<QqqqI", out, 16, c.epoch, c.current, c.committed, c.fail_frame, status)
        struct.pack_into("<II", out, 56, c.fail_code if status == 1 else 0, c.fail_code)
        return bytes(out)

    def frame(self, epoch: int, frame: int, statuses: list[list[int]], payload: np.ndarray) -> bytes:
        """begin, gate, publish, commit, packet (the reference harness's order,
        src/scan_trt_frame.cpp:546-553)."""
        self.begin(epoch, frame)
        self.gate(statuses)
        self.publish(payload)
        self.commit()
        return self.packet()


def outcome(packet: bytes) -> tuple[int, int, int, int]:
    """(frame, status, frame_error, fail_code) of a packet: status 0 ok,
    1 failed, 2 skipped after a failure."""
    frame, = struct.unpack_from("<q", packet, 24)
    status, = struct.unpack_from("<I", packet, 48)
    frame_error, fail_code = struct.unpack_from("<II", packet, 56)
    return frame, status, frame_error, fail_code


# ------------------------------------------------------------ model producer

def producer_allowed(i: int) -> int:
    """Bits a source may carry (reference cuda/model_producer.cu:57-59)."""
    if i < PRODUCER_PLUGINS:
        return (SCAN_INPUT_FAILURES | SCAN_RANGE_FAILURES) if i % 3 == 1 else CROSS_SCAN_NONFINITE_INPUT
    return FRAME_NONFINITE_INPUT if i == PRODUCER_PLUGINS else FRAME_NONFINITE_OUTPUT


def producer_aggregate(plugins: list[list[int]], tensors: list[np.ndarray]) -> tuple[int, int]:
    """(flags, done) of the aggregate; retires `plugins` in place.  tensors[0]
    is the image, tensors[1:] the six raw outputs."""
    bad_in = not np.all(np.abs(np.asarray(tensors[0], np.float32)) <= np.finfo(np.float32).max)
    bad_out = any(not np.all(np.abs(np.asarray(t, np.float32)) <= np.finfo(np.float32).max) for t in tensors[1:])
    sources = plugins + [[FRAME_NONFINITE_INPUT if bad_in else 0, SCAN_DONE],
                         [FRAME_NONFINITE_OUTPUT if bad_out else 0, SCAN_DONE]]
    flags = 0
    for i, s in enumerate(sources):
        if s[0]:
            flags |= POST_NUMERIC
        if s[1] != SCAN_DONE or s[0] & ~producer_allowed(i):
            flags |= POST_PROTOCOL
        s[0] = s[1] = 0
    return flags, PRODUCER_DONE
