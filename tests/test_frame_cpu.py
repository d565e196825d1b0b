"""CPU checks of the status consumers: the host model of the frame protocol
and of the producer aggregate reproduces the reference tests' known answers
(tests/scan_trt_tests.cpp:704-776, tests/model_producer_cuda_tests.cpp:144-200),
the library's host digest equals the model's, and the C ABI rejects bad calls
before any CUDA work."""
import ctypes

import numpy as np
import pytest

from oracle import frame_oracle as fo
from saccade_v1_b200 import _lib, frame

OK, FAILED, SKIPPED = 0, 1, 2
FAKE_STREAM = 0x5EED


def statuses(n=3):
    return [[0, fo.SCAN_DONE] for _ in range(n)]


def payload(seed, n=37):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


def test_valid_frames_commit_in_order():
    m = fo.FrameModel(epoch=7, count=37, capacity=8)
    for k in range(4):
        pk = m.frame(7, k, statuses(), payload(k))
        assert fo.outcome(pk) == (k, OK, 0, 0)
        assert m.records[k].published == 1 and m.records[k].digest == fo.digest(payload(k))
    assert m.c.committed == 3 and m.result_frames[m.c.committed_slot] == 3
    np.testing.assert_array_equal(m.results[m.c.committed_slot], payload(3))


def test_failure_latches_and_keeps_the_committed_payload():
    m = fo.FrameModel(epoch=1, count=37, capacity=8)
    m.frame(1, 0, statuses(), payload(0))
    bad = statuses()
    bad[1] = [1 << 1, fo.SCAN_DONE]  # scan plugin: non-finite delta
    assert fo.outcome(m.frame(1, 1, bad, payload(1))) == (1, FAILED, fo.NUMERIC, fo.NUMERIC)
    assert fo.outcome(m.frame(1, 2, statuses(), payload(2))) == (2, SKIPPED, 0, fo.NUMERIC)
    assert m.c.committed == 0 and m.c.fail_frame == 1 and m.records[2].published == 0
    np.testing.assert_array_equal(m.results[m.c.committed_slot], payload(0))


@pytest.mark.parametrize("index,status,error", [
    (1, [1 << 9, fo.SCAN_DONE], fo.NUMERIC),                      # flags with a finite payload (drive range)
    (1, [0, 0], fo.PROTOCOL),                                     # missing completion
    (1, [1 << 31, fo.SCAN_DONE], fo.NUMERIC | fo.PROTOCOL),       # unknown flag
    (0, [fo.CROSS_SCAN_NONFINITE_INPUT, fo.SCAN_DONE], fo.NUMERIC),  # expand flag
])
def test_invalid_status_blocks_publication(index, status, error):
    m = fo.FrameModel(epoch=3, count=37, capacity=4)
    st = statuses()
    st[index] = list(status)
    assert fo.outcome(m.frame(3, 0, st, payload(0))) == (0, FAILED, error, error)
    assert m.records[0].published == 0 and m.result_frames == [-1, -1]
    assert all(s == [0, 0] for s in st)  # every status retired


def test_protocol_errors():
    m = fo.FrameModel(epoch=3, count=5, capacity=4)
    assert fo.outcome(m.frame(3, 1, statuses(), payload(0, 5)))[1:] == (FAILED, fo.PROTOCOL, fo.PROTOCOL)  # out of order
    m = fo.FrameModel(epoch=3, count=5, capacity=4)
    assert fo.outcome(m.frame(4, 0, statuses(), payload(0, 5)))[1:] == (FAILED, fo.PROTOCOL, fo.PROTOCOL)  # epoch
    m = fo.FrameModel(epoch=3, count=5, capacity=4)
    assert fo.outcome(m.frame(3, 0, [], payload(0, 5)))[1:] == (FAILED, fo.PROTOCOL, fo.PROTOCOL)  # no status
    m = fo.FrameModel(epoch=3, count=5, capacity=4)
    st = statuses()
    m.frame(3, 0, st, payload(0, 5))
    assert fo.outcome(m.frame(3, 1, st, payload(1, 5)))[1:] == (FAILED, fo.PROTOCOL, fo.PROTOCOL)  # retired words


def test_producer_status_cases():
    tensors = [np.zeros(12, np.float32)] * 7
    fresh = lambda: [[0, fo.SCAN_DONE] for _ in range(fo.PRODUCER_PLUGINS)]
    p = fresh()
    assert fo.producer_aggregate(p, tensors) == (0, fo.PRODUCER_DONE)
    assert fo.producer_aggregate(p, tensors)[0] == fo.POST_PROTOCOL  # omitted producer: retired words
    for i in range(fo.PRODUCER_PLUGINS):
        scan = i % 3 == 1
        valid = fo.SCAN_INPUT_FAILURES | fo.SCAN_RANGE_FAILURES if scan else fo.CROSS_SCAN_NONFINITE_INPUT
        wrong = fo.CROSS_SCAN_NONFINITE_INPUT if scan else 1
        for source, want in (([valid, fo.SCAN_DONE], fo.POST_NUMERIC), ([0, 0], fo.POST_PROTOCOL),
                             ([0, fo.SCAN_DONE ^ 1], fo.POST_PROTOCOL), ([1 << 31, fo.SCAN_DONE], fo.POST_NUMERIC | fo.POST_PROTOCOL),
                             ([wrong, fo.SCAN_DONE], fo.POST_NUMERIC | fo.POST_PROTOCOL)):
            p = fresh()
            p[i] = list(source)
            assert fo.producer_aggregate(p, tensors)[0] == want, (i, source)
            assert all(s == [0, 0] for s in p)
    p = fresh()
    p[0], p[8] = [fo.CROSS_SCAN_NONFINITE_INPUT, fo.SCAN_DONE], [0, 0]
    assert fo.producer_aggregate(p, tensors)[0] == fo.POST_NUMERIC | fo.POST_PROTOCOL
    for t in range(7):
        for bad in (np.nan, np.inf, -np.inf):
            ts = [x.copy() for x in tensors]
            ts[t][-1] = bad
            assert fo.producer_aggregate(fresh(), ts)[0] == fo.POST_NUMERIC
    ts = [x.copy() for x in tensors]
    ts[0][-1], ts[6][-1] = np.finfo(np.float32).max, -np.finfo(np.float32).max
    assert fo.producer_aggregate(fresh(), ts)[0] == 0


@pytest.mark.parametrize("n", [0, 1, 37, 100003])
def test_library_digest_equals_model(n):
    x = payload(n, n)
    assert frame.scan_frame_digest(x) == fo.digest(x)
    if n:
        want = sum(fo.mix64((i << 32) | int(b)) for i, b in enumerate(x[:64].view(np.uint32))) & fo.M64
        assert fo.digest(x[:64]) == want


def test_frame_struct_sizes():
    assert frame.CONTROL_BYTES == 72 and frame.RECORD_BYTES == 144 and ctypes.sizeof(_lib.StatusList) == 136
    assert frame.PACKET_BYTES == fo.PACKET_BYTES == 12368


def test_frame_host_rejections():
    L = _lib.load()
    lst = _lib.StatusList()
    lst.count = 17
    rc = L.sacc_scan_frame_gate(0x1000, ctypes.byref(lst), None, 0, FAKE_STREAM)
    assert rc == _lib.SACC_EINVAL and "too many statuses" in _lib.last_error()
    lst.count = 1
    lst.status[0] = 0x2002
    rc = L.sacc_scan_frame_gate(0x1000, ctypes.byref(lst), None, 0, FAKE_STREAM)
    assert rc == _lib.SACC_EINVAL and "status is not 4-byte aligned" in _lib.last_error()
    assert L.sacc_scan_frame_begin(None, 1, 0, FAKE_STREAM) == _lib.SACC_EINVAL and "control is null" in _lib.last_error()
    assert L.sacc_scan_frame_commit(0x1000, 0) == _lib.SACC_EINVAL and "explicit non-default stream" in _lib.last_error()
    rc = L.sacc_scan_frame_publish(0x1000, 0x2000, 16, 0x2010, 0x3000, None, 0, FAKE_STREAM)
    assert rc == _lib.SACC_EINVAL and "results overlap payload" in _lib.last_error()
    rc = L.sacc_scan_frame_check_finite(0x2000, 4, 0x2008, 1, FAKE_STREAM)
    assert rc == _lib.SACC_EINVAL and "status overlaps data" in _lib.last_error()


def test_producer_host_rejections():
    L = _lib.load()
    raw = _lib.RawView()
    plugins = (ctypes.c_void_p * 9)(*[0x9000 + 8 * i for i in range(9)])
    ws = frame.model_producer_workspace_bytes()
    rc = L.sacc_model_producer_cuda(0x1000, 5, ctypes.byref(raw), plugins, 0x8000, 0xA000, ws, FAKE_STREAM, 0)
    assert rc == _lib.SACC_EINVAL and "incorrect model producer input/workspace capacity" in _lib.last_error()
    rc = L.sacc_model_producer_cuda(0x1000, 3 * 640 * 640, ctypes.byref(raw), plugins, 0x8000, 0xA000, ws, FAKE_STREAM, 0)
    assert rc == _lib.SACC_EINVAL and "F04 requires all six fixed-shape raw tensors" in _lib.last_error()
    for level in range(3):
        s = 8 << level
        raw.cls[level], raw.reg[level] = 0x100000 * (level + 1), 0x100000 * (level + 4) + 2
        raw.cls_elements[level], raw.reg_elements[level] = 80 * (640 // s) ** 2, 4 * (640 // s) ** 2
    rc = L.sacc_model_producer_cuda(0x1000, 3 * 640 * 640, ctypes.byref(raw), plugins, 0x8000, 0xA000, ws, FAKE_STREAM, 0)
    assert rc == _lib.SACC_EINVAL and "F04 requires aligned FP32 raw tensors" in _lib.last_error()
    rc = L.sacc_model_producer_cuda(0x1000, 3 * 640 * 640, ctypes.byref(raw), plugins, 0x8000, 0xA000, ws, FAKE_STREAM, 7)
    assert rc == _lib.SACC_EINVAL and "unknown model profile" in _lib.last_error()
    rc = L.sacc_model_producer_cuda(0x1000, 3 * 1280 * 768, ctypes.byref(raw), plugins, 0x8000, 0xA000, ws, FAKE_STREAM, 0)
    assert rc == _lib.SACC_EINVAL and "capacity" in _lib.last_error()
