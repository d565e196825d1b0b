"""GPU parity of the status consumers: the library's frame protocol (the five
single steps and the one-launch step) and model-producer aggregate against the
reference's own kernels (oracle/_ref/libref_frame.so, built from the reference
sources) and the host model, byte for byte: control block, records, result
versions, result frames, packets and retired statuses."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import saccade_v1_b200 as sb  # noqa: E402
from oracle import frame_oracle as fo  # noqa: E402
from oracle import ref_frame  # noqa: E402
from saccade_v1_b200 import frame as fr  # noqa: E402

DONE = fo.SCAN_DONE
FLT_MAX = float(np.finfo(np.float32).max)


def ref():
    R = ref_frame.load()
    if R is None:
        pytest.skip("oracle/_ref/libref_frame.so is not built")
    ref_frame.check(R.ref_frame_load())
    return R


def words(rows):
    return torch.tensor(np.array(rows, np.uint32).reshape(-1, 2).view(np.int32), device="cuda")


def host_words(t):
    return t.cpu().numpy().view(np.uint32).reshape(-1, 2).tolist()


class Lane:
    """Device buffers of one frame stream."""

    def __init__(self, control_bytes, record_bytes, count, capacity):
        self.ctl = torch.zeros(control_bytes, dtype=torch.uint8, device="cuda")
        self.st = torch.zeros((16, 2), dtype=torch.int32, device="cuda")
        self.records = torch.zeros(capacity * record_bytes, dtype=torch.uint8, device="cuda")
        self.results = torch.zeros(2 * count, dtype=torch.float32, device="cuda")
        self.rf = torch.zeros(2, dtype=torch.int64, device="cuda")
        self.packet = torch.zeros(fr.PACKET_BYTES, dtype=torch.uint8, device="cuda")


def scenario(rng, n_max=16):
    n = 0 if rng.random() < 0.05 else int(rng.integers(1, n_max + 1))
    st = [[0, DONE] for _ in range(n)]
    if n:
        i = int(rng.integers(n))
        r = rng.random()
        if r < 0.08:
            st[i] = [int(rng.choice([1, 1 << 5, 1 << 9, 1 << 13, fo.CROSS_SCAN_NONFINITE_INPUT, fo.FRAME_NONFINITE_INPUT,
                                     fo.FRAME_NONFINITE_OUTPUT])), DONE]
        elif r < 0.12:
            st[i] = [0, int(rng.choice([0, DONE ^ 1, 0x12345678]))]
        elif r < 0.14:
            st[i] = [1 << 31, DONE]
    return st


@pytest.mark.parametrize("count", [0, 1000, (1 << 20) + 3])
def test_frame_protocol_matches_reference_and_model(count):
    R = ref()
    s = torch.cuda.Stream()
    cap = 24
    ours, fused = Lane(fr.CONTROL_BYTES, fr.RECORD_BYTES, count, cap), Lane(fr.CONTROL_BYTES, fr.RECORD_BYTES, count, cap)
    theirs = Lane(R.ref_frame_control_bytes(), R.ref_frame_record_bytes(), count, cap)
    model = fo.FrameModel(epoch=0, count=count, capacity=cap)
    rng = np.random.default_rng(1000 + count)
    frames = 40 if count < 100000 else 16
    epoch, local = 0, 0
    for k in range(frames):
        if k % 8 == 0:  # a fresh stream every 8 frames (a latched failure skips the rest)
            epoch, local = 0x5EED0000 + k, 0
            with torch.cuda.stream(s):
                for lane in (ours, fused):
                    fr.scan_frame_initialize(lane.ctl, epoch, lane.rf, stream=s)
                ref_frame.check(R.ref_frame_initialize(theirs.ctl.data_ptr(), epoch, theirs.rf.data_ptr(), s.cuda_stream))
            model.initialize(epoch)
        st = scenario(rng)
        n = len(st)
        fno = local if rng.random() > 0.05 else local + int(rng.choice([-1, 1, 3]))
        ep = epoch if rng.random() > 0.03 else epoch + 1
        host = rng.standard_normal(count).astype(np.float32)
        with torch.cuda.stream(s):
            payload = torch.from_numpy(host).cuda()
            for lane in (ours, fused, theirs):
                if n:
                    lane.st[:n].copy_(words(st))
            fr.scan_frame_begin(ours.ctl, ep, fno, stream=s)
            fr.scan_frame_gate(ours.ctl, ours.st[:n], ours.records, cap, stream=s)
            fr.scan_frame_publish(ours.ctl, payload, ours.results, ours.rf, ours.records, cap, stream=s)
            fr.scan_frame_commit(ours.ctl, stream=s)
            fr.scan_frame_packet(ours.ctl, ours.packet, stream=s)
            fr.scan_frame_step(fused.ctl, ep, fno, fused.st[:n], payload, fused.results, fused.rf, fused.records, cap,
                               fused.packet, stream=s)
            t = theirs
            sp = ref_frame.ptrs([t.st.data_ptr() + 8 * i for i in range(n)])
            ref_frame.check(R.ref_frame_begin(t.ctl.data_ptr(), ep, fno, s.cuda_stream))
            ref_frame.check(R.ref_frame_gate(t.ctl.data_ptr(), sp, n, t.records.data_ptr(), cap, s.cuda_stream))
            ref_frame.check(R.ref_frame_publish(t.ctl.data_ptr(), payload.data_ptr() if count else None, count,
                                                t.results.data_ptr() if count else None, t.rf.data_ptr(),
                                                t.records.data_ptr(), cap, s.cuda_stream))
            ref_frame.check(R.ref_frame_commit(t.ctl.data_ptr(), s.cuda_stream))
            ref_frame.check(R.ref_frame_packet(t.ctl.data_ptr(), t.packet.data_ptr(), s.cuda_stream))
        s.synchronize()
        want_packet = model.frame(ep, fno, [list(x) for x in st], host)
        tag = f"frame {k} ({n} statuses, frame {fno}, epoch {'ok' if ep == epoch else 'bad'})"
        for name, lane in (("single steps", ours), ("one launch", fused)):
            assert torch.equal(lane.ctl[:60].cpu(), theirs.ctl[:60].cpu()), f"{name} control, {tag}"
            assert torch.equal(lane.records.cpu(), theirs.records.cpu()), f"{name} records, {tag}"
            assert torch.equal(lane.results.view(torch.int32), theirs.results.view(torch.int32)), f"{name} results, {tag}"
            assert torch.equal(lane.rf.cpu(), theirs.rf.cpu()), f"{name} result frames, {tag}"
            assert bytes(lane.packet.cpu().numpy()) == want_packet, f"{name} packet, {tag}"
            assert torch.equal(lane.st.cpu(), theirs.st.cpu()), f"{name} retired statuses, {tag}"
        assert bytes(theirs.packet.cpu().numpy()) == want_packet, f"reference packet vs model, {tag}"
        c = fr.read_control(fused.ctl.cpu().numpy())
        assert c["arrivals"] == 0 and c["digest_sum"] == 0
        m = model.c
        assert (c["current"], c["committed"], c["fail_frame"], c["fail_code"], c["committed_slot"]) == \
            (m.current, m.committed, m.fail_frame, m.fail_code, m.committed_slot), tag
        assert theirs.rf.cpu().tolist() == model.result_frames
        if 0 <= fno < cap:
            r = fr.read_record(fused.records.cpu().numpy(), fno)
            mr = model.records[fno]
            assert (r["flags"], r["done"], r["frame_status"], r["published"], r["digest"]) == \
                (mr.flags, mr.done, mr.frame_status, mr.published, mr.digest), tag
        local += 1
    np.testing.assert_array_equal(theirs.results.cpu().numpy().reshape(2, count).view(np.uint32),
                                  model.results.view(np.uint32))


@pytest.mark.parametrize("n", [0, 1, 4097, 1 << 20])
def test_digest_matches_reference(n):
    R = ref()
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    x[:: 97] = np.nan
    want = R.ref_frame_digest(x.ctypes.data if n else None, n)
    assert fr.scan_frame_digest(x) == want == fo.digest(x)


@pytest.mark.parametrize("count", [0, 1, 1000, (1 << 22) + 1])
def test_check_finite_matches_reference(count):
    R = ref()
    s = torch.cuda.Stream()
    cases = [(None, None)] + [(pos, bad) for pos in sorted({0, count // 2, max(count - 1, 0)}) if count
                              for bad in (np.nan, np.inf, -np.inf, FLT_MAX, -FLT_MAX)]
    for pos, bad in cases:
        with torch.cuda.stream(s):
            data = torch.zeros(count, dtype=torch.float32, device="cuda")
            if pos is not None:
                data[pos] = float(bad)
            mine, theirs = words([[0xFFFFFFFF, 0x12345678]]), words([[0xFFFFFFFF, 0x12345678]])
            fr.scan_frame_check_finite(data, mine, fo.FRAME_NONFINITE_OUTPUT, stream=s)
            ref_frame.check(R.ref_frame_check_finite(data.data_ptr() if count else None, count, theirs.data_ptr(),
                                                     fo.FRAME_NONFINITE_OUTPUT, s.cuda_stream))
        s.synchronize()
        finite = bad is None or np.isfinite(bad)
        want = [[0 if finite else fo.FRAME_NONFINITE_OUTPUT, DONE]]
        assert host_words(mine) == host_words(theirs) == want, (count, pos, bad)


def profile_tensors(seed=5, width=640, height=640):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    images = torch.randn(1, 3, height, width, device="cuda", generator=g) * 0.5
    cls = [torch.randn(1, 80, height // s, width // s, device="cuda", generator=g) for s in (8, 16, 32)]
    reg = [torch.randn(1, 4, height // s, width // s, device="cuda", generator=g) for s in (8, 16, 32)]
    return images, cls, reg


def run_producer(R, s, images, cls, reg, plugin_rows):
    mine, theirs = words(plugin_rows), words(plugin_rows)
    prod_m, prod_r = words([[0xA5A5A5A5, 0xA5A5A5A5]]), words([[0xA5A5A5A5, 0xA5A5A5A5]])
    ws_m = torch.zeros(fr.model_producer_workspace_bytes(), dtype=torch.uint8, device="cuda")
    ws_r = torch.zeros(R.ref_producer_workspace_bytes(), dtype=torch.uint8, device="cuda")
    with torch.cuda.stream(s):
        fr.model_producer_cuda(images, cls, reg, mine, prod_m, ws_m, stream=s)
        ref_frame.check(R.ref_model_producer(
            images.data_ptr(), images.numel(), ref_frame.ptrs([c.data_ptr() for c in cls]),
            ref_frame.ptrs([r.data_ptr() for r in reg]), ref_frame.sizes([c.numel() for c in cls]),
            ref_frame.sizes([r.numel() for r in reg]), ref_frame.ptrs([theirs.data_ptr() + 8 * i for i in range(9)]),
            prod_r.data_ptr(), ws_r.data_ptr(), ws_r.numel(), s.cuda_stream, 0))
    s.synchronize()
    assert host_words(mine) == host_words(theirs) == [[0, 0]] * 9, "every plugin status retired"
    got, want = host_words(prod_m)[0], host_words(prod_r)[0]
    assert got == want, (got, want)
    return got


def test_model_producer_status_cases_match_reference():
    R = ref()
    s = torch.cuda.Stream()
    images, cls, reg = profile_tensors()
    tensors = [images.cpu().numpy()] + [c.cpu().numpy() for c in cls] + [r.cpu().numpy() for r in reg]
    fresh = lambda: [[0, DONE] for _ in range(9)]
    assert run_producer(R, s, images, cls, reg, fresh()) == [0, fo.PRODUCER_DONE]
    assert run_producer(R, s, images, cls, reg, [[0, 0]] * 9) == [fo.POST_PROTOCOL, fo.PRODUCER_DONE]
    for i in range(9):
        scan = i % 3 == 1
        valid = fo.SCAN_INPUT_FAILURES | fo.SCAN_RANGE_FAILURES if scan else fo.CROSS_SCAN_NONFINITE_INPUT
        wrong = fo.CROSS_SCAN_NONFINITE_INPUT if scan else 1
        for source in ([valid, DONE], [0, 0], [0, DONE ^ 1], [1 << 31, DONE], [wrong, DONE]):
            rows = fresh()
            rows[i] = list(source)
            want, _ = fo.producer_aggregate([list(r) for r in rows], tensors)
            assert run_producer(R, s, images, cls, reg, rows) == [want, fo.PRODUCER_DONE], (i, source)
    rows = fresh()
    rows[0], rows[8] = [fo.CROSS_SCAN_NONFINITE_INPUT, DONE], [0, 0]
    assert run_producer(R, s, images, cls, reg, rows) == [fo.POST_NUMERIC | fo.POST_PROTOCOL, fo.PRODUCER_DONE]


def test_model_producer_finite_checks_match_reference():
    R = ref()
    s = torch.cuda.Stream()
    images, cls, reg = profile_tensors(6)
    flat = [images.view(-1)] + [c.view(-1) for c in cls] + [r.view(-1) for r in reg]
    fresh = lambda: [[0, DONE] for _ in range(9)]
    for t, x in enumerate(flat):
        for index in (0, x.numel() - 1):
            original = float(x[index])
            for bad in (np.nan, np.inf, -np.inf):
                x[index] = float(bad)
                assert run_producer(R, s, images, cls, reg, fresh()) == [fo.POST_NUMERIC, fo.PRODUCER_DONE], (t, index, bad)
            x[index] = original
    flat[0][-1], flat[6][-1] = FLT_MAX, -FLT_MAX
    assert run_producer(R, s, images, cls, reg, fresh()) == [0, fo.PRODUCER_DONE]


def test_model_producer_rejections():
    images, cls, reg = profile_tensors(7)
    plugins = words([[0, DONE]] * 9)
    producer = torch.zeros(2, dtype=torch.int32, device="cuda")
    ws = torch.zeros(fr.model_producer_workspace_bytes(), dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    with pytest.raises(sb.ScanInvalidArgument, match="current CUDA device|device memory"):
        fr.model_producer_cuda(images.cpu(), cls, reg, plugins, producer, ws, stream=s)
    with pytest.raises(sb.ScanInvalidArgument, match="overlapping model producer buffers"):
        fr.model_producer_cuda(images, cls, reg, plugins, plugins[0], ws, stream=s)
    with pytest.raises(sb.ScanInvalidArgument, match="incorrect model producer input/workspace capacity"):
        fr.model_producer_cuda(images, cls, reg, plugins, producer, ws, stream=s, profile="hr-1280x768")
    with pytest.raises(sb.ScanInvalidArgument, match="F04 requires all six fixed-shape raw tensors"):
        fr.model_producer_cuda(images, cls[::-1], reg, plugins, producer, ws, stream=s)
    assert host_words(plugins) == [[0, DONE]] * 9  # rejected before any GPU work


def test_frame_step_in_cuda_graph():
    """Five frames (status words re-armed by copies inside the graph) captured
    once; two replays from a fresh initialize give the single steps' bytes."""
    s = torch.cuda.Stream()
    count, cap, n = 4096, 8, 3
    rng = np.random.default_rng(9)
    rows = [[[0, DONE]] * n for _ in range(5)]
    rows[3] = [[0, DONE], [1 << 9, DONE], [0, DONE]]  # frame 3 fails, frame 4 is skipped
    with torch.cuda.stream(s):
        staged = [words(r) for r in rows]
        payloads = [torch.from_numpy(rng.standard_normal(count).astype(np.float32)).cuda() for _ in range(5)]
        g_lane, e_lane = Lane(fr.CONTROL_BYTES, fr.RECORD_BYTES, count, cap), Lane(fr.CONTROL_BYTES, fr.RECORD_BYTES, count, cap)
        packets = torch.zeros((5, fr.PACKET_BYTES), dtype=torch.uint8, device="cuda")
        e_packets = torch.zeros_like(packets)
        fr.scan_frame_initialize(e_lane.ctl, 77, e_lane.rf, stream=s)
        for k in range(5):
            e_lane.st[:n].copy_(staged[k])
            fr.scan_frame_begin(e_lane.ctl, 77, k, stream=s)
            fr.scan_frame_gate(e_lane.ctl, e_lane.st[:n], e_lane.records, cap, stream=s)
            fr.scan_frame_publish(e_lane.ctl, payloads[k], e_lane.results, e_lane.rf, e_lane.records, cap, stream=s)
            fr.scan_frame_commit(e_lane.ctl, stream=s)
            fr.scan_frame_packet(e_lane.ctl, e_packets[k], stream=s)
        fr.scan_frame_initialize(g_lane.ctl, 77, g_lane.rf, stream=s)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for k in range(5):
            g_lane.st[:n].copy_(staged[k])
            fr.scan_frame_step(g_lane.ctl, 77, k, g_lane.st[:n], payloads[k], g_lane.results, g_lane.rf, g_lane.records,
                               cap, packets[k], stream=s)
    for _ in range(2):
        with torch.cuda.stream(s):
            fr.scan_frame_initialize(g_lane.ctl, 77, g_lane.rf, stream=s)
            graph.replay()
        s.synchronize()
        assert torch.equal(packets, e_packets)
        assert torch.equal(g_lane.ctl[:60], e_lane.ctl[:60]) and torch.equal(g_lane.records, e_lane.records)
        assert torch.equal(g_lane.results, e_lane.results) and torch.equal(g_lane.rf, e_lane.rf)
    outcomes = [fo.outcome(bytes(p)) for p in packets.cpu().numpy()]
    assert [o[1] for o in outcomes] == [0, 0, 0, 1, 2]
