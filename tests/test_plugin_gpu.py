"""The plugin surface on the GPU: after bind(), enqueue must produce the same
bits and status words as the direct API (the reference's scan_trt_tests
compare every plugin call bit for bit with the direct S02 API,
docs/SCAN_TRT.md:46), including a failing call, and the three plugins chain
expand -> scan -> merge."""
import numpy as np
import pytest
import torch

from oracle.oracle import Shape, random_case

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as gu  # noqa: E402
import saccade_v1_b200 as sb  # noqa: E402
from saccade_v1_b200.plugin import (EXPAND, MERGE, SCAN, SCAN_F16, TENSOR_FLOAT, TENSOR_HALF, TENSOR_INT32,  # noqa: E402
                                    PluginError, ScanPlugin, TensorDesc)


def descs_for(k):
    s = k.shape
    dims = [(s.batch, s.length, s.channels), (s.batch, s.length, s.channels), (s.a_rows, s.state),
            (s.batch, s.length, s.state), (s.batch, s.length, s.c_width)] + ([(s.channels,)] if s.has_d else [])
    return [TensorDesc.of(d) for d in dims], [TensorDesc.of((s.batch, s.length, s.channels)),
                                              TensorDesc.of((2,), TENSOR_INT32)]


@pytest.mark.parametrize("bad", [False, True])
def test_plugin_enqueue_is_bitwise_the_direct_api(bad):
    k = random_case(Shape(4, 240, 256, 16, 1, 1, True), 0x5eed0600)
    if bad:
        k.delta[17] = np.inf
    p = ScanPlugin.create(*SCAN, [("has_d", 1)])
    p.bind()
    s = gu.stream()
    with torch.cuda.stream(s):
        ins = [gu.dev(x) for x in k.inputs()]
        y = torch.empty(k.u.size, device="cuda")
        st = gu.new_status()
        ind, outd = descs_for(k)
        p.enqueue(ind, outd, [t.data_ptr() for t in ins], [y.data_ptr(), st.data_ptr()], s)
    s.synchronize()
    direct_y, direct_st = gu.run_f32(k)
    assert gu.status_words(st) == direct_st
    assert np.array_equal(y.cpu().numpy().view(np.uint32), direct_y.view(np.uint32))


def test_plugin_descriptor_rejection_leaves_status():
    k = random_case(Shape(2, 8, 128, 16, 1, 1, True), 0x5eed0601)
    p = ScanPlugin.create(*SCAN, [("has_d", 1)])
    p.bind()
    s = gu.stream()
    with torch.cuda.stream(s):
        ins = [gu.dev(x) for x in k.inputs()]
        y = torch.empty(k.u.size, device="cuda")
        st = gu.new_status()
    s.synchronize()
    ind, outd = descs_for(k)
    ind[1] = TensorDesc.of((2, 9, 128))
    with pytest.raises(PluginError, match=r"saccade::SelectiveScan: delta \(2,9,128\) differs from u \(2,8,128\)"):
        p.enqueue(ind, outd, [t.data_ptr() for t in ins], [y.data_ptr(), st.data_ptr()], s)
    assert gu.status_words(st) == gu.STATUS_SENTINEL


def test_plugins_chain_expand_scan_merge():
    C, H, W = 8, 5, 5
    L = H * W
    x = np.random.default_rng(1).standard_normal(C * L).astype(np.float32)
    k = random_case(Shape(4, L, C, 4, 1, 1, True), 0x5eed0602)
    e = ScanPlugin.create(*EXPAND, [])
    sc = ScanPlugin.create(*SCAN, [("has_d", 1)])
    m = ScanPlugin.create(*MERGE, [("height", H), ("width", W)])
    for p in (e, sc, m):
        p.bind()
    s = gu.stream()
    with torch.cuda.stream(s):
        dx = gu.dev(x)
        tokens = torch.empty(4 * C * L, device="cuda")
        ins = [gu.dev(v) for v in k.inputs()]
        y = torch.empty(4 * L * C, device="cuda")
        out = torch.empty(C * L, device="cuda")
        sts = [gu.new_status() for _ in range(3)]
        e.enqueue([TensorDesc.of((1, C, H, W))], [TensorDesc.of((4, L, C)), TensorDesc.of((2,), TENSOR_INT32)],
                  [dx.data_ptr()], [tokens.data_ptr(), sts[0].data_ptr()], s)
        ind, outd = descs_for(k)
        sc.enqueue(ind, outd, [tokens.data_ptr()] + [t.data_ptr() for t in ins[1:]], [y.data_ptr(), sts[1].data_ptr()], s)
        m.enqueue([TensorDesc.of((4, L, C))], [TensorDesc.of((1, C, H, W)), TensorDesc.of((2,), TENSOR_INT32)],
                  [y.data_ptr()], [out.data_ptr(), sts[2].data_ptr()], s)
    s.synchronize()
    assert all(gu.status_words(t) == (0, sb.SCAN_DONE) for t in sts)
    # Same calls through the direct API give the same bits.
    k2 = k.copy()
    from oracle import oracle
    k2.u = oracle.cross_scan_expand(x, 1, C, H, W)
    y2, _ = gu.run_f32(k2)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), y2.view(np.uint32))


@pytest.mark.parametrize("bad", [False, True])
def test_fp16_plugin_enqueue_is_bitwise_the_direct_api(bad):
    """SelectiveScan v3 (FP16 u, delta, B, C, y; FP32 A, D) enqueues the same
    bits and status words as sacc_selective_scan_f16."""
    k = random_case(Shape(4, 240, 256, 16, 1, 1, True), 0x5eed0610)
    if bad:
        k.delta[17] = np.inf
    p = ScanPlugin.create(*SCAN_F16, [("has_d", 1)])
    p.bind()
    s = gu.stream()
    sh = sb.SelectiveScanShape(4, 240, 256, 16, 1, 1, True)
    with torch.cuda.stream(s):
        h = lambda x: torch.from_numpy(x).cuda().half()
        f = lambda x: torch.from_numpy(x).cuda()
        ins = [h(k.u), h(k.delta), f(k.a), h(k.b), h(k.c), f(k.d)]
        y = torch.empty(k.u.size, dtype=torch.float16, device="cuda")
        st = gu.new_status()
        ind, outd = descs_for(k)
        for i in (0, 1, 3, 4):
            ind[i].type = TENSOR_HALF
        outd[0].type = TENSOR_HALF
        p.enqueue(ind, outd, [t.data_ptr() for t in ins], [y.data_ptr(), st.data_ptr()], s)
        y2 = torch.empty_like(y)
        st2 = gu.new_status()
        sb.selective_scan_f16(sh, *ins, y2, st2, stream=s)
    s.synchronize()
    assert gu.status_words(st) == gu.status_words(st2)
    assert (gu.status_words(st)[0] != 0) == bad
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
    ind[0].type = TENSOR_FLOAT
    with pytest.raises(PluginError, match="input 0 is not linear FP16"):
        p.enqueue(ind, outd, [t.data_ptr() for t in ins], [y.data_ptr(), st.data_ptr()], s)


@pytest.mark.parametrize("dt,L", [("f16", 240), ("bf16", 60)])
def test_block_plugin_is_bitwise_the_block_api(dt, L):
    """saccade::MambaBlock v1 at the reference head's shapes (rank-1 C, no
    RMSNorm, residual), given TensorRT's workspace, enqueues the same bits as
    sacc_mamba_block_forward."""
    from oracle import mamba_oracle as mo
    from saccade_v1_b200.plugin import BLOCK, TENSOR_BF16
    tt = {"f16": torch.float16, "bf16": torch.bfloat16}[dt]
    act = TENSOR_HALF if dt == "f16" else TENSOR_BF16
    p = mo.random_block(31, 128, 256, 16, 16, 4, dt, norm=False, c_width=1)
    s = gu.stream()
    with torch.cuda.stream(s):
        w = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).cuda().to(
             tt if k in ("w_in", "w_x", "w_dt", "w_out") else torch.float32) for k, v in p.items()}
        x = (torch.randn(4, L, 128, device="cuda") * 0.5).to(tt)
        want = sb.mamba_block_forward(x, w, residual=True, stream=s)
        ins = [x, w["w_in"], w["conv_w"], w["conv_b"], w["w_x"], w["w_dt"], w["dt_bias"], w["A"], w["D"], w["w_out"]]
        descs = [TensorDesc.of(tuple(t.shape), TENSOR_FLOAT if t.dtype == torch.float32 else act) for t in ins]
        plug = ScanPlugin.create(*BLOCK, [("dt_rank", 16), ("residual", 1)])
        plug.bind()
        nbytes = plug.workspace_bytes(descs)
        ws = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
        out = torch.empty_like(x)
        plug.enqueue(descs, [TensorDesc.of(tuple(out.shape), act)], [t.data_ptr() for t in ins], [out.data_ptr()], s,
                     workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        with pytest.raises(PluginError, match="workspace"):
            plug.enqueue(descs, [TensorDesc.of(tuple(out.shape), act)], [t.data_ptr() for t in ins], [out.data_ptr()], s)
    s.synchronize()
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("dt,hw", [("f16", (12, 20)), ("bf16", (6, 10))])
def test_level_plugin_is_bitwise_the_level_api(dt, hw):
    """saccade::CrossScanMambaBlock v1 (a head level's expand -> block ->
    merge on the FP32 maps), given TensorRT's workspace, enqueues the same
    bits as sacc_cross_scan_block_forward."""
    from oracle import mamba_oracle as mo
    from saccade_v1_b200.plugin import LEVEL, TENSOR_BF16
    tt = {"f16": torch.float16, "bf16": torch.bfloat16}[dt]
    act = TENSOR_HALF if dt == "f16" else TENSOR_BF16
    p = mo.random_block(32, 128, 256, 16, 16, 4, dt, norm=False, c_width=1)
    s = gu.stream()
    with torch.cuda.stream(s):
        w = {k: torch.from_numpy(np.ascontiguousarray(v, np.float32)).cuda().to(
             tt if k in ("w_in", "w_x", "w_dt", "w_out") else torch.float32) for k, v in p.items()}
        x = torch.randn(1, 128, *hw, device="cuda") * 0.5
        want = sb.cross_scan_block_forward(x, w, dtype=tt, stream=s)
        ins = [x, w["w_in"], w["conv_w"], w["conv_b"], w["w_x"], w["w_dt"], w["dt_bias"], w["A"], w["D"], w["w_out"]]
        descs = [TensorDesc.of(tuple(t.shape), TENSOR_FLOAT if t.dtype == torch.float32 else act) for t in ins]
        plug = ScanPlugin.create(*LEVEL, [("dt_rank", 16), ("residual", 1)])
        plug.bind()
        ws = torch.empty(plug.workspace_bytes(descs) + 256, dtype=torch.uint8, device="cuda")
        out = torch.empty_like(x)
        plug.enqueue(descs, [TensorDesc.of(tuple(out.shape), TENSOR_FLOAT)], [t.data_ptr() for t in ins], [out.data_ptr()], s,
                     workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        with pytest.raises(PluginError, match="workspace"):
            plug.enqueue(descs, [TensorDesc.of(tuple(out.shape), TENSOR_FLOAT)], [t.data_ptr() for t in ins], [out.data_ptr()], s)
    s.synchronize()
    assert torch.equal(out.view(torch.int32), want.view(torch.int32))
