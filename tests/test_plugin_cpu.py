"""The plugin surface on the CPU: creator field parsing, output types and
shapes, format support, workspace, serialization and the enqueue rejections
that happen before any GPU work (reference src/scan_trt_plugin.cpp and its
tests/scan_trt_tests.cpp contract group)."""
import pytest

from saccade_v1_b200.plugin import (EXPAND, FIELD_OTHER, FORMAT_LINEAR, FORMAT_OTHER, MERGE, SCAN, SCAN_F16, TENSOR_FLOAT,
                                    TENSOR_HALF, TENSOR_INT32, TENSOR_OTHER, PluginError, ScanPlugin, TensorDesc)


def test_creator_accepts_exactly_the_advertised_fields():
    p = ScanPlugin.create(*SCAN, [("has_d", 1)])
    assert p.fields() == {"has_d": 1}
    assert ScanPlugin.create(*SCAN, [("has_d", 0)]).fields() == {"has_d": 0}
    assert ScanPlugin.create(*MERGE, [("height", 20), ("width", 32)]).fields() == {"height": 20, "width": 32}
    assert ScanPlugin.create(*EXPAND, []).fields() == {}


@pytest.mark.parametrize("fields,msg", [
    ([], "missing field has_d"),
    ([("has_d", 1), ("has_d", 0)], "duplicate field has_d"),
    ([("has_d", 1), ("height", 3)], "unknown field height"),
    ([("has_d", 2)], "has_d must be 0 or 1"),
    ([("has_d", None, 1, 1)], "field has_d must hold one INT32"),
    ([("has_d", 1, FIELD_OTHER, 1)], "field has_d must hold one INT32"),
    ([("has_d", 1, 1, 2)], "field has_d must hold one INT32"),
    ([(None, 1, 1, 1)], "unknown field (null)"),
])
def test_creator_rejections(fields, msg):
    with pytest.raises(PluginError, match=msg.replace("(", r"\(").replace(")", r"\)")) as e:
        ScanPlugin.create(*SCAN, fields)
    assert str(e.value).startswith("saccade::SelectiveScan creator: ")


def test_merge_creator_rejections_and_unknown_plugin():
    with pytest.raises(PluginError, match="height and width must be positive"):
        ScanPlugin.create(*MERGE, [("height", 0), ("width", 4)])
    with pytest.raises(PluginError, match="plugin creator not registered: saccade::SelectiveScan v4"):
        ScanPlugin.create("SelectiveScan", "4", [("has_d", 1)])


def test_output_types_and_shapes():
    p = ScanPlugin.create(*SCAN, [("has_d", 1)])
    assert p.output_types([TENSOR_FLOAT] * 6) == [TENSOR_FLOAT, TENSOR_INT32]
    with pytest.raises(PluginError, match="input 2 is not FP32"):
        p.output_types([TENSOR_FLOAT, TENSOR_FLOAT, TENSOR_INT32, TENSOR_FLOAT, TENSOR_FLOAT, TENSOR_FLOAT])
    dims = [(4, 960, 256), (4, 960, 256), (1, 16), (4, 960, 16), (4, 960, 1), (256,)]
    assert p.output_shapes(dims) == [(4, 960, 256), (2,)]
    with pytest.raises(PluginError, match="input dimensions disagree"):
        p.output_shapes([(4, 960, 256), (4, 961, 256), (1, 16), (4, 960, 16), (4, 960, 1), (256,)])
    with pytest.raises(PluginError, match="state must be a power of two"):
        p.output_shapes([(4, 9, 8), (4, 9, 8), (1, 3), (4, 9, 3), (4, 9, 1), (8,)])
    with pytest.raises(PluginError, match="A rows must be 1 or channels"):
        p.output_shapes([(4, 9, 8), (4, 9, 8), (2, 4), (4, 9, 4), (4, 9, 1), (8,)])
    with pytest.raises(PluginError, match="C width must be 1 or state"):
        p.output_shapes([(4, 9, 8), (4, 9, 8), (1, 4), (4, 9, 4), (4, 9, 2), (8,)])
    e = ScanPlugin.create(*EXPAND, [])
    assert e.output_shapes([(1, 128, 20, 32)]) == [(4, 640, 128), (2,)]
    m = ScanPlugin.create(*MERGE, [("height", 20), ("width", 32)])
    assert m.output_shapes([(4, 640, 128)]) == [(1, 128, 20, 32), (2,)]
    with pytest.raises(PluginError, match="y length differs from height"):
        m.output_shapes([(4, 641, 128)])


def test_formats_and_workspace():
    p = ScanPlugin.create(*SCAN, [("has_d", 0)])
    io = [TensorDesc.of((1,)) for _ in range(5)] + [TensorDesc.of((1,)), TensorDesc.of((2,), TENSOR_INT32)]
    assert all(p.supports_format(i, io, 5) for i in range(7))
    io[6] = TensorDesc.of((2,), TENSOR_FLOAT)
    assert not p.supports_format(6, io, 5)
    io[0] = TensorDesc.of((1,), TENSOR_FLOAT, FORMAT_OTHER)
    assert not p.supports_format(0, io, 5)
    io[1] = TensorDesc.of((1,), TENSOR_OTHER)
    assert not p.supports_format(1, io, 5)
    assert p.workspace_size() == 0


def test_enqueue_rejects_before_any_gpu_work():
    p = ScanPlugin.create(*SCAN, [("has_d", 1)])
    descs = [TensorDesc.of(d) for d in [(4, 9, 8), (4, 9, 8), (1, 4), (4, 9, 4), (4, 9, 1), (8,)]]
    outs = [TensorDesc.of((4, 9, 8)), TensorDesc.of((2,), TENSOR_INT32, FORMAT_LINEAR)]
    ptrs = [0x1000 * (i + 1) for i in range(6)]
    with pytest.raises(PluginError, match="an explicit non-default stream is required"):
        p.enqueue(descs, outs, ptrs, [0x9000, 0xA000], 0)
    with pytest.raises(PluginError, match="kernels are not loaded for any CUDA context"):
        p.enqueue(descs, outs, ptrs, [0x9000, 0xA000], 0x5EED)
    q = p.clone()
    assert q.fields() == {"has_d": 1}


H, F, I = TENSOR_HALF, TENSOR_FLOAT, TENSOR_INT32


@pytest.mark.parametrize("has_d", [0, 1])
def test_fp16_version_types_and_formats(has_d):
    """SelectiveScan v3: the same creator fields and shape rules as v2, FP16 u,
    delta, B, C and y, FP32 A and D, INT32 status."""
    p = ScanPlugin.create(*SCAN_F16, [("has_d", has_d)])
    assert p.fields() == {"has_d": has_d}
    ins = [H, H, F, H, H] + [F] * has_d
    assert p.output_types(ins) == [H, I]
    with pytest.raises(PluginError, match="input 0 is not FP16"):
        p.output_types([F] + ins[1:])
    with pytest.raises(PluginError, match="input 2 is not FP32"):
        p.output_types(ins[:2] + [H] + ins[3:])
    n = len(ins)
    io = [TensorDesc.of((1,), t) for t in ins] + [TensorDesc.of((1,), H), TensorDesc.of((2,), I)]
    assert all(p.supports_format(i, io, n) for i in range(n + 2))
    for pos, wrong in [(0, F), (2, H), (n, F), (n + 1, H)] + ([(5, H)] if has_d else []):
        bad = list(io)
        bad[pos] = TensorDesc.of((1,), wrong)
        assert not p.supports_format(pos, bad, n), pos
    dims = [(4, 240, 256), (4, 240, 256), (1, 16), (4, 240, 16), (4, 240, 1)] + [(256,)] * has_d
    assert p.output_shapes(dims) == [(4, 240, 256), (2,)]
    assert p.workspace_size() == 0


def test_fp16_version_enqueue_rejects_fp32_descriptors():
    p = ScanPlugin.create(*SCAN_F16, [("has_d", 1)])
    dims = [(4, 9, 8), (4, 9, 8), (1, 4), (4, 9, 4), (4, 9, 1), (8,)]
    descs = [TensorDesc.of(d) for d in dims]
    outs = [TensorDesc.of((4, 9, 8), H), TensorDesc.of((2,), I)]
    with pytest.raises(PluginError, match="kernels are not loaded|input 0 is not linear FP16|explicit non-default stream"):
        p.enqueue(descs, outs, [0x1000] * 6, [0x2000, 0x3000], 0x5EED)


# ---------------------------------------------------------------- MambaBlock plugin

from saccade_v1_b200.plugin import BLOCK, TENSOR_BF16  # noqa: E402

HEAD = [(4, 240, 128), (512, 128), (256, 4), (256,), (33, 256), (256, 16), (256,), (256, 16), (256,), (128, 256)]
FP32_IN = {2, 3, 6, 7, 8}


def head_types(act=TENSOR_HALF):
    return [TENSOR_FLOAT if i in FP32_IN else act for i in range(10)]


def test_block_creator_fields_and_rejections():
    p = ScanPlugin.create(*BLOCK, [("dt_rank", 16), ("residual", 1)])
    assert p.block_fields() == {"dt_rank": 16, "residual": 1}
    for fields, msg in (([("dt_rank", 16)], "missing field residual"), ([("dt_rank", 0), ("residual", 1)], "dt_rank must be positive"),
                        ([("dt_rank", 8), ("residual", 2)], "residual must be 0 or 1"),
                        ([("dt_rank", 8), ("residual", 1), ("has_d", 1)], "unknown field has_d")):
        with pytest.raises(PluginError, match=msg) as e:
            ScanPlugin.create(*BLOCK, fields)
        assert str(e.value).startswith("saccade::MambaBlock creator: ")


@pytest.mark.parametrize("act", [TENSOR_HALF, TENSOR_BF16])
def test_block_types_shapes_formats(act):
    p = ScanPlugin.create(*BLOCK, [("dt_rank", 16), ("residual", 1)])
    types = head_types(act)
    assert p.output_types(types, nb_out=1) == [act]
    with pytest.raises(PluginError, match="input 2 is not FP32"):
        p.output_types(types[:2] + [act] + types[3:], nb_out=1)
    with pytest.raises(PluginError, match="input 4 differs in type from x"):
        p.output_types(types[:4] + [TENSOR_FLOAT] + types[5:], nb_out=1)
    assert p.output_shapes(HEAD, nb_out=1, in_types=types) == [(4, 240, 128)]
    bad = list(HEAD)
    bad[4] = (40, 256)  # neither rank-1 (16 + 16 + 1) nor full (16 + 32) C
    with pytest.raises(PluginError, match="w_x"):
        p.output_shapes(bad, nb_out=1, in_types=types)
    io = [TensorDesc.of((1,), t) for t in types] + [TensorDesc.of((1,), act)]
    assert all(p.supports_format(i, io, 10) for i in range(11))
    wrong = list(io)
    wrong[10] = TensorDesc.of((1,), TENSOR_FLOAT)
    assert not p.supports_format(10, wrong, 10)
    wrong = list(io)
    wrong[7] = TensorDesc.of((1,), act)
    assert not p.supports_format(7, wrong, 10)


def test_block_workspace_needs_shapes():
    p = ScanPlugin.create(*BLOCK, [("dt_rank", 16), ("residual", 1)])
    assert p.workspace_size() == 0  # the shape-free query stays the scan plugins' 0
    descs = [TensorDesc.of(d, t) for d, t in zip(HEAD, head_types())]
    assert p.workspace_bytes(descs) > 4 * 240 * 256 * 2 * 4  # xz, u, y, ... of 960 tokens
    scan = ScanPlugin.create(*SCAN, [("has_d", 1)])
    assert scan.workspace_bytes([TensorDesc.of(d) for d in [(4, 9, 8), (4, 9, 8), (1, 4), (4, 9, 4), (4, 9, 1), (8,)]]) == 0


# ---------------------------------------------------------------- CrossScanMambaBlock plugin

from saccade_v1_b200.plugin import LEVEL  # noqa: E402

LEVEL_HEAD = [(1, 128, 12, 20)] + HEAD[1:]


def level_types(act=TENSOR_HALF):
    return [TENSOR_FLOAT] + head_types(act)[1:]


def test_level_creator_fields_and_rejections():
    p = ScanPlugin.create(*LEVEL, [("dt_rank", 16), ("residual", 1)])
    assert p.block_fields() == {"dt_rank": 16, "residual": 1}
    with pytest.raises(PluginError, match="missing field residual") as e:
        ScanPlugin.create(*LEVEL, [("dt_rank", 16)])
    assert str(e.value).startswith("saccade::CrossScanMambaBlock creator: ")


@pytest.mark.parametrize("act", [TENSOR_HALF, TENSOR_BF16])
def test_level_types_shapes_formats(act):
    """x and the output are the FP32 maps; w_in sets the activation type."""
    p = ScanPlugin.create(*LEVEL, [("dt_rank", 16), ("residual", 1)])
    types = level_types(act)
    assert p.output_types(types, nb_out=1) == [TENSOR_FLOAT]
    with pytest.raises(PluginError, match="input 0 is not FP32"):
        p.output_types([act] + types[1:], nb_out=1)
    with pytest.raises(PluginError, match="input 9 differs in type from w_in"):
        p.output_types(types[:9] + [TENSOR_FLOAT], nb_out=1)
    assert p.output_shapes(LEVEL_HEAD, nb_out=1, in_types=types) == [(1, 128, 12, 20)]
    with pytest.raises(PluginError, match=r"x must be \(batch, d_model, height, width\)"):
        p.output_shapes([(1, 240, 128)] + HEAD[1:], nb_out=1, in_types=types)
    bad = list(LEVEL_HEAD)
    bad[9] = (128, 128)  # w_out not (d_model, d_inner)
    with pytest.raises(PluginError, match="w_out"):
        p.output_shapes(bad, nb_out=1, in_types=types)
    io = [TensorDesc.of((1,), t) for t in types] + [TensorDesc.of((1,), TENSOR_FLOAT)]
    assert all(p.supports_format(i, io, 10) for i in range(11))
    for pos, t in ((0, act), (10, act), (4, TENSOR_FLOAT)):
        wrong = list(io)
        wrong[pos] = TensorDesc.of((1,), t)
        assert not p.supports_format(pos, wrong, 10)


def test_level_workspace_needs_shapes():
    p = ScanPlugin.create(*LEVEL, [("dt_rank", 16), ("residual", 1)])
    assert p.workspace_size() == 0
    descs = [TensorDesc.of(d, t) for d, t in zip(LEVEL_HEAD, level_types())]
    assert p.workspace_bytes(descs) > 4 * 240 * 256 * 2 * 3  # u, z, y of the four directions' 960 tokens
