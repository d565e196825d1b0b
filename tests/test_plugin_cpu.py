"""The plugin surface on the CPU: creator field parsing, output types and
shapes, format support, workspace, serialization and the enqueue rejections
that happen before any GPU work (reference src/scan_trt_plugin.cpp and its
tests/scan_trt_tests.cpp contract group)."""
import pytest

from saccade_v1_b200.plugin import (EXPAND, FIELD_OTHER, FORMAT_LINEAR, FORMAT_OTHER, MERGE, SCAN, TENSOR_FLOAT, TENSOR_INT32,
                                    TENSOR_OTHER, PluginError, ScanPlugin, TensorDesc)


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
    with pytest.raises(PluginError, match="plugin creator not registered: saccade::SelectiveScan v3"):
        ScanPlugin.create("SelectiveScan", "3", [("has_d", 1)])


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
