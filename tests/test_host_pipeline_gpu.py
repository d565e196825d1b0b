"""HostScanPipeline: pinned host batches streamed through the GPU in slices
(copies in both directions overlapping the scan) give the device path's
output bit for bit, ragged last slice included."""
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import saccade_v1_b200 as sb  # noqa: E402
from saccade_v1_b200.host_pipeline import HostScanPipeline  # noqa: E402


@pytest.mark.parametrize("layout,gate,batch,rows", [("BDL", False, 10, 4), ("BLD", True, 7, 3), ("BDL", True, 3, 8)])
def test_pipeline_equals_device_path(layout, gate, batch, rows):
    D, L, N = 256, 200, 16
    g = torch.Generator(device="cuda")
    g.manual_seed(5 + batch)
    bf = torch.bfloat16
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        shape_u = (batch, D, L) if layout == "BDL" else (batch, L, D)
        shape_b = (batch, 1, N, L) if layout == "BDL" else (batch, L, 1, N)
        u, dl = (torch.randn(shape_u, device="cuda", generator=g).to(bf) for _ in range(2))
        z = torch.randn(shape_u, device="cuda", generator=g).to(bf) if gate else None
        bm, cm = (torch.randn(shape_b, device="cuda", generator=g).to(bf) for _ in range(2))
        A = -(torch.rand(D, N, device="cuda", generator=g) * 3 + 0.1)
        Dv = torch.randn(D, device="cuda", generator=g)
        bias = torch.full((D,), -2.0, device="cuda")
        want = sb.selective_scan_ex(u, dl, A, bm, cm, D=Dv, z=z, delta_bias=bias, layout=layout, stream=s)
    s.synchronize()
    host = [x.cpu().pin_memory() if x is not None else None for x in (u, dl, bm, cm, z)]
    y_h = torch.zeros(shape_u, dtype=bf).pin_memory()
    pipe = HostScanPipeline(host[0], host[2], rows=rows, gate=gate)
    for _ in range(2):  # buffers reused across calls
        y_h.zero_()
        pipe.run(host[0], host[1], A, host[2], host[3], D=Dv, z=host[4], delta_bias=bias, y_h=y_h, layout=layout, stream=s)
        s.synchronize()
        assert torch.equal(y_h.view(torch.int16), want.cpu().view(torch.int16))


def test_pipeline_rejects_pageable_or_device_memory():
    u = torch.zeros(4, 128, 64, dtype=torch.bfloat16).pin_memory()
    b = torch.zeros(4, 1, 16, 64, dtype=torch.bfloat16).pin_memory()
    pipe = HostScanPipeline(u, b, rows=2)
    A = torch.zeros(128, 16, device="cuda")
    with pytest.raises(sb.ScanInvalidArgument, match="pinned"):
        pipe.run(u.clone(), u, A, b, b, y_h=u.clone())  # clone() is pageable
    with pytest.raises(sb.ScanInvalidArgument, match="pinned"):
        pipe.run(u.cuda(), u, A, b, b, y_h=u)
