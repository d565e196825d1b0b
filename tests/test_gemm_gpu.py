"""tcgen05 projection GEMM (sacc_gemm) against a torch FP32 reference of the same op.

C = A B^T (+ bias) (+ residual) with bf16/fp16 operands and FP32 accumulation:
the reference is (A.float() @ B.float().T + bias + residual) in FP32; the
tolerance covers the output rounding (2^-8 relative for bf16, 2^-11 for fp16)
plus FP32 summation-order differences (1e-5 relative to sum |a||b|).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import saccade_v1_b200 as sb  # noqa: E402


def check(c, ref, mag, out_dtype):
    rel = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 0.0}[out_dtype]
    tol = rel * ref.abs() + 1e-5 * mag + 1e-6
    err = (c.float() - ref).abs()
    bad = err > tol
    assert not bool(bad.any()), f"{int(bad.sum())} of {c.numel()} beyond tolerance, max err {float(err.max()):.3g}"


@pytest.mark.parametrize("shape", [(256, 512, 128), (200, 40, 256), (300, 1000, 520), (8192, 512, 128), (128, 64, 64),
                                   (1000, 256, 2048), (16384, 2048, 320), (5000, 700, 72), (20000, 1000, 512)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_matches_fp32_reference(shape, dt):
    m, n, k = shape
    g = torch.Generator(device="cuda")
    g.manual_seed(m * 7 + n * 3 + k)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = torch.randn(m, k, device="cuda", generator=g).to(dt)
        b = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(dt)
        c = sb.gemm(a, b, out_dtype=torch.float32, stream=s)
    s.synchronize()
    ref = a.float() @ b.float().T
    check(c, ref, a.float().abs() @ b.float().abs().T, torch.float32)
    assert sb.scan_fault() == 0


def test_gemm_bias_residual_and_16bit_out():
    m, n, k = 520, 384, 192
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
        b = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
        bias = torch.randn(n, device="cuda", generator=g)
        r = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
        c = sb.gemm(a, b, bias=bias, residual=r, stream=s)
    s.synchronize()
    ref = a.float() @ b.float().T + bias + r.float()
    check(c, ref, a.float().abs() @ b.float().abs().T + bias.abs() + r.float().abs(), torch.bfloat16)


def test_gemm_large_epilogue():
    """Large m, n, k (persistent tiles, many per CTA): row scale, bias, residual, 16-bit output, ragged m."""
    m, n, k = 16390, 2048, 256
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
        b = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).to(torch.bfloat16)
        bias = torch.randn(n, device="cuda", generator=g)
        r = torch.randn(m, n, device="cuda", generator=g).to(torch.bfloat16)
        rs = torch.rand(m, device="cuda", generator=g) + 0.5
        c = sb.gemm(a, b, bias=bias, residual=r, row_scale=rs, stream=s)
    s.synchronize()
    ref = (a.float() @ b.float().T) * rs[:, None] + bias + r.float()
    check(c, ref, (a.float().abs() @ b.float().abs().T) * rs[:, None] + bias.abs() + r.float().abs(), torch.bfloat16)
    assert sb.scan_fault() == 0


def test_gemm_strided_rows():
    """A as a column slice of a wider matrix (the x_proj dt slice feeding dt_proj)."""
    m, kfull, k, n = 333, 40, 16, 256
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        wide = torch.randn(m, kfull, device="cuda").to(torch.bfloat16)
        a = wide[:, :k]
        b = torch.randn(n, k, device="cuda").to(torch.bfloat16)
        c = sb.gemm(a, b, out_dtype=torch.float32, stream=s)
    s.synchronize()
    ref = a.float() @ b.float().T
    check(c, ref, a.float().abs() @ b.float().abs().T, torch.float32)


def test_gemm_rejections():
    a = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(8, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(sb.ScanInvalidArgument, match="multiples of 8"):
        sb.gemm(a, b, stream=torch.cuda.Stream())
    with pytest.raises(sb.ScanInvalidArgument, match="non-default stream"):
        sb.gemm(a[:, :8].contiguous(), b[:, :8].contiguous(), stream=0)
