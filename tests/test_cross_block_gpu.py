"""GPU parity of one Cross-Scan head level with the expand and merge fused into
the Mamba block (sacc_cross_scan_block_forward).

Checked against the binary64 oracle in the reference's order (expand, block
with the residual on the tokens, merge: oracle/mamba_oracle.py
cross_block_forward), and against the unfused composition of this library's
own calls (expand kernel, block, merge kernel).  The fused level runs in_proj
once per map position and the merge before out_proj (out_proj is linear), so
it agrees to rounding: |gpu - ref| <= 1e-3 + 1e-2 |ref|, the block's
tolerance for 16-bit activations against an FP32-or-better reference.
"""
import numpy as np
import pytest
import torch

from oracle import mamba_oracle as mo

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import gpu_util as gu  # noqa: E402
import saccade_v1_b200 as sb  # noqa: E402

TORCH = {"bf16": torch.bfloat16, "f16": torch.float16}


def to_dev(p, dt):
    out = {}
    for k, v in p.items():
        if k in ("w_in", "w_x", "w_dt", "w_out"):
            out[k] = torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device="cuda", dtype=TORCH[dt])
        else:
            out[k] = torch.from_numpy(np.ascontiguousarray(v, np.float32)).cuda()
    return out


def hr_params(seed, dt, norm=False, dt_rank=16):
    """The reference head's block: d_model 128, D 256, N 16, x_proj 256 -> dt_rank + 16 + 1 (rank-1 C)."""
    return mo.random_block(seed, 128, 256, 16, dt_rank, 4, dt, norm=norm, c_width=1)


def run_level(x_np, p, dt, residual=True):
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x = torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).cuda()
        out = sb.cross_scan_block_forward(x, to_dev(p, dt), residual=residual, dtype=TORCH[dt], stream=s)
    s.synchronize()
    return out.cpu().numpy()


def check(name, got, ref):
    err = np.abs(got.astype(np.float64) - ref)
    bad = ~(err <= 1e-3 + 1e-2 * np.abs(ref))
    assert not bad.any(), f"{name}: {int(bad.sum())}/{got.size} beyond 1e-3 + 1e-2|ref|, max err {err.max():.3g}"


def maps(seed, batch, h, w, c=128):
    return (np.random.default_rng(seed).standard_normal((batch, c, h, w)) * 0.5).astype(np.float32)


@pytest.mark.parametrize("h,w", [(6, 10), (12, 20), (24, 40)])
def test_hr_levels_match_oracle(h, w):
    """The three HR deploy levels (L = 60, 240, 960), one image, bf16."""
    p = hr_params(20 + h, "bf16")
    x = maps(h, 1, h, w)
    check(f"hr_{h}x{w}", run_level(x, p, "bf16"), mo.cross_block_forward(x, p, "bf16"))
    assert sb.scan_fault() == 0


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_two_images_odd_map_norm_and_no_residual(dt):
    """Two images, a 5 x 7 map (L = 35, odd rows for the output's FP32 stores),
    the RMSNorm fold, dt_rank 8, and the level without its residual."""
    p = hr_params(31, dt, norm=True, dt_rank=8)
    x = maps(7, 2, 5, 7)
    check(f"odd_{dt}", run_level(x, p, dt), mo.cross_block_forward(x, p, dt))
    check(f"odd_{dt}_nores", run_level(x, p, dt, residual=False), mo.cross_block_forward(x, p, dt, residual=False))


def test_full_width_c_and_wide_rank():
    """A full-width C and dt_rank 64 (delta through its own GEMM) on a 16 x 16 map."""
    p = mo.random_block(41, 128, 256, 16, 64, 4, "bf16", norm=False)
    x = maps(8, 1, 16, 16)
    check("full_c", run_level(x, p, "bf16"), mo.cross_block_forward(x, p, "bf16"))


def test_equals_unfused_composition():
    """expand kernel -> block on the bf16 tokens (no residual) -> + FP32 tokens
    -> merge kernel, all through this library, against the fused level."""
    h, w = 12, 20
    p = hr_params(51, "bf16")
    x_np = maps(9, 1, h, w)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x = torch.from_numpy(x_np).cuda()
        dev = to_dev(p, "bf16")
        fused = sb.cross_scan_block_forward(x, dev, stream=s)
        shape = sb.CrossScanShape(1, 128, h, w)
        tokens = torch.empty(4, h * w, 128, device="cuda")
        st = [gu.new_status() for _ in range(2)]
        sb.cross_scan_expand_cuda(shape, x, tokens, st[0], stream=s)
        r = sb.mamba_block_forward(tokens.to(torch.bfloat16), dev, residual=False, stream=s).float() + tokens
        unfused = torch.empty(1, 128, h, w, device="cuda")
        sb.cross_scan_merge_cuda(shape, r.contiguous(), unfused, st[1], stream=s)
    s.synchronize()
    assert [gu.status_words(t) for t in st] == [(0, sb.SCAN_DONE)] * 2
    check("fused_vs_unfused", fused.cpu().numpy(), unfused.cpu().numpy().astype(np.float64))


def test_workspace_reused_and_deterministic():
    p = hr_params(61, "bf16")
    x = torch.from_numpy(maps(10, 1, 6, 10)).cuda()
    dev = to_dev(p, "bf16")
    ws = torch.empty(sb.cross_scan_block_workspace(x, dev) + 256, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    outs = []
    for _ in range(2):
        ws.fill_(0xA5)
        with torch.cuda.stream(s):
            outs.append(sb.cross_scan_block_forward(x, dev, workspace=ws, stream=s))
        s.synchronize()
    assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32))


def test_rejections():
    p = to_dev(hr_params(71, "bf16"), "bf16")
    s = torch.cuda.Stream()
    x = torch.zeros(1, 128, 6, 10, device="cuda")
    with pytest.raises(sb.ScanInvalidArgument, match="float32"):
        sb.cross_scan_block_forward(x.half(), p, stream=s)
    with pytest.raises(sb.ScanInvalidArgument, match="overlaps"):
        sb.cross_scan_block_forward(x, p, out=x, stream=s)
    with pytest.raises(sb.ScanInvalidArgument, match="stream"):
        sb.cross_scan_block_forward(x, p, stream=torch.cuda.default_stream())
    bad = dict(p)
    bad["w_in"] = p["w_in"][:, :64].contiguous()  # d_model 64: not a multiple of 128
    with pytest.raises(sb.ScanInvalidArgument):
        sb.cross_scan_block_forward(torch.zeros(1, 64, 6, 10, device="cuda"), bad, stream=s)
