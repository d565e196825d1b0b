"""GPU parity of the fused Mamba block forward (sacc_mamba_block_forward).

The device pipeline (RMSNorm folded into the tcgen05 in_proj, conv1d + SiLU,
tcgen05 x_proj / dt_proj, bulk scan with D skip and SiLU(z) gate, tcgen05
out_proj with the residual) is compared with the binary64 block oracle
(oracle/mamba_oracle.py), which rounds to the activation dtype where the
device stores activations.  Tolerance (BASELINE, 16-bit activations against
an FP32-or-better reference): |gpu - ref| <= 1e-3 + 1e-2 |ref|.
"""
import numpy as np
import pytest
import torch

from oracle import mamba_oracle as mo

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

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


def run_block(x_np, p, dt, residual=True):
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        x = torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).to(device="cuda", dtype=TORCH[dt])
        y = sb.mamba_block_forward(x, to_dev(p, dt), residual=residual, stream=s)
    s.synchronize()
    return y.float().cpu().numpy()


def check(name, got, ref):
    err = np.abs(got.astype(np.float64) - ref)
    bad = ~(err <= 1e-3 + 1e-2 * np.abs(ref))
    assert not bad.any(), f"{name}: {int(bad.sum())}/{got.size} beyond 1e-3 + 1e-2|ref|, max err {err.max():.3g}"


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("norm", [True, False])
def test_block_matches_oracle_small(dt, norm):
    B, L, dm, D, N, R = 4, 32, 128, 256, 16, 8
    p = mo.random_block(10, dm, D, N, R, 4, dt, norm=norm)
    x = mo.rnd(np.random.default_rng(2).standard_normal((B, L, dm)) * 0.1, dt)
    got = run_block(x, p, dt)
    check(f"block_{dt}_{norm}", got, mo.block_forward(x, p, dt))
    assert sb.scan_fault() == 0


def test_block_without_residual_and_wide_dt_rank():
    B, L, dm, D, N, R = 2, 40, 256, 384, 16, 64
    p = mo.random_block(11, dm, D, N, R, 4, "bf16")
    x = mo.rnd(np.random.default_rng(3).standard_normal((B, L, dm)) * 0.1, "bf16")
    check("block_wide", run_block(x, p, "bf16", residual=False), mo.block_forward(x, p, "bf16", residual=False))


def test_config1_full_size_sampled_tracks():
    """256 tracks x 32 frames, d_model 128, D 256, N 16, dt_rank 8, fp16."""
    B, L, dm, D, N, R = 256, 32, 128, 256, 16, 8
    p = mo.random_block(12, dm, D, N, R, 4, "f16")
    x = mo.rnd(np.random.default_rng(4).standard_normal((B, L, dm)) * 0.1, "f16")
    got = run_block(x, p, "f16")
    pick = np.random.default_rng(5).integers(0, B, 12)
    check("config1_tracks", got[pick], mo.block_forward(x[pick], p, "f16"))


def test_block_rejections():
    x = torch.zeros(2, 8, 128, dtype=torch.float16, device="cuda")
    p = to_dev(mo.random_block(1, 128, 256, 16, 8, 4, "f16"), "f16")
    with pytest.raises(sb.ScanInvalidArgument, match="non-default stream"):
        sb.mamba_block_forward(x, p, stream=0)
    bad = dict(p, conv_w=torch.zeros(256, 3, device="cuda"))
    with pytest.raises(sb.ScanInvalidArgument, match="d_conv must be 4"):
        sb.mamba_block_forward(x, bad, stream=torch.cuda.Stream())


def test_config4_layer_sampled_tracks():
    """BASELINE config 4 layer shape (L 4096, d_model 1024, D 2048, N 16, dt_rank 64, bf16) on 8 tracks; two
    tracks against the oracle."""
    B, L, dm, D, N, R = 8, 4096, 1024, 2048, 16, 64
    p = mo.random_block(13, dm, D, N, R, 4, "bf16")
    x = mo.rnd(np.random.default_rng(6).standard_normal((B, L, dm)) * 0.1, "bf16")
    got = run_block(x, p, "bf16")
    pick = [1, 6]
    check("config4_tracks", got[pick], mo.block_forward(x[pick], p, "bf16"))
    assert sb.scan_fault() == 0


@pytest.mark.parametrize("L", [240, 64])
def test_block_rank1_c_reference_head_shapes(L):
    """The reference head's Mamba block (src/head_trt_network.cpp:192-230): 4 Cross-Scan directions x L tokens,
    d_model 128, d_inner 256, N 16, dt_rank 16, x_proj 256 -> 16 + 16 + 1 (one C per token), A shared by all
    channels (A_log of shape (1, 16)), no RMSNorm, residual; fp16 activations."""
    B, dm, D, N, R = 4, 128, 256, 16, 16
    p = mo.random_block(14, dm, D, N, R, 4, "f16", norm=False, c_width=1)
    p["A"] = np.tile(-np.exp(np.random.default_rng(15).uniform(-1, 1.5, (1, N))).astype(np.float32), (D, 1))
    x = mo.rnd(np.random.default_rng(16).standard_normal((B, L, dm)) * 0.5, "f16")
    check(f"head_rank1_L{L}", run_block(x, p, "f16"), mo.block_forward(x, p, "f16"))
    assert sb.scan_fault() == 0


def test_block_rejects_other_c_widths():
    p = to_dev(mo.random_block(1, 128, 256, 16, 8, 4, "f16", c_width=2), "f16")
    x = torch.zeros(2, 8, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(sb.ScanInvalidArgument, match="c_width must be 1 or d_state"):
        sb.mamba_block_forward(x, p, stream=torch.cuda.Stream())


@pytest.mark.parametrize("L", [6, 37, 60])
def test_block_lengths_not_multiple_of_8(L):
    B, dm, D, N, R = 3, 128, 256, 16, 8
    p = mo.random_block(17, dm, D, N, R, 4, "bf16")
    x = mo.rnd(np.random.default_rng(18).standard_normal((B, L, dm)) * 0.1, "bf16")
    check(f"block_L{L}", run_block(x, p, "bf16"), mo.block_forward(x, p, "bf16"))
    assert sb.scan_fault() == 0


def test_block_on_a_stream_that_is_not_current():
    """The wrapper's own workspace is taken for the launch stream, so a call on
    a stream other than the current one gives the same bits."""
    B, L, dm, D, N, R = 4, 32, 128, 256, 16, 8
    p = mo.random_block(13, dm, D, N, R, 4, "bf16", norm=False)
    x_np = mo.rnd(np.random.default_rng(6).standard_normal((B, L, dm)) * 0.1, "bf16")
    want = run_block(x_np, p, "bf16")
    s = torch.cuda.Stream()
    x = torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).to(device="cuda", dtype=torch.bfloat16)
    dev = to_dev(p, "bf16")
    torch.cuda.synchronize()
    out = torch.empty_like(x)
    y = sb.mamba_block_forward(x, dev, out=out, stream=s)  # the current stream stays the default one
    s.synchronize()
    assert np.array_equal(y.float().cpu().numpy(), want)


def test_fused_scan_graph_replay_new_inputs():
    """The reference head's block at the HR L = 960 level scans 8 units of 960 tokens, which takes the fused
    chunk-parallel launch (one cooperative launch whose parts hand their records over through flags in the
    workspace).  A CUDA graph captured once and replayed with new inputs in the same buffers must give the
    same bits as eager calls on those inputs: every replay reuses the captured launch's flag value, so the
    flags of the previous replay must not be taken for this one's."""
    B, L, dm, D, N, R = 4, 960, 128, 256, 16, 16
    p = mo.random_block(19, dm, D, N, R, 4, "f16", norm=False, c_width=1)
    dev = to_dev(p, "f16")
    rng = np.random.default_rng(20)
    xs = [torch.from_numpy(mo.rnd(rng.standard_normal((B, L, dm)) * 0.5, "f16").astype(np.float32)).to("cuda", torch.float16)
          for _ in range(3)]
    s = torch.cuda.Stream()
    x_static = xs[0].clone()
    out_static = torch.empty_like(x_static)
    ws = torch.empty(sb.mamba_block_workspace(x_static, dev) + 256, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        refs = [sb.mamba_block_forward(x, dev, stream=s) for x in xs]
        sb.mamba_block_forward(x_static, dev, out=out_static, workspace=ws, stream=s)  # warm-up before capture
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        sb.mamba_block_forward(x_static, dev, out=out_static, workspace=ws, stream=s)
    for i in (1, 2, 0, 2):
        x_static.copy_(xs[i])
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_static, refs[i]), f"replay with input {i} differs from the eager call"
    # The replayed output is also the block's result: direction 0 against the binary64 block oracle.
    check("hr_l960_graph", out_static.float().cpu().numpy()[:1], mo.block_forward(xs[2].float().cpu().numpy()[:1], p, "f16"))
    assert sb.scan_fault() == 0
