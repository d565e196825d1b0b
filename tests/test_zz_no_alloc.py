"""sacc_mamba_block_forward_noalloc (the block forward whose scratch is the
library's static device array) against sacc_mamba_block_forward (caller
workspace): two calls in a row on one stream, with different inputs, must each
match the workspace entry point within the block tests' tolerance
|a - b| <= 1e-3 + 1e-2 |b|; the second call reuses the scratch the first one
left behind.  Blocks that need more scratch than the static maximum are
rejected before any GPU work.  This file sorts last so that it also runs
after every other GPU test in one process."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

import saccade_v1_b200 as sb  # noqa: E402
from saccade_v1_b200 import _lib  # noqa: E402
from saccade_v1_b200.scan import _block_args  # noqa: E402

SCRATCH_MAX = 24 << 20  # SACC_NOALLOC_SCRATCH_BYTES


def weights(seed, dm, D, N, R, dt):
    r = np.random.default_rng(seed)
    u = lambda shape, fan: torch.from_numpy((r.uniform(-1, 1, shape) / np.sqrt(fan)).astype(np.float32)).cuda()
    p = {"w_in": u((2 * D, dm), dm).to(dt), "conv_w": u((D, 4), 4), "conv_b": u((D,), 4), "w_x": u((R + 2 * N, D), D).to(dt),
         "w_dt": u((D, R), R).to(dt), "w_out": u((dm, D), D).to(dt),
         "dt_bias": torch.from_numpy(np.log(np.expm1(np.exp(r.uniform(np.log(1e-3), np.log(1e-1), D)))).astype(np.float32)).cuda(),
         "A": -torch.arange(1, N + 1, dtype=torch.float32, device="cuda").repeat(D, 1),
         "D": torch.ones(D, device="cuda"),
         "norm_w": torch.from_numpy((1 + 0.1 * r.standard_normal(dm)).astype(np.float32)).cuda()}
    return p


def noalloc_call(x, p, out, stream):
    """Direct C-ABI call of sacc_mamba_block_forward_noalloc."""
    args = _block_args(x, p, 1e-5, True, out)
    rc = _lib.load().sacc_mamba_block_forward_noalloc(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream))
    assert rc == _lib.SACC_OK, _lib.last_error()


def close(a, b):
    a, b = a.float(), b.float()
    bad = ~((a - b).abs() <= 1e-3 + 1e-2 * b.abs())
    assert not bool(bad.any()), f"{int(bad.sum())}/{a.numel()} beyond 1e-3 + 1e-2|ref|"


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_noalloc_block_matches_workspace_entry_two_calls(dt):
    # 256 tracks x 32 frames, d_model 128, d_inner 256, N 16, dt_rank 8.
    B, L, dm, D, N, R = 256, 32, 128, 256, 16, 8
    p = weights(21, dm, D, N, R, dt)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.Generator(device="cuda")
        g.manual_seed(31)
        xs = [(torch.randn(B, L, dm, device="cuda", generator=g) * 0.1).to(dt) for _ in range(2)]
        assert sb.mamba_block_workspace(xs[0], p) <= SCRATCH_MAX
        got = [torch.empty_like(x) for x in xs]
        for x, y in zip(xs, got):  # two calls in a row, same scratch
            noalloc_call(x, p, y, s)
        ref = [sb.mamba_block_forward(x, p, stream=s) for x in xs]
    s.synchronize()
    for a, b in zip(got, ref):
        assert bool(torch.isfinite(a.float()).all())
        close(a, b)
    assert sb.scan_fault() == 0


def test_noalloc_rejects_blocks_beyond_the_static_scratch():
    B, L, dm, D, N, R = 512, 32, 128, 256, 16, 8
    p = weights(22, dm, D, N, R, torch.float16)
    x = torch.zeros(B, L, dm, dtype=torch.float16, device="cuda")
    assert sb.mamba_block_workspace(x, p) > SCRATCH_MAX
    y = torch.full_like(x, 7.0)
    s = torch.cuda.Stream()
    with pytest.raises(sb.ScanInvalidArgument, match=r"mamba_block_noalloc: needs \d+ bytes of scratch, more than the static maximum of 25165824"):
        sb.mamba_block_forward_noalloc(x, p, out=y, stream=s)
    s.synchronize()
    assert bool((y == 7.0).all())


def test_noalloc_fused_scan_path_two_inputs_and_graph_replay():
    """The reference head's block at its HR L = 960 level (4 directions x 960 tokens, d_inner 256, dt_rank 16,
    one C per token, fp16): few units over long sequences, so the scan runs as the fused chunk-parallel
    launch whose part records and hand-off flags live in the static scratch.  Two calls with different
    inputs, then a CUDA graph of the no-alloc call replayed with a third input, each against
    sacc_mamba_block_forward on the same input."""
    B, L, dm, D, N, R = 4, 960, 128, 256, 16, 16
    p = weights(23, dm, D, N, R, torch.float16)
    p.pop("norm_w")
    p["w_x"] = p["w_x"][: R + N + 1].contiguous()  # x_proj 256 -> 16 + 16 + 1: one C per token
    s = torch.cuda.Stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(41)
    with torch.cuda.stream(s):
        xs = [(torch.randn(B, L, dm, device="cuda", generator=g) * 0.5).to(torch.float16) for _ in range(3)]
        assert sb.mamba_block_workspace(xs[0], p) <= SCRATCH_MAX
        ref = [sb.mamba_block_forward(x, p, stream=s) for x in xs]
        got = [torch.empty_like(x) for x in xs[:2]]
        for x, y in zip(xs[:2], got):
            noalloc_call(x, p, y, s)
    s.synchronize()
    for a, b in zip(got, ref[:2]):
        assert bool(torch.isfinite(a.float()).all())
        close(a, b)
    x_static, y_static = xs[0].clone(), torch.empty_like(xs[0])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        noalloc_call(x_static, p, y_static, s)
    for i in (2, 1):
        x_static.copy_(xs[i])
        graph.replay()
        torch.cuda.synchronize()
        close(y_static, ref[i])
    assert sb.scan_fault() == 0
