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
