"""The batch-sharded C-ABI path (include/sacc_shard.h) on the GPUs of this process.

One host process drives n devices (the largest of 1, 2, 4, 8 that the machine
has): the batch of a BASELINE config-2-shaped scan (bf16, (B, D, L)) is split
with sacc_shard_rows, every device scans its rows (no collective on the scan
path), and one NCCL all-gather assembles y on every device.  Each device's
gathered output must equal the unsharded call's bits (the kernels are
deterministic per row and the shards run in the same launch mode).  A shard
rejected on the host leaves every device untouched.  NCCL's NVLS is switched
off for these runs.
"""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

import saccade_v1_b200 as sb  # noqa: E402
from saccade_v1_b200 import _lib  # noqa: E402

B, D, L, N = 16, 1536, 512, 16


def ndev():
    have = torch.cuda.device_count()
    return max(n for n in (1, 2, 4, 8) if n <= have)


def ex_args(u, dl, A, bm, cm, Dv, bias, y):
    a = _lib.ScanExArgs()
    a.batch, a.length, a.channels, a.state, a.groups, a.a_rows, a.c_width = u.shape[0], L, D, N, 1, D, N
    a.layout, a.dtype, a.delta_softplus, a.nseq = _lib.LAYOUT_BDL, _lib.DTYPE_BF16, 1, 0
    a.u, a.delta, a.b, a.c, a.z = u.data_ptr(), dl.data_ptr(), bm.data_ptr(), cm.data_ptr(), None
    a.a, a.d, a.delta_bias = A.data_ptr(), Dv.data_ptr(), bias.data_ptr()
    a.h0 = a.h_final = a.cu_seqlens = None
    a.y = y.data_ptr()
    return a


def inputs(device):
    g = torch.Generator(device="cuda:0")
    g.manual_seed(123)
    t = {"u": torch.randn(B, D, L, device="cuda:0", generator=g).to(torch.bfloat16),
         "dl": torch.randn(B, D, L, device="cuda:0", generator=g).to(torch.bfloat16),
         "bm": torch.randn(B, 1, N, L, device="cuda:0", generator=g).to(torch.bfloat16),
         "cm": torch.randn(B, 1, N, L, device="cuda:0", generator=g).to(torch.bfloat16),
         "A": -torch.arange(1, N + 1, dtype=torch.float32, device="cuda:0").repeat(D, 1),
         "Dv": torch.ones(D, device="cuda:0"), "bias": torch.full((D,), -3.0, device="cuda:0")}
    return {k: v.to(device) for k, v in t.items()}


def test_sharded_forward_gathers_the_unsharded_output():
    n = ndev()
    Lb = _lib.load()
    devs = (ctypes.c_int * n)(*range(n))
    group = ctypes.c_void_p()
    assert Lb.sacc_shard_group_create(n, devs, ctypes.byref(group)) == _lib.SACC_OK, _lib.last_error()
    try:
        full = inputs("cuda:0")
        s0 = torch.cuda.Stream(device=0)
        with torch.cuda.stream(s0):
            ref = sb.selective_scan_ex(full["u"], full["dl"], full["A"], full["bm"], full["cm"], D=full["Dv"],
                                       delta_bias=full["bias"], layout="BDL", stream=s0)
        s0.synchronize()
        args = (_lib.ScanExArgs * n)()
        streams = (ctypes.c_void_p * n)()
        gathers = (ctypes.c_void_p * n)()
        keep = []
        r0, rows = ctypes.c_uint64(0), ctypes.c_uint64(0)
        for i in range(n):
            assert Lb.sacc_shard_rows(B, n, i, ctypes.byref(r0), ctypes.byref(rows)) == _lib.SACC_OK
            dev = torch.device("cuda", i)
            t = inputs(dev)
            sl = slice(r0.value, r0.value + rows.value)
            shard = {k: (v[sl].contiguous() if k in ("u", "dl", "bm", "cm") else v) for k, v in t.items()}
            y = torch.empty_like(shard["u"])
            out = torch.full((B, D, L), 7.0, dtype=torch.bfloat16, device=dev)
            st = torch.cuda.Stream(device=dev)
            torch.cuda.synchronize(dev)
            args[i] = ex_args(shard["u"], shard["dl"], shard["A"], shard["bm"], shard["cm"], shard["Dv"], shard["bias"], y)
            streams[i], gathers[i] = st.cuda_stream, out.data_ptr()
            keep.append((shard, y, out, st))
        nbytes = keep[0][1].numel() * 2
        assert Lb.sacc_scan_sharded_forward(group, args, streams, gathers, nbytes) == _lib.SACC_OK, _lib.last_error()
        for i, (_, _, out, st) in enumerate(keep):
            st.synchronize()
            assert torch.equal(out.cpu().view(torch.int16), ref.cpu().view(torch.int16)), f"device {i}"
        # A rejected shard (state 3) leaves every device untouched.
        for _, y, out, _ in keep:
            y.fill_(5.0)
            out.fill_(7.0)
        torch.cuda.synchronize()
        args[n - 1].state = 3
        assert Lb.sacc_scan_sharded_forward(group, args, streams, gathers, nbytes) == _lib.SACC_EINVAL
        assert f"scan_sharded shard {n - 1}" in _lib.last_error()
        for i, (_, y, out, st) in enumerate(keep):
            st.synchronize()
            assert bool((y == 5.0).all()) and bool((out == 7.0).all()), f"device {i} got work from a rejected call"
    finally:
        torch.cuda.synchronize()
        assert Lb.sacc_shard_group_destroy(group) == _lib.SACC_OK, _lib.last_error()
    assert sb.scan_fault() == 0
