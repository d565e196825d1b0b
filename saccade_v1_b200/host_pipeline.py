"""Selective scan of host-resident batches (pinned memory in, pinned memory out).

The batch axis streams through the GPU in slices of `rows` sequences: the
host-to-device copy of slice i + 1, the scan of slice i and the device-to-host
copy of slice i - 1 run at the same time on three streams, through `depth`
sets of device buffers, so a call costs about the larger of its two PCIe
directions instead of their sum plus the scan.  Every slice is one ordinary
`selective_scan_ex` call on device buffers, so the output equals the device
path's bit for bit (rows are independent).

    pipe = HostScanPipeline(u_h, B_h, rows=4)          # buffers and streams, once
    pipe.run(u_h, delta_h, A, B_h, C_h, D=D, delta_bias=bias, y_h=y_h, layout="BDL", stream=s)

Host tensors: pinned (``pin_memory()``), contiguous, batch-major; A, D and
delta_bias are device tensors (parameters stay resident).  `run` only
enqueues: the caller's stream waits for the last copy, nothing synchronizes.
"""
from __future__ import annotations

import torch

from .scan import ScanInvalidArgument, selective_scan_ex


class HostScanPipeline:
    def __init__(self, u_like: torch.Tensor, b_like: torch.Tensor, *, rows: int = 4, depth: int = 2,
                 gate: bool = False, device=None):
        if rows < 1 or depth < 2:
            raise ScanInvalidArgument("HostScanPipeline: rows >= 1 and depth >= 2 are required")
        device = torch.device(device or "cuda")
        self.rows, self.depth = rows, depth
        row_u, row_b = tuple(u_like.shape[1:]), tuple(b_like.shape[1:])
        mk = lambda shape, dt: [torch.empty((rows,) + shape, dtype=dt, device=device) for _ in range(depth)]
        self.u, self.delta, self.y = mk(row_u, u_like.dtype), mk(row_u, u_like.dtype), mk(row_u, u_like.dtype)
        self.b, self.c = mk(row_b, b_like.dtype), mk(row_b, b_like.dtype)
        self.z = mk(row_u, u_like.dtype) if gate else None
        self.h2d, self.comp, self.d2h = (torch.cuda.Stream(device=device) for _ in range(3))
        ev = lambda: [torch.cuda.Event() for _ in range(depth)]
        self.ev_in, self.ev_scan, self.ev_out = ev(), ev(), ev()
        self.row_u, self.row_b = row_u, row_b

    def run(self, u, delta, A, B, C, D=None, z=None, delta_bias=None, *, y_h, layout: str = "BDL", stream=None):
        """Enqueues the scan of the whole host batch; returns y_h."""
        if tuple(u.shape[1:]) != self.row_u or tuple(B.shape[1:]) != self.row_b or (z is not None) != (self.z is not None):
            raise ScanInvalidArgument("HostScanPipeline: tensor shapes differ from the ones it was built for")
        for name, t in (("u", u), ("delta", delta), ("B", B), ("C", C), ("z", z), ("y_h", y_h)):
            if t is not None and (t.is_cuda or not t.is_pinned() or not t.is_contiguous()):
                raise ScanInvalidArgument(f"HostScanPipeline: {name} must be pinned, contiguous host memory")
        caller = stream or torch.cuda.current_stream()
        start = torch.cuda.Event()
        start.record(caller)
        for s in (self.h2d, self.comp, self.d2h):
            s.wait_event(start)
        batch = u.shape[0]
        for i, r0 in enumerate(range(0, batch, self.rows)):
            r1 = min(r0 + self.rows, batch)
            n, k = r1 - r0, i % self.depth
            with torch.cuda.stream(self.h2d):
                if i >= self.depth:
                    self.h2d.wait_event(self.ev_out[k])  # slice i - depth has left buffer set k
                for dst, src in ((self.u, u), (self.delta, delta), (self.b, B), (self.c, C), (self.z, z)):
                    if src is not None:
                        dst[k][:n].copy_(src[r0:r1], non_blocking=True)
                self.ev_in[k].record(self.h2d)
            with torch.cuda.stream(self.comp):
                self.comp.wait_event(self.ev_in[k])
                selective_scan_ex(self.u[k][:n], self.delta[k][:n], A, self.b[k][:n], self.c[k][:n], D,
                                  self.z[k][:n] if z is not None else None, delta_bias, layout=layout,
                                  out=self.y[k][:n], stream=self.comp)
                self.ev_scan[k].record(self.comp)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.ev_scan[k])
                y_h[r0:r1].copy_(self.y[k][:n], non_blocking=True)
                self.ev_out[k].record(self.d2h)
        for s in (self.h2d, self.comp, self.d2h):
            done = torch.cuda.Event()
            done.record(s)
            caller.wait_event(done)
        return y_h
