"""Selective-scan throughput benchmark (BASELINE config 2 on every GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one step = one selective-scan forward of BASELINE config 2 per GPU,
B=64 sequences x D=1536 channels x L=2048 tokens x N=16 states, bf16 u,
delta, B, C and y in Mamba's (B,D,L) layout, FP32 state, fused dt bias +
softplus and D skip.  Synthetic seeded inputs with config 0's distributions
(u, B, C, dt_pre ~ N(0,1), dt_bias = softplus^-1(logU[1e-3, 1e-1]),
A[d,n] = -(n+1), D = 1).  Inputs (1.2 GB) exceed the 126 MB L2, so no flush is
needed between steps.  N GPUs: batch sharding, every rank runs its own
64-sequence shard (weak scaling), no collective on the scan path.

metric "scan GB/s": algorithmic bytes (u, delta, y, B, C and the FP32
parameters, each counted once) / time.  `value` is device-timed with CUDA
events over K steps on the launching stream, max over ranks; `e2e` is the
same metric through the public API with the inputs copied from pinned host
memory and y copied back inside the timed region, with `e2e.pcie_roof` its
bound from the pinned copy rates measured on the same GPU.  `roofline`
compares the scan kernel against the measured HBM copy bandwidth
(MEASURED_PEAKS.json).

`secondary` (skipped with --no-secondary; `--only NAME` runs one alone) times
the other rows of the path on the device: config 3's L = 1 step, packed
re-scan and frame average, config 1's Mamba block, the reference ABI at the
HR deploy shapes (FP32, FP16 plugin v3, FP32 with casts; eager and from a
CUDA graph), the HR head block and the fused Cross-Scan head level (against
its unfused composition), the frame-end protocol, the projection GEMM and
config 4's four-layer stack.

--impl reference times the reference's own CPU implementation
(selective_scan_reference built from its sources into oracle/_ref) on all host
cores over a bounded sample of the same workload (one batch row per thread),
reported in the same unit by scaling with the state updates processed.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, D, L, N = 64, 1536, 2048, 16
METRIC = "scan GB/s (% HBM roofline) and tracks*frames/s at 1/2/4/8 B200"
UNIT = "GB/s"
FALLBACK_HBM = 6650.0


def algorithmic_bytes(batch=B, dim=D, length=L, state=N, elem=2) -> int:
    """u, delta, y (batch, D, L) + B, C (batch, N, L) in `elem` bytes; A (D,N), D, dt_bias in FP32."""
    return elem * (3 * batch * dim * length + 2 * batch * state * length) + 4 * (dim * state + 2 * dim)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def committed_traffic():
    """dram bytes per scan launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "scan_bulk_c2.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip())
    except OSError:
        pass
    return None


def committed_fma_cycles():
    """FMA-pipe cycles per warp and token of the scan from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "scan_bulk_c2.md")
    try:
        for line in open(path):
            if line.startswith("fma_pipe_cycles_per_warp_token:"):
                return float(line.split(":")[1].strip())
    except OSError:
        pass
    return None


def pipe_roof(torch, device, kernel_ms, sm_mhz, batch):
    """The scan's FP32 FMA-pipe roof: the measured FMA-pipe cycles per warp and
    token (packed f32x2 instructions count two) times the launch's warp-tokens,
    spread over every SM's four schedulers at the sampled SM clock; frac is that
    time over the launch's event-timed duration."""
    cycles = committed_fma_cycles()
    if cycles is None or not sm_mhz:
        return None
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    warp_tokens = batch * D * L / 32
    roof_ms = cycles * warp_tokens / (sms * 4) / (sm_mhz * 1e3)
    return {"pipe": "fp32 fma (packed pairs hold it two cycles)", "cycles_per_warp_token": cycles,
            "warp_tokens_per_launch": int(warp_tokens), "sm_mhz": sm_mhz, "roof_ms": round(roof_ms, 4),
            "kernel_ms": round(kernel_ms, 4), "frac": round(roof_ms / kernel_ms, 4),
            "source": "profiles/scan_bulk_c2.md (ncu: sm__pipe_fma_cycles_active per warp-token)"}


def pcie_roof(torch, device, u_host, y_dev, y_host, h2d, d2h, e2e_step_ms, max_over_ranks):
    """The `e2e` leg's PCIe roof on this GPU: pinned copies of one whole
    sequence-batch tensor timed host-to-device alone, device-to-host alone and
    both at once on two streams (best of five each).  The step cannot move its
    bytes faster than min(h2d, d2h) of them in both directions at the joint
    rate plus the rest in the larger direction alone; frac is that time over
    the measured e2e step.  Every rank measures its own link; the bound is the
    slowest rank's."""
    scratch = torch.empty(u_host.shape, dtype=u_host.dtype, device=device)
    s_in, s_out = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)

    def best(fn):
        fn()
        torch.cuda.synchronize(device)
        ts = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s_in)
            s_out.wait_event(a)
            fn()
            done = torch.cuda.Event()
            done.record(s_out)
            s_in.wait_event(done)
            b.record(s_in)
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return min(ts)

    def h2d_only():
        with torch.cuda.stream(s_in):
            scratch.copy_(u_host, non_blocking=True)

    def d2h_only():
        with torch.cuda.stream(s_out):
            y_host.copy_(y_dev, non_blocking=True)

    def both():
        h2d_only()
        d2h_only()

    n_in, n_out = u_host.numel() * u_host.element_size(), y_dev.numel() * y_dev.element_size()
    r_in = n_in / best(h2d_only) / 1e6
    r_out = n_out / best(d2h_only) / 1e6
    r_both = min(n_in, n_out) / best(both) / 1e6
    joint = min(h2d, d2h)
    rest, r_rest = (h2d - joint, r_in) if h2d >= d2h else (d2h - joint, r_out)
    bound_ms = max_over_ranks(joint / r_both / 1e6 + rest / r_rest / 1e6)
    del scratch
    return {"h2d_GBs": round(r_in, 1), "d2h_GBs": round(r_out, 1), "both_directions_GBs_each": round(r_both, 1),
            "bound_ms": round(bound_ms, 3), "e2e_ms_per_step": round(e2e_step_ms, 3),
            "frac": round(bound_ms / e2e_step_ms, 4),
            "model": "min(h2d, d2h) bytes at the joint rate + the rest at the larger direction's own rate"}


class NvmlClocks:
    """Samples SM clock and throttle reasons through NVML every 2 ms while the timed region runs (a query
    takes well under 0.1 ms, so short timed regions still get several samples)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, device_index: int):
        import pynvml
        pynvml.nvmlInit()
        self.nv = pynvml
        uuid = None
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            pass
        self.handle = None
        if uuid:
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.handle = None
        if self.handle is None:
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
        self.samples: list[tuple[float, int]] = []
        self.stop = threading.Event()

    def _run(self):
        nv, h = self.nv, self.handle
        while not self.stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=2)

    def summary(self):
        reasons = set()
        for _, mask in self.samples:
            for name, bit in self.REASONS.items():
                if mask & bit:
                    reasons.add(name)
        try:
            mx = float(self.nv.nvmlDeviceGetMaxClockInfo(self.handle, self.nv.NVML_CLOCK_SM))
        except Exception:
            mx = None
        sm = [c for c, _ in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml"}


def clock_sampler(device_index: int):
    try:
        return NvmlClocks(device_index)
    except Exception:
        return Clocks(device_index)


class Clocks:
    """Samples nvidia-smi every 200 ms while the timed region runs (used when NVML is unavailable)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.lines: list[str] = []
        self.proc = None
        target = str(device_index)
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            target = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            pass
        self.cmd = ["nvidia-smi", "-i", target, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                    "-lms", "200"]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_inputs(torch, device, seed: int, batch=B):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    bf = torch.bfloat16
    u = torch.randn(batch, D, L, device=device, generator=g).to(bf)
    delta = torch.randn(batch, D, L, device=device, generator=g).to(bf)
    bm = torch.randn(batch, 1, N, L, device=device, generator=g).to(bf)
    cm = torch.randn(batch, 1, N, L, device=device, generator=g).to(bf)
    rng = np.random.default_rng(seed)
    dtb = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
    bias = torch.from_numpy(np.log(np.expm1(dtb)).astype(np.float32)).to(device)
    A = -torch.arange(1, N + 1, dtype=torch.float32, device=device).repeat(D, 1).contiguous()
    Dv = torch.ones(D, dtype=torch.float32, device=device)
    return dict(u=u, delta=delta, B=bm, C=cm, bias=bias, A=A, D=Dv)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import saccade_v1_b200 as sb

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    sb.load_kernels()
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        t = make_inputs(torch, device, 1234 + rank, batch=args.batch)
        y = torch.empty_like(t["u"])
    stream.synchronize()

    def step():
        sb.selective_scan_ex(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], delta_bias=t["bias"],
                             layout="BDL", out=y, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        x = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        return float(x.item())

    for _ in range(args.warmup):
        step()
    stream.synchronize()

    # Device-timed region: K steps, per-launch events for the kernel duration.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(device)
    with clock_sampler(local_rank) as clocks:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        t1.record(stream)
        while not t1.query():  # poll (sleeping, GIL released) so that the clock sampler thread runs
            time.sleep(0.0002)
    torch.cuda.synchronize(device)
    barrier()
    total_ms = max_over_ranks(t0.elapsed_time(t1))
    kernel_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    kernel_ms = max_over_ranks(kernel_ms)

    # Output assembly (N > 1): scan + NCCL all-gather of every rank's y into
    # the full (N x 64)-sequence output on every rank; not part of `value`.
    gather = None
    if world > 1:
        from saccade_v1_b200.shard import gather_batch, shard_rows
        shard = shard_rows(args.batch * world, world, rank)
        gsteps = 5

        def gather_step():
            step()
            return gather_batch(y, shard, args.batch * world)

        with torch.cuda.stream(stream):
            gather_step()
        torch.cuda.synchronize(device)
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            g0.record(stream)
            for _ in range(gsteps):
                gather_step()
            g1.record(stream)
        g1.synchronize()
        barrier()
        gms = max_over_ranks(g0.elapsed_time(g1)) / gsteps
        gather = {"ms_per_step": round(gms, 4), "value": round(algorithmic_bytes(batch=args.batch) * world / (gms / 1e3) / 1e9, 2),
                  "unit": UNIT, "collective": "NCCL all_gather_into_tensor of y (bf16) over NVLink",
                  "gathered_bytes_per_rank": y.numel() * y.element_size() * world}

    # End to end through the public API: the step's inputs in pinned host
    # memory and its output back in pinned host memory, every byte crossing
    # PCIe inside the timed region.  HostScanPipeline streams the batch in
    # slices of 4 sequences, so the copies in both directions overlap each
    # other and the scan.
    from saccade_v1_b200.host_pipeline import HostScanPipeline
    host = {k: t[k].cpu().pin_memory() for k in ("u", "delta", "B", "C")}
    y_host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = y.numel() * y.element_size()
    e2e_steps = max(2, min(args.steps, 5))
    pipe = HostScanPipeline(host["u"], host["B"], rows=4, device=device)

    def e2e_step():
        pipe.run(host["u"], host["delta"], t["A"], host["B"], host["C"], D=t["D"], delta_bias=t["bias"],
                 y_h=y_host, layout="BDL", stream=stream)

    with torch.cuda.stream(stream):
        e2e_step()
    stream.synchronize()
    barrier()
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    pcie = pcie_roof(torch, device, host["u"], y, y_host, h2d, d2h, e2e_ms / e2e_steps, max_over_ranks)

    # Config 4 (4-layer stack, batch-sharded): every rank takes part.
    c4 = None
    if not args.no_secondary and not args.no_c4:
        c4 = c4_stack(torch, device, stream, rank, world, barrier, max_over_ranks)

    if rank != 0:
        return None
    nbytes = algorithmic_bytes(batch=args.batch)
    per_step_s = total_ms / 1e3 / args.steps
    value = nbytes * world / per_step_s / 1e9
    peak, peak_kind = peaks()
    achieved = nbytes / (kernel_ms / 1e3) / 1e9
    clock_summary = clocks.summary()
    cpu = cpu_baseline(args) if world == 1 and not args.no_cpu_baseline else None
    extra = secondary(torch, device, stream, peaks()[0]) if not args.no_secondary else None
    if extra is not None and c4 is not None:
        extra["c4_stack"] = c4
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, config-0 distributions)",
        "config": {"workload": f"C2 bulk selective scan: B={args.batch} D=1536 L=2048 N=16 bf16 (B,D,L), fp32 state, "
                               "dt_bias+softplus+D fused, per GPU", "global_batch": args.batch * world, "seq_len": L,
                   "d_inner": D, "d_state": N, "parallelism": f"batch-sharded x{world}",
                   "l2": "inputs 1.2 GB > 126 MB L2, no flush"},
        "tracks_frames_per_s": round(args.batch * world / per_step_s, 1),
        "e2e": {"value": round(nbytes * world / (e2e_ms / 1e3 / e2e_steps) / 1e9, 3), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps, "pcie_roof": pcie},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": committed_traffic(), "peak_kind": peak_kind,
                     "kernel": "scan (sacc_selective_scan_ex)", "algorithmic_bytes_per_launch": nbytes},
        "clocks": clock_summary,
        "pipe_roof": pipe_roof(torch, device, kernel_ms, clock_summary.get("sm_mhz"), args.batch),
        "gpu_launches": args.steps,
        "cpu_baseline": cpu,
        "secondary": extra,
        "with_allgather": gather,
    }
    return line


def time_device(torch, stream, fn, iters: int, warmup: int = 3) -> float:
    """Mean device time of fn() in microseconds, CUDA events on `stream`."""
    for _ in range(warmup):
        fn()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) * 1e3 / iters


def c3_inputs(torch, device, stream):
    """Config 3 tensors: 4096 tracks' activations (fp16) and carried state (256 x 16 FP32 each), plus the
    packed histories (lengths U{1..64}) of a full re-scan."""
    g = torch.Generator(device=device)
    g.manual_seed(77)
    T3, D3, N3 = 4096, 256, 16
    f16 = torch.float16
    with torch.cuda.stream(stream):
        t = {"u": torch.randn(T3, D3, device=device, generator=g).to(f16),
             "dl": torch.randn(T3, D3, device=device, generator=g).to(f16),
             "z": torch.randn(T3, D3, device=device, generator=g).to(f16),
             "bm": torch.randn(T3, N3, device=device, generator=g).to(f16),
             "cm": torch.randn(T3, N3, device=device, generator=g).to(f16),
             "A": -torch.arange(1, N3 + 1, dtype=torch.float32, device=device).repeat(D3, 1).contiguous(),
             "Dv": torch.ones(D3, device=device), "bias": torch.full((D3,), -4.6, device=device),
             "state": torch.randn(T3, D3, N3, device=device, generator=g) * 0.5}
        t["y"] = torch.empty_like(t["u"])
        lens = np.random.default_rng(3).integers(1, 65, T3)
        t["cu"] = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device=device)
        tot = int(lens.sum())
        for k in ("ur", "dr", "zr"):
            t[k] = torch.randn(1, tot, D3, device=device, generator=g).to(f16)
        for k in ("br", "cr"):
            t[k] = torch.randn(1, tot, 1, N3, device=device, generator=g).to(f16)
        t["yr"] = torch.empty_like(t["ur"])
        t["hr"] = torch.empty(T3, D3, N3, device=device)
    stream.synchronize()
    return t


def c3_step(torch, device, stream, peak):
    """Config 3: one per-frame L = 1 step of 4096 tracks' carried state."""
    import saccade_v1_b200 as sb
    t = c3_inputs(torch, device, stream)
    step = lambda: sb.selective_scan_step(t["u"], t["dl"], t["A"], t["bm"], t["cm"], t["state"], D=t["Dv"], z=t["z"],
                                          delta_bias=t["bias"], out=t["y"], stream=stream)
    us = time_device(torch, stream, step, 50)
    nbytes = 2 * t["state"].numel() * 4 + 4 * t["u"].numel() * 2 + 2 * t["bm"].numel() * 2 + 4 * (t["A"].numel() + 2 * 256)
    # L2-cold: in deployment one step runs per frame between other work that evicts the 126 MB L2, while back
    # to back the 64 MiB state partly stays there.  Each step is timed alone after writing a 256 MB buffer
    # (outside its event pair), so its state is read from HBM.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    cold = []
    for i in range(23):
        with torch.cuda.stream(stream):
            flush.fill_(i & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
        e1.synchronize()
        if i >= 3:
            cold.append(e0.elapsed_time(e1) * 1e3)
    del flush
    cold_us = statistics.median(cold)
    return {"us": round(us, 2), "tracks_frames_per_s": round(4096 / (us * 1e-6), 1),
            "GB_per_s": round(nbytes / (us * 1e-6) / 1e9, 1), "hbm_frac": round(nbytes / (us * 1e-6) / 1e9 / peak, 4),
            "l2_cold_us": round(cold_us, 2), "l2_cold_GB_per_s": round(nbytes / (cold_us * 1e-6) / 1e9, 1),
            "l2_cold_hbm_frac": round(nbytes / (cold_us * 1e-6) / 1e9 / peak, 4),
            "l2_cold_tracks_frames_per_s": round(4096 / (cold_us * 1e-6), 1),
            "note": "us / hbm_frac: 50 steps back to back (the state partly L2-resident); l2_cold_*: median of 20 "
                    "steps each timed alone after a 256 MB L2-evicting write",
            "bytes": nbytes, "workload": "4096 tracks, D=256, N=16, fp16 acts, fp32 carried state, gate+bias+D"}


def c3_rescan(torch, device, stream, peak):
    """Config 3: full packed re-scan of the 4096 histories with cu_seqlens, h0 -> h_final."""
    import saccade_v1_b200 as sb
    t = c3_inputs(torch, device, stream)
    rescan = lambda: sb.selective_scan_ex(t["ur"], t["dr"], t["A"], t["br"], t["cr"], D=t["Dv"], z=t["zr"],
                                          delta_bias=t["bias"], h0=t["state"], h_final=t["hr"], cu_seqlens=t["cu"],
                                          layout="BLD", out=t["yr"], stream=stream)
    us = time_device(torch, stream, rescan, 10)
    tok = t["ur"].shape[1]
    nbytes = 4 * tok * 256 * 2 + 2 * tok * 16 * 2 + 2 * t["state"].numel() * 4
    return {"us": round(us, 2), "tokens": tok, "GB_per_s": round(nbytes / (us * 1e-6) / 1e9, 1),
            "updates_per_s": round(tok * 256 * 16 / (us * 1e-6), 1),
            "workload": "4096 packed histories, lengths U{1..64}, BLD fp16, h0 -> h_final"}


def hr_deploy(torch, device, stream, peak):
    """Reference ABI at the HR deploy shapes (4 directions x L tokens x 256 channels, N = 16, FP32, shared A,
    rank-1 C, D): the reference's published 3-level total is 722.351 us (RTX 5070 Ti laptop GPU)."""
    import saccade_v1_b200 as sb
    g = torch.Generator(device=device)
    g.manual_seed(78)
    levels, calls, f16, casts = {}, [], [], []
    with torch.cuda.stream(stream):
        st = torch.zeros(2, dtype=torch.int32, device=device)
        for L_ in (960, 240, 60):
            shape = sb.SelectiveScanShape(4, L_, 256, 16, 1, 1, True)
            uu = torch.randn(4 * L_ * 256, device=device, generator=g) * 2
            dd = torch.rand(4 * L_ * 256, device=device, generator=g) * 9 - 6
            aa = -torch.rand(16, device=device, generator=g) * 3.95 - 0.05
            bb = torch.randn(4 * L_ * 16, device=device, generator=g)
            cc = torch.randn(4 * L_, device=device, generator=g)
            dv = torch.randn(256, device=device, generator=g)
            yy = torch.empty_like(uu)
            call = (lambda s_=shape, a_=(uu, dd, aa, bb, cc, dv, yy): sb.selective_scan_cuda(s_, *a_, st, stream=stream))
            levels[f"HR_L{L_}"] = round(time_device(torch, stream, call, 50), 2)
            calls.append(call)
            # FP16 engine: the plugin v3 path on FP16 activations, and the v2 path with the casts an FP16 engine
            # puts around an FP32 plugin (u, delta, B, C widened, y narrowed).
            hu, hd, hb, hc = uu.half(), dd.half(), bb.half(), cc.half()
            hy = torch.empty_like(hu)
            f16.append(lambda s_=shape, a_=(hu, hd, aa, hb, hc, dv, hy): sb.selective_scan_f16(s_, *a_, st, stream=stream))

            def cast_call(s_=shape, a_=(hu, hd, aa, hb, hc, dv), out=(yy, hy)):
                u_, d_, a32, b_, c_, dv_ = a_
                sb.selective_scan_cuda(s_, u_.float(), d_.float(), a32, b_.float(), c_.float(), dv_, out[0], st,
                                       stream=stream)
                out[1].copy_(out[0])
            casts.append(cast_call)
    total = time_device(torch, stream, lambda: [c() for c in calls], 50)
    with torch.cuda.stream(stream):
        total16 = time_device(torch, stream, lambda: [c() for c in f16], 50)
        total_cast = time_device(torch, stream, lambda: [c() for c in casts], 50)
    # The same calls replayed from a CUDA graph (how an engine enqueues them: no Python or host validation
    # between launches), so the figure is device time rather than host enqueue time at the small levels.
    graphs = {}
    for name, group in (("total_graph", calls), ("fp16_plugin_v3_total_graph", f16)):
        g_ = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_, stream=stream):
            for c in group:
                c()

        def replay(g_=g_):
            with torch.cuda.stream(stream):
                g_.replay()

        graphs[name] = round(time_device(torch, stream, replay, 100), 2)
        del g_
    stream.synchronize()
    return dict(levels, total=round(total, 2), fp16_plugin_v3_total=round(total16, 2),
                fp32_plugin_with_casts_total=round(total_cast, 2), **graphs, reference_published_total_us=722.351,
                note="reference figure is its own CUDA kernel on an RTX 5070 Ti laptop GPU; *_graph: the three "
                     "levels' calls replayed from one CUDA graph")


def frame_protocol(torch, device, stream):
    """Frame-end status handling per frame at the detector's shapes (T01 profile: image 3 x 640 x 640, payload
    84 x 8400 raw floats): nine plugin status words re-armed, the finite checks of the image and of the payload,
    then begin / gate (11 statuses) / publish / commit / packet as the reference's five launches, or as the
    library's one launch; eager and replayed from a CUDA graph."""
    from saccade_v1_b200 import frame as fr
    count, cap = 84 * 8400, 64
    g = torch.Generator(device=device)
    g.manual_seed(31)
    with torch.cuda.stream(stream):
        image = torch.randn(3 * 640 * 640, device=device, generator=g)
        payload = torch.randn(count, device=device, generator=g)
        done = np.array([[0, 0x4E414353]] * 11, np.uint32).view(np.int32)
        armed = torch.from_numpy(done).to(device)
        st = torch.zeros_like(armed)
        ctl, rec = fr.new_control(device), fr.new_records(cap, device)
        results = torch.empty(2 * count, device=device)
        rf = torch.empty(2, dtype=torch.int64, device=device)
        packet = torch.empty(fr.PACKET_BYTES, dtype=torch.uint8, device=device)
        fr.scan_frame_initialize(ctl, 1, rf, stream=stream)
    frame_no = [0]

    def checks():
        st.copy_(armed)
        fr.scan_frame_check_finite(image, st[9], fr.FRAME_NONFINITE_INPUT, stream=stream)
        fr.scan_frame_check_finite(payload, st[10], fr.FRAME_NONFINITE_OUTPUT, stream=stream)

    def single():
        checks()
        fr.scan_frame_begin(ctl, 1, frame_no[0], stream=stream)
        fr.scan_frame_gate(ctl, st, rec, cap, stream=stream)
        fr.scan_frame_publish(ctl, payload, results, rf, rec, cap, stream=stream)
        fr.scan_frame_commit(ctl, stream=stream)
        fr.scan_frame_packet(ctl, packet, stream=stream)
        frame_no[0] += 1

    def fused():
        checks()
        fr.scan_frame_step(ctl, 1, frame_no[0], st, payload, results, rf, rec, cap, packet, stream=stream)
        frame_no[0] += 1

    out = {}
    for name, fn in (("single_steps", single), ("one_launch", fused)):
        with torch.cuda.stream(stream):
            fr.scan_frame_initialize(ctl, 1, rf, stream=stream)
        frame_no[0] = 0
        out[f"{name}_us"] = round(time_device(torch, stream, fn, 200), 2)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fr.scan_frame_initialize(ctl, 1, rf, stream=stream)
        stream.synchronize()
        frame_no[0] = 0
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(10):
                fn()

        def replay():
            with torch.cuda.stream(stream):
                fr.scan_frame_initialize(ctl, 1, rf, stream=stream)
                graph.replay()

        out[f"{name}_us_graph"] = round(time_device(torch, stream, replay, 50) / 10, 2)
        del graph
    stream.synchronize()
    c = fr.read_control(ctl.cpu().numpy())
    assert c["fail_code"] == 0 and c["committed"] == 9, c  # every timed frame passed the gate and committed
    out["workload"] = ("per frame: 9 plugin statuses re-armed, finite checks of a 3 x 640 x 640 image and an "
                       "84 x 8400 payload, gate over 11 statuses, publish + digest of the payload, commit, packet")
    return out


def secondary(torch, device, stream, peak, only=None, gemm_m=64 * 4096):
    """Other rows of the hot path, device-timed on this GPU (not part of `value`); `only` runs one of them."""
    runs = {"c3_step": c3_step, "c3_rescan": c3_rescan, "hr_deploy_f32_us": hr_deploy,
            "c1_block": lambda *a: c1_block(*a[:3]), "hr_head_block": lambda *a: hr_head_block(*a[:3]),
            "hr_head_level": lambda *a: hr_head_level(*a[:3]),
            "gemm": lambda *a: gemm_probe(*a[:3], m=gemm_m),
            "frame_protocol": lambda *a: frame_protocol(*a[:3]),
            "c4_stack": lambda *a: c4_stack(*a[:3])}
    out = {}
    for name, fn in runs.items():
        if name == "c4_stack" and only != name:
            continue  # run on every rank by run_ours
        if only is None or name == only:
            out[name] = fn(torch, device, stream, peak)
            stream.synchronize()
    if "c3_step" in out and "c3_rescan" in out:
        us, us_r = out["c3_step"]["us"], out["c3_rescan"]["us"]
        out["c3_frame_avg_us"] = round(us + us_r / 30.0, 2)
        out["c3_tracks_frames_per_s"] = round(4096 / ((us + us_r / 30.0) * 1e-6), 1)
    return out


def c4_stack(torch, device, stream, rank=0, world=1, barrier=lambda: None, max_over_ranks=lambda v: v, forwards=2):
    """a 4-layer Mamba stack (d_model 1024, D 2048, N 16, d_conv 4, dt_rank 64, bf16, fp32
    state) over B = 512 tracks x L = 4096 frames, split by batch over the ranks (no collective inside the stack),
    then an NCCL all-gather of the last layer's output.  Device-timed, max over ranks; every rank takes the
    same steps."""
    import saccade_v1_b200 as sb
    from saccade_v1_b200.shard import gather_batch, shard_rows
    B4, L4, dm, D4, N4, R4, layers = 512, 4096, 1024, 2048, 16, 64, 4
    shard = shard_rows(B4, world, rank)
    bf = torch.bfloat16
    g = torch.Generator(device=device)
    g.manual_seed(4000 + rank)
    with torch.cuda.stream(stream):
        params = []
        for li in range(layers):
            p = synthetic_block(400 + li, dm, D4, N4, R4)
            params.append({k: (torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device=device, dtype=bf)
                               if k in ("w_in", "w_x", "w_dt", "w_out") else
                               torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device)) for k, v in p.items()})
        x = torch.randn(shard.size, L4, dm, device=device, generator=g, dtype=bf) * 0.1
        bufs = [torch.empty_like(x), torch.empty_like(x)]
        ws = torch.empty(sb.mamba_block_workspace(x, params[0]) + 256, dtype=torch.uint8, device=device)

        def forward():
            h = x
            for li in range(layers):
                out = bufs[li % 2]
                sb.mamba_block_forward(h, params[li], out=out, workspace=ws, stream=stream)
                h = out
            return h

        forward()
    stream.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(forwards):
        with torch.cuda.stream(stream):
            h = forward()
    e1.record(stream)
    e1.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / forwards
    gms = None
    if world > 1:
        with torch.cuda.stream(stream):
            gather_batch(h, shard, B4)
        torch.cuda.synchronize(device)
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            g0.record(stream)
            full = gather_batch(h, shard, B4)
            g1.record(stream)
        g1.synchronize()
        barrier()
        gms = max_over_ranks(g0.elapsed_time(g1))
        del full
    tokens = B4 * L4
    flop = layers * 2 * tokens * (dm * 2 * D4 + D4 * (R4 + 2 * N4) + R4 * D4 + D4 * dm)
    res = {"ms_per_forward": round(ms, 3), "tracks_frames_per_s": round(tokens / (ms / 1e3), 1),
           "gemm_tflops": round(flop / (ms / 1e3) / 1e12, 1), "ranks": world, "tracks_per_rank": shard.size,
           "allgather_ms": None if gms is None else round(gms, 3),
           "tracks_frames_per_s_with_allgather": round(tokens / ((ms + (gms or 0.0)) / 1e3), 1),
           "workload": "4 layers, d_model 1024, D 2048, N 16, dt_rank 64, bf16, B=512 x L=4096, batch-sharded"}
    del x, bufs, ws, params
    torch.cuda.empty_cache()
    return res


def synthetic_block(seed, d_model, d_inner, d_state, dt_rank, d_conv=4):
    """Seeded block weights: uniform +-1/sqrt(fan_in), A = -(1..N), D = 1,
    dt_bias = softplus^-1(logU[1e-3, 1e-1]), RMSNorm weight ~ 1 + N(0, 0.01)."""
    r = np.random.default_rng(seed)
    u = lambda shape, fan: (r.uniform(-1, 1, shape) / np.sqrt(fan)).astype(np.float32)
    return {"w_in": u((2 * d_inner, d_model), d_model), "conv_w": u((d_inner, d_conv), d_conv),
            "conv_b": u((d_inner,), d_conv), "w_x": u((dt_rank + 2 * d_state, d_inner), d_inner),
            "w_dt": u((d_inner, dt_rank), dt_rank),
            "dt_bias": np.log(np.expm1(np.exp(r.uniform(np.log(1e-3), np.log(1e-1), d_inner)))).astype(np.float32),
            "A": -np.tile(np.arange(1, d_state + 1, dtype=np.float32), (d_inner, 1)),
            "D": np.ones(d_inner, np.float32), "w_out": u((d_model, d_inner), d_inner),
            "norm_w": (1.0 + 0.1 * r.standard_normal(d_model)).astype(np.float32)}


def c1_block(torch, device, stream):
    """one Mamba block forward over 256 tracks x 32 frames (fp16), graph-captured."""
    import saccade_v1_b200 as sb
    B1, L1, dm, D1, N1, R1 = 256, 32, 128, 256, 16, 8
    p = synthetic_block(12, dm, D1, N1, R1)
    with torch.cuda.stream(stream):
        dev = {k: (torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device=device, dtype=torch.float16)
                   if k in ("w_in", "w_x", "w_dt", "w_out") else torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device))
               for k, v in p.items()}
        x = (torch.randn(B1, L1, dm, device=device) * 0.1).to(torch.float16)
        y = torch.empty_like(x)
        ws = torch.empty(sb.mamba_block_workspace(x, dev) + 256, dtype=torch.uint8, device=device)
        fwd = lambda: sb.mamba_block_forward(x, dev, out=y, workspace=ws, stream=stream)
        fwd()
    stream.synchronize()
    eager_us = time_device(torch, stream, fwd, 50)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fwd()

    def replay():
        with torch.cuda.stream(stream):  # CUDAGraph.replay launches on the current stream
            g.replay()

    graph_us = time_device(torch, stream, replay, 200)
    flops = 2 * B1 * L1 * (dm * 2 * D1 + D1 * (R1 + 2 * N1) + R1 * D1 + D1 * dm)
    return {"us_graph": round(graph_us, 2), "us_eager": round(eager_us, 2),
            "tracks_frames_per_s": round(B1 / (graph_us * 1e-6), 1), "gflop": round(flops / 1e9, 3),
            "kernels_per_forward": 6,  # RMSNorm prep in one launch; dt_proj runs inside the scan at dt_rank 8
            "workload": "256 tracks x 32 frames, d_model 128, D 256, N 16, dt_rank 8, fp16, RMSNorm + residual"}


def hr_head_block(torch, device, stream):
    """The reference head's Mamba block at its three HR deploy levels (4 Cross-Scan directions x L = 960 / 240 /
    60 tokens, d_model 128, d_inner 256, N 16, dt_rank 16, rank-1 C, A shared by the channels, no RMSNorm,
    residual; fp16), one forward per level replayed from one CUDA graph."""
    import saccade_v1_b200 as sb
    dm, D1, N1, R1 = 128, 256, 16, 16
    p = synthetic_block(21, dm, D1, N1, R1)
    r = np.random.default_rng(22)
    p["w_x"] = p["w_x"][:R1 + N1 + 1]  # x_proj 256 -> 16 + 16 + 1
    p["A"] = np.tile(-np.exp(r.uniform(-1, 1.5, (1, N1))).astype(np.float32), (D1, 1))
    del p["norm_w"]
    with torch.cuda.stream(stream):
        dev = {k: (torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device=device, dtype=torch.float16)
                   if k in ("w_in", "w_x", "w_dt", "w_out") else torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device))
               for k, v in p.items()}
        levels = []
        for L_ in (960, 240, 60):
            x = (torch.randn(4, L_, dm, device=device) * 0.5).to(torch.float16)
            y = torch.empty_like(x)
            ws = torch.empty(sb.mamba_block_workspace(x, dev) + 256, dtype=torch.uint8, device=device)
            levels.append((L_, x, y, ws))
        fwd = lambda lv: sb.mamba_block_forward(lv[1], dev, out=lv[2], workspace=lv[3], stream=stream)
        for lv in levels:
            fwd(lv)
    stream.synchronize()
    out = {f"L{lv[0]}_us_eager": round(time_device(torch, stream, lambda lv=lv: fwd(lv), 50), 2) for lv in levels}
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for lv in levels:
            fwd(lv)

    def replay():
        with torch.cuda.stream(stream):
            g.replay()

    out["three_levels_us_graph"] = round(time_device(torch, stream, replay, 200), 2)
    out["workload"] = ("reference head block x 3 HR levels: (4, L, 128) fp16, d_inner 256, N 16, dt_rank 16, "
                       "rank-1 C, shared A, residual, no RMSNorm")
    return out


def hr_head_level(torch, device, stream):
    """The reference head's steps 3-5 at its three HR deploy levels (maps 24 x 40, 12 x 20, 6 x 10, d_model 128):
    Cross-Scan expand, the Mamba block on the four directions (d_inner 256, N 16, dt_rank 16, rank-1 C, shared A,
    residual on the tokens), merge.  Fused: sacc_cross_scan_block_forward per level.  Unfused, for comparison:
    this library's expand kernel, an fp16 cast, the block, an FP32 cast and the merge kernel.  fp16 activations,
    FP32 maps in and out; each variant's three levels replayed from one CUDA graph."""
    import saccade_v1_b200 as sb
    dm, D1, N1, R1 = 128, 256, 16, 16
    p = synthetic_block(21, dm, D1, N1, R1)
    r = np.random.default_rng(22)
    p["w_x"] = p["w_x"][:R1 + N1 + 1]  # x_proj 256 -> 16 + 16 + 1
    p["A"] = np.tile(-np.exp(r.uniform(-1, 1.5, (1, N1))).astype(np.float32), (D1, 1))
    del p["norm_w"]
    f16 = torch.float16
    with torch.cuda.stream(stream):
        dev = {k: (torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device=device, dtype=f16)
                   if k in ("w_in", "w_x", "w_dt", "w_out") else torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device))
               for k, v in p.items()}
        levels = []
        for h, w in ((24, 40), (12, 20), (6, 10)):
            x = torch.randn(1, dm, h, w, device=device) * 0.5
            shape = sb.CrossScanShape(1, dm, h, w)
            tok = torch.empty(4, h * w, dm, device=device)
            lv = {"x": x, "out": torch.empty_like(x), "out2": torch.empty_like(x), "shape": shape, "tok": tok,
                  "tok16": torch.empty(4, h * w, dm, device=device, dtype=f16), "r16": torch.empty(4, h * w, dm, device=device, dtype=f16),
                  "r": torch.empty_like(tok), "st": torch.zeros(2, dtype=torch.int32, device=device),
                  "ws": torch.empty(sb.cross_scan_block_workspace(x, dev, dtype=f16) + 256, dtype=torch.uint8, device=device)}
            lv["ws_b"] = torch.empty(sb.mamba_block_workspace(lv["tok16"], dev) + 256, dtype=torch.uint8, device=device)
            levels.append(lv)

        def fused(lv):
            sb.cross_scan_block_forward(lv["x"], dev, dtype=f16, out=lv["out"], workspace=lv["ws"], stream=stream)

        def unfused(lv):
            sb.cross_scan_expand_cuda(lv["shape"], lv["x"], lv["tok"], lv["st"], stream=stream)
            lv["tok16"].copy_(lv["tok"])
            sb.mamba_block_forward(lv["tok16"], dev, out=lv["r16"], workspace=lv["ws_b"], stream=stream)
            lv["r"].copy_(lv["r16"])
            sb.cross_scan_merge_cuda(lv["shape"], lv["r"], lv["out2"], lv["st"], stream=stream)

        for lv in levels:
            fused(lv)
            unfused(lv)
    stream.synchronize()
    out = {}
    for name, fn in (("fused", fused), ("unfused", unfused)):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for lv in levels:
                fn(lv)

        def replay():
            with torch.cuda.stream(stream):
                g.replay()

        out[f"{name}_three_levels_us_graph"] = round(time_device(torch, stream, replay, 200), 2)
        del g
    stream.synchronize()
    diff = max(float((lv["out"] - lv["out2"]).abs().max()) for lv in levels)
    out["max_abs_diff_fused_vs_unfused"] = round(diff, 5)
    flop_fused = sum(2 * lv["x"].shape[2] * lv["x"].shape[3] * (dm * 2 * D1 + 4 * D1 * (R1 + 2 * N1) + D1 * dm) for lv in levels)
    flop_unfused = sum(2 * 4 * lv["x"].shape[2] * lv["x"].shape[3] * (dm * 2 * D1 + D1 * (R1 + 2 * N1) + D1 * dm) for lv in levels)
    out["gemm_mflop_fused"] = round(flop_fused / 1e6, 1)
    out["gemm_mflop_unfused"] = round(flop_unfused / 1e6, 1)
    out["workload"] = ("reference head steps 3-5 x 3 HR levels (maps 24x40, 12x20, 6x10, d_model 128 FP32): expand, block "
                       "(d_inner 256, N 16, dt_rank 16, rank-1 C, shared A, residual on the tokens, fp16), merge")
    return out


def gemm_probe(torch, device, stream, m=64 * 4096):
    """The tcgen05 projection GEMM at the config-4 in_proj shape of one 8-GPU shard (bf16 in, bf16 out;
    m = 64 tracks x 4096 tokens, n = 2 x d_inner, k = d_model)."""
    import saccade_v1_b200 as sb
    n, k = 4096, 1024
    with torch.cuda.stream(stream):
        a = torch.randn(m, k, device=device).to(torch.bfloat16)
        b = (torch.randn(n, k, device=device) / 32).to(torch.bfloat16)
        c = torch.empty(m, n, device=device, dtype=torch.bfloat16)
        run = lambda: sb.gemm(a, b, out=c, stream=stream)
    us = time_device(torch, stream, run, 5, warmup=2)
    tflops = 2 * m * n * k / (us * 1e-6) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        peak = 1590.0
    del a, b, c
    return {"shape_mnk": [m, n, k], "us": round(us, 1), "tflops": round(tflops, 1), "peak_tflops": peak,
            "frac": round(tflops / peak, 4), "bound": "tensor"}


def reference_sample(threads: int):
    """One bounded sample of the workload in the reference ABI: `threads` batch rows of (L, D) FP32."""
    from oracle import oracle
    rows = max(1, min(threads, B))
    rng = np.random.default_rng(99)
    u = rng.standard_normal((rows, L, D), dtype=np.float32)
    dtb = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), D))
    bias = np.log(np.expm1(dtb)).astype(np.float32)
    delta = (rng.standard_normal((rows, L, D), dtype=np.float32) + bias).astype(np.float32)  # dt_pre + dt_bias in FP32
    b = rng.standard_normal((rows, L, N), dtype=np.float32)
    c = rng.standard_normal((rows, L, N), dtype=np.float32)
    a = -np.tile(np.arange(1, N + 1, dtype=np.float32), (D, 1))
    d = np.ones(D, np.float32)
    shape = oracle.Shape(rows, L, D, N, D, N, True)
    return oracle, shape, [np.ascontiguousarray(x) for x in (u, delta, a, b, c, d)], rows


def time_reference(threads: int):
    """Runs the reference's selective_scan_reference once over the sample; returns (seconds, rows, kind)."""
    import ctypes
    oracle, shape, ins, rows = reference_sample(threads)
    y = np.zeros(rows * L * D, np.float64)
    R = oracle.ref_lib()
    f32 = ctypes.POINTER(ctypes.c_float)
    ptrs = [x.ctypes.data_as(f32) for x in ins]
    t0 = time.perf_counter()
    if R is not None:
        rc = R.sacc_ref_selective_scan_threads(ctypes.byref(shape.c()), *ptrs,
                                               y.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), threads)
        kind = "reference"
    else:  # the reference build did not travel: the C restatement, one thread
        k = oracle.Case(shape, *ins)
        rc, _, _ = oracle.scan_ref(k)
        kind = "port"
        threads = 1
    dt = time.perf_counter() - t0
    if rc != 0:
        raise RuntimeError(f"reference scan failed with status {rc}")
    return dt, rows, kind, threads


def cpu_baseline(args):
    threads = os.cpu_count() or 1
    dt, rows, kind, used = time_reference(threads)
    value = algorithmic_bytes(batch=rows) / dt / 1e9
    return {"value": round(value, 4), "unit": UNIT, "cores": used, "kind": kind,
            "sample": f"{rows} of {B} batch rows (L={L}, D={D}, N={N}), one row per thread, FP32 reference ABI; "
                      f"value scaled by the C2 bf16 algorithmic bytes of the rows processed; {dt:.2f} s"}


def run_reference(args):
    threads = os.cpu_count() or 1
    times = []
    for i in range(args.warmup + args.steps):
        dt, rows, kind, used = time_reference(threads)
        if i >= args.warmup:
            times.append(dt)
    per = statistics.mean(times)
    value = algorithmic_bytes(batch=rows) / per / 1e9
    sample = (f"{rows} of {B} batch rows (L={L}, D={D}, N={N}) per step, one row per thread, FP32 reference ABI; "
              f"scaled by the C2 bf16 algorithmic bytes of the rows processed")
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64 (reference binary64 on f32 inputs)",
        "data": "synthetic (seeded, config-0 distributions)",
        "config": {"workload": "C2 bulk selective scan: B=64 D=1536 L=2048 N=16, sample on host cores",
                   "global_batch": B, "seq_len": L, "d_inner": D, "d_state": N, "parallelism": f"{used} host threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": used, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip the config-3 and deploy-shape timings")
    ap.add_argument("--batch", type=int, default=B, help="sequences per GPU (config 2: 64; smaller only for profiling)")
    ap.add_argument("--no-c4", action="store_true", help="skip the config-4 stack (52 GB on one GPU)")
    ap.add_argument("--only", choices=["c3_step", "c3_rescan", "hr_deploy_f32_us", "c1_block", "hr_head_block", "hr_head_level",
                                       "frame_protocol", "gemm",
                                       "c4_stack"],
                    help="run one secondary measurement alone on cuda:0 and print it (for profiling)")
    ap.add_argument("--gemm-m", type=int, default=64 * 4096, help="rows of the GEMM probe (smaller only for profiling)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        # NCCL's initialisation log (communicator size and rank per process) stays on, so a run's output shows
        # that every rank joined one communicator of `world` ranks; NCCL reads these once, before torch loads it.
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    import torch
    import torch.distributed as dist
    if args.only:
        device = torch.device("cuda", 0)
        stream = torch.cuda.Stream(device)
        print(json.dumps(secondary(torch, device, stream, peaks()[0], only=args.only, gemm_m=args.gemm_m)), flush=True)
        return
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
