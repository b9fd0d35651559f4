"""Benchmark of the Conv3d hot path on B200.

Workload ("trunk"): the UNet3D trunk sweep at batch 4 per GPU, bf16, NDHWC —
k3 pad1 convs 1->24 and 24->24 at 64x128x128, 48->48 at 32x64x64, 96->96 at
16x32x32, 192->192 at 8x16x16, and k1 convs 48->24, 96->48, 192->96 at the
matching levels. One step = forward, dW (+db) and dX of every layer, seeded
synthetic N(0,1) inputs / grad_out and default-init weights.

Metric: conv TFLOP/s over fwd+dW+dX (algorithmic FLOPs 2*V*Cin*Cout*k^3 per
leg; padding MACs not counted), whole job. With N GPUs each rank runs its own
batch-4 sweep (weak scaling, batch-sharded data parallel) and the fp32 dW/db
of every layer are all-reduced over NCCL on a side stream while dX runs.

Usage:  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Prints ONE JSON line on rank 0.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rdna4-conv3d-wmma_b200"))

import torch  # noqa: E402

# name, cin, cout, (D, H, W), k
TRUNK = [
    ("k3 1->24", 1, 24, (64, 128, 128), 3),
    ("k3 24->24", 24, 24, (64, 128, 128), 3),
    ("k3 48->48", 48, 48, (32, 64, 64), 3),
    ("k3 96->96", 96, 96, (16, 32, 32), 3),
    ("k3 192->192", 192, 192, (8, 16, 16), 3),
    ("k1 48->24", 48, 24, (64, 128, 128), 1),
    ("k1 96->48", 96, 48, (32, 64, 64), 1),
    ("k1 192->96", 192, 96, (16, 32, 32), 1),
]
# ConvTranspose3d k=2 s=2 p=0 (name, cin, cout, input (D, H, W));
# timed after the trunk, reported beside it, not part of `value`
TCONV = [
    ("T k2s2 192->96", 192, 96, (8, 16, 16)),
    ("T k2s2 96->48", 96, 48, (16, 32, 32)),
    ("T k2s2 48->24", 48, 24, (32, 64, 64)),
]
BATCH = 4
METRIC = "conv TFLOP/s (fwd/dW/dX) vs bf16 peak; UNet3D ms/sample at 1/2/4/8 B200"


def layer_flops(cin, cout, spatial, k, batch=BATCH):
    d, h, w = spatial
    return 2.0 * batch * d * h * w * cin * cout * k ** 3   # pad=(k-1)/2 keeps the output size


def layer_bytes(cin, cout, spatial, k, batch=BATCH, leg="fwd"):
    """Minimum HBM bytes of one leg (bf16 activations, fp32 dW)."""
    d, h, w = spatial
    v = batch * d * h * w
    wbytes = cin * cout * k ** 3
    if leg == "dw":
        return 2 * v * (cin + cout) + 4 * wbytes
    return 2 * v * (cin + cout) + 2 * wbytes


def tconv_bytes(cin, cout, spatial, leg, batch=BATCH):
    """Minimum HBM bytes of one k2s2 transpose-conv leg (bf16, fp32 dW)."""
    d, h, w = spatial
    v = batch * d * h * w
    if leg == "dw":
        return 2 * v * cin + 2 * 8 * v * cout + 4 * 8 * cin * cout
    return 2 * v * cin + 2 * 8 * v * cout + 2 * 8 * cin * cout


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"],
                "bf16_tflops_sustained": j.get("bf16_tflops_sustained", j["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# distributed set-up
# ---------------------------------------------------------------------------
def init_dist(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU baseline: the reference's CPU path (stock PyTorch fp32 conv3d)
# ---------------------------------------------------------------------------
def cpu_sample_pass(layers, frac_d):
    """fwd + dW + dX of every layer on CPU fp32, batch 1, depth cut to frac_d."""
    import torch.nn.functional as F
    flops = 0.0
    t0 = time.perf_counter()
    for name, cin, cout, (d, h, w), k in layers:
        dd = max(2, int(round(d * frac_d)))
        g = torch.Generator().manual_seed(0)
        x = torch.randn(1, cin, dd, h, w, generator=g)
        wt = torch.randn(cout, cin, k, k, k, generator=g) / (cin * k ** 3) ** 0.5
        pad = (k - 1) // 2
        y = F.conv3d(x, wt, None, 1, pad)
        go = torch.randn_like(y)
        torch.nn.grad.conv3d_weight(x, wt.shape, go, 1, pad)
        torch.nn.grad.conv3d_input(x.shape, wt, go, 1, pad)
        flops += 3 * layer_flops(cin, cout, (dd, h, w), k, batch=1)
    return flops, time.perf_counter() - t0


def cpu_baseline(layers, budget_s=15.0, frac_d=1 / 16):
    cores = torch.get_num_threads()
    cpu_sample_pass(layers, frac_d)  # warm-up
    rates, t_start = [], time.perf_counter()
    while len(rates) < 5 or (time.perf_counter() - t_start < budget_s and len(rates) < 50):
        fl, dt = cpu_sample_pass(layers, frac_d)
        rates.append(fl / dt / 1e12)
        if time.perf_counter() - t_start > 2 * budget_s:
            break
    return {"value": round(statistics.median(rates), 5), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": (f"stock torch fp32 F.conv3d + conv3d_weight + conv3d_input on CPU (the reference's "
                       f"CPU path, conv3d_wmma.py:1437-1438,1299-1314) over every trunk layer at batch 1 and "
                       f"{frac_d:.4g} of the depth; median of {len(rates)} passes; os.cpu_count()="
                       f"{os.cpu_count()}")}


def run_reference_arm(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    frac = 1 / 32
    for _ in range(args.warmup):
        cpu_sample_pass(TRUNK, frac)
    fl_tot, t_tot = 0.0, 0.0
    for _ in range(args.steps):
        fl, dt = cpu_sample_pass(TRUNK, frac)
        fl_tot += fl
        t_tot += dt
    val = fl_tot / t_tot / 1e12
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 5), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t_tot / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "trunk sweep (BASELINE configs[1]) fwd+dW+dX, CPU sample",
                   "batch": 1, "depth_fraction": frac, "layers": [t[0] for t in TRUNK]},
        "cpu_baseline": {"value": round(val, 5), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": (f"each step: stock torch fp32 conv3d fwd+dW+dX on CPU (the reference's CPU "
                                    f"path) over every trunk layer at batch 1 and {frac:.4g} of the depth")},
        "e2e": {"value": round(val, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
class Layer:
    def __init__(self, spec, device, seed):
        import torch.nn as nn
        self.name, self.cin, self.cout, self.spatial, self.k = spec
        self.pad = (self.k - 1) // 2
        d, h, w = self.spatial
        g = torch.Generator(device=device).manual_seed(seed)
        cl = torch.channels_last_3d
        self.x = torch.randn(BATCH, self.cin, d, h, w, device=device, generator=g).to(
            torch.bfloat16).contiguous(memory_format=cl)
        self.go = torch.randn(BATCH, self.cout, d, h, w, device=device, generator=g).to(
            torch.bfloat16).contiguous(memory_format=cl)
        conv = nn.Conv3d(self.cin, self.cout, self.k, padding=self.pad)
        self.w = conv.weight.detach().to(device=device, dtype=torch.bfloat16)
        self.b = conv.bias.detach().to(device=device, dtype=torch.bfloat16)
        self.flops = layer_flops(self.cin, self.cout, self.spatial, self.k)


def run_step(layers, reducer, ev=None, legs=("fwd", "dw", "dx")):
    """fwd, dW(+db) and dX of every layer through the package's launch path."""
    cw = sys.modules["rdna4_conv3d.conv3d_wmma"]
    p3 = lambda p: (p, p, p)  # noqa: E731
    outs = []
    pending = []
    for i, L in enumerate(layers):
        y = dw = db = dx = handle = None
        if ev is not None:
            ev[i][0].record()
        if "fwd" in legs:
            y = cw._launch_fwd(L.x, L.w, L.b, p3(L.pad))
        if ev is not None:
            ev[i][1].record()
        if "dw" in legs:
            dw, db = cw._launch_wgrad(L.x, L.go, L.w.shape, p3(L.pad), True)
            handle = reducer.reduce_async([dw, db]) if reducer is not None else None
        if ev is not None:
            ev[i][2].record()
        if "dx" in legs:
            dx = cw._launch_dgrad(L.go, L.w, L.x.shape, p3(L.pad))
        if ev is not None:
            ev[i][3].record()
        if handle is not None:
            pending.append(handle)
        outs.append((y, dw, db, dx))
    # the reductions ran on a side stream under the later legs; the step
    # waits for them once, at its end
    for handle in pending:
        handle.wait()
    return outs


class TLayer:
    def __init__(self, spec, device, seed):
        import torch.nn as nn
        self.name, self.cin, self.cout, self.spatial = spec
        d, h, w = self.spatial
        g = torch.Generator(device=device).manual_seed(seed)
        cl = torch.channels_last_3d
        self.x = torch.randn(BATCH, self.cin, d, h, w, device=device, generator=g).to(
            torch.bfloat16).contiguous(memory_format=cl)
        self.go = torch.randn(BATCH, self.cout, 2 * d, 2 * h, 2 * w, device=device, generator=g).to(
            torch.bfloat16).contiguous(memory_format=cl)
        conv = nn.ConvTranspose3d(self.cin, self.cout, 2, stride=2)
        self.w = conv.weight.detach().to(device=device, dtype=torch.bfloat16)
        self.b = conv.bias.detach().to(device=device, dtype=torch.bfloat16)
        self.flops = 2.0 * BATCH * d * h * w * self.cin * self.cout * 8


def time_tconv(device, steps, warmup, peaks, names=None):
    """fwd / dX / dW(+db) of BASELINE configs[2] through the package's launch
    path, CUDA events per leg; per leg: us, TFLOP/s and HBM GB/s of the
    minimum bytes against the measured copy bandwidth."""
    cw = sys.modules["rdna4_conv3d.conv3d_wmma"]
    layers = [TLayer(spec, device, seed=500 + i) for i, spec in enumerate(TCONV) if names is None or spec[0] in names]

    def step(evs=None):
        for i, L in enumerate(layers):
            if evs is not None:
                evs[i][0].record()
            cw.transpose_k2s2_fwd(L.x, L.w, L.b)
            if evs is not None:
                evs[i][1].record()
            cw.transpose_k2s2_dx(L.x.shape, L.w, L.go)
            if evs is not None:
                evs[i][2].record()
            cw.transpose_k2s2_dw(L.x, L.w.shape, L.go, True)
            if evs is not None:
                evs[i][3].record()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    # a step is ~0.2 ms: keep warming up for at least 0.25 s so that a fresh
    # process is timed after the SM clocks have ramped, not during the ramp
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < 0.25:
        step()
        torch.cuda.synchronize()
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in layers] for _ in range(steps)]
    for s_ in range(steps):
        step(evs[s_])
    torch.cuda.synchronize()
    from rdna4_conv3d import _native
    rows = []
    for i, L in enumerate(layers):
        desc = _native.make_desc(BATCH, *L.spatial, L.cin, L.cout, 2, (0, 0, 0), torch.bfloat16, 0)
        row = {"layer": L.name, "gflop_per_leg": round(L.flops / 1e9, 3)}
        for j, (leg, code) in enumerate((("fwd", _native.LEG_TFWD), ("dx", _native.LEG_TDX),
                                         ("dw", _native.LEG_TDW))):
            ms = sum(ev[i][j].elapsed_time(ev[i][j + 1]) for ev in evs) / steps
            gbs = tconv_bytes(L.cin, L.cout, L.spatial, leg) / (ms / 1e3) / 1e9
            row[leg + "_us"] = round(ms * 1e3, 2)
            row[leg + "_tflops"] = round(L.flops / (ms / 1e3) / 1e12, 2)
            row[leg + "_hbm_gbs"] = round(gbs, 1)
            row[leg + "_hbm_frac"] = round(gbs / peaks["hbm_gbs"], 4)
            row[leg + "_kernel"] = "tcgen05" if _native.plan_kernel(desc, code) == _native.KERNEL_TC else "simt"
        rows.append(row)
    return rows


def run_e2e(layers, host, steps, warmup, world):
    """Public-API legs with inputs copied from pinned host memory and results
    read back every step (wmma_fwd / wmma_dw / wmma_dx).

    Three streams: host->device copies of a layer's x and dY run on one copy
    stream, the three legs on the compute stream, the device->host reads of
    y, dX and dW on a second copy stream, ordered by events, so layer i's
    uploads and layer i-1's downloads overlap layer i's kernels. The bound is
    the PCIe link: the step moves h2d + d2h bytes, one direction each.
    """
    from rdna4_conv3d import wmma_dw, wmma_dx, wmma_fwd
    h2d = sum(hx.numel() * 2 + hg.numel() * 2 for hx, hg, _ in host)
    d2h = 0
    for L in layers:
        d2h += L.x.numel() * 2 // L.cin * L.cout + L.x.numel() * 2 + L.w.numel() * 2
    out_bufs = []
    for L in layers:
        cl = torch.channels_last_3d
        yb = torch.empty((BATCH, L.cout) + L.spatial, dtype=torch.bfloat16, pin_memory=True, memory_format=cl)
        dxb = torch.empty(L.x.shape, dtype=torch.bfloat16, pin_memory=True, memory_format=cl)
        dwb = torch.empty(L.w.shape, dtype=torch.bfloat16, pin_memory=True)
        out_bufs.append((yb, dxb, dwb))
    # device input buffers, one pair per layer, refilled every step
    dev_in = [(torch.empty_like(hx, device="cuda"), torch.empty_like(hg, device="cuda")) for hx, hg, _ in host]
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    n = len(layers)
    uploaded = [torch.cuda.Event() for _ in range(n)]
    consumed = [torch.cuda.Event() for _ in range(n)]
    computed = [torch.cuda.Event() for _ in range(n)]
    for e in consumed:
        e.record(comp)
    cl = torch.channels_last_3d

    def step():
        for i, (L, (hx, hg, _), (yb, dxb, dwb), (dx_in, dg_in)) in enumerate(zip(layers, host, out_bufs, dev_in)):
            with torch.cuda.stream(up):
                up.wait_event(consumed[i])           # last step's kernels are done with the buffers
                dx_in.copy_(hx, non_blocking=True)
                dg_in.copy_(hg, non_blocking=True)
                uploaded[i].record(up)
            comp.wait_event(uploaded[i])
            x = dx_in.contiguous(memory_format=cl)       # already NDHWC: no copy
            go = dg_in.contiguous(memory_format=cl)
            y = wmma_fwd(x, L.w, L.b, 1, L.pad)
            dw = wmma_dw(x, L.w, go, 1, L.pad)
            dx = wmma_dx(x, L.w, go, 1, L.pad)
            consumed[i].record(comp)
            computed[i].record(comp)
            with torch.cuda.stream(down):
                down.wait_event(computed[i])
                yb.copy_(y, non_blocking=True)
                dxb.copy_(dx, non_blocking=True)
                dwb.copy_(dw, non_blocking=True)
            for t in (y, dw, dx, x, go):
                t.record_stream(down)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    up.wait_stream(comp)
    for _ in range(steps):
        step()
    comp.wait_stream(down)
    comp.wait_stream(up)
    e1.record(comp)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    barrier(world)
    return ms, h2d, d2h


def pcie_floor_ms(h2d, d2h, probe_bytes=512 << 20):
    """Time of the step's copies alone at the link's measured rate: one pinned
    buffer copied host->device and another device->host at the same time."""
    hu = torch.empty(probe_bytes, dtype=torch.uint8, pin_memory=True)
    hd = torch.empty(probe_bytes, dtype=torch.uint8, pin_memory=True)
    du = torch.empty(probe_bytes, dtype=torch.uint8, device="cuda")
    dd = torch.empty(probe_bytes, dtype=torch.uint8, device="cuda")
    su, sd = torch.cuda.Stream(), torch.cuda.Stream()
    best_u = best_d = 0.0
    for _ in range(3):
        eu = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ed = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize()
        eu[0].record(su)
        ed[0].record(sd)
        with torch.cuda.stream(su):
            du.copy_(hu, non_blocking=True)
        with torch.cuda.stream(sd):
            hd.copy_(dd, non_blocking=True)
        eu[1].record(su)
        ed[1].record(sd)
        torch.cuda.synchronize()
        best_u = max(best_u, probe_bytes / (eu[0].elapsed_time(eu[1]) / 1e3))
        best_d = max(best_d, probe_bytes / (ed[0].elapsed_time(ed[1]) / 1e3))
    return max(h2d / best_u, d2h / best_d) * 1e3, best_u / 1e9, best_d / 1e9


# ---------------------------------------------------------------------------
# UNet3D training step
# ---------------------------------------------------------------------------
UNET_SPATIAL = (64, 128, 128)
DEPTH_SHARD_SPATIAL = (128, 256, 256)


def _unet_step_fn(net, opt):
    from rdna4_conv3d.losses import cross_entropy

    def step(x, tgt, loss_scale=1.0):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = cross_entropy(net(x), tgt) * loss_scale
        loss.backward()
        opt.step()
        return loss.detach()
    return step


def _graph_step(net, opt, x, tgt, warmup, loss_scale=1.0):
    """Capture one whole training step (forward, backward, Adam) in a CUDA
    graph over static input / label buffers; returns (replay, loss buffer).
    Warm-up runs eagerly on a side stream first (plan tuning, NCCL set-up)."""
    from rdna4_conv3d.losses import cross_entropy
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(max(warmup, 3)):
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = cross_entropy(net(x), tgt) * loss_scale
            loss.backward()
            opt.step()
    # the last warm-up loss holds its autograd graph, whose gradient
    # accumulators would keep the side stream as their stream during capture
    del loss
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    opt.zero_grad(set_to_none=True)
    with torch.cuda.graph(g):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            static_loss = cross_entropy(net(x), tgt) * loss_scale
        static_loss.backward()
        opt.step()
    return g, static_loss


def time_unet(dev, base, batch, steps, warmup, world, rank, graph=False):
    """fwd + bwd + Adam of UNet3D (AMP bf16) at `batch` samples per GPU,
    batch-sharded data parallel over the ranks (GradSync: bucketed gradient
    all-reduce overlapped with the backward pass). Device time with CUDA
    events (max over ranks), then the same steps end to end: input and labels
    copied from pinned host memory and the loss read back every step.
    ``graph``: the step is captured once in a CUDA graph and replayed (the
    host then only launches the graph)."""
    from rdna4_conv3d import _native
    from rdna4_conv3d.distributed import GradSync
    from rdna4_conv3d.unet3d import conv_flops_per_sample, unet3d
    cl = torch.channels_last_3d
    torch.manual_seed(0)
    net = unet3d(base, wmma=True, device=dev)
    sync = GradSync(net) if world > 1 else None
    opt = torch.optim.Adam(net.parameters(), lr=1e-3, fused=True, capturable=graph)
    step = _unet_step_fn(net, opt)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(batch, 1, *UNET_SPATIAL, device=dev, generator=g).contiguous(memory_format=cl)
    tgt = torch.randint(0, 4, (batch,) + UNET_SPATIAL, device=dev, generator=g)
    if graph:
        cg, static_loss = _graph_step(net, opt, x, tgt, warmup)

        def step(xx, tt, loss_scale=1.0):  # noqa: F811  (graphed step: refill the static inputs, replay)
            if xx is not x:
                x.copy_(xx, non_blocking=True)
                tgt.copy_(tt, non_blocking=True)
            cg.replay()
            return static_loss.detach()
    for _ in range(max(warmup, 3)):
        step(x, tgt)
    torch.cuda.synchronize()
    barrier(world)
    n0 = _native.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        loss = step(x, tgt)
    e1.record()
    host_ms = (time.perf_counter() - h0) * 1e3 / steps
    torch.cuda.synchronize()
    launches = (_native.launch_count() - n0) // steps
    ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    barrier(world)

    # end to end: pinned host input/labels in, loss out, every step
    hx = torch.empty(x.shape, dtype=x.dtype, pin_memory=True, memory_format=cl)
    ht = torch.empty(tgt.shape, dtype=tgt.dtype, pin_memory=True)
    hx.copy_(x)
    ht.copy_(tgt)
    hl = torch.empty(steps, dtype=torch.float32, pin_memory=True)
    torch.cuda.synchronize()
    barrier(world)
    e0.record()
    for i in range(steps):
        xd = hx.to(dev, non_blocking=True)
        td = ht.to(dev, non_blocking=True)
        hl[i:i + 1].copy_(step(xd, td).float().reshape(1), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1), world) / steps
    barrier(world)
    flops = 3.0 * conv_flops_per_sample(net, UNET_SPATIAL) * batch * world
    res = {"base": base, "input": [batch, 1, *UNET_SPATIAL], "batch_per_gpu": batch, "global_batch": batch * world,
           "cuda_graph": bool(graph),
           "ms_per_step": round(ms, 3), "ms_per_sample": round(ms / (batch * world), 3),
           "conv_tflops": round(flops / (ms / 1e3) / 1e12, 2), "host_issue_ms_per_step": round(host_ms, 3),
           "e2e_ms_per_step": round(ms_e2e, 3), "e2e_ms_per_sample": round(ms_e2e / (batch * world), 3),
           "h2d_bytes_per_step": int(hx.numel() * hx.element_size() + ht.numel() * ht.element_size()),
           "d2h_bytes_per_step": 4,
           "native_launches_per_step": None if graph else int(launches),
           "loss_last": round(float(hl[-1]), 5)}
    if graph:
        del cg
    if sync is not None:
        sync.remove()
    del net, opt, x, tgt
    torch.cuda.empty_cache()
    return res


def time_depth_shard(dev, base, steps, warmup, world, rank, graph=False):
    """One 1x1x128x256x256 volume per step, D-sharded over the ranks (halo
    exchange per k3 conv, whole-volume BatchNorm statistics); on one GPU the
    plain unsharded model. ms per sample = per step. ``graph``: the step
    (halo exchanges and gradient all-reduces included) is captured once in a
    CUDA graph and replayed."""
    import torch.distributed as dist

    from rdna4_conv3d.distributed import GradSync, depth_shard_model
    from rdna4_conv3d.unet3d import unet3d
    cl = torch.channels_last_3d
    torch.manual_seed(0)
    net = unet3d(base, wmma=True, device=dev)
    sync = None
    if world > 1:
        sync = GradSync(depth_shard_model(net), average=False)
    opt = torch.optim.Adam(net.parameters(), lr=1e-3, fused=True, capturable=graph)
    step = _unet_step_fn(net, opt)
    d, h, w = DEPTH_SHARD_SPATIAL
    dl = d // world
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(1, 1, d, h, w, device=dev, generator=g)[:, :, rank * dl:(rank + 1) * dl]
    x = x.contiguous(memory_format=cl)
    tgt = torch.randint(0, 4, (1, d, h, w), device=dev, generator=g)[:, rank * dl:(rank + 1) * dl].contiguous()
    cg = None
    if graph:
        cg, static_loss = _graph_step(net, opt, x, tgt, warmup, 1.0 / world)

        def step(xx, tt, loss_scale=1.0):  # noqa: F811  (graphed step)
            cg.replay()
            return static_loss.detach()
    for _ in range(max(warmup, 3)):
        step(x, tgt, 1.0 / world)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        loss = step(x, tgt, 1.0 / world)
    e1.record()
    host_ms = (time.perf_counter() - h0) * 1e3 / steps
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    loss = loss.clone()
    if world > 1:
        dist.all_reduce(loss)
    barrier(world)
    res = {"base": base, "volume": [1, 1, d, h, w], "planes_per_gpu": dl, "cuda_graph": bool(graph),
           "ms_per_sample": round(ms, 3), "host_issue_ms_per_step": round(host_ms, 3),
           "loss_last": round(float(loss), 5)}
    if cg is not None:
        del cg
    if sync is not None:
        sync.remove()
    del net, opt, x, tgt
    torch.cuda.empty_cache()
    return res


def cpu_unet_baseline(base=24, spatial=(16, 32, 32), budget_s=10.0):
    """Stock fp32 UNet3D fwd + bwd + Adam on the host cores (the reference's
    CPU path: nn.Conv3d on CPU tensors), batch 1 on a reduced volume; the
    per-sample time is scaled to the full 64x128x128 volume by the ratio of
    conv FLOPs."""
    import torch.nn.functional as F

    from rdna4_conv3d.unet3d import conv_flops_per_sample, unet3d
    torch.manual_seed(0)
    net = unet3d(base, wmma=False)
    opt = torch.optim.Adam(net.parameters(), lr=1e-3)
    x = torch.randn(1, 1, *spatial).contiguous(memory_format=torch.channels_last_3d)
    tgt = torch.randint(0, 4, (1,) + spatial)

    def step():
        opt.zero_grad(set_to_none=True)
        F.cross_entropy(net(x), tgt).backward()
        opt.step()
    step()
    times, t_start = [], time.perf_counter()
    while len(times) < 5 or (time.perf_counter() - t_start < budget_s and len(times) < 30):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    scale = conv_flops_per_sample(net, UNET_SPATIAL) / conv_flops_per_sample(net, spatial)
    return {"ms_per_sample": round(med * scale * 1e3, 1), "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"stock torch fp32 UNet3D base {base} fwd+bwd+Adam on CPU, batch 1 at "
                       f"{'x'.join(map(str, spatial))}, median of {len(times)} steps, scaled to 64x128x128 by "
                       f"conv FLOPs (x{scale:.0f})")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-tconv", action="store_true", help="skip the ConvTranspose3d k2s2 legs (configs[2])")
    ap.add_argument("--only", default=None, help="run one trunk layer, e.g. 'k3 24->24', or one transpose-conv "
                                                 "layer, e.g. 'T k2s2 48->24' (profiling)")
    ap.add_argument("--legs", default="fwd,dw,dx", help="comma list of legs to run (profiling)")
    ap.add_argument("--no-unet", action="store_true", help="skip the UNet3D training steps (configs[3]/[4])")
    ap.add_argument("--no-depth-shard", action="store_true", help="skip the depth-sharded volume")
    ap.add_argument("--unet-only", action="store_true", help="only the UNet3D steps (one JSON line)")
    ap.add_argument("--no-graph", action="store_true", help="skip the CUDA-graph UNet steps (eager depth shard)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        return run_reference_arm(args)

    world, rank, local = init_dist(args.gpus)
    dev = torch.device("cuda", local)
    from rdna4_conv3d import _native
    from rdna4_conv3d.conv3d_wmma import conv3d_kernels
    _native.lib()

    if args.unet_only:
        u_steps = max(3, args.steps)
        res = {"base24": time_unet(dev, 24, BATCH, u_steps, args.warmup, world, rank)}
        if not args.no_graph:
            res["base24_graph"] = time_unet(dev, 24, BATCH, u_steps, args.warmup, world, rank, graph=True)
        if not args.no_depth_shard:
            res["base32"] = time_unet(dev, 32, BATCH, u_steps, args.warmup, world, rank)
            res["depth_shard_base32"] = time_depth_shard(dev, 32, max(2, min(args.steps, 5)), 3, world, rank,
                                                         graph=not args.no_graph)
        if rank == 0:
            print(json.dumps({"impl": "ours", "n_gpus": world, "unet": res}), flush=True)
        if world > 1:
            import torch.distributed as dist
            barrier(world)
            dist.destroy_process_group()
        return 0

    if args.only in [t[0] for t in TCONV]:
        # one transpose-conv layer (profiling): its legs only, one JSON line of per-leg times
        rows = time_tconv(dev, args.steps, args.warmup, load_peaks(), names=[args.only])
        if rank == 0:
            print(json.dumps({"impl": "ours", "only": args.only, "tconv_layers": rows}), flush=True)
        return 0

    specs = [t for t in TRUNK if args.only is None or t[0] == args.only]
    if not specs:
        raise SystemExit(f"unknown layer {args.only!r}; choose from {[t[0] for t in TRUNK]}")
    legs = tuple(args.legs.split(","))
    layers = [Layer(spec, dev, seed=1000 * rank + i) for i, spec in enumerate(specs)]
    reducer = None
    if world > 1:
        from rdna4_conv3d.distributed import GradAllReducer
        reducer = GradAllReducer()

    step_flops = sum(len(legs) * L.flops for L in layers)
    # the clocks sampler starts before the warm-up, so the GPU does not sit
    # idle (and drop its clocks) between the warm-up and the timed steps
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    for _ in range(args.warmup):
        run_step(layers, reducer, legs=legs)
    torch.cuda.synchronize()

    # per step, per layer: events around the fwd / dW / dX legs; the host runs
    # ahead of the GPU (no synchronize inside the timed loop), so a leg's time
    # is the GPU's and holds no host launch latency
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in layers]
           for _ in range(args.steps)]
    leg_ms = [[0.0, 0.0, 0.0] for _ in layers]
    barrier(world)
    torch.cuda.synchronize()
    n_launch0 = _native.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    h0 = time.perf_counter()
    for s in range(args.steps):
        run_step(layers, reducer, evs[s], legs=legs)
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps  # host time to issue a step
    t1.record()
    torch.cuda.synchronize()
    for ev in evs:
        for i in range(len(layers)):
            for j in range(3):
                leg_ms[i][j] += ev[i][j].elapsed_time(ev[i][j + 1])
    launches = _native.launch_count() - n_launch0
    clocks = sampler.stop()
    ms_total = max_over_ranks(t0.elapsed_time(t1), world)
    barrier(world)

    ms_step = ms_total / args.steps
    value = step_flops * world * args.steps / (ms_total / 1e3) / 1e12
    peaks = load_peaks()

    # per-layer breakdown (this rank) and the dominant kernel
    breakdown = []
    dom = None
    for L, lm in zip(layers, leg_ms):
        fam = conv3d_kernels((BATCH, L.cin) + L.spatial, L.cout, L.k, L.pad)
        row = {"layer": L.name, "gflop_per_leg": round(L.flops / 1e9, 3)}
        for j, leg in enumerate(("fwd", "dw", "dx")):
            if leg not in legs:
                continue
            ms = lm[j] / args.steps
            row[leg + "_us"] = round(ms * 1e3, 2)
            row[leg + "_tflops"] = round(L.flops / (ms / 1e3) / 1e12, 2) if ms > 0 else None
            row[leg + "_kernel"] = fam[leg]
            if dom is None or ms > dom[0]:
                dom = (ms, L, leg)
        breakdown.append(row)
    ms_dom, Ld, leg_d = dom
    ai = Ld.flops / layer_bytes(Ld.cin, Ld.cout, Ld.spatial, Ld.k, leg=leg_d)
    # the legs run inside a ms-scale step at full SM clock (the clocks record
    # shows it), so the denominator is the burst GEMM peak; the sustained,
    # power-capped figure is kept beside it for reference
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    traffic_tab = load_traffic()
    tkey = f"{Ld.name} {leg_d}"
    if ai >= ridge:
        achieved = Ld.flops / (ms_dom / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                "peak_sustained": peaks["bf16_tflops_sustained"],
                "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4)}
    else:
        achieved = layer_bytes(Ld.cin, Ld.cout, Ld.spatial, Ld.k, leg=leg_d) / (ms_dom / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4)}
    roof["traffic"] = traffic_tab.get(tkey)
    roof["kernel"] = f"{tkey} ({breakdown[layers.index(Ld)][leg_d + '_kernel']})"
    roof["peak_src"] = f"{peaks['src']} (burst bf16 GEMM / copy bandwidth)"

    e2e = None
    if not args.no_e2e and args.only is None and len(legs) == 3:
        host = []
        for L in layers:
            # pinned host copies in the kernels' NDHWC layout (channels_last_3d strides kept)
            cl = torch.channels_last_3d
            hx = torch.empty(L.x.shape, dtype=L.x.dtype, pin_memory=True, memory_format=cl)
            hg = torch.empty(L.go.shape, dtype=L.go.dtype, pin_memory=True, memory_format=cl)
            hx.copy_(L.x)
            hg.copy_(L.go)
            host.append((hx, hg, None))
        e2e_steps = max(1, min(args.steps, 3))
        ms_e2e, h2d, d2h = run_e2e(layers, host, e2e_steps, 1, world)
        floor_ms, bw_u, bw_d = pcie_floor_ms(h2d, d2h)
        e2e = {"value": round(step_flops * world * e2e_steps / (ms_e2e / 1e3) / 1e12, 3), "unit": "TFLOP/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "ms_per_step": round(ms_e2e / e2e_steps, 3),
               "path": "public API wmma_fwd/wmma_dw/wmma_dx, pinned host inputs copied in and results copied "
                       "back inside the timed region; uploads, kernels and downloads on three streams",
               "pcie_floor_ms": round(floor_ms, 3), "pcie_gbs_h2d_d2h": [round(bw_u, 1), round(bw_d, 1)]}

    tconv = None
    if args.only is None and len(legs) == 3 and not args.no_tconv:
        tconv = time_tconv(dev, min(args.steps, 5), 2, peaks)

    unet = None
    if args.only is None and len(legs) == 3 and not args.no_unet:
        # BASELINE configs[3] (base 24, 4 samples per GPU) at every N, and
        # configs[4] (base 32, 4 per GPU = global batch 32 at N = 8; and the
        # depth-sharded 1x1x128x256x256 volume)
        u_steps = max(3, min(args.steps, 10))
        unet = {"base24": time_unet(dev, 24, BATCH, u_steps, 3, world, rank),
                "base32": time_unet(dev, 32, BATCH, u_steps, 3, world, rank)}
        if not args.no_graph:
            # the whole step (gradient all-reduces included at N > 1) in one
            # CUDA graph: the eager step is bound by the host's issue rate
            unet["base24_graph"] = time_unet(dev, 24, BATCH, u_steps, 3, world, rank, graph=True)
            unet["base32_graph"] = time_unet(dev, 32, BATCH, u_steps, 3, world, rank, graph=True)
        if not args.no_depth_shard:
            unet["depth_shard_base32"] = time_depth_shard(dev, 32, max(2, min(args.steps, 5)), 3, world, rank,
                                                          graph=not args.no_graph)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.only is None:
        cpu = cpu_baseline(TRUNK)
        if unet is not None:
            unet["cpu_baseline_base24"] = cpu_unet_baseline(24)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "trunk sweep (BASELINE configs[1]): k3 1->24, 24->24, 48->48, 96->96, "
                                   "192->192 and k1 48->24, 96->48, 192->96, fwd+dW+dX",
                       "batch_per_gpu": BATCH, "global_batch": BATCH * world, "dtype": "bf16",
                       "parallelism": f"dp{world}" if world > 1 else "single",
                       "l2": "no flush: each step streams ~1.7 GB of activations, far above the 126 MB L2"},
            "gflop_per_step_per_gpu": round(step_flops / 1e9, 2),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": int(launches),
            "clocks": clocks, "host_issue_ms_per_step": round(host_ms, 3), "layers": breakdown,
            "tconv_layers": tconv,
            "tconv_note": "BASELINE configs[2] (ConvTranspose3d k2s2, batch 4, bf16), timed after the trunk "
                          "with CUDA events per leg; not part of value; hbm_frac against the measured copy "
                          "bandwidth for the minimum bytes of each leg",
            "unet": unet,
            "unet_note": "BASELINE configs[3]/[4]: UNet3D fwd+bwd+Adam (AMP bf16, fused Adam), seeded synthetic "
                         "N(0,1) input and uniform labels, random init; ms_per_sample = device step time (max "
                         "over ranks) / global batch; e2e_* copies input and labels from pinned host memory and "
                         "reads the loss back every step; not part of value",
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        barrier(world)
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
