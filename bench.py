#!/usr/bin/env python
"""DDPM hot-path benchmark (driver contract: one JSON line on rank 0).

Workload: DDPM forward+backward at B=1 per GPU,
C=64, 256x256, K=3, dilations (1,3,5), seeded default init, x, y and the
upstream gradient ~ N(0,1), synthetic data. One "step" = forward + backward of
the whole module (generator/filter kernels and the 3x3 fuse conv, all on this
library's kernels), plus, for N>1 GPUs, the NCCL gradient all-reduce of the
batch-sharded data-parallel step (per-GPU batch fixed => weak scaling).

Timing: W warm-up steps, then exactly K timed steps bracketed by barrier +
synchronize; each step is timed with CUDA events on the launching stream and
an L2 flush (a 256 MiB write) runs between steps outside the events. The
device-time ``value`` replays the step as one CUDA graph with inputs resident
in HBM; ``e2e`` runs the public API eagerly with the H2D copy of x, y and the
upstream gradient from pinned host memory and the D2H read of the loss inside
the timed region (the gradient's copy on a side stream overlapping the
forward; the Python collector paused while timing). The max over ranks is
reported.

``--impl reference`` times the reference's CPU algorithm (the oracle port of
``unfold_impl.DDPM`` in oracle/) on this host's cores for the same config.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "DDPM fwd+bwd ms @B1 C64 256² K3; dyn-filter HBM TB/s vs ~8 TB/s peak"
WORKLOAD = "configs[3] DDPM training step (fwd+bwd)"  # both arms, same workload
C, H, W, K = 64, 256, 256, 3
DILATIONS = (1, 3, 5)
# 256^2 K3 FP32 fused training step, RTX 5090 (README.md:161-162).
PUBLISHED_FP32_MS = 3.66
L2_FLUSH_BYTES = 256 * 1024**2
DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16}
DTYPE_TAG = {"fp32": "f32", "bf16": "bf16"}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--dtype", choices=list(DTYPES), default="fp32",
                    help="headline dtype (the other one is reported under 'extra')")
    ap.add_argument("--batch", type=int, default=1, help="per-GPU batch")
    ap.add_argument("--path", choices=["auto", "fused", "materialised"], default="auto")
    ap.add_argument("--no-graph", action="store_true", help="time eager steps for 'value'")
    ap.add_argument("--skip-extra", action="store_true", help="headline dtype only")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU oracle baseline leg")
    ap.add_argument("--profile-kernel", default=None,
                    help="only launch this library kernel (ncu capture target)")
    ap.add_argument("--profile-iters", type=int, default=3)
    return ap.parse_args(argv)


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi clocks/throttle sampling every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [v.strip() for v in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": smax,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# --------------------------------------------------------------- workload --
def build_model(dtype, path, device):
    from dynamicconvolutionoperator_b200 import DDPM
    from dynamicconvolutionoperator_b200 import _kernels

    torch.manual_seed(0)  # identical replicated init on every rank
    fused = {"auto": None, "fused": True, "materialised": False}[path]
    model = DDPM(C, K, fused_generator_training=fused).to(device=device, dtype=dtype)
    probe = torch.empty((1, C, H, W), dtype=dtype, device="meta")
    taken = "fused" if (model._use_fused_training(probe) and
                        _kernels.fused_generator_supported(C, K, dtype)) else "materialised"
    return model, taken


def make_inputs(batch, dtype, rank):
    gen = torch.Generator().manual_seed(1000 + rank)
    shape = (batch, C, H, W)
    return [torch.randn(shape, generator=gen).to(dtype) for _ in range(3)]  # x, y, upstream


def step_fn(model, x, y, g, allreduce):
    # x and y take part in autograd (dX and dY are computed), as in the
    # reference's training benchmarks (gpu_bench.py:275-300).
    # g is the upstream gradient of the module output (d loss / d out for
    # loss = <out, g>): backward starts from it directly, and the loss value
    # read back to the host is the one dot product
    x = x.detach().requires_grad_(True)
    y = y.detach().requires_grad_(True)
    out = model(x, y)
    out.backward(g)
    if allreduce is not None:
        allreduce()
    with torch.no_grad():
        return torch.dot(out.reshape(-1), g.reshape(-1)).float()


def time_steps(run, steps, flush, stream):
    """Per-step CUDA-event durations (ms) with an L2 flush between steps."""
    times = []
    for _ in range(steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run()
        e1.record(stream)
        times.append((e0, e1))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


def measure_dtype(args, dtype, device, rank, world, dist, timed_clocks=False):
    from dynamicconvolutionoperator_b200 import _lib
    from dynamicconvolutionoperator_b200.data_parallel import GradAllReducer

    model, taken = build_model(dtype, args.path, device)
    hx, hy, hg = [t.pin_memory() for t in make_inputs(args.batch, dtype, rank)]
    x, y, g = [t.to(device) for t in (hx, hy, hg)]
    reducer = GradAllReducer(model) if world > 1 else None
    allreduce = reducer.all_reduce if reducer is not None else None
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def zero():
        for p in model.parameters():
            p.grad = None

    # eager warm-up, and the number of library launches per step
    for _ in range(max(args.warmup, 1)):
        zero()
        step_fn(model, x, y, g, allreduce)
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    zero()
    step_fn(model, x, y, g, allreduce)
    torch.cuda.synchronize()
    launches_per_step = _lib.launch_count() - n0

    use_graph = not args.no_graph
    if use_graph:
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                zero()
                step_fn(model, x, y, g, None)
        stream.wait_stream(side)
        zero()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step_fn(model, x, y, g, None)

        def run():
            graph.replay()
            if allreduce is not None:
                allreduce()
    else:
        def run():
            zero()
            step_fn(model, x, y, g, allreduce)

    for _ in range(args.warmup):
        run()
    sampler = ClockSampler(device.index if device.index is not None else 0)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    if timed_clocks:
        sampler.start()
    times = time_steps(run, args.steps, flush, stream)
    clocks = sampler.stop() if timed_clocks else None
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = sum(times) / len(times)

    # ---- end to end through the public API: H2D inputs, fwd+bwd, D2H loss ----
    # x and y are copied on the compute stream (the forward starts with them);
    # the upstream gradient g is copied on a side stream that starts once those
    # two copies are done (sharing the PCIe link with them would only delay the
    # forward) and overlaps the forward, as a training loop's input pipeline
    # would; the compute stream waits for it before the loss, so every copy
    # lies inside the timed region.
    host_loss = torch.empty((), dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(device)

    def e2e_step():
        zero()
        xe = hx.to(device, non_blocking=True)
        ye = hy.to(device, non_blocking=True)
        copy_stream.wait_stream(stream)
        with torch.cuda.stream(copy_stream):
            ge = hg.to(device, non_blocking=True)
        x_ = xe.detach().requires_grad_(True)
        y_ = ye.detach().requires_grad_(True)
        out = model(x_, y_)
        stream.wait_stream(copy_stream)
        ge.record_stream(stream)
        out.backward(ge)
        if allreduce is not None:
            allreduce()
        with torch.no_grad():
            loss = torch.dot(out.reshape(-1), ge.reshape(-1)).float()
        host_loss.copy_(loss, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e2e_times = []
    gc.disable()  # a collector pause inside a timed step is host jitter, not work
    try:
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            e2e_step()
            e1.record(stream)
            e1.synchronize()
            e2e_times.append(e0.elapsed_time(e1))
    finally:
        gc.enable()
    if dist is not None:
        dist.barrier()
    e2e_ms = sum(e2e_times) / len(e2e_times)
    if use_graph:
        del graph
    in_bytes = sum(t.numel() * t.element_size() for t in (hx, hy, hg))
    return {
        "ms": ms,
        "e2e_ms": e2e_ms,
        "h2d_bytes": in_bytes,
        "d2h_bytes": host_loss.element_size(),
        "launches_per_step": launches_per_step,
        "path": taken,
        "clocks": clocks,
        "model": model,
        "inputs": (x, y),
    }


# ---------------------------------------------------------------- roofline --
def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# DRAM bytes (read + write) per launch at this configuration, from the ncu
# captures summarised in profiles/<kernel>_256.md, keyed by (kernel, dtype);
# None where no capture exists. Outputs still resident in L2 when a captured
# launch ends are not counted as writes.
NCU_TRAFFIC_BYTES: dict[tuple[str, str], float] = {
    # staged paths: the main kernel only (the staging copies are HBM-bound
    # passes of their own, profiles/staging_256.md)
    ("gencat_fwd", "torch.float32"): 115258624,
    ("gencat_fwd", "torch.bfloat16"): 42377472,
    ("gencat_bwd_x", "torch.float32"): 91352320,
    ("gencat_bwd_x", "torch.bfloat16"): 45780224,
    ("gencat_bwd_yw", "torch.float32"): 114652928,
    ("gencat_bwd_yw", "torch.bfloat16"): 73122816,
    ("fuseconv_fwd", "torch.float32"): 75615744,
    ("fuseconv_fwd", "torch.bfloat16"): 36270848,
    ("fuseconv_dgrad", "torch.float32"): 27409920,
    ("fuseconv_dgrad", "torch.bfloat16"): 9356288,
    # dout pre-pass + TMA main kernel (the split reduction is not captured)
    ("fuseconv_wgrad", "torch.float32"): 16783872 + 89954560,
    ("fuseconv_wgrad", "torch.bfloat16"): 8395264 + 42037760,
    ("dyncat_fwd", "torch.float32"): 491269632,
    ("dyncat_bwd", "torch.float32"): 466273536 + 593169408,
    ("dyncat_bwd", "torch.bfloat16"): 201383936 + 271141376,
}


def library_kernels(model, x, y, dtype, device):
    """Thunks launching each library kernel of the step on its own, with the
    operands it sees inside the step, and each kernel's roofline work unit:
    (thunk, bound, algorithmic bytes or FLOPs per launch)."""
    from dynamicconvolutionoperator_b200 import _lib

    n = x.shape[0]
    elt = x.element_size()
    ncp = n * C * H * W
    with torch.no_grad():
        taps = model.generator(y).reshape(n, 3, C, K * K, H, W).contiguous()
    out = torch.empty((n, 4 * C, H, W), dtype=dtype, device=device)
    gout = torch.randn((n, 4 * C, H, W), device=device).to(dtype)
    gx = torch.empty_like(x)
    gk = torch.empty_like(taps)
    code = _lib.dtype_code(dtype)
    sh = _lib.stream_handle(device)
    from dynamicconvolutionoperator_b200 import _kernels

    gen_w = model.generator.weight.detach()
    gen_b = model.generator.bias.detach()
    packed = _kernels.pack_generator_weight(gen_w, gen_b, C, K, use_cache=False)
    out2 = torch.empty_like(out)
    gy = torch.empty_like(y)
    gw = torch.empty((3 * C * K * K, C), dtype=dtype, device=device)
    gb = torch.empty(3 * C * K * K, dtype=dtype, device=device)
    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, C, H, W, K))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    gen_flops = 2 * (3 * C * K * K) * C * n * H * W
    from dynamicconvolutionoperator_b200 import _fuseconv

    fuse_w = model.fuse.weight.detach()
    fuse_b = model.fuse.bias.detach()
    fpacked = _fuseconv.pack_fuse_weight(fuse_w, use_cache=False)
    fout = torch.empty_like(x)
    fgout = torch.randn_like(x)
    fgx = torch.empty_like(out)
    fuse_flops = 2 * (4 * C) * C * 9 * n * H * W
    fgw = torch.empty_like(fuse_w)
    fgb = torch.empty_like(fuse_b)
    fws_bytes = int(_lib.load().ddpm_fuseconv_bwd_weight_workspace_bytes(n, 4 * C, C, H, W))
    fws = torch.empty(fws_bytes, dtype=torch.uint8, device=device)
    sy_bytes = int(_lib.load().ddpm_gencat_stage_bytes(n, C, H, W, K, *DILATIONS, code))
    sy = torch.empty(sy_bytes, dtype=torch.uint8, device=device)

    # as in the training step: one staging call (x and y) in the forward, timed with
    # it; the forward, dX and dY + dW read the staged operands
    _lib.call("ddpm_gencat_stage", x.data_ptr(), y.data_ptr(), sy.data_ptr(), sy_bytes, n, C, H,
              W, K, *DILATIONS, code, sh)

    # as in the step: the generator forward also writes the fuse conv's staged
    # planes of its output (C % 8 == 0), so the fuse forward needs no staging
    fp_bytes = int(_lib.load().ddpm_fuseconv_stage_bytes(n, 4 * C, H, W, code))
    fplanes = torch.empty(fp_bytes, dtype=torch.uint8, device=device)

    def fwd():
        _lib.call("ddpm_gencat_stage", x.data_ptr(), y.data_ptr(), sy.data_ptr(), sy_bytes, n, C,
                  H, W, K, *DILATIONS, code, sh)
        _lib.call("ddpm_gencat_fwd_staged_planes", sy.data_ptr(), sy_bytes, packed.data_ptr(),
                  gen_b.data_ptr(), out2.data_ptr(), fplanes.data_ptr(), fp_bytes,
                  n, C, H, W, K, *DILATIONS, code, sh)

    # fuse conv as in the step: the data gradient stages grad_out as operand
    # planes (timed with it); the forward reads the planes the generator wrote
    fwd()
    gp_bytes = int(_lib.load().ddpm_fuseconv_stage_bytes(n, C, H, W, code))
    gplanes = torch.empty(gp_bytes, dtype=torch.uint8, device=device)

    def fuse_fwd():
        _lib.call("ddpm_fuseconv_fwd_staged", fplanes.data_ptr(), fp_bytes, fpacked.data_ptr(),
                  fuse_b.data_ptr(), fout.data_ptr(), n, 4 * C, C, H, W, code, sh)

    def fuse_dgrad():
        _lib.call("ddpm_fuseconv_stage", fgout.data_ptr(), gplanes.data_ptr(), gp_bytes, n, C, H,
                  W, code, sh)
        _lib.call("ddpm_fuseconv_bwd_data_staged", gplanes.data_ptr(), gp_bytes,
                  fpacked.data_ptr(), fgx.data_ptr(), n, 4 * C, C, H, W, code, sh)

    def bwd_x():
        _lib.call("ddpm_gencat_bwd_x_staged", sy.data_ptr(), sy_bytes, packed.data_ptr(),
                  gen_b.data_ptr(), gout.data_ptr(), gx.data_ptr(), n, C, H, W, K, *DILATIONS,
                  code, sh)

    def bwd_yw():
        _lib.call("ddpm_gencat_bwd_yw_staged", sy.data_ptr(), sy_bytes, packed.data_ptr(),
                  gout.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                  ws_bytes, n, C, H, W, K, *DILATIONS, code, sh)

    keep = (taps, out, gout, gx, gk, packed, out2, gy, gw, gb, ws, fpacked, fout, fgout, fgx,
            fgw, fgb, fws, sy, fplanes, gplanes)
    return keep, {
        "fuseconv_fwd": (fuse_fwd, "tensor", fuse_flops),
        "fuseconv_wgrad": (
            lambda: _lib.call("ddpm_fuseconv_bwd_weight", out.data_ptr(), fgout.data_ptr(),
                              fgw.data_ptr(), fgb.data_ptr(), fws.data_ptr(), fws_bytes,
                              n, 4 * C, C, H, W, code, sh),
            "tensor", fuse_flops,
        ),
        "fuseconv_dgrad": (fuse_dgrad, "tensor", fuse_flops),
        "gencat_bwd_x": (bwd_x, "tensor", gen_flops),
        "gencat_bwd_yw": (bwd_yw, "tensor", 2 * gen_flops),
        "gencat_fwd": (fwd, "tensor", 2 * (3 * C * K * K) * C * n * H * W),
        "dyncat_fwd": (
            lambda: _lib.call("ddpm_dyncat_fwd", x.data_ptr(), code, taps.data_ptr(), code,
                              out.data_ptr(), n, C, H, W, K, *DILATIONS, sh),
            "hbm", (3 * K * K + 5) * ncp * elt,
        ),
        "dyncat_bwd": (
            lambda: _lib.call("ddpm_dyncat_bwd", x.data_ptr(), code, taps.data_ptr(),
                              gout.data_ptr(), code, gx.data_ptr(), gk.data_ptr(),
                              n, C, H, W, K, *DILATIONS, sh),
            "hbm", (6 * K * K + 9) * ncp * elt,
        ),
    }


def kernel_roofline(model, x, y, dtype, steps, device):
    """Time the library's kernels of the step in isolation (CUDA events, L2
    flushed before every launch) and return per-kernel roofline entries."""
    hbm, tflops, src = load_peaks()
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    keep, kernels = library_kernels(model, x, y, dtype, device)
    res = {}
    for name, (fn, bound, work) in kernels.items():
        for _ in range(3):
            fn()
        ts = time_steps(fn, max(steps, 5), flush, stream)
        t = sum(ts) / len(ts)
        if bound == "hbm":
            achieved, peak, unit = work / (t * 1e-3) / 1e9, hbm, "GB/s"
        else:
            achieved, peak, unit = work / (t * 1e-3) / 1e12, tflops, "TFLOP/s"
        traffic = NCU_TRAFFIC_BYTES.get((name, str(dtype)))
        res[name] = {
            "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic, "work": work,
            "ms": round(t, 5), "peak_source": src,
        }
    del keep
    return res


def profile_kernel(args):
    """Launch one library kernel ``--profile-iters`` times at the bench config
    (the target of the committed ncu captures; prints nothing but 'ok')."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    dtype = DTYPES[args.dtype]
    model, _ = build_model(dtype, args.path, device)
    x, y, _ = [t.to(device) for t in make_inputs(args.batch, dtype, 0)]
    keep, kernels = library_kernels(model, x, y, dtype, device)
    fn = kernels[args.profile_kernel][0]
    for _ in range(args.profile_iters):
        fn()
    torch.cuda.synchronize()
    del keep
    print("ok")
    return 0


# -------------------------------------------------------------- CPU legs --
def cpu_step_time(dtype, batch, budget_s=15.0, max_steps=10, warmup=1):
    """Oracle (reference CPU algorithm) fwd+bwd ms per full step on host cores."""
    from oracle import ddpm_oracle as orc

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    model = orc.make_model(C, K, dtype=dtype, seed=0)
    x, y, g = orc.make_inputs((batch, C, H, W), dtype=dtype, seed=1000)

    def one():
        xr = x.clone().requires_grad_(True)
        yr = y.clone().requires_grad_(True)
        model.zero_grad(set_to_none=True)
        out = model(xr, yr)
        (out.float() * g.float()).sum().backward()

    for _ in range(warmup):
        one()
    times, t_start = [], time.perf_counter()
    while len(times) < max_steps and (time.perf_counter() - t_start) < budget_s:
        t0 = time.perf_counter()
        one()
        times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), cores, len(times)


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    dtype = DTYPES[args.dtype]
    ms, cores, n = cpu_step_time(dtype, args.batch, budget_s=120.0,
                                 max_steps=max(1, min(args.steps, 10)),
                                 warmup=max(0, min(args.warmup, 1)))
    sample = (f"{n} full fwd+bwd steps (median) of B={args.batch} C={C} {H}x{W} K={K} "
              f"{args.dtype}, oracle port of unfold_impl.DDPM on {cores} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(ms, 3), "unit": "ms",
        "n_gpus": args.gpus, "steps": n, "warmup": min(args.warmup, 1), "ms_per_step": round(ms, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
        "dtype": DTYPE_TAG[args.dtype], "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch_per_gpu": args.batch,
                   "global_batch": args.batch, "channels": C, "height": H, "width": W, "kernel_size": K,
                   "dilations": list(DILATIONS), "parallelism": "cpu"},
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# -------------------------------------------------------------------- main --
def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.profile_kernel:
        return profile_kernel(args)

    # The fuse conv runs in true FP32 for the fp32 step: TF32 would put the
    # output outside the FP32 parity tolerance, which is measured the same way.
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    headline = measure_dtype(args, DTYPES[args.dtype], device, rank, world, dist,
                             timed_clocks=True)
    extra = {}
    if not args.skip_extra:
        other = "bf16" if args.dtype == "fp32" else "fp32"
        m = measure_dtype(args, DTYPES[other], device, rank, world, dist)
        extra[other] = {"ms_per_step": round(m["ms"], 4), "e2e_ms": round(m["e2e_ms"], 4),
                        "path": m["path"]}
        del m
    roof = kernel_roofline(headline["model"], *headline["inputs"], DTYPES[args.dtype],
                           args.steps, device)

    def gather_max(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    ms = gather_max(headline["ms"])
    e2e_ms = gather_max(headline["e2e_ms"])
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cms, cores, n = cpu_step_time(DTYPES[args.dtype], args.batch)
        cpu = {"value": round(cms, 3), "unit": "ms", "cores": cores, "kind": "port",
               "sample": f"{n} full fwd+bwd steps (median) of the same workload, oracle port "
                         f"of unfold_impl.DDPM, {args.dtype}"}
    # dominant kernel among those the headline step launches
    in_step = {"fused": ("gencat_fwd", "gencat_bwd_x", "gencat_bwd_yw"),
               "materialised": ("dyncat_fwd", "dyncat_bwd")}[headline["path"]]
    in_step = in_step + ("fuseconv_fwd", "fuseconv_dgrad", "fuseconv_wgrad")
    dominant = max((k for k in roof if k in in_step), key=lambda k: roof[k]["ms"])
    if rank == 0:
        px = args.batch * world * H * W
        line = {
            "metric": METRIC,
            "value": round(ms, 4),
            "unit": "ms",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": False,
            "scaling": "weak",
            "vs_baseline": round(ms / PUBLISHED_FP32_MS, 4) if args.dtype == "fp32" else None,
            "dtype": DTYPE_TAG[args.dtype],
            "data": "synthetic",
            "config": {
                "workload": WORKLOAD,
                "batch_per_gpu": args.batch, "global_batch": args.batch * world,
                "channels": C, "height": H, "width": W, "kernel_size": K,
                "dilations": list(DILATIONS), "path": headline["path"],
                "parallelism": f"dp{world}", "cuda_graph": not args.no_graph,
                "l2": "flushed between steps (256 MiB write)",
                "cudnn_tf32": bool(torch.backends.cudnn.allow_tf32),
            },
            "mpixel_per_s": round(px / (ms * 1e-3) / 1e6, 2),
            "e2e": {"value": round(e2e_ms, 4), "unit": "ms",
                    "h2d_bytes_per_step": headline["h2d_bytes"],
                    "d2h_bytes_per_step": headline["d2h_bytes"]},
            "gpu_launches": int(headline["launches_per_step"] * args.steps),
            "roofline": {k: v for k, v in roof[dominant].items() if k != "work"}
            | {"kernel": dominant},
            "kernels": roof,
            "clocks": headline["clocks"],
            "cpu_baseline": cpu,
            "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
