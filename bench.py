#!/usr/bin/env python
"""DDPM hot-path benchmark (driver contract: one JSON line on rank 0).

Headline workload: batch-sharded DDPM training,
global batch 64 split over the N ranks (64/N samples per GPU: strong
scaling), C=64, 256x256, K=3, dilations (1,3,5), bf16, seeded default init
replicated on every rank, x, y and the upstream gradient ~ N(0,1), synthetic
data. One "step" = forward + backward of the whole module on the rank's shard
(generator/filter kernels and the 3x3 fuse conv, all on this library's
kernels) plus, for N>1, the NCCL all-reduce (average) of the parameter
gradients, launched from the backward so it overlaps the generator backward.

Also measured and reported under ``extra``: configs[3] (B=1 per GPU, fp32 and
bf16; weak scaling at N>1) with the same step structure, and the per-kernel
rooflines at B=1 in both dtypes (``kernels``, ``kernels_bf16``).

Timing: W warm-up steps, then exactly K timed steps bracketed by barrier +
synchronize; each step is timed with CUDA events on the launching stream and
an L2 flush (a 256 MiB write) runs between steps outside the events. The
device-time ``value`` replays the step (all-reduce included) as one CUDA graph
with inputs resident in HBM; ``e2e`` runs the public API eagerly with the H2D
copy of x, y and the upstream gradient from pinned host memory and the D2H read
of the loss inside the timed region (micro-batches of the shard: the copy of
micro-batch i+1 overlaps the compute of micro-batch i, gradients accumulate,
the all-reduce runs once; the Python collector paused while timing). The max
over ranks is reported.

``--impl reference`` times the reference's CPU algorithm (the oracle port of
``unfold_impl.DDPM`` in oracle/) on this host's cores for the same config: a
bounded sample of one-sample steps, scaled to the global batch.
``--memory`` prints the temporary peak memory of one training step (the
reference's ``gpu_memory_bench.py`` measurement).
"""

from __future__ import annotations

import argparse
import contextlib
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
WORKLOADS = {
    "sharded": "configs[4] batch-sharded DDPM training step (fwd+bwd + gradient all-reduce)",
    "b1": "configs[3] DDPM training step (fwd+bwd)",
}
C, H, W, K = 64, 256, 256, 3
DILATIONS = (1, 3, 5)
GLOBAL_BATCH = 64
# Published absolute number for the configs[3] fp32 step: 256^2 K3 FP32 fused
# training, RTX 5090 (reference README.md:161-162).
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
    ap.add_argument("--workload", choices=list(WORKLOADS), default="sharded",
                    help="headline: configs[4] (sharded, default) or configs[3] (b1)")
    ap.add_argument("--global-batch", type=int, default=GLOBAL_BATCH,
                    help="configs[4] global batch (split over the ranks)")
    ap.add_argument("--dtype", choices=list(DTYPES), default=None,
                    help="headline dtype (default: bf16 for sharded, fp32 for b1)")
    ap.add_argument("--path", choices=["auto", "fused", "materialised"], default="auto")
    ap.add_argument("--no-graph", action="store_true", help="time eager steps for 'value'")
    ap.add_argument("--skip-extra", action="store_true", help="headline workload only")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU oracle baseline leg")
    ap.add_argument("--no-triton", action="store_true",
                    help="skip timing the reference's Triton path on the GPU")
    ap.add_argument("--memory", action="store_true",
                    help="print the temporary peak memory of one training step and exit")
    ap.add_argument("--launch-list", action="store_true",
                    help="one eager step of the workload inside cudaProfilerStart/Stop (for "
                         "ncu --profile-from-start off) and exit")
    ap.add_argument("--triton-ref", action="store_true",
                    help="time the reference's own Triton path (baseline/_ref) on cuda:0 for "
                         "--workload/--dtype and exit (run by the main bench as a subprocess)")
    ap.add_argument("--inference", action="store_true",
                    help="print the configs[2] inference lines (fused and materialised) only")
    ap.add_argument("--crossover", action="store_true",
                    help="time fused vs materialised training steps over image sizes and exit")
    ap.add_argument("--profile-kernel", default=None,
                    help="only launch this library kernel (ncu capture target)")
    ap.add_argument("--profile-iters", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1, help="per-GPU batch of --profile-kernel")
    args = ap.parse_args(argv)
    if args.dtype is None:
        args.dtype = "bf16" if args.workload == "sharded" else "fp32"
    return args


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
    """x, y and the upstream gradient of this rank's shard, seeded per rank
    (the shards of one global batch), generated on the host."""
    gen = torch.Generator().manual_seed(1000 + rank)
    shape = (batch, C, H, W)
    return [torch.randn(shape, generator=gen).to(dtype) for _ in range(3)]


def step_fn(model, x, y, g, allreduce, loss=True):
    # x and y take part in autograd (dX and dY are computed), as in the
    # reference's training benchmarks (gpu_bench.py:275-300).
    # g is the upstream gradient of the module output (d loss / d out for
    # loss = <out, g>): backward starts from it directly. With ``loss`` the
    # loss value (the one dot product) is formed for a read-back to the host;
    # the training step itself never needs it.
    x = x.detach().requires_grad_(True)
    y = y.detach().requires_grad_(True)
    out = model(x, y)
    out.backward(g)
    if allreduce is not None:
        allreduce()
    if not loss:
        return None
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


def measure(args, dtype, batch, device, rank, world, dist, timed_clocks=False, micro=None):
    """Device-timed step (CUDA graph, inputs in HBM) and end-to-end step
    (public API, host buffers) of ``batch`` samples on this rank, with the
    gradient all-reduce at world > 1. ``micro``: the end-to-end step's
    micro-batch size (copies of the next micro-batch overlap the compute)."""
    from dynamicconvolutionoperator_b200 import _lib
    from dynamicconvolutionoperator_b200.data_parallel import GradAllReducer

    model, taken = build_model(dtype, args.path, device)
    hx, hy, hg = [t.pin_memory() for t in make_inputs(batch, dtype, rank)]
    x, y, g = [t.to(device) for t in (hx, hy, hg)]
    reducer = GradAllReducer(model, overlap=True) if world > 1 else None
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
    graph = None
    allreduce_in_graph = False
    if use_graph:
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                zero()
                step_fn(model, x, y, g, allreduce)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        zero()
        graph = torch.cuda.CUDAGraph()
        # the whole step, the overlapped NCCL all-reduce included, as one graph
        # (the loss read-back belongs to the end-to-end step below)
        with torch.cuda.graph(graph):
            step_fn(model, x, y, g, allreduce, loss=False)
        allreduce_in_graph = allreduce is not None

        def run():
            graph.replay()
    else:
        def run():
            zero()
            step_fn(model, x, y, g, allreduce, loss=False)

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
    if graph is not None:
        del graph  # before any later destroy_process_group: it holds NCCL calls
        graph = None
        zero()

    # ---- end to end through the public API: H2D inputs, fwd+bwd, D2H loss ----
    # All H2D copies of the step are queued on a copy stream at the start of
    # the timed region, micro-batch by micro-batch; the compute stream starts
    # micro-batch i's forward once its x and y copies are done and its
    # backward once its upstream-gradient copy is, so the copies overlap the
    # compute. Gradients accumulate over the micro-batches
    # (every one but the last under no_sync), the all-reduce runs once, and
    # the summed loss is read back. Every copy lies inside the timed region.
    mb = micro or batch
    if batch % mb:
        mb = batch
    bounds = [(i, i + mb) for i in range(0, batch, mb)]
    host_loss = torch.empty((), dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(device)

    def e2e_step():
        zero()
        copy_stream.wait_stream(stream)
        ready_xy, ready_g = [], []
        with torch.cuda.stream(copy_stream):
            for a, b in bounds:
                x[a:b].copy_(hx[a:b], non_blocking=True)
                y[a:b].copy_(hy[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                ready_xy.append(ev)
                # the upstream gradient is needed only by the backward: its copy
                # overlaps the micro-batch's forward
                g[a:b].copy_(hg[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_stream)
                ready_g.append(ev)
        loss = torch.zeros((), dtype=torch.float32, device=device)
        for i, (a, b) in enumerate(bounds):
            stream.wait_event(ready_xy[i])
            last = i == len(bounds) - 1
            ctx = reducer.no_sync() if (reducer is not None and not last) else contextlib.nullcontext()
            with ctx:
                xe = x[a:b].detach().requires_grad_(True)
                ye = y[a:b].detach().requires_grad_(True)
                out = model(xe, ye)
                stream.wait_event(ready_g[i])
                out.backward(g[a:b])
            with torch.no_grad():
                loss += torch.dot(out.reshape(-1), g[a:b].reshape(-1)).float()
        if allreduce is not None:
            allreduce()
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
    in_bytes = sum(t.numel() * t.element_size() for t in (hx, hy, hg))
    if reducer is not None:
        reducer.remove_hooks()
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
        "micro_batch": mb,
        "allreduce_in_graph": allreduce_in_graph,
    }


# ---------------------------------------------------------------- roofline --
def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


# DRAM bytes (read + write) per launch at B=1 C=64 256x256 K=3, from the ncu
# captures summarised in profiles/<kernel>_256.md, keyed by (kernel, dtype);
# None where no capture exists. Outputs still resident in L2 when a captured
# launch ends are not counted as writes.
NCU_TRAFFIC_BYTES: dict[tuple[str, str], float] = {
    # staged paths: the main kernel only (the staging copies are HBM-bound
    # passes of their own, profiles/staging_256.md)
    ("gencat_fwd", "torch.float32"): 115258624,
    ("gencat_fwd", "torch.bfloat16"): 19198976 + 13590272,  # 16-bit x cells
    ("gencat_bwd_x", "torch.float32"): 86148096 + 5298688,  # channel-last grad_out
    ("gencat_bwd_x", "torch.bfloat16"): 45455616 + 169728,  # channel-last grad_out
    # channel-last grad_out, D_y drained by TMA reductions
    ("gencat_bwd_yw", "torch.float32"): 105654784 + 8497664,
    ("gencat_bwd_yw", "torch.bfloat16"): 61231104 + 1570816,  # 16-bit x cells
    ("fuseconv_fwd", "torch.float32"): 75615744,
    ("fuseconv_fwd", "torch.bfloat16"): 36270848,
    ("fuseconv_dgrad", "torch.float32"): 27409920,
    ("fuseconv_dgrad", "torch.bfloat16"): 9356288,
    # dout pre-pass + TMA main kernel (the split reduction is not captured)
    ("fuseconv_wgrad", "torch.float32"): 16783872 + 89954560,
    ("fuseconv_wgrad", "torch.bfloat16"): 8395264 + 42037760,
    # the TMA-fed filter kernels (dyncat_tma.cu): forward; dK + dX
    ("dyncat_fwd", "torch.float32"): 469865984 + 57570304,
    ("dyncat_fwd", "torch.bfloat16"): 234918144 + 22441472,
    ("dyncat_bwd", "torch.float32"): 67156992 + 394124544 + 516594944 + 16864000,
    ("dyncat_bwd", "torch.bfloat16"): 33578496 + 167493632 + 258332928 + 7923456,
}


def library_kernels(model, x, y, dtype, device, materialised=True):
    """Thunks launching each library kernel of the step on its own, with the
    operands it sees inside the step, and each kernel's roofline work unit:
    (thunk, bound, algorithmic bytes or FLOPs per launch). ``materialised``
    adds the materialised-path filter kernels (their taps tensor is 27 C
    planes per sample)."""
    from dynamicconvolutionoperator_b200 import _lib

    n = x.shape[0]
    elt = x.element_size()
    ncp = n * C * H * W
    if materialised:
        with torch.no_grad():
            taps = model.generator(y).reshape(n, 3, C, K * K, H, W).contiguous()
        gk = torch.empty_like(taps)
    else:
        taps = gk = None
    out = torch.empty((n, 4 * C, H, W), dtype=dtype, device=device)
    gout = torch.randn((n, 4 * C, H, W), device=device).to(dtype)
    gx = torch.empty_like(x)
    code = _lib.dtype_code(dtype)
    sh = _lib.stream_handle(device)
    from dynamicconvolutionoperator_b200 import _kernels

    gen_w = model.generator.weight.detach()
    gen_b = model.generator.bias.detach()
    packed = _kernels.pack_generator_weight(gen_w, gen_b, C, K)
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
    fpacked = _fuseconv.pack_fuse_weight(fuse_w)
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

    # as in the step: at C=64 the fuse conv hands the generator backward its
    # gradient channel-last, and the *_nhwc entry points read it so
    nhwc = C == 64
    gout_g = gout.contiguous(memory_format=torch.channels_last) if nhwc else gout
    sfx = "_nhwc" if nhwc else ""

    def bwd_x():
        _lib.call("ddpm_gencat_bwd_x_staged" + sfx, sy.data_ptr(), sy_bytes, packed.data_ptr(),
                  gen_b.data_ptr(), gout_g.data_ptr(), gx.data_ptr(), n, C, H, W, K, *DILATIONS,
                  code, sh)

    def bwd_yw():
        _lib.call("ddpm_gencat_bwd_yw_staged" + sfx, sy.data_ptr(), sy_bytes, packed.data_ptr(),
                  gout_g.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                  ws_bytes, n, C, H, W, K, *DILATIONS, code, sh)

    keep = (taps, out, gout, gout_g, gx, gk, packed, out2, gy, gw, gb, ws, fpacked, fout, fgout,
            fgx, fgw, fgb, fws, sy, fplanes, gplanes)
    kernels = {
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
    if not materialised:
        del kernels["dyncat_fwd"], kernels["dyncat_bwd"]
    return keep, kernels


def kernel_roofline(model, x, y, dtype, steps, device, materialised=True):
    """Time the library's kernels of the step in isolation (CUDA events, L2
    flushed before every launch) and return per-kernel roofline entries.
    ``traffic`` is the DRAM bytes of the B=1 ncu capture times the batch
    (every kernel's traffic grows in proportion to the samples processed)."""
    hbm, tflops, src = load_peaks()
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    n = x.shape[0]
    keep, kernels = library_kernels(model, x, y, dtype, device, materialised)
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
        if traffic is not None:
            traffic = int(traffic * n)
        res[name] = {
            "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "traffic": traffic, "work": work,
            "ms": round(t, 5), "peak_source": src,
        }
    del keep
    return res


def profile_k5_forward(args, device, dtype):
    """The fused K=5 forward of configs[2] (B=``--batch``, C=64, 128x128,
    dilations 1/3/5): staging plus ``ddpm_gencat_fwd_staged``, launched
    ``--profile-iters`` times."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    ks, hw = 5, 128
    torch.manual_seed(0)
    gen = torch.nn.Conv2d(C, 3 * C * ks * ks, 1).to(device=device, dtype=dtype)
    g = torch.Generator().manual_seed(9)
    x, y = (torch.randn((args.batch, C, hw, hw), generator=g).to(dtype).to(device)
            for _ in range(2))
    n = args.batch
    code = _lib.dtype_code(dtype)
    sh = _lib.stream_handle(device)
    packed = _kernels.pack_generator_weight(gen.weight.detach(), gen.bias.detach(), C, ks)
    sb = int(_lib.load().ddpm_gencat_stage_bytes(n, C, hw, hw, ks, *DILATIONS, code))
    st = torch.empty(sb, dtype=torch.uint8, device=device)
    out = torch.empty((n, 4 * C, hw, hw), dtype=dtype, device=device)
    for _ in range(args.profile_iters):
        _lib.call("ddpm_gencat_stage", x.data_ptr(), y.data_ptr(), st.data_ptr(), sb, n, C, hw, hw,
                  ks, *DILATIONS, code, sh)
        _lib.call("ddpm_gencat_fwd_staged", st.data_ptr(), sb, packed.data_ptr(),
                  gen.bias.data_ptr(), out.data_ptr(), n, C, hw, hw, ks, *DILATIONS, code, sh)
    torch.cuda.synchronize()


def profile_kernel(args):
    """Launch one library kernel ``--profile-iters`` times at B=``--batch``
    C=64 256x256 K=3 (the target of the committed ncu captures; prints
    nothing but 'ok'); ``gencat_fwd_k5``: the fused K=5 forward at 128x128."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    dtype = DTYPES[args.dtype]
    if args.profile_kernel == "gencat_fwd_k5":
        profile_k5_forward(args, device, dtype)
        print("ok")
        return 0
    model, _ = build_model(dtype, args.path, device)
    x, y, _ = [t.to(device) for t in make_inputs(args.batch, dtype, 0)]
    keep, kernels = library_kernels(model, x, y, dtype, device,
                                    materialised=args.profile_kernel.startswith("dyncat"))
    fn = kernels[args.profile_kernel][0]
    for _ in range(args.profile_iters):
        fn()
    torch.cuda.synchronize()
    del keep
    print("ok")
    return 0


# -------------------------------------------------------------- CPU legs --
def cpu_sample_time(dtype, steps, warmup, budget_s=None):
    """Median ms of one-sample forward+backward steps of the oracle port of
    ``unfold_impl.DDPM`` (the reference's CPU algorithm) on all host cores."""
    from oracle import ddpm_oracle as orc

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    model = orc.make_model(C, K, dtype=dtype, seed=0)
    x, y, g = orc.make_inputs((1, C, H, W), dtype=dtype, seed=1000)

    def one():
        xr = x.clone().requires_grad_(True)
        yr = y.clone().requires_grad_(True)
        model.zero_grad(set_to_none=True)
        out = model(xr, yr)
        out.backward(g)

    for _ in range(warmup):
        one()
    times, t_start = [], time.perf_counter()
    while len(times) < max(steps, 1):
        if budget_s is not None and times and time.perf_counter() - t_start > budget_s:
            break
        t0 = time.perf_counter()
        one()
        times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), cores, len(times)


def workload_config(args, world):
    """The ``config`` object both arms print: the workload, not how it ran."""
    if args.workload == "sharded":
        glob, per = args.global_batch, args.global_batch // world
        scaling = "strong"
    else:
        glob, per = world, 1
        scaling = "weak"
    return {
        "workload": WORKLOADS[args.workload] + f", {args.dtype}",
        "global_batch": glob, "batch_per_gpu": per,
        "channels": C, "height": H, "width": W, "kernel_size": K,
        "dilations": list(DILATIONS), "parallelism": f"dp{world}",
        "l2": "flushed between steps (256 MiB write)",
    }, scaling


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    cfg, scaling = workload_config(args, world)
    per_ms, cores, n = cpu_sample_time(DTYPES[args.dtype], args.steps, args.warmup)
    ms = per_ms * cfg["global_batch"]
    sample = (f"{n} timed one-sample fwd+bwd steps (median {per_ms:.1f} ms, after {args.warmup} "
              f"warm-up) of C={C} {H}x{W} K={K} {args.dtype}, oracle port of unfold_impl.DDPM "
              f"on {cores} host threads, x {cfg['global_batch']} samples of the global batch")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(ms, 3), "unit": "ms",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": False, "scaling": scaling, "vs_baseline": None,
        "dtype": DTYPE_TAG[args.dtype], "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ memory --
def memory_peaks(device, resolution=H):
    """Temporary peak memory of one B=1 C=64 K=3 training step, measured like
    the reference's ``gpu_memory_bench.py:54-73`` (``max_memory_allocated``
    minus the allocation before the step; loss = out.square().mean())."""
    from dynamicconvolutionoperator_b200 import DDPM

    res = []
    for dname in ("fp32", "bf16"):
        dtype = DTYPES[dname]
        for path in ("fused", "materialised"):
            torch.manual_seed(0)
            module = DDPM(C, K, fused_generator_training=path == "fused")
            module = module.to(device=device, dtype=dtype).train()
            x = torch.randn(1, C, resolution, resolution, device=device, dtype=dtype,
                            requires_grad=True)
            y = torch.randn_like(x, requires_grad=True)

            def step():
                module.zero_grad(set_to_none=True)
                x.grad = None
                y.grad = None
                module(x, y).square().mean().backward()

            for _ in range(2):
                step()
            torch.cuda.synchronize()
            module.zero_grad(set_to_none=True)
            x.grad = None
            y.grad = None
            torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats(device)
            base = torch.cuda.memory_allocated(device)
            step()
            torch.cuda.synchronize()
            peak = torch.cuda.max_memory_allocated(device)
            res.append({"dtype": dname, "path": path, "resolution": resolution,
                        "baseline_mib": round(base / 2**20, 1),
                        "temporary_peak_mib": round((peak - base) / 2**20, 1)})
            del module, x, y
            torch.cuda.empty_cache()
    return res


# ------------------------------------------------- reference Triton on GPU --
REF_DIR = REPO / "baseline" / "_ref"


def triton_reference_leg(args, device):
    """The reference's stock CUDA path, ``triton_impl.DDPM`` on CUDA tensors
    (its Triton kernels and cuDNN, ``triton_impl.py:305-392``), on this GPU for
    the same workload: the "existing kernel" comparison. Eager forward +
    backward from the upstream gradient, CUDA events, L2 flushed between steps;
    Triton's JIT and autotuning happen in the warm-up. Returns a dict."""
    if not (REF_DIR / "triton_impl.py").is_file():
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    sys.path.insert(0, str(REF_DIR))
    import triton_impl  # the reference's module, unmodified

    if triton_impl._load_triton_ops() is None:
        return {"unavailable": "the reference's Triton kernels do not import on this box"}
    cfg, _ = workload_config(args, 1)
    dtype = DTYPES[args.dtype]
    torch.manual_seed(0)
    model = triton_impl.DDPM(C, K).to(device=device, dtype=dtype)
    x, y, g = [t.to(device) for t in make_inputs(cfg["batch_per_gpu"], dtype, 0)]
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    def run():
        for p in model.parameters():
            p.grad = None
        step_fn(model, x, y, g, None)

    for _ in range(max(args.warmup, 2)):
        run()
    torch.cuda.synchronize()
    ts = time_steps(run, args.steps, flush, stream)
    return {"ms_per_step": round(sum(ts) / len(ts), 4), "batch": cfg["batch_per_gpu"],
            "dtype": args.dtype, "workload": cfg["workload"],
            "cudnn_tf32": bool(torch.backends.cudnn.allow_tf32),
            "timing": "eager fwd+bwd, CUDA events, L2 flushed between steps"}


def run_triton_legs(args, legs, timeout_s=180, budget_s=360):
    """Each reference Triton measurement in its own process (a failure there
    cannot touch this process's CUDA context), each bounded in time and all of
    them together too, so the bench line always comes out."""
    out = {}
    t_start = time.monotonic()
    for name, extra in legs:
        left = budget_s - (time.monotonic() - t_start)
        if left < 30:
            out[name] = {"unavailable": f"skipped: the {budget_s} s budget of these legs ran out"}
            continue
        timeout_s = min(timeout_s, left)
        cmd = [sys.executable, str(REPO / "bench.py"), "--triton-ref", "--steps", str(args.steps),
               "--warmup", str(args.warmup)] + extra
        try:
            res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s,
                                 env=dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0"))
            lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
            if res.returncode == 0 and lines:
                out[name] = json.loads(lines[-1])["triton_ref"]
            else:
                tail = (res.stderr or res.stdout).strip().splitlines()[-1:] or ["no output"]
                out[name] = {"unavailable": f"exit {res.returncode}: {tail[0][:300]}"}
        except subprocess.TimeoutExpired:
            out[name] = {"unavailable": f"did not finish within {timeout_s:.0f} s"}
    return out


# ------------------------------------------------------ inference (cfg[2]) --
def inference_lines(args, device):
    """DDPM inference (forward only, no autograd), B=1, C=64,
    128x128, K=3 and K=5, fp32 and bf16, through the fused generator path
    (``fused_generator_inference=True``, the default) and the materialised
    path (the 1x1 generator as cuBLAS GEMMs, then this library's filter kernels);
    graph-replayed device time, L2 flushed between steps."""
    from dynamicconvolutionoperator_b200 import DDPM

    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    out = {}
    for ks in (3, 5):
        for dname in ("fp32", "bf16"):
            dtype = DTYPES[dname]
            line = {}
            for path in ("fused", "materialised"):
                torch.manual_seed(0)
                model = DDPM(C, ks, fused_generator_inference=path == "fused")
                model = model.to(device=device, dtype=dtype).eval()
                gen = torch.Generator().manual_seed(9)
                x, y = (torch.randn((1, C, 128, 128), generator=gen).to(dtype).to(device)
                        for _ in range(2))
                with torch.no_grad():
                    side = torch.cuda.Stream(device)
                    side.wait_stream(stream)
                    with torch.cuda.stream(side):
                        for _ in range(3):
                            model(x, y)
                    stream.wait_stream(side)
                    torch.cuda.synchronize()
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph):
                        model(x, y)
                for _ in range(args.warmup):
                    graph.replay()
                ts = time_steps(graph.replay, max(args.steps, 10), flush, stream)
                line[f"{path}_ms"] = round(statistics.median(ts), 4)
                del graph, model
            out[f"K{ks}_{dname}"] = line
    return {"workload": "configs[2] DDPM inference, B=1, C=64, 128x128", **out}


# --------------------------------------------------------------- crossover --
CROSSOVER_SIZES = {3: (32, 48, 64, 96, 128, 192, 256), 5: (32, 64, 128, 256)}


def crossover(args, device):
    """Fused vs materialised training step (B=1, C=64, K=3 and K=5) at square
    image sizes, both dtypes: graph-replayed device time, L2 flushed between
    steps. The measurement behind the module's automatic training-path choice."""
    from dynamicconvolutionoperator_b200 import DDPM

    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    rows = []
    for ks, dname, hw in ((k, d, s) for k in CROSSOVER_SIZES for d in ("fp32", "bf16")
                          for s in CROSSOVER_SIZES[k]):
        dtype = DTYPES[dname]
        row = {"ks": ks, "dtype": dname, "hw": hw, "tokens": hw * hw}
        for path in ("fused", "materialised"):
            torch.manual_seed(0)
            model = DDPM(C, ks, fused_generator_training=path == "fused")
            model = model.to(device=device, dtype=dtype)
            gen = torch.Generator().manual_seed(7)
            x, y, g = (torch.randn((1, C, hw, hw), generator=gen).to(dtype).to(device)
                       for _ in range(3))

            def zero():
                for p in model.parameters():
                    p.grad = None

            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                for _ in range(3):
                    zero()
                    step_fn(model, x, y, g, None)
            stream.wait_stream(side)
            torch.cuda.synchronize()
            zero()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step_fn(model, x, y, g, None)
            for _ in range(args.warmup):
                graph.replay()
            ts = time_steps(graph.replay, max(args.steps, 10), flush, stream)
            row[path + "_ms"] = round(statistics.median(ts), 4)
            del graph, model
        row["fused_faster"] = row["fused_ms"] < row["materialised_ms"]
        rows.append(row)
    return rows


# -------------------------------------------------------------------- main --
def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.profile_kernel:
        return profile_kernel(args)

    if args.triton_ref:
        # the reference's stock path with PyTorch's defaults (cuDNN may use
        # TF32, the faster setting for its fuse conv)
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        print(json.dumps({"triton_ref": triton_reference_leg(args, device)}), flush=True)
        return 0
    # The fuse conv runs without TF32 for the fp32 step: TF32 would put the
    # output outside the FP32 parity tolerance, which is measured the same way.
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.memory:
        print(json.dumps({"memory": memory_peaks(device)}), flush=True)
        return 0
    if args.crossover:
        print(json.dumps({"crossover": crossover(args, device)}), flush=True)
        return 0
    if args.inference:
        print(json.dumps({"configs[2]_inference": inference_lines(args, device)}), flush=True)
        return 0

    if args.launch_list:
        cfg, _ = workload_config(args, world)
        dtype = DTYPES[args.dtype]
        model, _ = build_model(dtype, args.path, device)
        x, y, g = [t.to(device) for t in make_inputs(cfg["batch_per_gpu"], dtype, rank)]
        for _ in range(max(args.warmup, 1)):
            for p in model.parameters():
                p.grad = None
            step_fn(model, x, y, g, None)
        torch.cuda.synchronize()
        for p in model.parameters():
            p.grad = None
        torch.cuda.profiler.start()
        step_fn(model, x, y, g, None, loss=False)  # the device-timed step
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print("ok")
        return 0
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def gather_max(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    memory = memory_peaks(device) if (world == 1 and not args.skip_extra) else None
    cfg, scaling = workload_config(args, world)
    if args.workload == "sharded" and args.global_batch % world:
        raise SystemExit(f"global batch {args.global_batch} does not split over {world} GPUs")
    per = cfg["batch_per_gpu"]
    dtype = DTYPES[args.dtype]
    headline = measure(args, dtype, per, device, rank, world, dist, timed_clocks=True,
                       micro=4 if per >= 8 else None)
    head_roof = kernel_roofline(headline["model"], *headline["inputs"], dtype, args.steps, device,
                                materialised=(headline["path"] == "materialised"
                                              or args.workload == "b1"))
    ms = gather_max(headline["ms"])
    e2e_ms = gather_max(headline["e2e_ms"])
    head_info = {k: headline[k] for k in ("h2d_bytes", "d2h_bytes", "launches_per_step", "path",
                                          "clocks", "micro_batch", "allreduce_in_graph")}
    del headline
    torch.cuda.empty_cache()

    # configs[3] (B=1 per GPU) in both dtypes, with the per-kernel rooflines
    extra, kernels = {}, {}
    if args.workload == "b1":
        kernels[args.dtype] = head_roof
    if not args.skip_extra:
        for dname in ("fp32", "bf16"):
            if args.workload == "b1" and dname == args.dtype:
                continue
            m = measure(args, DTYPES[dname], 1, device, rank, world, dist)
            kernels[dname] = kernel_roofline(m["model"], *m["inputs"], DTYPES[dname], args.steps,
                                             device)
            entry = {"workload": WORKLOADS["b1"] + f", {dname}", "batch_per_gpu": 1,
                     "global_batch": world, "scaling": "weak",
                     "ms_per_step": round(gather_max(m["ms"]), 4),
                     "e2e_ms": round(gather_max(m["e2e_ms"]), 4), "path": m["path"],
                     "h2d_bytes_per_step": m["h2d_bytes"]}
            if dname == "fp32":
                entry["vs_published_rtx5090_fp32_ms"] = round(entry["ms_per_step"] /
                                                              PUBLISHED_FP32_MS, 4)
            extra[f"configs[3]_{dname}"] = entry
            del m
            torch.cuda.empty_cache()

    if world == 1 and not args.skip_extra:
        extra["configs[2]_inference"] = inference_lines(args, device)
        torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        steps = 10 if args.workload == "sharded" else 5
        per_ms, cores, n = cpu_sample_time(dtype, steps, 1, budget_s=20.0)
        cpu = {"value": round(per_ms * cfg["global_batch"], 3), "unit": "ms", "cores": cores,
               "kind": "port",
               "sample": f"{n} one-sample fwd+bwd steps (median {per_ms:.1f} ms) of the same "
                         f"workload, oracle port of unfold_impl.DDPM, {args.dtype}, "
                         f"x {cfg['global_batch']} samples"}
    triton = None
    if rank == 0 and world == 1 and not args.skip_extra and not args.no_triton:
        legs = [(f"{args.workload}_{args.dtype}", ["--workload", args.workload, "--dtype",
                                                   args.dtype])]
        legs += [(f"configs[3]_{d}", ["--workload", "b1", "--dtype", d]) for d in ("fp32", "bf16")
                 if not (args.workload == "b1" and d == args.dtype)]
        triton = run_triton_legs(args, legs)
    # dominant kernel among those the headline step launches
    in_step = {"fused": ("gencat_fwd", "gencat_bwd_x", "gencat_bwd_yw"),
               "materialised": ("dyncat_fwd", "dyncat_bwd")}[head_info["path"]]
    in_step = in_step + ("fuseconv_fwd", "fuseconv_dgrad", "fuseconv_wgrad")
    dominant = max((k for k in head_roof if k in in_step), key=lambda k: head_roof[k]["ms"])
    if rank == 0:
        px = cfg["global_batch"] * H * W
        line = {
            "metric": METRIC,
            "value": round(ms, 4),
            "unit": "ms",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": False,
            "scaling": scaling,
            # a published number exists for the configs[3] fp32 step only
            "vs_baseline": (round(ms / PUBLISHED_FP32_MS, 4)
                            if (args.workload == "b1" and args.dtype == "fp32") else None),
            "dtype": DTYPE_TAG[args.dtype],
            "data": "synthetic",
            "config": cfg,
            "run": {"value_step": "forward + backward of the module on the shard (+ the "
                                  "gradient all-reduce at N > 1) as one CUDA graph; the loss "
                                  "read-back is part of e2e",
                    "path": head_info["path"], "cuda_graph": not args.no_graph,
                    "allreduce_in_graph": head_info["allreduce_in_graph"],
                    "allreduce": ("NCCL average over 2 flat buckets (fuse, generator), "
                                  "launched from the backward" if world > 1 else None),
                    "e2e_micro_batch": head_info["micro_batch"],
                    "cudnn_tf32": bool(torch.backends.cudnn.allow_tf32)},
            "mpixel_per_s": round(px / (ms * 1e-3) / 1e6, 2),
            "e2e": {"value": round(e2e_ms, 4), "unit": "ms",
                    "h2d_bytes_per_step": head_info["h2d_bytes"],
                    "d2h_bytes_per_step": head_info["d2h_bytes"]},
            "gpu_launches": int(head_info["launches_per_step"] * args.steps),
            "roofline": {k: v for k, v in head_roof[dominant].items() if k != "work"}
            | {"kernel": dominant, "batch": per},
            "kernels_headline": head_roof,
            "kernels": kernels.get("fp32"),
            "kernels_bf16": kernels.get("bf16"),
            "clocks": head_info["clocks"],
            "cpu_baseline": cpu,
            "triton_b200": triton,
            "memory": memory,
            "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
