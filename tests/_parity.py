"""Parity harness: the CUDA DDPM against the CPU oracle (float64 gold).

Tolerance policy:
  * fp32: output, dX, dY max-abs <= 2e-3; parameter gradients max-abs
    normalised by max|gold| <= 2e-3 (parameter grads reach |g| ~ 2e3 at 256^2,
    where even the fp32 reference differs from float64 by ~4e-3 absolute).
  * bf16: output, dX, dY max-abs <= 3e-2 and RMSE <= 5e-3; parameter
    gradients normalised max-abs <= 3e-2 and normalised RMSE <= 5e-3.
Gold = the oracle run in float64 on the dtype-rounded inputs and weights, so
the comparison measures the kernels' error, not the input rounding.
"""

from __future__ import annotations

import torch

from oracle import ddpm_oracle as orc

TOL = {
    torch.float32: {"max_abs": 2e-3, "rmse": None, "norm_max": 2e-3, "norm_rmse": None},
    torch.bfloat16: {"max_abs": 3e-2, "rmse": 5e-3, "norm_max": 3e-2, "norm_rmse": 5e-3},
    torch.float16: {"max_abs": 3e-2, "rmse": 5e-3, "norm_max": 3e-2, "norm_rmse": 5e-3},
}


def build_pair(channels, ks, dtype, seed=0, **ddpm_kwargs):
    """(oracle model on CPU in ``dtype``, DDPM on cuda with identical weights)."""
    from dynamicconvolutionoperator_b200 import DDPM

    ref = orc.make_model(channels, ks, dtype=dtype, seed=seed)
    dev = DDPM(channels, ks, **ddpm_kwargs)
    dev.load_state_dict(ref.state_dict())
    return ref, dev.to(device="cuda", dtype=dtype)


def run_device(model, x, y, grad=None):
    x = x.cuda().detach().requires_grad_(grad is not None)
    y = y.cuda().detach().requires_grad_(grad is not None)
    if grad is None:
        with torch.no_grad():
            return model(x, y).cpu(), None
    out = model(x, y)
    names = ["x", "y"] + [n for n, _ in model.named_parameters()]
    grads = torch.autograd.grad(out, [x, y, *model.parameters()], grad.cuda())
    return out.detach().cpu(), {k: g.cpu() for k, g in zip(names, grads)}


def compare(dev_out, dev_grads, gold_out, gold_grads, dtype):
    """Error stats per tensor; returns (stats, failures)."""
    tol = TOL[dtype]
    stats, fails = {}, []
    items = [("out", dev_out, gold_out)]
    if dev_grads is not None:
        items += [(k, dev_grads[k], gold_grads[k]) for k in gold_grads]
    for name, a, e in items:
        s = orc.error_stats(a, e)
        s["norm_rmse"] = s["rmse"] / s["ref_max"]
        stats[name] = s
        # written as "not (err <= tol)" so that a NaN error fails
        if name in ("out", "x", "y"):
            if not s["max_abs"] <= tol["max_abs"]:
                fails.append(f"{name}: max_abs {s['max_abs']:.3e} > {tol['max_abs']}")
            if tol["rmse"] is not None and not s["rmse"] <= tol["rmse"]:
                fails.append(f"{name}: rmse {s['rmse']:.3e} > {tol['rmse']}")
        else:
            if not s["norm_max"] <= tol["norm_max"]:
                fails.append(f"{name}: norm_max {s['norm_max']:.3e} > {tol['norm_max']}")
            if tol["norm_rmse"] is not None and not s["norm_rmse"] <= tol["norm_rmse"]:
                fails.append(f"{name}: norm_rmse {s['norm_rmse']:.3e} > {tol['norm_rmse']}")
    return stats, fails


def ddpm_parity(shape, ks, dtype, grad=True, seed=0, input_seed=1, **ddpm_kwargs):
    """Run DDPM on cuda and the float64 oracle on CPU; returns (stats, failures)."""
    n, c, h, w = shape
    prev_tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False  # keep the cuDNN fuse conv in true fp32
    try:
        ref, dev = build_pair(c, ks, dtype, seed=seed, **ddpm_kwargs)
        x, y, g = orc.make_inputs(shape, dtype=dtype, seed=input_seed, grad_seed=input_seed + 1)
        dev_out, dev_grads = run_device(dev, x, y, g if grad else None)
        gold_out, gold_grads = orc.run_reference(
            ref, x, y, grad=g if grad else None, dtype=torch.float64
        )
    finally:
        torch.backends.cudnn.allow_tf32 = prev_tf32
    return compare(dev_out, dev_grads, gold_out, gold_grads, dtype)
