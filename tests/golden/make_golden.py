"""Generate the golden fixtures under tests/golden/ from the REAL reference.

Run in the build container, where the reference checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/DynamicConvolutionOperator

It imports the reference's own ``unfold_impl.DDPM`` (the math oracle,
``unfold_impl.py:5-42``) and records, on CPU:

* ``reftests.npz`` — the reference unit-test fixtures re-run verbatim
  (``test_triton_impl.py:10-56``: seed 123, shapes [2,3,5,7] for K in {1,3,5}
  forward, [2,4,5,7] K=3 forward+backward with loss ``square().mean()``):
  full inputs, state dicts, outputs and gradients.
* ``cfg1.npz``: C=32, 48x48, K=3, fp32 inference; full
  output, plus checksums of the seeded inputs/weights.
* ``cfg2_<dtype>_k<K>.npz``: [2,24,15,17], fp32 and
  bf16, K in {1,3,5}, forward+backward with an N(0,1) upstream gradient; full
  output/dx/dy and fingerprints of every parameter gradient.

Inputs and weights for cfg1/cfg2 come from the oracle's seeded constructors
(``oracle.ddpm_oracle.make_model`` / ``make_inputs``); the fixtures store
checksums of them so a test can tell a changed RNG from a changed formula.
The GPU box never runs this script; it only reads the .npz files.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import ddpm_oracle as orc  # noqa: E402


def fingerprint(t: torch.Tensor, prefix: str) -> dict[str, np.ndarray]:
    a = t.detach().double().reshape(-1)
    idx = torch.linspace(0, a.numel() - 1, steps=min(256, a.numel())).round().long()
    return {
        f"{prefix}__shape": np.array(t.shape, dtype=np.int64),
        f"{prefix}__sum": np.array(a.sum().item()),
        f"{prefix}__abssum": np.array(a.abs().sum().item()),
        f"{prefix}__sumsq": np.array(a.square().sum().item()),
        f"{prefix}__amax": np.array(a.abs().max().item()),
        f"{prefix}__idx": idx.numpy(),
        f"{prefix}__samples": a[idx].numpy(),
    }


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().numpy()


def ref_models(ref_mod, channels, kernel_size, seed, dtype=torch.float32):
    torch.manual_seed(seed)
    return ref_mod.DDPM(channels, kernel_size).to(dtype)


def grads_of(model, x, y, upstream=None, loss_square_mean=False):
    x = x.detach().clone().requires_grad_(True)
    y = y.detach().clone().requires_grad_(True)
    out = model(x, y)
    tensors = [x, y] + list(model.parameters())
    names = ["x", "y"] + [n for n, _ in model.named_parameters()]
    if loss_square_mean:
        grads = torch.autograd.grad(out.square().mean(), tensors)
    else:
        grads = torch.autograd.grad(out, tensors, upstream)
    return out.detach(), dict(zip(names, grads))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout directory")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import unfold_impl  # the reference math module

    torch.set_num_threads(8)

    # ---- reference unit-test fixtures (test_triton_impl.py:10-56) ----------
    rec: dict[str, np.ndarray] = {}
    for ks in (1, 3, 5):
        torch.manual_seed(123)
        ref = unfold_impl.DDPM(3, ks)
        x = torch.randn(2, 3, 5, 7)
        y = torch.randn_like(x)
        with torch.no_grad():
            out = ref(x, y)
        p = f"fwd_k{ks}"
        rec[f"{p}__x"], rec[f"{p}__y"], rec[f"{p}__out"] = f32(x), f32(y), f32(out)
        for k, v in ref.state_dict().items():
            rec[f"{p}__sd__{k}"] = f32(v)
    torch.manual_seed(123)
    ref = unfold_impl.DDPM(4, 3)
    x = torch.randn(2, 4, 5, 7)
    y = torch.randn_like(x)
    out, grads = grads_of(ref, x, y, loss_square_mean=True)
    rec["bwd__x"], rec["bwd__y"], rec["bwd__out"] = f32(x), f32(y), f32(out)
    for k, v in ref.state_dict().items():
        rec[f"bwd__sd__{k}"] = f32(v)
    for k, v in grads.items():
        rec[f"bwd__grad__{k}"] = f32(v)
    np.savez_compressed(HERE / "reftests.npz", **rec)

    # ---- cfg1: C=32, 48x48, K=3, fp32 inference ----------------------------
    ref = ref_models(unfold_impl, 32, 3, seed=0)
    x, y, _ = orc.make_inputs((1, 32, 48, 48), seed=1)
    with torch.no_grad():
        out = ref(x, y)
    rec = {"out": f32(out)}
    rec.update(fingerprint(x, "x"))
    rec.update(fingerprint(y, "y"))
    for k, v in ref.state_dict().items():
        rec.update(fingerprint(v, f"sd__{k}"))
    np.savez_compressed(HERE / "cfg1.npz", **rec)

    # ---- cfg2: [2,24,15,17], fp32/bf16, K in {1,3,5}, fwd+bwd ---------------
    for dtype, tag in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        for ks in (1, 3, 5):
            ref = ref_models(unfold_impl, 24, ks, seed=123, dtype=dtype)
            x, y, g = orc.make_inputs((2, 24, 15, 17), dtype=dtype, seed=456, grad_seed=789)
            out, grads = grads_of(ref, x, y, upstream=g)
            rec = {"out": f32(out), "grad__x": f32(grads["x"]), "grad__y": f32(grads["y"])}
            for name in ("x", "y", "g"):
                rec.update(fingerprint({"x": x, "y": y, "g": g}[name], f"in__{name}"))
            for k, v in ref.state_dict().items():
                rec.update(fingerprint(v, f"sd__{k}"))
            for k, v in grads.items():
                if k not in ("x", "y"):
                    rec.update(fingerprint(v, f"grad__{k}"))
            np.savez_compressed(HERE / f"cfg2_{tag}_k{ks}.npz", **rec)

    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
    return 0


if __name__ == "__main__":
    sys.exit(main())
