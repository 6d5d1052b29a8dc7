"""Helpers to read the golden fixtures written by tests/golden/make_golden.py."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


def tensor(rec: dict, key: str) -> torch.Tensor:
    return torch.from_numpy(np.array(rec[key]))


def state_dict(rec: dict, prefix: str) -> dict[str, torch.Tensor]:
    p = f"{prefix}__sd__"
    return {k[len(p):]: torch.from_numpy(v) for k, v in rec.items() if k.startswith(p)}


def check_fingerprint(rec: dict, prefix: str, t: torch.Tensor, rtol: float, atol: float) -> None:
    """Compare a tensor with a stored fingerprint (shape, sums, sampled values)."""
    a = t.detach().double().reshape(-1).cpu()
    assert tuple(rec[f"{prefix}__shape"]) == tuple(t.shape), prefix
    idx = torch.from_numpy(rec[f"{prefix}__idx"])
    samples = torch.from_numpy(rec[f"{prefix}__samples"])
    scale = float(rec[f"{prefix}__amax"])
    torch.testing.assert_close(a[idx], samples, rtol=rtol, atol=atol + rtol * scale, msg=prefix)
    n = a.numel()
    for key, val in (("sum", a.sum()), ("abssum", a.abs().sum()), ("sumsq", a.square().sum())):
        ref = float(rec[f"{prefix}__{key}"])
        tol = atol * n + rtol * (abs(ref) + scale * n)
        assert abs(val.item() - ref) <= tol, (prefix, key, val.item(), ref)
