"""Full DDPM forward(+backward) on the GPU against the float64 oracle, at the
BASELINE configs, through both the materialised and the fused paths.

Tolerances are those of the north star (see tests/_parity.py): fp32 2e-3
max-abs; bf16 3e-2 max-abs and 5e-3 RMSE; parameter gradients normalised by
their largest gold magnitude.
"""

from __future__ import annotations

import pytest
import torch

from tests import _golden as gold
from tests._parity import ddpm_parity

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16]


def _assert_ok(stats, fails):
    assert not fails, "\n".join(fails) + f"\n{stats}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("ks", [1, 3, 5])
@pytest.mark.parametrize("fused", [False, True])
def test_cfg2_regression_training(dtype, ks, fused):
    """[2,24,15,17], K in {1,3,5}, fwd+bwd, every gradient."""
    stats, fails = ddpm_parity((2, 24, 15, 17), ks, dtype, seed=123, input_seed=456,
                               fused_generator_training=fused)
    _assert_ok(stats, fails)


@pytest.mark.parametrize("dtype", DTYPES)
def test_cfg2_matches_reference_golden_output(dtype):
    """The GPU output sits within tolerance of the reference's own CPU output
    recorded in tests/golden (same seeds, same dtype)."""
    from dynamicconvolutionoperator_b200 import DDPM
    from oracle import ddpm_oracle as orc

    tag = "fp32" if dtype == torch.float32 else "bf16"
    rec = gold.load(f"cfg2_{tag}_k3.npz")
    ref = orc.make_model(24, 3, dtype=dtype, seed=123)
    dev = DDPM(24, 3).cuda().to(dtype)
    dev.load_state_dict(ref.state_dict())
    x, y, _ = orc.make_inputs((2, 24, 15, 17), dtype=dtype, seed=456, grad_seed=789)
    torch.backends.cudnn.allow_tf32 = False
    with torch.no_grad():
        out = dev(x.cuda(), y.cuda()).float().cpu()
    tol = 2e-3 if dtype == torch.float32 else 3e-2
    assert (out - gold.tensor(rec, "out")).abs().max().item() <= tol


def test_cfg1_inference_matches_golden():
    """C=32 48x48 K=3 fp32 inference vs the reference's output."""
    from dynamicconvolutionoperator_b200 import DDPM
    from oracle import ddpm_oracle as orc

    rec = gold.load("cfg1.npz")
    ref = orc.make_model(32, 3, seed=0)
    dev = DDPM(32, 3).cuda()
    dev.load_state_dict(ref.state_dict())
    x, y, _ = orc.make_inputs((1, 32, 48, 48), seed=1)
    torch.backends.cudnn.allow_tf32 = False
    for fused in (True, False):
        dev.fused_generator_inference = fused
        with torch.no_grad():
            out = dev(x.cuda(), y.cuda()).cpu()
        assert (out - gold.tensor(rec, "out")).abs().max().item() <= 2e-3


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("ks", [3, 5])
@pytest.mark.parametrize("fused", [True, False])
def test_cfg3_inference_128(dtype, ks, fused):
    """B=1 C=64 128x128, K in {3,5}, fused vs materialised."""
    stats, fails = ddpm_parity((1, 64, 128, 128), ks, dtype, grad=False, seed=20,
                               input_seed=21, fused_generator_inference=fused)
    _assert_ok(stats, fails)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("fused", [True, False])
def test_cfg4_training_256(dtype, fused):
    """B=1 C=64 256x256 K=3, fwd+bwd, every gradient."""
    stats, fails = ddpm_parity((1, 64, 256, 256), 3, dtype, seed=30, input_seed=31,
                               fused_generator_training=fused)
    _assert_ok(stats, fails)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("ks", [1, 3])
def test_cudnn_fuse_path_training(dtype, ks):
    """``native_fuse=False``: the fuse conv through cuDNN (bias folded into the
    contraction for 16-bit outputs), every gradient within tolerance."""
    stats, fails = ddpm_parity((2, 24, 15, 17), ks, dtype, seed=7, input_seed=8,
                               native_fuse=False)
    _assert_ok(stats, fails)
