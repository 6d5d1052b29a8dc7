"""Host-side contract of the drop-in DDPM (CPU, no GPU needed).

Mirrors the reference's own unit tests for the API (``test_triton_impl.py:58-65``)
and the constructor / input checks (``triton_impl.py:36-44, 280-283``).
"""

from __future__ import annotations

import pytest
import torch

from dynamicconvolutionoperator_b200 import DDPM, fused_dynamic_cat
from dynamicconvolutionoperator_b200 import triton_impl as drop_in
from oracle import ddpm_oracle as orc


def test_rejects_invalid_shapes():
    model = DDPM(4, 3)
    with pytest.raises(ValueError, match="identical shapes"):
        model(torch.randn(1, 4, 5, 5), torch.randn(1, 4, 4, 5))


def test_rejects_even_kernel():
    with pytest.raises(ValueError, match="positive odd"):
        DDPM(4, 2)


@pytest.mark.parametrize("ks", [0, -1, 4])
def test_rejects_bad_kernel_sizes(ks):
    with pytest.raises(ValueError, match="positive odd"):
        DDPM(4, ks)


def test_rejects_bad_dim():
    with pytest.raises(ValueError, match="dim must be positive"):
        DDPM(0, 3)


def test_rejects_non_nchw_and_channel_mismatch():
    model = DDPM(4, 3)
    with pytest.raises(ValueError, match="NCHW"):
        model(torch.randn(4, 5, 5), torch.randn(4, 5, 5))
    with pytest.raises(ValueError, match="expected 4 channels"):
        model(torch.randn(1, 3, 5, 5), torch.randn(1, 3, 5, 5))


def test_cpu_tensors_fail_loudly():
    """No CPU fallback: CPU tensors that pass the input checks raise."""
    model = DDPM(4, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        model(torch.randn(1, 4, 5, 5), torch.randn(1, 4, 5, 5))
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_dynamic_cat(torch.randn(1, 2, 3, 3), torch.randn(1, 3, 2, 9, 3, 3), 3, (1, 3, 5))


@pytest.mark.parametrize("ks", [1, 3, 5])
def test_state_dict_interchange_with_unfold_reference(ks):
    """Parameter names/shapes match the reference (``unfold_impl.py:15,19``)."""
    ref = orc.make_model(6, ks, seed=11)
    new = DDPM(6, ks)
    new.load_state_dict(ref.state_dict())
    back = orc.UnfoldDDPM(6, ks)
    back.load_state_dict(new.state_dict())
    for k, v in ref.state_dict().items():
        torch.testing.assert_close(back.state_dict()[k], v, rtol=0, atol=0)
    assert new.generator.weight.shape == (3 * 6 * ks * ks, 6, 1, 1)
    assert new.fuse.weight.shape == (6, 24, 3, 3)


def test_ctor_keeps_reference_attributes():
    m = DDPM(8, 3, spatial_tile_size=11, max_generated_bytes=0, recompute=False,
             fused_generator_inference=False, fused_generator_training=True)
    assert (m.dim, m.kernel_size, m.spatial_tile_size, m.max_generated_bytes) == (8, 3, 11, 0)
    assert m.recompute is False and m.fused_generator_inference is False
    assert m.fused_generator_training is True and m.dilations == (1, 3, 5)
    assert drop_in.DDPM is DDPM


def test_fuse_bias_fold_matches_conv2d():
    """The bias-folded fuse conv equals ``nn.Conv2d`` (values and gradients)."""
    from dynamicconvolutionoperator_b200.ddpm import _fuse_single_rounding

    gen = torch.Generator().manual_seed(3)
    cat = torch.randn(2, 16, 7, 9, generator=gen, dtype=torch.float64, requires_grad=True)
    wt = torch.randn(4, 16, 3, 3, generator=gen, dtype=torch.float64, requires_grad=True)
    b = torch.randn(4, generator=gen, dtype=torch.float64, requires_grad=True)
    g = torch.randn(2, 4, 7, 9, generator=gen, dtype=torch.float64)
    got = _fuse_single_rounding(cat, wt, b)
    ref = torch.nn.functional.conv2d(cat, wt, b, 1, 1)
    torch.testing.assert_close(got, ref, rtol=1e-12, atol=1e-12)
    for a, e in zip(torch.autograd.grad(got, (cat, wt, b), g),
                    torch.autograd.grad(ref, (cat, wt, b), g)):
        torch.testing.assert_close(a, e, rtol=1e-12, atol=1e-12)


def test_training_crossover_follows_the_b200_measurement():
    """The reference's rule (``triton_impl.py:313-316``: fuse above 16384
    tokens) was measured on an RTX 5090; on B200 the K = 3 fused step wins at
    every measured size in FP32 and above 4096 tokens in 16-bit types; the
    K = 5 one above 1024 tokens in every dtype."""
    from dynamicconvolutionoperator_b200 import _kernels

    for tokens in (1, 1024, 16384, 65536):
        assert _kernels.auto_fuse_training(tokens, 64, 3, torch.float32)
    for dt in (torch.bfloat16, torch.float16):
        assert _kernels.auto_fuse_training(4097, 64, 3, dt)
        assert _kernels.auto_fuse_training(16384, 64, 3, dt)
        assert not _kernels.auto_fuse_training(4096, 64, 3, dt)
    for dt in (torch.float32, torch.bfloat16):
        assert _kernels.auto_fuse_training(1025, 64, 5, dt)
        assert not _kernels.auto_fuse_training(1024, 64, 5, dt)


def test_fused_kernel_limits():
    """Forward: C <= 64, K in {1, 3} with halo (K/2) * max(dilation) <= 8 or
    K = 5 with halo <= 16; fused training at every such K (the fully fused
    backward kernels at K <= 3, the reference's limit, ``triton_impl.py:320``;
    at K = 5 fused dX, and fused dY + dW for 16-bit data with rows of a
    multiple of 8 pixels, FP32 taking a materialised dK for dY / dW)."""
    from dynamicconvolutionoperator_b200 import _kernels

    ok = _kernels.fused_generator_supported
    assert ok(64, 3, torch.float32) and ok(1, 1, torch.bfloat16, (1, 1, 1))
    assert not ok(65, 3, torch.float32)
    assert ok(64, 5, torch.float32) and ok(64, 5, torch.bfloat16, (1, 8, 4))
    assert not ok(64, 5, torch.float32, (1, 9, 4)) and not ok(64, 7, torch.bfloat16)
    assert ok(64, 3, torch.float16, (1, 3, 8)) and not ok(64, 3, torch.float16, (1, 3, 9))
    assert not ok(64, 3, torch.float64)
    assert [k for k in (1, 3, 5, 7) if _kernels.fused_training_supported(k)] == [1, 3, 5]
    assert _kernels.FUSED_TRAINING_KERNEL_SIZES == (1, 3)
    dyw = _kernels._fused_dyw_ok
    assert dyw(3, torch.float32, 17, (1, 3, 5)) and dyw(5, torch.float16, 64, (1, 8, 4))
    assert not dyw(5, torch.float32, 64, (1, 3, 5)) and not dyw(5, torch.bfloat16, 60, (1, 3, 5))


@pytest.mark.parametrize(
    "hw,ks,requested,expect",
    [((128, 128), 3, None, True), ((128, 127), 3, None, True), ((32, 32), 3, None, True),
     ((256, 256), 5, None, True), ((256, 256), 5, False, False),
     ((256, 256), 3, False, False), ((8, 8), 3, True, True), ((8, 8), 7, True, False)],
)
def test_module_training_path_choice(hw, ks, requested, expect):
    """``fused_generator_training``: None follows the crossover, True / False
    force the path, and K > 5 always materialises."""
    m = DDPM(4, ks, fused_generator_training=requested)
    assert m._use_fused_training(torch.empty(1, 4, *hw)) is expect
