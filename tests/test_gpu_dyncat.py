"""Materialised dynamic filter kernels (ddpm_dyncat_fwd / ddpm_dyncat_bwd)
against the oracle's closed-form math in float64 (``_triton_kernels.py:21-254``).

Edge cases follow the reference's own coverage (non-power-of-2 channels,
non-square borders, cross-tile neighbourhoods: ``gpu_validate.py:39-41``) plus
1x1 images, images smaller than the dilation halo, multi-tile planes with
ragged edges, K up to 7, custom dilations and the autocast dtype pair.
"""

from __future__ import annotations

import pytest
import torch

from oracle import ddpm_oracle as orc

pytestmark = pytest.mark.gpu

SHAPES = [(2, 3, 5, 7), (2, 24, 15, 17), (1, 4, 1, 1), (1, 2, 3, 200), (3, 5, 33, 130),
          # rows of whole 16-byte vectors (W % 8 == 0): the TMA-fed kernels for
          # K = 3 -- ragged tiles in both directions, images narrower than a
          # tile and smaller than the dilation halo
          (2, 3, 40, 136), (2, 5, 9, 8), (1, 3, 17, 264)]
TOLS = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (8e-3, 2e-3), torch.float16: (1e-3, 1e-4)}


def _inputs(shape, ks, xdt, kdt, seed=0):
    gen = torch.Generator().manual_seed(seed)
    n, c, h, w = shape
    x = torch.randn(shape, generator=gen).to(xdt)
    k = torch.randn((n, 3, c, ks * ks, h, w), generator=gen).to(kdt)
    g = torch.randn((n, 4 * c, h, w), generator=gen).to(kdt)
    return x, k, g


def _check(actual, gold, dtype):
    rtol, atol = TOLS[dtype]
    torch.testing.assert_close(actual.double().cpu(), gold, rtol=rtol, atol=atol)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ks", [1, 3, 5, 7])
@pytest.mark.parametrize(
    "xdt,kdt",
    [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
     (torch.float16, torch.float16), (torch.float32, torch.bfloat16)],
)
def test_dyncat_forward_backward(shape, ks, xdt, kdt):
    from dynamicconvolutionoperator_b200 import fused_dynamic_cat

    dil = (1, 3, 5)
    x, k, g = _inputs(shape, ks, xdt, kdt)
    xd = x.cuda().requires_grad_(True)
    kd = k.cuda().requires_grad_(True)
    out = fused_dynamic_cat(xd, kd, ks, dil)
    assert out.dtype == kdt and out.shape == (shape[0], 4 * shape[1], *shape[2:])
    gx, gk = torch.autograd.grad(out, (xd, kd), g.cuda())
    gold_out = orc.dynamic_cat(x.double(), k.double(), ks, dil)
    gold_gx, gold_gk = orc.dynamic_cat_backward(x.double(), k.double(), g.double(), ks, dil)
    _check(out, gold_out, kdt)
    _check(gx, gold_gx, xdt if xdt != torch.float32 else kdt)
    _check(gk, gold_gk, kdt)


@pytest.mark.parametrize("dil", [(2, 1, 4), (1, 1, 1), (7, 2, 3)])
def test_dyncat_custom_dilations(dil):
    from dynamicconvolutionoperator_b200 import fused_dynamic_cat

    x, k, g = _inputs((2, 6, 19, 23), 3, torch.float32, torch.float32, seed=3)
    xd = x.cuda().requires_grad_(True)
    kd = k.cuda().requires_grad_(True)
    out = fused_dynamic_cat(xd, kd, 3, dil)
    gx, gk = torch.autograd.grad(out, (xd, kd), g.cuda())
    _check(out, orc.dynamic_cat(x.double(), k.double(), 3, dil), torch.float32)
    ggx, ggk = orc.dynamic_cat_backward(x.double(), k.double(), g.double(), 3, dil)
    _check(gx, ggx, torch.float32)
    _check(gk, ggk, torch.float32)


def test_dyncat_only_requested_grads():
    from dynamicconvolutionoperator_b200 import fused_dynamic_cat

    x, k, g = _inputs((1, 4, 9, 9), 3, torch.float32, torch.float32)
    kd = k.cuda().requires_grad_(True)
    out = fused_dynamic_cat(x.cuda(), kd, 3, (1, 3, 5))
    (gk,) = torch.autograd.grad(out, (kd,), g.cuda())
    _, ggk = orc.dynamic_cat_backward(x.double(), k.double(), g.double(), 3, (1, 3, 5))
    _check(gk, ggk, torch.float32)


def test_dyncat_large_plane_bf16():
    """128x128 C=64 (BASELINE configs[2] filter shape), fwd + bwd."""
    from dynamicconvolutionoperator_b200 import fused_dynamic_cat

    x, k, g = _inputs((1, 64, 128, 128), 3, torch.bfloat16, torch.bfloat16, seed=5)
    xd = x.cuda().requires_grad_(True)
    kd = k.cuda().requires_grad_(True)
    out = fused_dynamic_cat(xd, kd, 3, (1, 3, 5))
    gx, gk = torch.autograd.grad(out, (xd, kd), g.cuda())
    _check(out, orc.dynamic_cat(x.double(), k.double(), 3), torch.bfloat16)
    ggx, ggk = orc.dynamic_cat_backward(x.double(), k.double(), g.double(), 3)
    _check(gx, ggx, torch.bfloat16)
    _check(gk, ggk, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("width", [20, 24])
def test_dyncat_backward_ignores_taps_that_feed_padding(dtype, width):
    """A tap value at pixel p whose source p + off lies outside the image only
    meets the zero padding, so it never reaches grad_x, even when it is not
    finite (the reference folds its products into the discarded border)."""
    from dynamicconvolutionoperator_b200 import fused_dynamic_cat

    ks, dil = 3, (1, 3, 5)
    x, k, g = _inputs((1, 3, 12, width), ks, dtype, dtype, seed=7)
    n, c, h, w = x.shape
    rows = torch.arange(h).view(h, 1)
    cols = torch.arange(w).view(1, w)
    for b, d in enumerate(dil):
        for ki in range(ks):
            for kj in range(ks):
                dy, dx = (ki - ks // 2) * d, (kj - ks // 2) * d
                outside = ((rows + dy < 0) | (rows + dy >= h) | (cols + dx < 0) | (cols + dx >= w))
                k[:, b, :, ki * ks + kj][:, :, outside] = float("inf")
    xd = x.cuda().requires_grad_(True)
    out = fused_dynamic_cat(xd, k.cuda(), ks, dil)
    (gx,) = torch.autograd.grad(out, (xd,), g.cuda())
    gold_gx, _ = orc.dynamic_cat_backward(x.double(), k.double(), g.double(), ks, dil)
    assert torch.isfinite(gold_gx).all()
    assert torch.isfinite(gx).all()
    _check(gx, gold_gx, dtype)


def _misaligned(t):
    """The same values one element past a 16-byte boundary: the library's
    vector kernels need 16-byte aligned rows, so this selects the scalar ones."""
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
    out = buf[1:].view(t.shape)
    out.copy_(t)
    assert out.data_ptr() % 16 != 0
    return out


@pytest.mark.parametrize("shape", [(1, 3, 21, 136), (2, 2, 9, 264), (1, 4, 16, 8), (1, 2, 5, 40)])
@pytest.mark.parametrize("ks", [1, 3, 5])
@pytest.mark.parametrize("dil", [(1, 3, 5), (7, 2, 4)])
@pytest.mark.parametrize(
    "xdt,kdt",
    [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
     (torch.float16, torch.float16), (torch.float32, torch.bfloat16)],
)
def test_dyncat_grad_x_vector_kernel_matches_scalar(shape, ks, dil, xdt, kdt):
    """grad_x from aligned tensors (the vector kernel for 16-bit taps, rows a
    multiple of 16 bytes) is bit-identical to the scalar kernel's (same sum,
    same order) and matches the oracle; shapes cover ragged column tiles,
    8-wide images and tap shifts wider than one vector, for the dilations with
    a compile-time instance (1, 3, 5) and for run-time ones."""
    from dynamicconvolutionoperator_b200 import fused_dynamic_cat

    x, k, g = _inputs(shape, ks, xdt, kdt, seed=11)
    kc, gc = k.cuda(), g.cuda()
    grads = []
    for kk in (kc, _misaligned(kc)):
        xd = x.cuda().requires_grad_(True)
        out = fused_dynamic_cat(xd, kk, ks, dil)
        (gx,) = torch.autograd.grad(out, (xd,), gc)
        grads.append(gx)
    assert torch.equal(grads[0], grads[1])
    gold_gx, _ = orc.dynamic_cat_backward(x.double(), k.double(), g.double(), ks, dil)
    _check(grads[0], gold_gx, xdt if xdt != torch.float32 else kdt)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_dyncat_largest_accepted_data_gradient_halo(dtype):
    """Halo 39, the largest the data gradient stages (232,368 bytes of shared
    memory for its three planes), runs and matches the oracle."""
    from dynamicconvolutionoperator_b200 import fused_dynamic_cat

    ks, dil = 3, (1, 39, 5)
    x, k, g = _inputs((1, 2, 20, 24), ks, dtype, dtype, seed=13)
    xd = x.cuda().requires_grad_(True)
    kd = k.cuda().requires_grad_(True)
    out = fused_dynamic_cat(xd, kd, ks, dil)
    gx, gk = torch.autograd.grad(out, (xd, kd), g.cuda())
    _check(out, orc.dynamic_cat(x.double(), k.double(), ks, dil), dtype)
    ggx, ggk = orc.dynamic_cat_backward(x.double(), k.double(), g.double(), ks, dil)
    _check(gx, ggx, dtype)
    _check(gk, ggk, dtype)


@pytest.mark.parametrize("shape", [(2, 24, 37, 264), (1, 64, 256, 256), (3, 5, 16, 128)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_tma_kernels_match_register_kernels_bit_for_bit(shape, dtype):
    """K = 3, dilations (1, 3, 5), W % 8 == 0: the TMA-fed forward, dK and dX
    compute the same sums in the same order as the register-fed kernels, so
    the two paths agree bit for bit (the register-fed ones are checked against
    the oracle above)."""
    from dynamicconvolutionoperator_b200 import _lib, fused_dynamic_cat

    x, k, g = _inputs(shape, 3, dtype, dtype, seed=11)
    xd, kd, gd = x.cuda(), k.cuda(), g.cuda()

    def run():
        xr = xd.clone().requires_grad_(True)
        kr = kd.clone().requires_grad_(True)
        out = fused_dynamic_cat(xr, kr, 3, (1, 3, 5))
        gx, gk = torch.autograd.grad(out, (xr, kr), gd)
        return out, gx, gk

    n0 = _lib.launch_count()
    tma = run()
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 3  # forward, dK, dX: one launch each
    _lib.call("ddpm_test_disable_tma", 1)
    try:
        ref = run()
    finally:
        _lib.call("ddpm_test_disable_tma", 0)
    for a, b, name in zip(tma, ref, ("out", "grad_x", "grad_k")):
        assert torch.equal(a, b), f"{name} differs between the TMA and register kernels"
    assert _lib.device_status(reset=True) == 0
