"""Fused generator + dynamic filter (ddpm_gencat_*) against the oracle.

The oracle restates the reference's fused semantics (``_triton_kernels.py:
268-420``): taps = W*y + b accumulated in FP32, rounded to the I/O dtype for
bf16/fp16 (``:332-335``), then multiplied with shifted x. Shapes cover the
reference's regression set (C=24 -> channel padding, 15x17 borders, tiles that
straddle the image edge), a 1x1 image, C=3, and the 128x128 C=64 config.
"""

from __future__ import annotations

import pytest
import torch

from oracle import ddpm_oracle as orc

pytestmark = pytest.mark.gpu

SHAPES = [(2, 24, 15, 17), (1, 3, 5, 7), (1, 4, 1, 1), (2, 16, 9, 40), (1, 64, 48, 48),
          (1, 64, 128, 128), (3, 40, 33, 30)]
# Error budget: fp32 operands carried as bf16 hi+lo pairs (~1e-5 relative per
# product); bf16/fp16 taps may round one ulp apart where the FP32 sum lands
# near a rounding boundary, plus the output rounding.
TOL = {torch.float32: (1e-4, 1e-4), torch.bfloat16: (1e-2, 3e-2), torch.float16: (2e-3, 4e-3)}


def _case(shape, ks, dtype, seed=0):
    n, c, h, w = shape
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=gen).to(dtype)
    y = torch.randn(shape, generator=gen).to(dtype)
    bound = 1.0 / c**0.5
    wt = ((torch.rand((3 * c * ks * ks, c, 1, 1), generator=gen) * 2 - 1) * bound).to(dtype)
    b = ((torch.rand(3 * c * ks * ks, generator=gen) * 2 - 1) * bound).to(dtype)
    return x, y, wt, b


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ks", [1, 3, 5])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_gencat_forward(shape, ks, dtype):
    from dynamicconvolutionoperator_b200 import fused_generator_dynamic_cat

    x, y, wt, b = _case(shape, ks, dtype)
    with torch.no_grad():
        out = fused_generator_dynamic_cat(x.cuda(), y.cuda(), wt.cuda(), b.cuda(), ks, (1, 3, 5))
    torch.cuda.synchronize()
    gold = orc.fused_generator_cat(x, y, wt, b, ks, quantize=True)
    rtol, atol = TOL[dtype]
    c = shape[1]
    torch.testing.assert_close(out[:, :c].cpu(), x, rtol=0, atol=0)
    torch.testing.assert_close(out.float().cpu(), gold.float(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("shape", [(2, 24, 15, 17), (1, 64, 48, 48), (3, 40, 33, 30)])
@pytest.mark.parametrize("ks", [1, 3, 5])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gencat_forward_unstaged_abi(shape, ks, dtype):
    """ddpm_gencat_fwd staging tiles from x and y itself (the public module
    path stages the operands once and calls ddpm_gencat_fwd_staged)."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    x, y, wt, b = _case(shape, ks, dtype)
    n, c, h, w = shape
    xd, yd, wd, bd = x.cuda(), y.cuda(), wt.cuda(), b.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    out = torch.full((n, 4 * c, h, w), float("nan"), dtype=dtype, device="cuda")
    _lib.call("ddpm_gencat_fwd", xd.data_ptr(), yd.data_ptr(), packed.data_ptr(), bd.data_ptr(),
              out.data_ptr(), n, c, h, w, ks, 1, 3, 5, _lib.dtype_code(dtype),
              _lib.stream_handle(out.device))
    torch.cuda.synchronize()
    gold = orc.fused_generator_cat(x, y, wt, b, ks, quantize=True)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.float().cpu(), gold.float(), rtol=rtol, atol=atol)


def test_gencat_custom_dilations_and_repeat_calls():
    """Custom dilations; repeated calls reuse the cached packed weight and an
    in-place weight update invalidates it."""
    from dynamicconvolutionoperator_b200 import fused_generator_dynamic_cat

    x, y, wt, b = _case((2, 32, 20, 24), 3, torch.float32, seed=3)
    xd, yd, wd, bd = x.cuda(), y.cuda(), wt.cuda(), b.cuda()
    dil = (2, 1, 4)
    with torch.no_grad():
        o1 = fused_generator_dynamic_cat(xd, yd, wd, bd, 3, dil)
        o2 = fused_generator_dynamic_cat(xd, yd, wd, bd, 3, dil)
        wd.mul_(0.5)
        o3 = fused_generator_dynamic_cat(xd, yd, wd, bd, 3, dil)
    torch.testing.assert_close(o1, o2, rtol=0, atol=0)
    gold1 = orc.fused_generator_cat(x, y, wt, b, 3, dil)
    gold3 = orc.fused_generator_cat(x, y, wt * 0.5, b, 3, dil)
    torch.testing.assert_close(o1.cpu(), gold1, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(o3.cpu(), gold3, rtol=1e-4, atol=1e-4)


def test_gencat_multiple_tiles_per_cta():
    """More tiles than SMs: every persistent CTA loops over several tiles and
    the TMEM / weight rings wrap many times."""
    from dynamicconvolutionoperator_b200 import fused_generator_dynamic_cat

    x, y, wt, b = _case((4, 64, 96, 128), 3, torch.bfloat16, seed=9)
    with torch.no_grad():
        out = fused_generator_dynamic_cat(x.cuda(), y.cuda(), wt.cuda(), b.cuda(), 3, (1, 3, 5))
    gold = orc.fused_generator_cat(x, y, wt, b, 3, quantize=True)
    rtol, atol = TOL[torch.bfloat16]
    torch.testing.assert_close(out.float().cpu(), gold.float(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("shape", [(2, 24, 15, 17), (1, 64, 48, 48), (3, 40, 33, 30),
                                   (1, 8, 1, 1), (1, 16, 9, 130), (1, 32, 19, 21)])
@pytest.mark.parametrize("ks", [1, 3, 5])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_gencat_forward_writes_fuse_planes(shape, ks, dtype):
    """ddpm_gencat_fwd_staged_planes: the same output as ddpm_gencat_fwd_staged,
    and planes byte-identical to ddpm_fuseconv_stage of that output (padding
    frame included: both buffers start as filler bytes)."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    x, y, wt, b = _case(shape, ks, dtype, seed=9)
    n, c, h, w = shape
    xd, yd, wd, bd = x.cuda(), y.cuda(), wt.cuda(), b.cuda()
    lib = _lib.load()
    code = _lib.dtype_code(dtype)
    st = _lib.stream_handle(xd.device)
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    sb = int(lib.ddpm_gencat_stage_bytes(n, c, h, w, ks, 1, 3, 5, code))
    staged = torch.empty(sb, dtype=torch.uint8, device="cuda")
    _lib.call("ddpm_gencat_stage", xd.data_ptr(), yd.data_ptr(), staged.data_ptr(), sb,
              n, c, h, w, ks, 1, 3, 5, code, st)
    ref = torch.full((n, 4 * c, h, w), float("nan"), dtype=dtype, device="cuda")
    _lib.call("ddpm_gencat_fwd_staged", staged.data_ptr(), sb, packed.data_ptr(), bd.data_ptr(),
              ref.data_ptr(), n, c, h, w, ks, 1, 3, 5, code, st)
    pb = int(lib.ddpm_fuseconv_stage_bytes(n, 4 * c, h, w, code))
    planes = torch.full((pb,), 0x5A, dtype=torch.uint8, device="cuda")
    out = torch.full_like(ref, float("nan"))
    _lib.call("ddpm_gencat_fwd_staged_planes", staged.data_ptr(), sb, packed.data_ptr(),
              bd.data_ptr(), out.data_ptr(), planes.data_ptr(), pb,
              n, c, h, w, ks, 1, 3, 5, code, st)
    gold = torch.full((pb,), 0xA5, dtype=torch.uint8, device="cuda")
    _lib.call("ddpm_fuseconv_stage", ref.data_ptr(), gold.data_ptr(), pb, n, 4 * c, h, w, code, st)
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, rtol=0, atol=0, equal_nan=True)
    assert torch.equal(planes, gold)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gencat_k5_halo_limits_and_tiles(dtype):
    """K = 5: the largest halo the forward covers ((K/2) * 8 = 16, dilations
    (1, 8, 4)) against the oracle on a shape with more tiles than SMs, and a
    halo of 18 rejected as unsupported before anything is launched."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib, fused_generator_dynamic_cat

    x, y, wt, b = _case((2, 64, 40, 72), 5, dtype, seed=4)
    dil = (1, 8, 4)
    with torch.no_grad():
        out = fused_generator_dynamic_cat(x.cuda(), y.cuda(), wt.cuda(), b.cuda(), 5, dil)
    gold = orc.fused_generator_cat(x, y, wt, b, 5, dil, quantize=True)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.float().cpu(), gold.float(), rtol=rtol, atol=atol)
    assert not _kernels.fused_generator_supported(64, 5, dtype, (1, 9, 4))
    rc = _lib.load().ddpm_gencat_fwd_staged(1, 1, 1, 1, 1, 1, 64, 8, 8, 5, 1, 9, 4,
                                            _lib.dtype_code(dtype), None)
    assert rc == -2


def test_gencat_forward_fuse_planes_rejects_ragged_channels():
    """The planes variant needs whole 8-channel groups per branch (C % 8 == 0)."""
    from dynamicconvolutionoperator_b200 import _lib

    rc = _lib.load().ddpm_gencat_fwd_staged_planes(1, 1, 1, 1, 1, 256, 1 << 20, 1, 3, 8, 8, 3,
                                                    1, 3, 5, 0, None)
    assert rc == -2
