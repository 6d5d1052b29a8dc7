"""Fused generator backward kernels against the oracle (float64 autograd of
the fused semantics, ``_triton_kernels.py:911-1053``)."""

from __future__ import annotations

import pytest
import torch

from oracle import ddpm_oracle as orc
from tests.test_gpu_gencat import SHAPES, _case

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-4, 2e-4), torch.bfloat16: (1e-2, 3e-2), torch.float16: (2e-3, 4e-3)}


def _gold_grads(x, y, wt, b, g, ks, dil):
    """d<fused_cat, g>/d(x, y, W, b) in float64 with the I/O-dtype tap rounding."""
    io = x.dtype
    x64 = x.double().requires_grad_(True)
    y64 = y.double().requires_grad_(True)
    w64 = wt.double().requires_grad_(True)
    b64 = b.double().requires_grad_(True)
    taps = orc.generated_taps(y64, w64, b64, ks)
    if io in (torch.bfloat16, torch.float16):
        # straight-through rounding: forward value rounded, gradient identity
        taps = taps + (taps.detach().to(io).double() - taps.detach())
    out = orc.dynamic_cat(x64, taps, ks, dil)
    return torch.autograd.grad(out, (x64, y64, w64, b64), g.double())


def _stage_y(yd, ks, dil):
    """Staged copy of y through the C ABI (ddpm_gencat_stage_y)."""
    from dynamicconvolutionoperator_b200 import _lib

    n, c, h, w = yd.shape
    code = _lib.dtype_code(yd.dtype)
    nb = int(_lib.load().ddpm_gencat_stage_y_bytes(n, c, h, w, ks, *dil, code))
    assert nb > 0
    staged = torch.full((nb,), 0xAB, dtype=torch.uint8, device=yd.device)  # no reliance on zeros
    _lib.call("ddpm_gencat_stage_y", yd.data_ptr(), staged.data_ptr(), nb, n, c, h, w, ks, *dil,
              code, _lib.stream_handle(yd.device))
    return staged, nb


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ks", [1, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("staged", [False, True])
def test_gencat_bwd_x(shape, ks, dtype, staged):
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    x, y, wt, b = _case(shape, ks, dtype)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(5)).to(dtype)
    gx_gold, *_ = _gold_grads(x, y, wt, b, g, ks, (1, 3, 5))
    yd, wd, bd, gd = y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks, use_cache=False)
    gx = torch.full((n, c, h, w), float("nan"), dtype=dtype, device="cuda")
    stream = _lib.stream_handle(gx.device)
    if staged:
        sy, nb = _stage_y(yd, ks, (1, 3, 5))
        _lib.call("ddpm_gencat_bwd_x_staged", sy.data_ptr(), nb, packed.data_ptr(), bd.data_ptr(),
                  gd.data_ptr(), gx.data_ptr(), n, c, h, w, ks, 1, 3, 5, _lib.dtype_code(dtype),
                  stream)
    else:
        _lib.call("ddpm_gencat_bwd_x", yd.data_ptr(), packed.data_ptr(), bd.data_ptr(),
                  gd.data_ptr(), gx.data_ptr(), n, c, h, w, ks, 1, 3, 5, _lib.dtype_code(dtype),
                  stream)
    torch.cuda.synchronize()
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(gx.double().cpu(), gx_gold, rtol=rtol, atol=atol)


@pytest.mark.parametrize("shape,ks,dil", [((2, 24, 15, 17), 3, (1, 3, 5)), ((1, 64, 9, 130), 3, (2, 1, 4)),
                                          ((1, 5, 4, 3), 1, (1, 1, 1))])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_stage_y_layout(shape, ks, dil, dtype):
    """Staged y = y channel-last, zero padded by the halo, ones channel at C,
    [part][n][Hp][G][Wp][8]; fp32 as bf16 hi + residual (hi + lo == y to
    within bf16 of the residual)."""
    n, c, h, w = shape
    y = torch.randn(shape, generator=torch.Generator().manual_seed(3)).to(dtype)
    staged, nb = _stage_y(y.cuda(), ks, dil)
    torch.cuda.synchronize()
    G = (c + 1 + 15) // 16 * 2
    ph = (ks // 2) * max(dil)
    Hp, Wp = h + 2 * ph, (w + 127) // 128 * 128 + 16
    parts = 2 if dtype == torch.float32 else 1
    assert nb == parts * n * Hp * G * Wp * 16
    want = torch.zeros((n, G * 8, Hp, Wp), dtype=torch.float64)
    want[:, :c, ph:ph + h, 8:8 + w] = y.double()
    want[:, c] = 1.0
    # [n][Hp][G][Wp][8] -> [n][G*8][Hp][Wp]
    planes = staged.cpu().view(torch.bfloat16 if dtype != torch.float16 else torch.float16)
    planes = planes.view(parts, n, Hp, G, Wp, 8).permute(0, 1, 3, 5, 2, 4).reshape(parts, n, G * 8, Hp, Wp)
    got = planes[0].double() + (planes[1].double() if parts == 2 else 0.0)
    # fp32: |y - hi| <= 2^-8 |y| and the residual is rounded to bf16 again
    tol = 2.0 ** -15 * want.abs().max().item() if dtype == torch.float32 else 0.0
    assert (got - want).abs().max().item() <= tol


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ks", [1, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gencat_bwd_yw(shape, ks, dtype):
    """dY, dW and db from the on-chip dK (split partials + reduce)."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    x, y, wt, b = _case(shape, ks, dtype)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(6)).to(dtype)
    _, gy_gold, gw_gold, gb_gold = _gold_grads(x, y, wt, b, g, ks, (1, 3, 5))
    xd, yd, wd, bd, gd = x.cuda(), y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks, use_cache=False)
    gy = torch.empty_like(yd)
    gw = torch.empty((3 * c * ks * ks, c), dtype=dtype, device="cuda")
    gb = torch.empty(3 * c * ks * ks, dtype=dtype, device="cuda")
    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.call("ddpm_gencat_bwd_yw", xd.data_ptr(), yd.data_ptr(), packed.data_ptr(), gd.data_ptr(),
              gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(), ws_bytes,
              n, c, h, w, ks, 1, 3, 5, _lib.dtype_code(dtype), _lib.stream_handle(gy.device))
    torch.cuda.synchronize()
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(gy.double().cpu(), gy_gold, rtol=rtol, atol=atol)
    # parameter gradients sum over all pixels: compare normalised by their scale
    for got, gold in ((gw.reshape(gw_gold.shape), gw_gold), (gb, gb_gold)):
        scale = gold.abs().max().item() + 1e-12
        err = (got.double().cpu() - gold).abs().max().item() / scale
        assert err <= (2e-4 if dtype == torch.float32 else 1e-2), err


def test_fused_autograd_matches_oracle_all_grads():
    """End to end through fused_generator_dynamic_cat + autograd (fp32)."""
    from dynamicconvolutionoperator_b200 import fused_generator_dynamic_cat

    shape, ks = (2, 24, 16, 40), 3
    x, y, wt, b = _case(shape, ks, torch.float32, seed=12)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(13))
    gold = _gold_grads(x, y, wt, b, g, ks, (1, 3, 5))
    ts = [t.cuda().requires_grad_(True) for t in (x, y, wt, b)]
    out = fused_generator_dynamic_cat(*ts, ks, (1, 3, 5))
    grads = torch.autograd.grad(out, ts, g.cuda())
    for got, ref in zip(grads, gold):
        scale = max(ref.abs().max().item(), 1.0)
        assert (got.double().cpu() - ref).abs().max().item() <= 2e-4 * scale
