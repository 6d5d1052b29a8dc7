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


def _stage(xd, yd, ks, dil):
    """Staged operands through the C ABI (ddpm_gencat_stage); xd may be None."""
    from dynamicconvolutionoperator_b200 import _lib

    n, c, h, w = yd.shape
    code = _lib.dtype_code(yd.dtype)
    nb = int(_lib.load().ddpm_gencat_stage_bytes(n, c, h, w, ks, *dil, code))
    assert nb > 0
    staged = torch.full((nb,), 0xAB, dtype=torch.uint8, device=yd.device)  # no reliance on zeros
    _lib.call("ddpm_gencat_stage", xd.data_ptr() if xd is not None else None, yd.data_ptr(),
              staged.data_ptr(), nb, n, c, h, w, ks, *dil, code, _lib.stream_handle(yd.device))
    return staged, nb


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ks", [1, 3, 5])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("staged", [False, True])
def test_gencat_bwd_x(shape, ks, dtype, staged):
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    x, y, wt, b = _case(shape, ks, dtype)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(5)).to(dtype)
    gx_gold, *_ = _gold_grads(x, y, wt, b, g, ks, (1, 3, 5))
    yd, wd, bd, gd = y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    gx = torch.full((n, c, h, w), float("nan"), dtype=dtype, device="cuda")
    stream = _lib.stream_handle(gx.device)
    if staged:
        sy, nb = _stage(None, yd, ks, (1, 3, 5))
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
def test_stage_layout(shape, ks, dil, dtype):
    """y plane = y channel-last, zero padded by the halo, ones channel at C,
    [part][n][G][Hp][Wp][8]; fp32 as bf16 hi + residual (hi + lo == y to
    within bf16 of the residual). x plane = 16-byte cells [n][ceil(C/k)][H][W][k]:
    fp32 as FP32 (k = 4), 16-bit data in its own type (k = 8, the same bits)."""
    n, c, h, w = shape
    gen = torch.Generator().manual_seed(3)
    y = torch.randn(shape, generator=gen).to(dtype)
    x = torch.randn(shape, generator=gen).to(dtype)
    staged, nb = _stage(x.cuda(), y.cuda(), ks, dil)
    torch.cuda.synchronize()
    G = (c + 1 + 15) // 16 * 2
    ph = (ks // 2) * max(dil)
    Hp, Wp = h + 2 * ph, (w + 127) // 128 * 128 + 16
    parts = 2 if dtype == torch.float32 else 1
    part_bytes = n * G * Hp * Wp * 16
    x_off = (parts * part_bytes + 255) // 256 * 256
    xcell = 4 if dtype == torch.float32 else 8
    cq = (c + xcell - 1) // xcell
    assert nb == x_off + n * cq * h * w * 16
    want = torch.zeros((n, G * 8, Hp, Wp), dtype=torch.float64)
    want[:, :c, ph:ph + h, 8:8 + w] = y.double()
    want[:, c] = 1.0
    # [part][n][G][Hp][Wp][8] -> [part][n][G*8][Hp][Wp]
    raw = staged.cpu()
    planes = raw[:parts * part_bytes].view(torch.bfloat16)
    planes = planes.view(parts, n, G, Hp, Wp, 8).permute(0, 1, 2, 5, 3, 4).reshape(parts, n, G * 8, Hp, Wp)
    got = planes[0].double() + (planes[1].double() if parts == 2 else 0.0)
    # fp32: |y - hi| <= 2^-8 |y| and the residual is rounded to bf16 again
    tol = 2.0 ** -15 * want.abs().max().item() if dtype == torch.float32 else 0.0
    assert (got - want).abs().max().item() <= tol
    xp = raw[x_off:x_off + n * cq * h * w * 16].view(dtype).view(n, cq, h, w, xcell)
    xp = xp.permute(0, 1, 4, 2, 3).reshape(n, cq * xcell, h, w)
    bits = torch.int16 if xcell == 8 else torch.int32  # compare the bits
    assert torch.equal(xp[:, :c].view(bits), x.view(bits))
    assert not xp[:, c:].view(bits).any()


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ks", [1, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("staged", [False, True])
def test_gencat_bwd_yw(shape, ks, dtype, staged):
    """dY, dW and db from the on-chip dK (split partials + reduce); staged: x
    and y read from the staged operands by TMA."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    x, y, wt, b = _case(shape, ks, dtype)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(6)).to(dtype)
    _, gy_gold, gw_gold, gb_gold = _gold_grads(x, y, wt, b, g, ks, (1, 3, 5))
    xd, yd, wd, bd, gd = x.cuda(), y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    gy = torch.full_like(yd, float("nan"))
    gw = torch.full((3 * c * ks * ks, c), float("nan"), dtype=dtype, device="cuda")
    gb = torch.full((3 * c * ks * ks,), float("nan"), dtype=dtype, device="cuda")
    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    stream = _lib.stream_handle(gy.device)
    if staged:
        st, nb = _stage(xd, yd, ks, (1, 3, 5))
        _lib.call("ddpm_gencat_bwd_yw_staged", st.data_ptr(), nb, packed.data_ptr(),
                  gd.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                  ws_bytes, n, c, h, w, ks, 1, 3, 5, _lib.dtype_code(dtype), stream)
    else:
        _lib.call("ddpm_gencat_bwd_yw", xd.data_ptr(), yd.data_ptr(), packed.data_ptr(),
                  gd.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                  ws_bytes, n, c, h, w, ks, 1, 3, 5, _lib.dtype_code(dtype), stream)
    torch.cuda.synchronize()
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(gy.double().cpu(), gy_gold, rtol=rtol, atol=atol)
    # parameter gradients sum over all pixels: compare normalised by their scale
    for got, gold in ((gw.reshape(gw_gold.shape), gw_gold), (gb, gb_gold)):
        scale = gold.abs().max().item() + 1e-12
        err = (got.double().cpu() - gold).abs().max().item() / scale
        assert err <= (2e-4 if dtype == torch.float32 else 1e-2), err


@pytest.mark.parametrize("ks", [3, 5])
def test_fused_autograd_matches_oracle_all_grads(ks):
    """End to end through fused_generator_dynamic_cat + autograd (fp32). At
    K = 5 the forward is fused and the backward recomputes the taps with the
    1x1 generator convolution (cuDNN, TF32 off here) and takes the filter's
    gradients from ddpm_dyncat_bwd."""
    from dynamicconvolutionoperator_b200 import fused_generator_dynamic_cat

    shape = (2, 24, 16, 40)
    x, y, wt, b = _case(shape, ks, torch.float32, seed=12)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(13))
    gold = _gold_grads(x, y, wt, b, g, ks, (1, 3, 5))
    ts = [t.cuda().requires_grad_(True) for t in (x, y, wt, b)]
    with torch.backends.cudnn.flags(enabled=True, allow_tf32=False):
        out = fused_generator_dynamic_cat(*ts, ks, (1, 3, 5))
        grads = torch.autograd.grad(out, ts, g.cuda())
    for got, ref in zip(grads, gold):
        scale = max(ref.abs().max().item(), 1.0)
        assert (got.double().cpu() - ref).abs().max().item() <= 2e-4 * scale


def test_fused_k5_autograd_partial_grads_bf16():
    """K = 5, bf16, only some inputs requiring gradients: the recompute
    backward returns None for the others and matches the oracle for the rest."""
    from dynamicconvolutionoperator_b200 import fused_generator_dynamic_cat

    shape, ks = (1, 16, 12, 20), 5
    x, y, wt, b = _case(shape, ks, torch.bfloat16, seed=14)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(15)).bfloat16()
    gold = _gold_grads(x, y, wt, b, g, ks, (1, 3, 5))
    xd, yd, wd, bd = x.cuda(), y.cuda().requires_grad_(True), wt.cuda().requires_grad_(True), b.cuda()
    out = fused_generator_dynamic_cat(xd, yd, wd, bd, ks, (1, 3, 5))
    gy, gw = torch.autograd.grad(out, (yd, wd), g.cuda())
    for got, ref in ((gy, gold[1]), (gw, gold[2])):
        scale = max(ref.abs().max().item(), 1.0)
        assert (got.double().cpu() - ref).abs().max().item() <= 3e-2 * scale


@pytest.mark.parametrize("shape", [(1, 64, 20, 24), (2, 40, 19, 24)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_max_halo_and_ragged_gradient_tiles(shape, dtype):
    """Dilation halo 8, the largest supported (C=64 needs single-buffered x
    halos in the fp32 forward and the 16-bit dY+dW pass to fit shared
    memory), and 16-bit gradient tiles copied by TMA with ragged rows, columns
    and channel groups (C=40): forward and every gradient through autograd,
    plus the unstaged forward entry point."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib, fused_generator_dynamic_cat

    ks, dil = 3, (8, 1, 8)
    x, y, wt, b = _case(shape, ks, dtype, seed=21)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(22)).to(dtype)
    gold_out = orc.fused_generator_cat(x, y, wt, b, ks, dil, quantize=True)
    gold = _gold_grads(x, y, wt, b, g, ks, dil)
    ts = [t.cuda().requires_grad_(True) for t in (x, y, wt, b)]
    out = fused_generator_dynamic_cat(*ts, ks, dil)
    grads = torch.autograd.grad(out, ts, g.cuda())
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.detach().float().cpu(), gold_out.float(), rtol=rtol, atol=atol)
    for got, ref in zip(grads[:2], gold[:2]):
        torch.testing.assert_close(got.double().cpu(), ref, rtol=rtol, atol=atol)
    for got, ref in zip(grads[2:], gold[2:]):
        scale = ref.abs().max().item() + 1e-12
        err = (got.double().cpu() - ref).abs().max().item() / scale
        assert err <= (2e-4 if dtype == torch.float32 else 1e-2), err

    with torch.no_grad():
        xd, yd, wd, bd = (t.detach() for t in ts)
        packed = _kernels.pack_generator_weight(wd, bd, c, ks)
        o2 = torch.full((n, 4 * c, h, w), float("nan"), dtype=dtype, device="cuda")
        _lib.call("ddpm_gencat_fwd", xd.data_ptr(), yd.data_ptr(), packed.data_ptr(),
                  bd.data_ptr(), o2.data_ptr(), n, c, h, w, ks, *dil, _lib.dtype_code(dtype),
                  _lib.stream_handle(o2.device))
        torch.cuda.synchronize()
    torch.testing.assert_close(o2.float().cpu(), gold_out.float(), rtol=rtol, atol=atol)


@pytest.mark.parametrize("shape", [(2, 64, 15, 40), (1, 64, 33, 136)])
@pytest.mark.parametrize("ks", [1, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_channel_last_grad_out_matches_nchw(shape, ks, dtype):
    """The *_staged_nhwc backward entry points read grad_out channel-last
    ([N][H][W][4C], C = 64) and give dX bit for bit and dY, dW, db to FP32
    summation order of the NCHW entry points (FP32 included: two 128-byte
    channel boxes per dX unit, vector loads in the dY+dW builders)."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    x, y, wt, b = _case(shape, ks, dtype)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(8)).to(dtype)
    xd, yd, wd, bd = x.cuda(), y.cuda(), wt.cuda(), b.cuda()
    gd = g.cuda()
    gd_cl = gd.contiguous(memory_format=torch.channels_last)
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    st, nb = _stage(xd, yd, ks, (1, 3, 5))
    code = _lib.dtype_code(dtype)
    stream = _lib.stream_handle(xd.device)
    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
    res = {}
    for sfx, gg in (("", gd), ("_nhwc", gd_cl)):
        gx = torch.full_like(xd, float("nan"))
        gy = torch.full_like(yd, float("nan"))
        gw = torch.full((3 * c * ks * ks, c), float("nan"), dtype=dtype, device="cuda")
        gb = torch.full((3 * c * ks * ks,), float("nan"), dtype=dtype, device="cuda")
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        _lib.call("ddpm_gencat_bwd_x_staged" + sfx, st.data_ptr(), nb, packed.data_ptr(),
                  bd.data_ptr(), gg.data_ptr(), gx.data_ptr(), n, c, h, w, ks, 1, 3, 5, code,
                  stream)
        _lib.call("ddpm_gencat_bwd_yw_staged" + sfx, st.data_ptr(), nb, packed.data_ptr(),
                  gg.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                  ws_bytes, n, c, h, w, ks, 1, 3, 5, code, stream)
        res[sfx] = (gx, gy, gw, gb)
    torch.cuda.synchronize()
    ref, got = res[""], res["_nhwc"]
    assert torch.equal(got[0], ref[0]), "dX differs"
    for a, r in zip(got[1:], ref[1:]):
        assert torch.isfinite(a).all()
        scale = r.double().abs().max().item() + 1e-12
        assert (a.double() - r.double()).abs().max().item() / scale <= 1e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_k5_bwd_x_channel_last_and_max_halo(dtype):
    """K = 5 dX: the channel-last entry point matches the NCHW one bit for bit,
    and the largest halo (16, dilations (1, 8, 4)) matches the oracle on a
    shape whose rows span two 128-pixel tiles."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    shape, ks, dil = (1, 64, 13, 150), 5, (1, 8, 4)
    x, y, wt, b = _case(shape, ks, dtype, seed=21)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(22)).to(dtype)
    gx_gold, *_ = _gold_grads(x, y, wt, b, g, ks, dil)
    xd, yd, wd, bd, gd = x.cuda(), y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    st, nb = _stage(None, yd, ks, dil)
    code = _lib.dtype_code(dtype)
    stream = _lib.stream_handle(yd.device)
    out = {}
    for sfx, gg in (("", gd), ("_nhwc", gd.contiguous(memory_format=torch.channels_last))):
        gx = torch.full_like(xd, float("nan"))
        _lib.call("ddpm_gencat_bwd_x_staged" + sfx, st.data_ptr(), nb, packed.data_ptr(),
                  bd.data_ptr(), gg.data_ptr(), gx.data_ptr(), n, c, h, w, ks, *dil, code, stream)
        out[sfx] = gx
    torch.cuda.synchronize()
    assert torch.equal(out[""], out["_nhwc"])
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out[""].double().cpu(), gx_gold, rtol=rtol, atol=atol)


def test_channel_last_grad_out_rejected_outside_its_limits():
    """C != 64 returns DDPM_ERR_UNSUPPORTED before anything is launched."""
    from dynamicconvolutionoperator_b200 import _lib

    lib = _lib.load()
    t = torch.zeros(16, dtype=torch.uint8, device="cuda")
    p = t.data_ptr()
    stream = _lib.stream_handle(t.device)
    for c, code in ((32, 0), (48, 1)):
        rc = lib.ddpm_gencat_bwd_x_staged_nhwc(p, 16, p, p, p, p, 1, c, 8, 16, 3, 1, 3, 5, code,
                                               stream)
        assert rc == -2, (c, code, rc)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_channel_last_dyw_many_tiles_per_cta(dtype):
    """dY + dW with the gradient tile by TMA (channel-last and NCHW) against the
    unstaged pass at B=2, 256^2: about 28 tiles per CTA, so the gradient
    buffer is refilled while earlier tiles are in flight. (A release of that
    buffer before every thread's loads had completed once corrupted a few
    tiles of dY and dW here, and only here.)"""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    shape, ks = (2, 64, 256, 256), 3
    x, y, wt, b = _case(shape, ks, dtype, seed=31)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(32)).to(dtype)
    xd, yd, wd, bd, gd = x.cuda(), y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    st, nb = _stage(xd, yd, ks, (1, 3, 5))
    code = _lib.dtype_code(dtype)
    stream = _lib.stream_handle(xd.device)
    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
    res = {}
    for name in ("unstaged", "staged", "staged_nhwc"):
        gy = torch.full_like(yd, float("nan"))
        gw = torch.full((3 * c * ks * ks, c), float("nan"), dtype=dtype, device="cuda")
        gb = torch.full((3 * c * ks * ks,), float("nan"), dtype=dtype, device="cuda")
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        if name == "unstaged":
            _lib.call("ddpm_gencat_bwd_yw", xd.data_ptr(), yd.data_ptr(), packed.data_ptr(),
                      gd.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                      ws_bytes, n, c, h, w, ks, 1, 3, 5, code, stream)
        else:
            gg = gd.contiguous(memory_format=torch.channels_last) if name.endswith("nhwc") else gd
            _lib.call("ddpm_gencat_bwd_yw_" + name, st.data_ptr(), nb, packed.data_ptr(),
                      gg.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                      ws_bytes, n, c, h, w, ks, 1, 3, 5, code, stream)
        res[name] = (gy.double(), gw.double(), gb.double())
    torch.cuda.synchronize()
    for name in ("staged", "staged_nhwc"):
        for got, ref in zip(res[name], res["unstaged"]):
            scale = ref.abs().max().item()
            assert (got - ref).abs().max().item() <= 2e-2 * scale, name


@pytest.mark.parametrize("shape,dil", [((1, 64, 40, 48), (1, 3, 5)), ((2, 24, 17, 40), (1, 3, 5)),
                                       ((1, 64, 24, 136), (1, 3, 5)), ((1, 64, 13, 152), (1, 8, 4)),
                                       ((2, 16, 21, 24), (6, 2, 1))])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_k5_fused_dyw_matches_oracle(shape, dil, dtype):
    """K = 5 fused dY + dW (16-bit, staged, gradient tile by TMA; octet sets
    of <= 4 per CTA, an x halo of 16 + 2R columns: 36 at halo 10, 48 at the
    largest halo 16 with one x buffer, 28 at halo 6 with two) against the
    float64 oracle, through the NCHW entry and, at C = 64, the channel-last
    one."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    ks = 5
    x, y, wt, b = _case(shape, ks, dtype, seed=41)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(42)).to(dtype)
    _, gy_gold, gw_gold, gb_gold = _gold_grads(x, y, wt, b, g, ks, dil)
    xd, yd, wd, bd, gd = x.cuda(), y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    st, nb = _stage(xd, yd, ks, dil)
    code = _lib.dtype_code(dtype)
    stream = _lib.stream_handle(xd.device)
    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
    assert ws_bytes > 0
    variants = [("", gd)] + ([("_nhwc", gd.contiguous(memory_format=torch.channels_last))]
                             if c == 64 else [])
    for sfx, gg in variants:
        gy = torch.full_like(yd, float("nan"))
        gw = torch.full((3 * c * ks * ks, c), float("nan"), dtype=dtype, device="cuda")
        gb = torch.full((3 * c * ks * ks,), float("nan"), dtype=dtype, device="cuda")
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        _lib.call("ddpm_gencat_bwd_yw_staged" + sfx, st.data_ptr(), nb, packed.data_ptr(),
                  gg.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(), ws.data_ptr(),
                  ws_bytes, n, c, h, w, ks, *dil, code, stream)
        torch.cuda.synchronize()
        for got, ref in ((gy, gy_gold), (gw.view(-1, c, 1, 1), gw_gold), (gb, gb_gold)):
            scale = max(ref.abs().max().item(), 1.0)
            assert (got.double().cpu() - ref).abs().max().item() <= 3e-2 * scale, sfx


def test_k5_fused_dyw_limits():
    """FP32 and unstaged operands are not fused dY + dW shapes at K = 5
    (DDPM_ERR_UNSUPPORTED before any launch); 16-bit data is, at every halo
    the forward covers, when its rows allow the gradient tile's tensor map."""
    from dynamicconvolutionoperator_b200 import _kernels, _lib

    lib = _lib.load()
    for code in (0,):
        rc = lib.ddpm_gencat_bwd_yw_staged(1, 1 << 20, 1, 1, 1, 1, 1, 1, 1 << 20,
                                           1, 64, 16, 16, 5, 1, 3, 5, code, None)
        assert rc == -2
    assert _kernels._fused_dyw_ok(5, torch.bfloat16, 48, (1, 8, 4))
    assert _kernels._fused_dyw_ok(5, torch.bfloat16, 48, (1, 3, 5))
    assert not _kernels._fused_dyw_ok(5, torch.bfloat16, 44, (1, 3, 5))
    assert not _kernels._fused_dyw_ok(5, torch.float32, 48, (1, 3, 5))

