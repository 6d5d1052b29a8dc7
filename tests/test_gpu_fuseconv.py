"""Native 3x3 fuse convolution (forward and data gradient) against a float64
reference of the same convolution (``nn.Conv2d(4C, C, 3, 1, 1)``,
reference ``triton_impl.py:294``), through the C ABI."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

# (n, cin, cout, h, w): DDPM shapes (cin = 4 * cout) plus ragged edges
SHAPES = [
    (2, 96, 24, 15, 17),
    (1, 12, 3, 5, 7),
    (1, 256, 64, 64, 64),
    (3, 160, 40, 33, 130),
    (1, 256, 64, 256, 256),
    (1, 64, 16, 1, 1),
    (2, 200, 50, 9, 257),
]
# fp32: bf16 hi + lo operands (~1e-5 relative per product); 16-bit: one output
# rounding of the FP32 accumulator (half an ulp) plus accumulation order.
TOL = {torch.float32: (2e-5, 2e-4), torch.bfloat16: (8e-3, 2e-2), torch.float16: (1e-3, 4e-3)}


def _inputs(shape, dtype, seed=0):
    n, cin, cout, h, w = shape
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn((n, cin, h, w), generator=gen).to(dtype)
    bound = 1.0 / (cin * 9) ** 0.5
    wt = ((torch.rand((cout, cin, 3, 3), generator=gen) * 2 - 1) * bound).to(dtype)
    b = ((torch.rand(cout, generator=gen) * 2 - 1) * bound).to(dtype)
    g = torch.randn((n, cout, h, w), generator=gen).to(dtype)
    return x, wt, b, g


def _pack(wt, cin, cout, dtype):
    from dynamicconvolutionoperator_b200 import _lib

    nbytes = int(_lib.load().ddpm_fuseconv_pack_bytes(cin, cout, _lib.dtype_code(dtype)))
    packed = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("ddpm_fuseconv_pack", wt.data_ptr(), cin, cout, _lib.dtype_code(dtype),
              packed.data_ptr(), nbytes, _lib.stream_handle(packed.device))
    return packed


def _stage(src):
    """src as staged planes (ddpm_fuseconv_stage); filler bytes, so nothing
    relies on the buffer starting at zero."""
    from dynamicconvolutionoperator_b200 import _lib

    n, c, h, w = src.shape
    code = _lib.dtype_code(src.dtype)
    nbytes = int(_lib.load().ddpm_fuseconv_stage_bytes(n, c, h, w, code))
    assert nbytes > 0
    planes = torch.full((nbytes,), 0x5A, dtype=torch.uint8, device="cuda")
    _lib.call("ddpm_fuseconv_stage", src.data_ptr(), planes.data_ptr(), nbytes, n, c, h, w, code,
              _lib.stream_handle(planes.device))
    return planes, nbytes


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fuseconv_forward(shape, dtype):
    """Unstaged and staged-plane forward: both within tolerance of float64,
    and equal to each other bit for bit (same operands, same MMA order)."""
    from dynamicconvolutionoperator_b200 import _lib

    n, cin, cout, h, w = shape
    x, wt, b, _ = _inputs(shape, dtype)
    xd, wd, bd = x.cuda(), wt.cuda(), b.cuda()
    packed = _pack(wd, cin, cout, dtype)
    out = torch.full((n, cout, h, w), float("nan"), dtype=dtype, device="cuda")
    _lib.call("ddpm_fuseconv_fwd", xd.data_ptr(), packed.data_ptr(), bd.data_ptr(),
              out.data_ptr(), n, cin, cout, h, w, _lib.dtype_code(dtype),
              _lib.stream_handle(out.device))
    planes, nbytes = _stage(xd)
    out_s = torch.full_like(out, float("nan"))
    _lib.call("ddpm_fuseconv_fwd_staged", planes.data_ptr(), nbytes, packed.data_ptr(),
              bd.data_ptr(), out_s.data_ptr(), n, cin, cout, h, w, _lib.dtype_code(dtype),
              _lib.stream_handle(out.device))
    torch.cuda.synchronize()
    gold = F.conv2d(xd.double(), wd.double(), bd.double(), 1, 1)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(out.double(), gold, rtol=rtol, atol=atol)
    torch.testing.assert_close(out_s, out, rtol=0, atol=0)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fuseconv_bwd_data(shape, dtype):
    from dynamicconvolutionoperator_b200 import _lib

    n, cin, cout, h, w = shape
    x, wt, _, g = _inputs(shape, dtype, seed=1)
    wd, gd = wt.cuda(), g.cuda()
    packed = _pack(wd, cin, cout, dtype)
    gx = torch.full((n, cin, h, w), float("nan"), dtype=dtype, device="cuda")
    _lib.call("ddpm_fuseconv_bwd_data", gd.data_ptr(), packed.data_ptr(), gx.data_ptr(),
              n, cin, cout, h, w, _lib.dtype_code(dtype), _lib.stream_handle(gx.device))
    planes, nbytes = _stage(gd)
    gx_s = torch.full_like(gx, float("nan"))
    _lib.call("ddpm_fuseconv_bwd_data_staged", planes.data_ptr(), nbytes, packed.data_ptr(),
              gx_s.data_ptr(), n, cin, cout, h, w, _lib.dtype_code(dtype),
              _lib.stream_handle(gx.device))
    torch.cuda.synchronize()
    gold = torch.nn.grad.conv2d_input((n, cin, h, w), wd.double(), gd.double(), 1, 1)
    rtol, atol = TOL[dtype]
    torch.testing.assert_close(gx.double(), gold, rtol=rtol, atol=atol)
    torch.testing.assert_close(gx_s, gx, rtol=0, atol=0)


def test_fuseconv_rejects_unsupported():
    from dynamicconvolutionoperator_b200 import _lib

    lib = _lib.load()
    assert lib.ddpm_fuseconv_pack_bytes(257, 64, 0) == 0
    rc = lib.ddpm_fuseconv_fwd(None, None, None, None, 1, 256, 65, 4, 4, 0, None)
    assert rc == -2


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fuseconv_bwd_weight(shape, dtype):
    """Weight and bias gradient vs float64 (normalised by the largest gold
    magnitude: they sum over every pixel)."""
    from dynamicconvolutionoperator_b200 import _lib

    n, cin, cout, h, w = shape
    x, wt, _, g = _inputs(shape, dtype, seed=2)
    xd, gd = x.cuda(), g.cuda()
    gw = torch.full((cout, cin, 3, 3), float("nan"), dtype=dtype, device="cuda")
    gb = torch.full((cout,), float("nan"), dtype=dtype, device="cuda")
    nbytes = int(_lib.load().ddpm_fuseconv_bwd_weight_workspace_bytes(n, cin, cout, h, w))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("ddpm_fuseconv_bwd_weight", xd.data_ptr(), gd.data_ptr(), gw.data_ptr(),
              gb.data_ptr(), ws.data_ptr(), nbytes, n, cin, cout, h, w, _lib.dtype_code(dtype),
              _lib.stream_handle(xd.device))
    torch.cuda.synchronize()
    gold_w = torch.nn.grad.conv2d_weight(xd.double(), (cout, cin, 3, 3), gd.double(), 1, 1)
    gold_b = gd.double().sum(dim=(0, 2, 3))
    tol = 2e-5 if dtype == torch.float32 else 1e-2
    for got, gold in ((gw, gold_w), (gb, gold_b)):
        scale = gold.abs().max().item() + 1e-12
        err = (got.double() - gold).abs().max().item() / scale
        assert err <= tol, err


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fuseconv_bwd_combined(shape, dtype):
    """ddpm_fuseconv_bwd (data + weight/bias gradient in one call; for widths
    that are a multiple of 8 the data gradient reads grad_out from the weight
    gradient's channel-last copy) equals ddpm_fuseconv_bwd_data and
    ddpm_fuseconv_bwd_weight bit for bit."""
    from dynamicconvolutionoperator_b200 import _lib

    n, cin, cout, h, w = shape
    x, wt, b, g = _inputs(shape, dtype, seed=2)
    xd, wd, gd = x.cuda(), wt.cuda(), g.cuda()
    packed = _pack(wd, cin, cout, dtype)
    code = _lib.dtype_code(dtype)
    st = _lib.stream_handle(xd.device)
    nb = int(_lib.load().ddpm_fuseconv_bwd_weight_workspace_bytes(n, cin, cout, h, w))
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    gx_ref = torch.full_like(xd, float("nan"))
    gw_ref = torch.full_like(wd, float("nan"))
    gb_ref = torch.full((cout,), float("nan"), dtype=dtype, device="cuda")
    _lib.call("ddpm_fuseconv_bwd_data", gd.data_ptr(), packed.data_ptr(), gx_ref.data_ptr(),
              n, cin, cout, h, w, code, st)
    _lib.call("ddpm_fuseconv_bwd_weight", xd.data_ptr(), gd.data_ptr(), gw_ref.data_ptr(),
              gb_ref.data_ptr(), ws.data_ptr(), nb, n, cin, cout, h, w, code, st)
    gx = torch.full_like(gx_ref, float("nan"))
    gw = torch.full_like(gw_ref, float("nan"))
    gb = torch.full_like(gb_ref, float("nan"))
    ws.fill_(0x5A)
    _lib.call("ddpm_fuseconv_bwd", xd.data_ptr(), gd.data_ptr(), packed.data_ptr(), gx.data_ptr(),
              gw.data_ptr(), gb.data_ptr(), ws.data_ptr(), nb, n, cin, cout, h, w, code, st)
    torch.cuda.synchronize()
    torch.testing.assert_close(gx, gx_ref, rtol=0, atol=0)
    torch.testing.assert_close(gw, gw_ref, rtol=0, atol=0)
    torch.testing.assert_close(gb, gb_ref, rtol=0, atol=0)


@pytest.mark.parametrize("shape", [(2, 256, 64, 15, 24), (1, 256, 64, 32, 136), (1, 32, 16, 9, 40)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_fuseconv_bwd_nhwc_matches_nchw(shape, dtype):
    """ddpm_fuseconv_bwd_nhwc writes grad_x channel-last with the values of
    ddpm_fuseconv_bwd bit for bit (and the same weight / bias gradients)."""
    from dynamicconvolutionoperator_b200 import _lib

    n, cin, cout, h, w = shape
    x, wt, b, g = _inputs(shape, dtype, seed=9)
    xd, wd, gd = x.cuda(), wt.cuda(), g.cuda()
    packed = _pack(wd, cin, cout, dtype)
    code = _lib.dtype_code(dtype)
    st = _lib.stream_handle(xd.device)
    nb = int(_lib.load().ddpm_fuseconv_bwd_weight_workspace_bytes(n, cin, cout, h, w))
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    outs = {}
    for name in ("ddpm_fuseconv_bwd", "ddpm_fuseconv_bwd_nhwc"):
        cl = name.endswith("nhwc")
        gx = torch.full_like(xd, float("nan"),
                             memory_format=torch.channels_last if cl else torch.contiguous_format)
        gw = torch.full_like(wd, float("nan"))
        gb = torch.full((cout,), float("nan"), dtype=dtype, device="cuda")
        _lib.call(name, xd.data_ptr(), gd.data_ptr(), packed.data_ptr(), gx.data_ptr(),
                  gw.data_ptr(), gb.data_ptr(), ws.data_ptr(), nb, n, cin, cout, h, w, code, st)
        outs[name] = (gx, gw, gb)
    torch.cuda.synchronize()
    ref, got = outs["ddpm_fuseconv_bwd"], outs["ddpm_fuseconv_bwd_nhwc"]
    assert got[0].is_contiguous(memory_format=torch.channels_last)
    for a, r in zip(got, ref):
        assert torch.equal(a, r)  # value comparison, layout-independent
