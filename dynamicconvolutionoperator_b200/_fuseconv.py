"""Native 3x3 fuse convolution of the DDPM (``nn.Conv2d(4C, C, 3, 1, 1)``).

The reference leaves this convolution to cuDNN (``triton_impl.py:294, 392``).
On B200 that call runs true FP32 on cuDNN's FFT / SIMT kernels (about 2 ms of
a 3 ms training step at 256^2) and, for bf16 / fp16 outputs, adds the bias
after the convolution has been rounded (two roundings). ``fuse_conv`` runs it
on the library's tensor-core kernels instead (``ddpm_fuseconv_*`` in
``include/ddpm_b200.h``): FP32 as bf16 hi + lo operands, the bias added to the
FP32 accumulator before a single output rounding. Same parameters, same
autograd contract as ``nn.Conv2d``.

The backward runs on the same library: data gradient (shifted-window GEMM)
and weight / bias gradient (split spatial reduction into FP32 partials).

The forward and the data gradient first stage their source tensor (x, resp.
grad_out) once as zero-padded channel-group planes (``ddpm_fuseconv_stage``),
which the staged kernels read with one TMA copy per K slab; the results equal
the unstaged entry points bit for bit.
"""

from __future__ import annotations

import torch

from . import _lib
from ._gradbuf import grad_buffer
from ._kernels import FUSE_PLANES_ATTR

FUSE_MAX_CIN = 256
FUSE_MAX_COUT = 64


def fuse_conv_supported(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                        conv: torch.nn.Conv2d | None = None) -> bool:
    """Shapes and dtypes the native kernels cover: a 3x3 convolution with
    stride 1, padding 1 (zeros), dilation 1 and one group. With ``conv`` its
    configuration is checked too, so a replaced ``fuse`` module of another
    configuration goes to its own forward instead."""
    if conv is not None and not (
        tuple(conv.stride) == (1, 1)
        and tuple(conv.padding) == (1, 1)
        and tuple(conv.dilation) == (1, 1)
        and conv.groups == 1
        and conv.padding_mode == "zeros"
    ):
        return False
    return (
        x.is_cuda
        and x.ndim == 4
        and x.dtype in _lib.DTYPE_CODE
        and weight.dtype == x.dtype
        and (bias is None or bias.dtype == x.dtype)
        and weight.ndim == 4
        and tuple(weight.shape[2:]) == (3, 3)
        and weight.shape[1] == x.shape[1]
        and weight.shape[0] <= FUSE_MAX_COUT
        and weight.shape[1] <= FUSE_MAX_CIN
    )


def nhwc_grad_ok(cat: torch.Tensor) -> bool:
    """Whether the gradient of a fused generator output ``cat`` [N, 4C, H, W]
    can travel channel-last to the generator's backward (C == 64)."""
    return cat.shape[1] == 256


def pack_fuse_weight(weight: torch.Tensor) -> torch.Tensor:
    """The weight in the kernels' shared-memory operand layout (forward and
    data-gradient images). Packed on every forward (one small launch): a copy
    cached across calls would miss writes through ``param.data``, which leave
    the version counter untouched."""
    cout, cin = weight.shape[0], weight.shape[1]
    code = _lib.dtype_code(weight.dtype)
    nbytes = int(_lib.load().ddpm_fuseconv_pack_bytes(cin, cout, code))
    packed = torch.empty(nbytes, dtype=torch.uint8, device=weight.device)
    w = weight.contiguous()
    _lib.call("ddpm_fuseconv_pack", w.data_ptr(), cin, cout, code, packed.data_ptr(), nbytes,
              _lib.stream_handle(weight.device))
    return packed


def _stage_planes(src: torch.Tensor) -> tuple[torch.Tensor, int]:
    """``src`` [N, C, H, W] as the staged operand planes (``ddpm_fuseconv_stage``)."""
    n, c, h, w = src.shape
    code = _lib.dtype_code(src.dtype)
    nbytes = int(_lib.load().ddpm_fuseconv_stage_bytes(n, c, h, w, code))
    planes = torch.empty(nbytes, dtype=torch.uint8, device=src.device)
    _lib.call("ddpm_fuseconv_stage", src.data_ptr(), planes.data_ptr(), nbytes, n, c, h, w, code,
              _lib.stream_handle(src.device))
    return planes, nbytes


class _FuseConv(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, planes_in):
        x = x.contiguous()
        n, cin, h, w = x.shape
        cout = weight.shape[0]
        packed = pack_fuse_weight(weight)
        out = torch.empty((n, cout, h, w), dtype=x.dtype, device=x.device)
        b = bias.contiguous() if bias is not None else None
        # the producer's own planes of x when it wrote them, else one staging pass
        planes, nbytes = planes_in[:2] if planes_in is not None else _stage_planes(x)
        _lib.call("ddpm_fuseconv_fwd_staged", planes.data_ptr(), nbytes, packed.data_ptr(),
                  b.data_ptr() if b is not None else None, out.data_ptr(),
                  n, cin, cout, h, w, _lib.dtype_code(x.dtype), _lib.stream_handle(x.device))
        ctx.save_for_backward(x, weight)
        ctx.bias = bias  # the parameter itself (its gradient buffer is looked up by identity)
        ctx.packed = packed
        ctx.has_bias = bias is not None
        # x came from the fused generator forward (its planes): the gradient of x
        # goes to that generator's backward, which reads it channel-last where
        # its producer said so (the fully fused backward kernels, K <= 3)
        ctx.grad_nhwc = planes_in is not None and planes_in[2] and nhwc_grad_ok(x)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, weight = ctx.saved_tensors
        g = grad_out.contiguous()
        n, cin, h, w = x.shape
        cout = weight.shape[0]
        gx = gw = gb = None
        need_b = ctx.has_bias and ctx.needs_input_grad[2]
        if ctx.needs_input_grad[0] and (ctx.needs_input_grad[1] or need_b):
            # both in one call: the data gradient reads grad_out from the
            # channel-last copy the weight gradient makes anyway
            nhwc = ctx.grad_nhwc
            gx = (torch.empty_like(x, memory_format=torch.channels_last) if nhwc
                  else torch.empty_like(x))
            gw = (grad_buffer(weight, weight.shape, x.dtype, x.device)
                  if ctx.needs_input_grad[1] else torch.empty_like(weight))
            gb = grad_buffer(ctx.bias, (cout,), x.dtype, x.device) if need_b else None
            nbytes = int(_lib.load().ddpm_fuseconv_bwd_weight_workspace_bytes(n, cin, cout, h, w))
            ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
            _lib.call("ddpm_fuseconv_bwd_nhwc" if nhwc else "ddpm_fuseconv_bwd", x.data_ptr(), g.data_ptr(), ctx.packed.data_ptr(),
                      gx.data_ptr(), gw.data_ptr(), gb.data_ptr() if gb is not None else None,
                      ws.data_ptr(), nbytes, n, cin, cout, h, w, _lib.dtype_code(x.dtype),
                      _lib.stream_handle(x.device))
            return gx, (gw if ctx.needs_input_grad[1] else None), gb, None
        if ctx.needs_input_grad[0]:
            gx = torch.empty_like(x)
            planes, nbytes = _stage_planes(g)
            _lib.call("ddpm_fuseconv_bwd_data_staged", planes.data_ptr(), nbytes,
                      ctx.packed.data_ptr(), gx.data_ptr(), n, cin, cout, h, w,
                      _lib.dtype_code(x.dtype), _lib.stream_handle(x.device))
        if ctx.needs_input_grad[1] or need_b:
            gw = (grad_buffer(weight, weight.shape, x.dtype, x.device)
                  if ctx.needs_input_grad[1] else torch.empty_like(weight))
            gb = grad_buffer(ctx.bias, (cout,), x.dtype, x.device) if need_b else None
            nbytes = int(_lib.load().ddpm_fuseconv_bwd_weight_workspace_bytes(n, cin, cout, h, w))
            ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
            _lib.call("ddpm_fuseconv_bwd_weight", x.data_ptr(), g.data_ptr(), gw.data_ptr(),
                      gb.data_ptr() if gb is not None else None, ws.data_ptr(), nbytes,
                      n, cin, cout, h, w, _lib.dtype_code(x.dtype),
                      _lib.stream_handle(x.device))
            if not ctx.needs_input_grad[1]:
                gw = None
        return gx, gw, gb, None


def fuse_conv(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """``F.conv2d(x, weight, bias, 1, 1)`` for a 3x3 weight on the native kernels."""
    _lib.load()
    # Staged planes written by the producer of x (the fused generator forward),
    # valid while x is unmodified; taken off x so they are freed after use.
    planes_in = None
    held = getattr(x, FUSE_PLANES_ATTR, None)
    if held is not None:
        delattr(x, FUSE_PLANES_ATTR)
        if held[2] == x._version and x.is_contiguous():
            planes_in = (held[0], held[1], held[3])
    return _FuseConv.apply(x, weight, bias, planes_in)


__all__ = ["fuse_conv", "fuse_conv_supported", "pack_fuse_weight"]
