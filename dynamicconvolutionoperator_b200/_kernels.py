"""Autograd front-ends of the sm_100a DDPM kernels.

Drop-in for the reference's ``_triton_kernels.py`` public surface
(``fused_dynamic_cat``, ``fused_generator_dynamic_cat``; reference
``_triton_kernels.py:869-870`` and ``:1056-1065``). Each op launches the
C-ABI entry points of ``libddpm_b200.so`` on torch's current CUDA stream;
outputs and workspaces come from the PyTorch caching allocator. There is no
Triton and no CPU or eager-PyTorch fallback: non-CUDA tensors raise.
"""

from __future__ import annotations

import torch

from . import _lib


def _require_cuda(*tensors: torch.Tensor) -> None:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                "the DDPM B200 kernels require CUDA tensors; got a tensor on "
                f"{t.device} (the reference's CPU paths are not part of this build)"
            )
        if t.device != dev:
            raise RuntimeError(f"all tensors must be on one device, got {dev} and {t.device}")


def _dil(dilations) -> tuple[int, int, int]:
    d = tuple(int(v) for v in dilations)
    if len(d) != 3:
        raise ValueError(f"exactly three dilations are required, got {dilations!r}")
    return d


class _DynamicCat(torch.autograd.Function):
    """Materialised dynamic filter (reference ``_DynamicCat``, ``_triton_kernels.py:814-866``).

    Saves ``(x, kernels)``; backward returns ``(grad_x, grad_kernels, None, None)``.
    The output has ``kernels.dtype`` (reference ``:820-822``).
    """

    @staticmethod
    def forward(ctx, x, kernels, kernel_size, dilations):
        x = x.contiguous()
        kernels = kernels.contiguous()
        _require_cuda(x, kernels)
        n, c, h, w = x.shape
        ks = int(kernel_size)
        d0, d1, d2 = _dil(dilations)
        expect = (n, 3, c, ks * ks, h, w)
        if tuple(kernels.shape) != expect:
            raise ValueError(f"kernels must have shape {expect}, got {tuple(kernels.shape)}")
        out = torch.empty((n, 4 * c, h, w), dtype=kernels.dtype, device=x.device)
        with torch.cuda.device(x.device):
            _lib.call(
                "ddpm_dyncat_fwd",
                x.data_ptr(), _lib.dtype_code(x.dtype),
                kernels.data_ptr(), _lib.dtype_code(kernels.dtype),
                out.data_ptr(),
                n, c, h, w, ks, d0, d1, d2,
                _lib.stream_handle(x.device),
            )
        ctx.save_for_backward(x, kernels)
        ctx.kernel_size = ks
        ctx.dilations = (d0, d1, d2)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x, kernels = ctx.saved_tensors
        grad_out = grad_out.to(kernels.dtype).contiguous()
        n, c, h, w = x.shape
        need_x, need_k = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        grad_x = torch.empty_like(x) if need_x else None
        grad_k = torch.empty_like(kernels) if need_k else None
        if need_x or need_k:
            d0, d1, d2 = ctx.dilations
            with torch.cuda.device(x.device):
                _lib.call(
                    "ddpm_dyncat_bwd",
                    x.data_ptr(), _lib.dtype_code(x.dtype),
                    kernels.data_ptr(), grad_out.data_ptr(), _lib.dtype_code(kernels.dtype),
                    grad_x.data_ptr() if need_x else None,
                    grad_k.data_ptr() if need_k else None,
                    n, c, h, w, ctx.kernel_size, d0, d1, d2,
                    _lib.stream_handle(x.device),
                )
        return grad_x, grad_k, None, None


def fused_dynamic_cat(x, kernels, kernel_size, dilations):
    """``cat([x, d1, d3, d5])`` from materialised taps (reference ``_triton_kernels.py:869``)."""
    return _DynamicCat.apply(x, kernels, kernel_size, dilations)


# ------------------------------------------------------------------ policy --
# Limits of the fused generator kernels of this build (tcgen05 tiles hold the
# padded channel count in shared memory and TMEM).
FUSED_MAX_CHANNELS = 64
FUSED_KERNEL_SIZES = (1, 3)


def fused_generator_supported(channels: int, kernel_size: int, dtype: torch.dtype) -> bool:
    """Whether the fused generator+filter kernels cover this configuration."""
    return False


def fused_training_supported(kernel_size: int) -> bool:
    """The flash-style recompute backward covers K <= 3, like the reference
    (``triton_impl.py:320``)."""
    return kernel_size in FUSED_KERNEL_SIZES


def auto_fuse_training(tokens: int, channels: int, kernel_size: int, dtype: torch.dtype) -> bool:
    """Auto crossover between the fused and materialised training paths.

    The reference fuses above 16384 spatial tokens (and at exactly 16384 for
    FP32), measured on an RTX 5090 (``triton_impl.py:313-316``).
    """
    return tokens > 16384 or (tokens == 16384 and dtype == torch.float32)


def fused_generator_dynamic_cat(x, y, weight, bias, kernel_size, dilations):
    """Fused 1x1 generator + dynamic filter (reference ``_triton_kernels.py:1056``)."""
    raise NotImplementedError("fused generator kernels are not built in this version")


__all__ = ["fused_dynamic_cat", "fused_generator_dynamic_cat"]
