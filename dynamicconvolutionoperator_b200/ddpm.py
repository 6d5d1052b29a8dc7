"""Drop-in ``DDPM`` (Dynamic Dilated Pyramid Module) for B200.

Mirrors the reference's ``triton_impl.DDPM`` (``triton_impl.py:247-392``):
same constructor arguments and validation messages, same parameters and
state-dict keys (``generator.weight [3CK^2, C, 1, 1]``, ``generator.bias``,
``fuse.weight [C, 4C, 3, 3]``, ``fuse.bias``), same ``forward(x, y)`` and
autograd contract, so state dicts interchange with the reference's
``unfold_impl.DDPM`` and ``triton_impl.DDPM`` in both directions.

What changed is the GPU body: the Triton kernels, autotune tables and the
silent CPU fallback (``triton_impl.py:23-33, 353-354``) are replaced by the
sm_100a kernels of ``libddpm_b200.so``. CUDA tensors always take the native
path; CPU tensors raise (the reference's CPU branches are not part of this
build). The final 3x3 ``fuse`` convolution (a cuDNN call in the reference,
``triton_impl.py:294, 392``) runs on the library's own tensor-core kernels for
C <= 64 (``native_fuse=True``, the default) and on cuDNN otherwise. Under
autocast the module runs on the same native kernels in the autocast dtype
(inputs and parameters cast once, differentiably).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from . import _fuseconv, _kernels

_DEFAULT_DILATIONS = (1, 3, 5)


def _check_inputs(x: torch.Tensor, y: torch.Tensor, channels: int) -> None:
    """Input contract of the reference (``triton_impl.py:36-44``), same messages."""
    if x.ndim != 4 or y.ndim != 4:
        raise ValueError(f"x and y must be NCHW tensors, got {x.shape=} and {y.shape=}")
    if x.shape != y.shape:
        raise ValueError(f"x and y must have identical shapes, got {x.shape=} and {y.shape=}")
    if x.shape[1] != channels:
        raise ValueError(f"expected {channels} channels, got {x.shape[1]}")
    if x.device != y.device:
        raise ValueError(f"x and y must be on the same device, got {x.device} and {y.device}")


def _autocast_enabled() -> bool:
    try:
        return torch.is_autocast_enabled("cuda")
    except TypeError:  # older signature
        return torch.is_autocast_enabled()


class DDPM(nn.Module):
    """Dynamic Dilated Pyramid Module with sm_100a fused and materialised paths.

    Args:
        dim: Input/output channel count.
        kernel_size: Odd dynamic depthwise kernel size.
        spatial_tile_size: Kept for API compatibility (the reference's CPU
            streaming tile, ``triton_impl.py:253-254``); unused on the GPU.
        max_generated_bytes: Kept for API compatibility (CPU budget,
            ``triton_impl.py:255-257``); unused on the GPU.
        recompute: Kept for API compatibility (CPU checkpointing).
        fused_generator_inference: Fuse the 1x1 generator with the dynamic
            filter (taps never reach HBM) when gradients are disabled.
        fused_generator_training: ``None`` (default) picks the path from the
            measured crossover, ``True`` always uses the flash-style recompute
            training path, ``False`` always materialises the taps.
        native_fuse: Run the 3x3 ``fuse`` convolution on this library's
            tensor-core kernels (C <= 64; single rounding of conv + bias, no
            TF32). ``False`` keeps the reference's cuDNN call.
    """

    def __init__(
        self,
        dim: int,
        kernel_size: int = 3,
        *,
        spatial_tile_size: int = 4096,
        max_generated_bytes: int = 256 * 1024**2,
        recompute: bool = True,
        fused_generator_inference: bool = True,
        fused_generator_training: bool | None = None,
        native_fuse: bool = True,
    ) -> None:
        super().__init__()
        if kernel_size < 1 or kernel_size % 2 == 0:
            raise ValueError(f"kernel_size must be a positive odd integer, got {kernel_size}")
        if dim < 1:
            raise ValueError(f"dim must be positive, got {dim}")

        self.dim = dim
        self.kernel_size = kernel_size
        self.spatial_tile_size = spatial_tile_size
        self.max_generated_bytes = max_generated_bytes
        self.recompute = recompute
        self.fused_generator_inference = fused_generator_inference
        self.fused_generator_training = fused_generator_training
        self.native_fuse = native_fuse
        self.dilations = _DEFAULT_DILATIONS
        self.generator = nn.Conv2d(dim, 3 * dim * kernel_size**2, 1)
        self.fuse = nn.Conv2d(4 * dim, dim, 3, 1, 1)

    # ------------------------------------------------------------ dispatch --
    def _fused_generator_ok(self, x: torch.Tensor, y: torch.Tensor,
                            weight: torch.Tensor, bias: torch.Tensor | None) -> bool:
        """Dtype/bias preconditions of the fused generator path (reference
        ``triton_impl.py:322-329``) plus this build's kernel limits."""
        return (
            x.dtype == y.dtype == weight.dtype
            and bias is not None
            and bias.dtype == x.dtype
            and _kernels.fused_generator_supported(self.dim, self.kernel_size, x.dtype,
                                                   self.dilations)
        )

    def _use_fused_training(self, x: torch.Tensor) -> bool:
        requested = self.fused_generator_training
        if requested is None:
            requested = _kernels.auto_fuse_training(
                x.shape[0] * x.shape[2] * x.shape[3], self.dim, self.kernel_size, x.dtype
            )
        return bool(requested) and _kernels.fused_training_supported(self.kernel_size)

    def _cuda_cat(self, x: torch.Tensor, y: torch.Tensor, weight: torch.Tensor,
                  bias: torch.Tensor | None, fuse_planes: bool = False) -> torch.Tensor:
        """GPU path selection (replaces ``DDPM._cuda_cat``, ``triton_impl.py:305-348``)
        with the generator's ``weight`` and ``bias`` (the parameters, or their
        autocast copies). ``fuse_planes``: the native fuse conv will consume the
        output, so the fused forward may also write it as the fuse conv's
        staged planes."""
        grad = torch.is_grad_enabled()
        fuse_training = grad and self._use_fused_training(x)
        want_fused = (self.fused_generator_inference and not grad) or fuse_training
        if want_fused and self._fused_generator_ok(x, y, weight, bias):
            return _kernels.fused_generator_dynamic_cat(
                x, y, weight, bias, self.kernel_size, self.dilations, _fuse_planes=fuse_planes,
            )
        kernels = _kernels.generator_taps(y, weight, bias).reshape(
            x.shape[0],
            len(self.dilations),
            self.dim,
            self.kernel_size**2,
            x.shape[2],
            x.shape[3],
        )
        return _kernels.fused_dynamic_cat(x, kernels, self.kernel_size, self.dilations)

    def forward(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        _check_inputs(x, y, self.dim)
        if not x.is_cuda:
            raise RuntimeError(
                "DDPM (B200 build) runs on CUDA tensors only; got tensors on "
                f"{x.device}. The reference's CPU paths are not part of this build."
            )
        gen, fuse = self.generator, self.fuse
        params = (gen.weight, gen.bias, fuse.weight, fuse.bias)
        if _autocast_enabled():
            # Under autocast both convolutions of the module run in the autocast
            # dtype (as nn.Conv2d does under autocast), so the whole module runs
            # on the native kernels in that dtype: inputs and parameters are
            # cast once (differentiably: gradients reach the FP32 parameters)
            # and autocast is off inside. The reference instead declines its
            # fused path under autocast (``triton_impl.py:325``); the output
            # dtype is the autocast dtype on both.
            ac = torch.get_autocast_dtype("cuda")
            with torch.autocast("cuda", enabled=False):
                x, y, *params = (t.to(ac) if t is not None and t.is_floating_point() else t
                                 for t in (x, y, *params))
                return self._forward_cuda(x, y, *params, autocast_dtype=ac)
        return self._forward_cuda(x, y, *params)

    def _forward_cuda(self, x, y, gen_w, gen_b, fuse_w, fuse_b, autocast_dtype=None):
        fuse = self.fuse
        if not _is_standard_fuse(fuse):
            # a replaced fuse module of another kind or configuration runs its
            # own forward (under the caller's autocast, if there was one)
            cat_out = self._cuda_cat(x, y, gen_w, gen_b)
            with torch.autocast("cuda", enabled=autocast_dtype is not None,
                                dtype=autocast_dtype or torch.bfloat16):
                return fuse(cat_out)
        native = self.native_fuse and fuse_w.dtype == x.dtype
        cat_out = self._cuda_cat(x, y, gen_w, gen_b, fuse_planes=native)
        if native and _fuseconv.fuse_conv_supported(cat_out, fuse_w, fuse_b, fuse):
            return _fuseconv.fuse_conv(cat_out, fuse_w, fuse_b)
        if (
            cat_out.dtype in (torch.bfloat16, torch.float16)
            and fuse_w.dtype == cat_out.dtype
            and fuse_b is not None
        ):
            return _fuse_single_rounding(cat_out, fuse_w, fuse_b)
        return F.conv2d(cat_out, fuse_w, fuse_b, 1, 1)


def _is_standard_fuse(fuse: nn.Module) -> bool:
    """``fuse`` is the module's own kind of layer: a 3x3 ``nn.Conv2d`` with
    stride 1, padding 1 (zeros), dilation 1 and one group."""
    return (
        type(fuse) is nn.Conv2d
        and tuple(fuse.kernel_size) == (3, 3)
        and tuple(fuse.stride) == (1, 1)
        and tuple(fuse.padding) == (1, 1)
        and tuple(fuse.dilation) == (1, 1)
        and fuse.groups == 1
        and fuse.padding_mode == "zeros"
    )


_BIAS_LANES = 8  # extra input channels carrying the folded bias (keeps Cin % 8 == 0)


def _fuse_single_rounding(cat: torch.Tensor, weight: torch.Tensor,
                          bias: torch.Tensor) -> torch.Tensor:
    """The 3x3 ``fuse`` conv with its bias folded into the cuDNN contraction.

    ``nn.Conv2d`` on cuDNN adds the bias after the convolution has been
    rounded to the 16-bit output type, so a bf16 output is rounded twice
    (up to one ulp, 0.031 for |out| in [4, 8)). Here the bias rides in the
    contraction as a constant-one input channel whose only non-zero weight is
    the centre tap, so cuDNN's FP32 accumulator holds conv + bias and the
    output is rounded once. Same result up to that rounding, same gradients
    (the bias gradient is the ones channel's centre-tap weight gradient).
    """
    n, _, h, w = cat.shape
    c_out = weight.shape[0]
    lanes = cat.new_zeros((n, _BIAS_LANES, h, w))
    lanes[:, 0].fill_(1)
    # [C, 8, 3, 3]: bias at input lane 0, centre tap (1, 1); zeros elsewhere
    bias_block = torch.nn.functional.pad(bias.reshape(c_out, 1, 1, 1),
                                         (1, 1, 1, 1, 0, _BIAS_LANES - 1))
    return torch.nn.functional.conv2d(torch.cat((cat, lanes), 1),
                                      torch.cat((weight, bias_block), 1), None, 1, 1)


__all__ = ["DDPM"]
