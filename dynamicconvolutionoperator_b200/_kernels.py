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
from ._gradbuf import grad_buffer, grads_written


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
        grad_x, grad_k = _dyncat_backward(x, kernels, grad_out, ctx.kernel_size, ctx.dilations,
                                          ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return grad_x, grad_k, None, None


def _dyncat_backward(x, kernels, grad_out, ks, dilations, need_x, need_k):
    """(grad_x, grad_kernels) of the materialised filter (``ddpm_dyncat_bwd``)."""
    grad_out = grad_out.to(kernels.dtype).contiguous()
    n, c, h, w = x.shape
    grad_x = torch.empty_like(x) if need_x else None
    grad_k = torch.empty_like(kernels) if need_k else None
    if need_x or need_k:
        d0, d1, d2 = dilations
        with torch.cuda.device(x.device):
            _lib.call(
                "ddpm_dyncat_bwd",
                x.data_ptr(), _lib.dtype_code(x.dtype),
                kernels.data_ptr(), grad_out.data_ptr(), _lib.dtype_code(kernels.dtype),
                grad_x.data_ptr() if need_x else None,
                grad_k.data_ptr() if need_k else None,
                n, c, h, w, ks, d0, d1, d2,
                _lib.stream_handle(x.device),
            )
    return grad_x, grad_k


def fused_dynamic_cat(x, kernels, kernel_size, dilations):
    """``cat([x, d1, d3, d5])`` from materialised taps (reference ``_triton_kernels.py:869``)."""
    return _DynamicCat.apply(x, kernels, kernel_size, dilations)


# ------------------------------------------------------------------ policy --
# Limits of the fused generator kernels of this build (tcgen05 tiles hold the
# padded channel count in shared memory and TMEM).
FUSED_MAX_CHANNELS = 64
# Kernel sizes of the fused forward, and of the fully fused (flash-style
# recompute) backward kernels in every dtype. At K = 5 the fused backward
# kernels cover 16-bit data (``_fused_dyw_ok``); FP32 pairs the fused forward
# and dX kernels with a materialised dK (``_k5_backward``). The reference
# fuses training for K <= 3 only (``triton_impl.py:320``).
FUSED_KERNEL_SIZES = (1, 3, 5)
FUSED_TRAINING_KERNEL_SIZES = (1, 3)
FUSED_BACKWARD_AVAILABLE = True

# Largest dilation halo (K // 2) * max(dilations) of the fused forward per K:
# the x halo tile spans 8 (K <= 3) or 16 (K = 5) pixels beyond the tile.
FUSED_MAX_HALO = {1: 8, 3: 8, 5: 16}


def fused_generator_supported(channels: int, kernel_size: int, dtype: torch.dtype,
                              dilations=(1, 3, 5)) -> bool:
    """Whether the fused generator+filter forward covers this configuration."""
    return (
        channels <= FUSED_MAX_CHANNELS
        and kernel_size in FUSED_KERNEL_SIZES
        and dtype in _lib.DTYPE_CODE
        and (kernel_size // 2) * max(dilations) <= FUSED_MAX_HALO[kernel_size]
    )


# Largest dilation halo of the fused dY + dW kernel at K = 5: the forward's
# (its x halo of 16 channels x (8 + 2R) rows x (16 + 2R) 16-bit cells, 60 KB
# at R = 16, fits beside the operand rings).
FUSED_DYW_MAX_HALO_K5 = 16


def _fused_dyw_ok(kernel_size: int, dtype: torch.dtype, width: int, dilations) -> bool:
    """Whether the fused dY + dW kernel covers this backward: K <= 3 always;
    K = 5 for 16-bit data (halos up to 16) whose rows allow the gradient
    tile's tensor map (W % 8 == 0). FP32 has no room for the wider K = 5 halo
    beside its hi / lo operand rings."""
    return kernel_size in FUSED_TRAINING_KERNEL_SIZES or (
        kernel_size == 5 and dtype != torch.float32 and width % 8 == 0
        and 2 * max(dilations) <= FUSED_DYW_MAX_HALO_K5)


def fused_training_supported(kernel_size: int) -> bool:
    """Whether the fused generator path can train at this kernel size: K <= 3
    with the fully fused backward, K = 5 with the split one (fused dX,
    materialised dK). The reference stops at K <= 3 (``triton_impl.py:320``)."""
    return FUSED_BACKWARD_AVAILABLE and kernel_size in FUSED_KERNEL_SIZES


def auto_fuse_training(tokens: int, channels: int, kernel_size: int, dtype: torch.dtype) -> bool:
    """Auto crossover between the fused and materialised training paths.

    The reference fuses above 16384 spatial tokens (and at exactly 16384 for
    FP32), a threshold it measured on an RTX 5090 (``triton_impl.py:313-316``).
    Measured on B200 with this library's kernels and the GEMM generator of the
    materialised path (``bench.py --crossover``: B=1, C=64, square images,
    CUDA-graph replays, L2 flushed): K = 3 FP32 fuses faster at every size
    (0.170 against 0.186 ms at 32^2, 0.590 against 1.98 ms at 256^2); K = 3
    16-bit training is faster materialised up to 64^2 (4096 tokens: 0.137
    against 0.129 ms bf16, both launch-bound) and fused from 96^2 on (0.350
    against 0.459 ms at 256^2); K = 5 is faster materialised at 32^2 (0.277
    against 0.252 ms FP32, 0.160 against 0.150 ms bf16) and fused from 64^2
    on (bf16 0.645 against 1.10 ms, FP32 3.58 against 4.87 ms at 256^2). So:
    K <= 3 FP32 always fuses, K <= 3 16-bit types above 4096 tokens, K = 5
    above 1024 tokens.
    """
    if kernel_size > 3:
        return tokens > 1024
    return dtype == torch.float32 or tokens > 4096


# ------------------------------------------------------- weight packing ----
def pack_generator_weight(weight: torch.Tensor, bias: torch.Tensor, channels: int,
                          kernel_size: int) -> torch.Tensor:
    """Packed copy of the generator weight and bias in the fused kernels'
    operand layout (all three images: forward, dX and dY).

    Packed on every forward (one small launch: 0.85 MB bf16 / 1.5 MB fp32 at
    C=64, K=3). A copy cached across calls cannot tell when the weight changed:
    writes through ``param.data`` (``dist.broadcast(p.data)``, EMA or legacy
    optimizer code) leave the parameter's version counter untouched, so a
    cache keyed on it would keep serving stale weights. The backward reuses the
    forward's copy, which is what the forward computed with.
    """
    w2 = weight.reshape(weight.shape[0], -1).contiguous()
    b1 = bias.contiguous()
    code = _lib.dtype_code(weight.dtype)
    nbytes = int(_lib.load().ddpm_gencat_pack_bytes(channels, kernel_size, code))
    packed = torch.empty(nbytes, dtype=torch.uint8, device=weight.device)
    _lib.call("ddpm_gencat_pack", w2.data_ptr(), b1.data_ptr(), channels, kernel_size, code,
              packed.data_ptr(), nbytes, _lib.stream_handle(weight.device))
    return packed


def _stage_operands(x, y, kernel_size, dilations):
    """x and y staged once as the tensor-core operand copies the fused kernels
    read by TMA (``ddpm_gencat_stage``); valid while x and y are unchanged."""
    n, c, h, w = x.shape
    d0, d1, d2 = _dil(dilations)
    code = _lib.dtype_code(x.dtype)
    nb = int(_lib.load().ddpm_gencat_stage_bytes(n, c, h, w, int(kernel_size), d0, d1, d2, code))
    staged = torch.empty(nb, dtype=torch.uint8, device=x.device)
    _lib.call("ddpm_gencat_stage", x.data_ptr(), y.data_ptr(), staged.data_ptr(), nb,
              n, c, h, w, int(kernel_size), d0, d1, d2, code, _lib.stream_handle(x.device))
    return staged


# Attribute of a cat output that carries its fuse-conv staged planes (written by
# the forward itself) to the fuse conv: (planes, nbytes, output version,
# whether the output's backward reads its gradient channel-last).
FUSE_PLANES_ATTR = "_ddpm_fuse_planes"


def _launch_gencat_fwd(x, y, packed, bias, kernel_size, dilations, staged=None,
                       fuse_planes=False):
    """The forward output; with ``fuse_planes`` (C % 8 == 0) the forward also
    writes the output as the fuse conv's staged planes and attaches them to it
    (``FUSE_PLANES_ATTR``), which saves the fuse conv its staging pass."""
    n, c, h, w = x.shape
    out = torch.empty((n, 4 * c, h, w), dtype=x.dtype, device=x.device)
    d0, d1, d2 = _dil(dilations)
    if staged is None:
        staged = _stage_operands(x, y, kernel_size, dilations)
    code = _lib.dtype_code(x.dtype)
    stream = _lib.stream_handle(x.device)
    if fuse_planes and c % 8 == 0:
        nbytes = int(_lib.load().ddpm_fuseconv_stage_bytes(n, 4 * c, h, w, code))
        planes = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        _lib.call(
            "ddpm_gencat_fwd_staged_planes",
            staged.data_ptr(), staged.numel(), packed.data_ptr(), bias.data_ptr(),
            out.data_ptr(), planes.data_ptr(), nbytes,
            n, c, h, w, int(kernel_size), d0, d1, d2, code, stream,
        )
        setattr(out, FUSE_PLANES_ATTR, (planes, nbytes, out._version,
                                        _fused_dyw_ok(int(kernel_size), x.dtype, w,
                                                      _dil(dilations))))
        return out
    _lib.call(
        "ddpm_gencat_fwd_staged",
        staged.data_ptr(), staged.numel(), packed.data_ptr(), bias.data_ptr(), out.data_ptr(),
        n, c, h, w, int(kernel_size), d0, d1, d2, code, stream,
    )
    return out


def _prepare(x, y, weight, bias, kernel_size, dilations):
    x, y = x.contiguous(), y.contiguous()
    bias = bias.contiguous()
    _require_cuda(x, y, weight, bias)
    n, c, h, w = x.shape
    if not (x.dtype == y.dtype == weight.dtype == bias.dtype):
        raise RuntimeError("fused generator path needs x, y, weight and bias of one dtype")
    if weight.shape[0] != 3 * c * kernel_size**2 or weight.numel() != weight.shape[0] * c:
        raise ValueError(f"generator weight must be [3*C*K^2, C(,1,1)], got {tuple(weight.shape)}")
    if not fused_generator_supported(c, kernel_size, x.dtype, _dil(dilations)):
        raise RuntimeError(
            f"fused generator kernels support C <= {FUSED_MAX_CHANNELS}, K in "
            f"{FUSED_KERNEL_SIZES} and a dilation halo <= {FUSED_MAX_HALO} (per K); got "
            f"C={c}, K={kernel_size}, dilations={tuple(dilations)}"
        )
    return x, y, bias


class _GeneratorDynamicCat(torch.autograd.Function):
    """Fused generator + filter (reference ``_GeneratorDynamicCat``,
    ``_triton_kernels.py:911-1053``): saves only ``(x, y, weight, bias)``."""

    @staticmethod
    def forward(ctx, x, y, weight, bias, kernel_size, dilations, fuse_planes=False):
        bias_param = bias
        x, y, bias = _prepare(x, y, weight, bias, kernel_size, dilations)
        with torch.cuda.device(x.device):
            packed = pack_generator_weight(weight, bias, x.shape[1], kernel_size)
            staged = _stage_operands(x, y, kernel_size, dilations)
            out = _launch_gencat_fwd(x, y, packed, bias, kernel_size, dilations, staged,
                                     fuse_planes)
        ctx.save_for_backward(x, y, weight, bias)
        ctx.bias = bias_param  # the parameter itself (gradient buffers are looked up by identity)
        ctx.packed = packed
        ctx.staged = staged  # reused by the backward (depends on x and y only)
        ctx.kernel_size = int(kernel_size)
        ctx.dilations = _dil(dilations)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if ctx.kernel_size not in FUSED_TRAINING_KERNEL_SIZES:
            # K = 5: the fused dY + dW kernel where it applies (all three
            # gradients, or dX alone), else dK materialised
            x = ctx.saved_tensors[0]
            need_x, need_y, need_w, need_b = ctx.needs_input_grad[:4]
            some = need_y or need_w or need_b
            fused = _fused_dyw_ok(ctx.kernel_size, x.dtype, x.shape[3], ctx.dilations) and (
                (need_y and need_w and need_b) or not some)
            if not fused:
                return _k5_backward(ctx, grad_out)
        x, y, weight, bias = ctx.saved_tensors
        packed = ctx.packed
        n, c, h, w = x.shape
        ks = ctx.kernel_size
        d0, d1, d2 = ctx.dilations
        code = _lib.dtype_code(x.dtype)
        need_x, need_y, need_w, need_b = ctx.needs_input_grad[:4]
        grad_x = torch.empty_like(x) if need_x else None
        grad_y = torch.empty_like(y) if need_y else None
        grad_w = grad_b = None
        if need_w or need_b:
            # into the caller's gradient buffers where it attached some (the
            # data-parallel reducer's flat buckets), else fresh tensors
            rows = 3 * c * ks * ks
            grad_w = (grad_buffer(weight, (rows, c), x.dtype, x.device) if need_w
                      else torch.empty((rows, c), dtype=x.dtype, device=x.device))
            grad_b = (grad_buffer(ctx.bias, (rows,), x.dtype, x.device) if need_b
                      else torch.empty(rows, dtype=x.dtype, device=x.device))
        full = need_y and grad_w is not None
        # a channel-last grad_out (the module's fuse conv writes it so for a
        # C = 64 generator output) is read as is; anything else as NCHW
        nhwc = (grad_out.dtype == x.dtype and c == 64
                and not grad_out.is_contiguous()
                and grad_out.is_contiguous(memory_format=torch.channels_last)
                and (full or not (need_y or grad_w is not None)))
        if not nhwc:
            grad_out = grad_out.to(x.dtype).contiguous()
        sfx = "_nhwc" if nhwc else ""
        with torch.cuda.device(x.device):
            stream = _lib.stream_handle(x.device)
            # the operands staged by the forward (x and y, channel-last operand
            # copies): the backward kernels stage their tiles with bulk / TMA copies
            staged = ctx.staged
            sb = staged.numel()
            # dY + dW/db first: once the weight gradients are written, a
            # listener (the data-parallel reducer) may start their all-reduce,
            # which then runs while dX computes
            if full:
                ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
                ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
                _lib.call("ddpm_gencat_bwd_yw_staged" + sfx, staged.data_ptr(), sb,
                          packed.data_ptr(),
                          grad_out.data_ptr(), grad_y.data_ptr(), grad_w.data_ptr(),
                          grad_b.data_ptr(), ws.data_ptr(), ws_bytes,
                          n, c, h, w, ks, d0, d1, d2, code, stream)
            elif need_y or grad_w is not None:
                ws = None
                ws_bytes = 0
                if grad_w is not None:
                    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
                    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
                _lib.call("ddpm_gencat_bwd_yw", x.data_ptr(), y.data_ptr(), packed.data_ptr(),
                          grad_out.data_ptr(), grad_y.data_ptr() if need_y else None,
                          grad_w.data_ptr() if grad_w is not None else None,
                          grad_b.data_ptr() if grad_b is not None else None,
                          ws.data_ptr() if ws is not None else None, ws_bytes,
                          n, c, h, w, ks, d0, d1, d2, code, stream)
            if need_w and need_b:
                grads_written((weight, ctx.bias), (grad_w, grad_b))
            if need_x:
                _lib.call("ddpm_gencat_bwd_x_staged" + sfx, staged.data_ptr(), sb,
                          packed.data_ptr(),
                          bias.data_ptr(), grad_out.data_ptr(), grad_x.data_ptr(),
                          n, c, h, w, ks, d0, d1, d2, code, stream)
        gw = grad_w.view_as(weight) if (grad_w is not None and need_w) else None
        gb = grad_b if need_b else None
        return grad_x, grad_y, gw, gb, None, None, None


# ------------------------------------------------ materialised generator ----
def _augmented(y: torch.Tensor) -> torch.Tensor:
    """y as ``[N, k, H*W]`` with a constant-one channel at index C (the bias
    column of the GEMM) and zero channels up to k = round8(C + 1)."""
    n, c, h, w = y.shape
    k = (c + 1 + 7) // 8 * 8
    p = h * w
    parts = [y.reshape(n, c, p), y.new_ones((n, 1, p))]
    if k > c + 1:
        parts.append(y.new_zeros((n, k - c - 1, p)))
    return torch.cat(parts, 1)


def _augmented_weight(weight: torch.Tensor, bias: torch.Tensor | None, k: int) -> torch.Tensor:
    rows, c = weight.shape[0], weight.numel() // weight.shape[0]
    parts = [weight.reshape(rows, c)]
    parts.append(bias.reshape(rows, 1) if bias is not None else weight.new_zeros((rows, 1)))
    if k > c + 1:
        parts.append(weight.new_zeros((rows, k - c - 1)))
    return torch.cat(parts, 1)


def _generator_grads(grad, y, weight, ya, need_y, need_wb):
    """dY = W^T grad and (dW | db) = grad . ya^T of the GEMM generator (the
    per-sample products summed in FP32; one product for N = 1)."""
    n, c = y.shape[0], y.shape[1]
    rows = weight.shape[0]
    gy = gwa = None
    if need_y:
        gy = torch.matmul(weight.reshape(rows, c).t(), grad).view_as(y)
    if need_wb:
        gwa = torch.matmul(grad, ya.transpose(1, 2))
        acc = torch.float32 if grad.dtype in (torch.bfloat16, torch.float16) else grad.dtype
        gwa = (gwa[0] if n == 1 else gwa.sum(0, dtype=acc)).to(grad.dtype)
    return gy, gwa


class _GeneratorGemm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, weight, bias):
        ya = _augmented(y)
        ctx.save_for_backward(y, weight, ya)
        ctx.has_bias = bias is not None
        return torch.matmul(_augmented_weight(weight, bias, ya.shape[1]), ya)

    @staticmethod
    def backward(ctx, grad):
        y, weight, ya = ctx.saved_tensors
        need_y, need_w, need_b = ctx.needs_input_grad
        gy, gwa = _generator_grads(grad.contiguous(), y, weight, ya, need_y, need_w or need_b)
        c = y.shape[1]
        gw = gwa[:, :c].reshape(weight.shape) if need_w else None
        gb = gwa[:, c].contiguous() if (need_b and ctx.has_bias) else None
        return gy, gw, gb


def generator_taps(y: torch.Tensor, weight: torch.Tensor,
                   bias: torch.Tensor | None) -> torch.Tensor:
    """The 1x1 generator convolution ``F.conv2d(y, weight, bias)`` of the
    materialised path (reference ``triton_impl.py:340-347``) as one batched
    GEMM on cuBLAS, ``[N, 3CK^2, H*W]``, with the bias folded in as a
    constant-one input channel (one rounding of W.y + b, as in the fused
    path); its backward is two GEMMs (dY = W^T dK; dW and db together from dK
    times the augmented y). Measured on B200 at C=64, 128^2, K=5: forward
    0.060 ms bf16 / 0.306 ms fp32 against 0.214 / 0.574 ms for the cuDNN
    convolution, whose 1x1 kernel choice is an sm_75 one; backward 0.088 /
    0.67 ms against 0.120 / 1.41 ms."""
    return _GeneratorGemm.apply(y, weight, bias)


def _k5_backward(ctx, grad_out):
    """Backward of the fused forward at K = 5 where the fused dY + dW kernel
    does not apply (FP32, whose hi / lo operand rings leave no room for the
    K = 5 halo; rows the gradient tile's tensor map cannot address; a subset of
    the gradients): dX by the fused recompute kernel
    (``ddpm_gencat_bwd_x_staged``: the taps never reach HBM), dK = shifted x *
    g_b written once by ``ddpm_dyncat_bwd`` (tap gradient only, no taps read),
    and dY, dW, db from dK by cuBLAS GEMMs (dY = W^T dK; dW and db together
    from dK times the augmented y, whose constant-one channel gives db). Only
    (x, y, weight, bias) were saved, as in the fused path."""
    x, y, weight, bias = ctx.saved_tensors
    n, c, h, w = x.shape
    ks = ctx.kernel_size
    d0, d1, d2 = ctx.dilations
    code = _lib.dtype_code(x.dtype)
    need_x, need_y, need_w, need_b = ctx.needs_input_grad[:4]
    grad_out = grad_out.to(x.dtype).contiguous()
    grad_x = torch.empty_like(x) if need_x else None
    gy = gw = gb = None
    rows = 3 * c * ks * ks
    with torch.cuda.device(x.device):
        stream = _lib.stream_handle(x.device)
        if need_y or need_w or need_b:
            dk = torch.empty((n, rows, h, w), dtype=x.dtype, device=x.device)
            _lib.call("ddpm_dyncat_bwd", x.data_ptr(), code, None, grad_out.data_ptr(), code,
                      None, dk.data_ptr(), n, c, h, w, ks, d0, d1, d2, stream)
            gy, gwa = _generator_grads(dk.view(n, rows, h * w), y, weight,
                                       _augmented(y) if (need_w or need_b) else None,
                                       need_y, need_w or need_b)
            if gwa is not None:
                gw = gwa[:, :c].contiguous()
                gb = gwa[:, c].contiguous()
            del dk
        if need_x:
            staged = ctx.staged
            _lib.call("ddpm_gencat_bwd_x_staged", staged.data_ptr(), staged.numel(),
                      ctx.packed.data_ptr(), bias.data_ptr(), grad_out.data_ptr(),
                      grad_x.data_ptr(), n, c, h, w, ks, d0, d1, d2, code, stream)
    gw = gw.view_as(weight) if need_w else None
    return grad_x, gy if need_y else None, gw, gb if need_b else None, None, None, None


def fused_generator_dynamic_cat(x, y, weight, bias, kernel_size, dilations, *,
                                _fuse_planes=False):
    """Fused 1x1 generator + dynamic filter (reference ``_triton_kernels.py:1056-1065``).

    Differentiable w.r.t. x, y, weight and bias; without gradients it is a
    single launch (plus the weight packing). ``_fuse_planes`` (used by
    the DDPM module when its native fuse conv consumes the output) has the
    forward also write the fuse conv's staged planes.
    """
    if torch.is_grad_enabled() and any(t.requires_grad for t in (x, y, weight, bias)):
        return _GeneratorDynamicCat.apply(x, y, weight, bias, kernel_size, dilations,
                                          _fuse_planes)
    x, y, bias = _prepare(x, y, weight, bias, kernel_size, dilations)
    with torch.cuda.device(x.device):
        packed = pack_generator_weight(weight, bias, x.shape[1], kernel_size)
        return _launch_gencat_fwd(x, y, packed, bias, kernel_size, dilations,
                                  fuse_planes=_fuse_planes)


__all__ = ["fused_dynamic_cat", "fused_generator_dynamic_cat"]
