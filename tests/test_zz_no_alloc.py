"""The no-allocation backward entry point (``ddpm_gencat_bwd_yw_static``)
against the workspace entry point (``ddpm_gencat_bwd_yw``), through the C ABI.

The static variant keeps its dW/db partials in a fixed 8 MiB device array and
caps the spatial split count to fit; it computes dY with the separate dY
kernel while the workspace entry builds dK once for dY and dW and sums the
channel groups' dY shares with FP32 atomics, so all outputs agree to
summation-order rounding. It is called twice in a row to show that the
shared scratch needs no clearing between calls (those two agree exactly).
"""

from __future__ import annotations

import pytest
import torch

from tests.test_gpu_gencat import _case

pytestmark = pytest.mark.gpu

# (n, c, h, w): the last shape needs more than 8 MiB of partials at the
# workspace path's split count, so the static variant runs with fewer splits.
SHAPES = [(2, 24, 15, 17), (1, 64, 128, 128)]
# max |static - workspace| / max |workspace| for dY, dW and db
PARAM_TOL = {torch.float32: 1e-4, torch.bfloat16: 1e-2}


def _inputs(shape, ks, dtype):
    from dynamicconvolutionoperator_b200 import _kernels

    x, y, wt, b = _case(shape, ks, dtype)
    n, c, h, w = shape
    g = torch.randn((n, 4 * c, h, w), generator=torch.Generator().manual_seed(7)).to(dtype)
    xd, yd, wd, bd, gd = x.cuda(), y.cuda(), wt.cuda(), b.cuda(), g.cuda()
    packed = _kernels.pack_generator_weight(wd, bd, c, ks)
    return xd, yd, packed, gd


STATIC_SCRATCH_BYTES = 8 << 20


def _partials_bytes(n, c, h, w, ks):
    """Bytes of dW/db partials the workspace entry's split plan uses (its
    split count, uncapped): channel-group batches of at most 512 accumulator
    columns share the SMs, the rest of the SMs split the spatial tiles."""
    cp = (c + 15) // 16 * 16
    nw = (c + 1 + 15) // 16 * 16
    ng = (cp // 16) * ((3 * ks * ks + 7) // 8)
    gb = min(512 // nw, ng)
    nbatches = (ng + gb - 1) // gb
    tiles = n * ((h + 7) // 8) * ((w + 15) // 16)
    splits = min(max(torch.cuda.get_device_properties(0).multi_processor_count // nbatches, 1),
                 tiles)
    return splits * ng * 128 * nw * 4


def _outputs(yd, c, ks):
    kk = 3 * c * ks * ks
    return (torch.full_like(yd, float("nan")),
            torch.full((kk, c), float("nan"), dtype=yd.dtype, device=yd.device),
            torch.full((kk,), float("nan"), dtype=yd.dtype, device=yd.device))


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("ks", [1, 3])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_static_scratch_matches_workspace_entry(shape, ks, dtype):
    from dynamicconvolutionoperator_b200 import _lib

    n, c, h, w = shape
    xd, yd, packed, gd = _inputs(shape, ks, dtype)
    code = _lib.dtype_code(dtype)
    stream = _lib.stream_handle(yd.device)

    gy_ref, gw_ref, gb_ref = _outputs(yd, c, ks)
    ws_bytes = int(_lib.load().ddpm_gencat_bwd_workspace_bytes(n, c, h, w, ks))
    need = _partials_bytes(n, c, h, w, ks)
    assert need <= ws_bytes  # the workspace covers the plan's partials
    if shape == SHAPES[-1]:
        # the case that must run the static entry with a capped split count
        assert need > STATIC_SCRATCH_BYTES
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.call("ddpm_gencat_bwd_yw", xd.data_ptr(), yd.data_ptr(), packed.data_ptr(),
              gd.data_ptr(), gy_ref.data_ptr(), gw_ref.data_ptr(), gb_ref.data_ptr(),
              ws.data_ptr(), ws_bytes, n, c, h, w, ks, 1, 3, 5, code, stream)

    results = []
    for _ in range(2):
        gy, gw, gb = _outputs(yd, c, ks)
        _lib.call("ddpm_gencat_bwd_yw_static", xd.data_ptr(), yd.data_ptr(), packed.data_ptr(),
                  gd.data_ptr(), gy.data_ptr(), gw.data_ptr(), gb.data_ptr(),
                  n, c, h, w, ks, 1, 3, 5, code, stream)
        results.append((gy, gw, gb))
    torch.cuda.synchronize()

    for gy, gw, gb in results:
        for got, ref in ((gy, gy_ref), (gw, gw_ref), (gb, gb_ref)):
            assert torch.isfinite(got).all()
            scale = ref.double().abs().max().item() + 1e-12
            err = (got.double() - ref.double()).abs().max().item() / scale
            assert err <= PARAM_TOL[dtype], err
    # same plan, same summation order: the two static calls agree exactly
    for a, b in zip(results[0], results[1]):
        assert torch.equal(a, b)


def test_static_scratch_argument_errors():
    from dynamicconvolutionoperator_b200 import _lib

    lib = _lib.load()
    yd = torch.zeros((1, 8, 4, 4), device="cuda")
    gw = torch.zeros((3 * 8 * 9, 8), device="cuda")
    stream = _lib.stream_handle(yd.device)
    p = yd.data_ptr()
    # grad_weight without grad_bias
    rc = lib.ddpm_gencat_bwd_yw_static(p, p, p, p, None, gw.data_ptr(), None,
                                       1, 8, 4, 4, 3, 1, 3, 5, 0, stream)
    assert rc == -1 and b"grad_bias" in lib.ddpm_last_error()
    # outside the fused limits (C > 64)
    rc = lib.ddpm_gencat_bwd_yw_static(p, p, p, p, p, None, None,
                                       1, 65, 4, 4, 3, 1, 3, 5, 0, stream)
    assert rc == -2
