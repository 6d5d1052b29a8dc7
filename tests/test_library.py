"""The C-ABI shared library loads and exports every declared entry point (CPU).

No compute call is made here; only argument validation paths that return
before touching the GPU are exercised.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from dynamicconvolutionoperator_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "ddpm_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"DDPM_API\s+[\w\s\*]+?\b(ddpm_\w+)\s*\(", text)


def test_header_and_binding_agree():
    decl = set(declared_symbols())
    assert decl, "no declarations parsed from the header"
    assert decl == set(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert _lib.load().ddpm_version() >= 100


def test_argument_errors_return_codes_without_gpu():
    lib = _lib.load()
    rc = lib.ddpm_dyncat_fwd(None, 0, None, 0, None, 1, 1, 1, 1, 3, 1, 3, 5, None)
    assert rc == -1
    assert b"null" in lib.ddpm_last_error()
    rc = lib.ddpm_dyncat_fwd(1, 0, 1, 0, 1, 1, 1, 1, 1, 2, 1, 3, 5, None)
    assert rc == -1
    assert b"odd" in lib.ddpm_last_error()
    rc = lib.ddpm_dyncat_fwd(1, 7, 1, 0, 1, 1, 1, 1, 1, 3, 1, 3, 5, None)
    assert rc == -1
    with pytest.raises(RuntimeError, match="dtype"):
        _lib.call("ddpm_dyncat_bwd", 1, 9, 1, 1, 0, 1, 1, 1, 1, 1, 1, 3, 1, 3, 5, None)


def test_dyncat_bwd_rejects_halos_the_data_gradient_cannot_stage():
    """The data gradient stages its tile's three gradient planes with the
    dilation halo; halos above 39 do not fit a CTA and are refused up front
    (the tap gradient alone, and the forward, go to 64)."""
    lib = _lib.load()
    f32 = _lib.dtype_code(torch.float32)
    args = (1, f32, 1, 1, f32)
    rc = lib.ddpm_dyncat_bwd(*args, 1, 1, 1, 1, 8, 8, 3, 1, 40, 5, None)
    assert rc != 0 and b"halo 40" in lib.ddpm_last_error()
    rc = lib.ddpm_dyncat_bwd(*args, 1, None, 1, 1, 8, 8, 3, 1, 65, 5, None)
    assert rc != 0 and b"halo" in lib.ddpm_last_error()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape,ks,dil", [((2, 24, 15, 17), 3, (1, 3, 5)), ((1, 64, 256, 256), 5, (1, 8, 4)),
                                          ((1, 5, 4, 3), 1, (1, 1, 1))])
def test_stage_bytes_follow_the_staged_layout(dtype, shape, ks, dil):
    """ddpm_gencat_stage_bytes (host arithmetic only): the y plane
    [part][n][G][Hp][Wp][8] in 16-byte rows, then, 256-byte aligned, the x
    plane of 16-byte cells holding 4 FP32 channels (fp32) or 8 channels in the
    input type (bf16 / fp16); 0 for a halo the fused kernels do not cover."""
    lib = _lib.load()
    code = _lib.dtype_code(dtype)
    n, c, h, w = shape
    G = (c + 1 + 15) // 16 * 2
    ph = (ks // 2) * max(dil)
    pw = 8 if ks <= 3 else 16
    Hp, Wp = h + 2 * ph, (w + 127) // 128 * 128 + 2 * pw
    parts = 2 if dtype == torch.float32 else 1
    x_off = (parts * n * G * Hp * Wp * 16 + 255) // 256 * 256
    xcell = 4 if dtype == torch.float32 else 8
    want = x_off + n * ((c + xcell - 1) // xcell) * h * w * 16
    assert lib.ddpm_gencat_stage_bytes(n, c, h, w, ks, *dil, code) == want
    if ks > 1:  # halos (K // 2) * 9 = 9 (K = 3, limit 8) and 18 (K = 5, limit 16)
        assert lib.ddpm_gencat_stage_bytes(n, c, h, w, ks, 1, 9, 4, code) == 0
