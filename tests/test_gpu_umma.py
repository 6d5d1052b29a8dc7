"""tcgen05 UMMA layout self-test through the C ABI (``ddpm_umma_selftest``).

Checks the operand layouts the fused kernels are built on against a float64
matmul: K-major, MN-major, K-major read from an arbitrary row offset of a
staged tile (the shifted-window trick of the dX kernel), and an MN-major B
whose K window starts at an arbitrary row (the weight-gradient kernel).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant,n,k,shift", [
    (0, 64, 64, 0), (0, 144, 64, 0), (0, 48, 32, 0), (0, 256, 128, 0),
    (1, 64, 64, 0), (1, 128, 32, 0),
    (2, 64, 64, 5), (2, 64, 64, 13), (2, 16, 16, 1),
    (3, 64, 128, 0), (3, 64, 128, 7), (3, 64, 64, 9), (3, 192, 32, 3),
])
def test_umma_layouts(variant, n, k, shift):
    from dynamicconvolutionoperator_b200 import _lib

    gen = torch.Generator().manual_seed(variant * 1000 + n + k + shift)
    b_mn = variant == 3
    a = torch.randn(128 if b_mn else 128 + shift, k, generator=gen).to(torch.bfloat16)
    b = torch.randn(n, k + shift if b_mn else k, generator=gen).to(torch.bfloat16)
    ad, bd = a.cuda(), b.cuda()
    d = torch.full((128, n), float("nan"), device="cuda")
    _lib.call("ddpm_umma_selftest", variant, ad.data_ptr(), bd.data_ptr(), d.data_ptr(),
              n, k, shift, _lib.stream_handle(d.device))
    torch.cuda.synchronize()
    if b_mn:
        ref = a.double() @ b[:, shift:shift + k].double().T
    else:
        ref = a[shift:shift + 128].double() @ b.double().T
    torch.testing.assert_close(d.cpu().double(), ref, rtol=1e-4, atol=1e-3)
