"""The failure path of the tensor-core kernels, exercised on the GPU without a
fault: every mbarrier wait inside them is bounded, and a wait that runs out
records a code in the device status word, makes every role of the CTA unwind
and free its tensor memory, and lets the launch return.

The test hook ``ddpm_test_skip_arrive`` has one producer thread of the fused
generator forward withhold an arrival, so one wait runs out (after its 2 s
limit). The call must return, the status must carry the code, and the next
normal call on the same device must pass parity against the oracle.
"""

from __future__ import annotations

import time

import pytest
import torch

from tests._parity import compare

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_wait_that_runs_out_reports_and_the_device_stays_usable(dtype):
    from dynamicconvolutionoperator_b200 import DDPM, _lib
    from oracle import ddpm_oracle as orc

    shape = (1, 16, 8, 32)
    ref = orc.make_model(16, 3, dtype=dtype, seed=50)
    model = DDPM(16, 3).cuda().to(dtype)
    model.load_state_dict(ref.state_dict())
    x, y, _ = orc.make_inputs(shape, dtype=dtype, seed=51)
    xd, yd = x.cuda(), y.cuda()
    assert _lib.device_status(reset=True) == 0

    _lib.call("ddpm_test_skip_arrive", 1)
    try:
        t0 = time.monotonic()
        with torch.no_grad():
            model(xd, yd)  # the fused forward: one CTA's wait runs out
        code = _lib.device_status(reset=True)  # synchronises
        elapsed = time.monotonic() - t0
    finally:
        _lib.call("ddpm_test_skip_arrive", 0)
    assert code != 0, "the wait that ran out recorded no status"
    assert elapsed < 60, f"the failing launch took {elapsed:.1f} s to unwind"

    # the context is intact: the same call now runs normally and matches the oracle
    with torch.no_grad():
        out = model(xd, yd).cpu()
    assert _lib.device_status(reset=True) == 0
    gold, _ = orc.run_reference(ref, x, y, dtype=torch.float64)
    stats, fails = compare(out, None, gold, None, dtype)
    assert not fails, "\n".join(fails) + f"\n{stats}"
