"""Full DDPM forward(+backward) on the GPU against the float64 oracle, at the
BASELINE configs, through both the materialised and the fused paths.

Tolerances are those of the north star (see tests/_parity.py): fp32 2e-3
max-abs; bf16 3e-2 max-abs and 5e-3 RMSE; parameter gradients normalised by
their largest gold magnitude.
"""

from __future__ import annotations

import pytest
import torch

from tests import _golden as gold
from tests._parity import compare, ddpm_parity, run_device

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16]


def _assert_ok(stats, fails):
    assert not fails, "\n".join(fails) + f"\n{stats}"


@pytest.mark.parametrize("dtype", DTYPES + [torch.float16])
@pytest.mark.parametrize("ks", [1, 3, 5])
@pytest.mark.parametrize("fused", [False, True])
def test_cfg2_regression_training(dtype, ks, fused):
    """[2,24,15,17], K in {1,3,5}, fwd+bwd, every gradient."""
    stats, fails = ddpm_parity((2, 24, 15, 17), ks, dtype, seed=123, input_seed=456,
                               fused_generator_training=fused)
    _assert_ok(stats, fails)


@pytest.mark.parametrize("dtype", DTYPES)
def test_cfg2_matches_reference_golden_output(dtype):
    """The GPU output sits within tolerance of the reference's own CPU output
    recorded in tests/golden (same seeds, same dtype)."""
    from dynamicconvolutionoperator_b200 import DDPM
    from oracle import ddpm_oracle as orc

    tag = "fp32" if dtype == torch.float32 else "bf16"
    rec = gold.load(f"cfg2_{tag}_k3.npz")
    ref = orc.make_model(24, 3, dtype=dtype, seed=123)
    dev = DDPM(24, 3).cuda().to(dtype)
    dev.load_state_dict(ref.state_dict())
    x, y, _ = orc.make_inputs((2, 24, 15, 17), dtype=dtype, seed=456, grad_seed=789)
    torch.backends.cudnn.allow_tf32 = False
    with torch.no_grad():
        out = dev(x.cuda(), y.cuda()).float().cpu()
    tol = 2e-3 if dtype == torch.float32 else 3e-2
    assert (out - gold.tensor(rec, "out")).abs().max().item() <= tol


def test_cfg1_inference_matches_golden():
    """C=32 48x48 K=3 fp32 inference vs the reference's output."""
    from dynamicconvolutionoperator_b200 import DDPM
    from oracle import ddpm_oracle as orc

    rec = gold.load("cfg1.npz")
    ref = orc.make_model(32, 3, seed=0)
    dev = DDPM(32, 3).cuda()
    dev.load_state_dict(ref.state_dict())
    x, y, _ = orc.make_inputs((1, 32, 48, 48), seed=1)
    torch.backends.cudnn.allow_tf32 = False
    for fused in (True, False):
        dev.fused_generator_inference = fused
        with torch.no_grad():
            out = dev(x.cuda(), y.cuda()).cpu()
        assert (out - gold.tensor(rec, "out")).abs().max().item() <= 2e-3


@pytest.mark.parametrize("dtype", DTYPES + [torch.float16])
@pytest.mark.parametrize("ks", [3, 5])
@pytest.mark.parametrize("fused", [True, False])
def test_cfg3_inference_128(dtype, ks, fused):
    """B=1 C=64 128x128, K in {3,5}, fused vs materialised."""
    stats, fails = ddpm_parity((1, 64, 128, 128), ks, dtype, grad=False, seed=20,
                               input_seed=21, fused_generator_inference=fused)
    _assert_ok(stats, fails)


@pytest.mark.parametrize("dtype", DTYPES + [torch.float16])
@pytest.mark.parametrize("fused", [True, False])
def test_cfg4_training_256(dtype, fused):
    """B=1 C=64 256x256 K=3, fwd+bwd, every gradient."""
    stats, fails = ddpm_parity((1, 64, 256, 256), 3, dtype, seed=30, input_seed=31,
                               fused_generator_training=fused)
    _assert_ok(stats, fails)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("ks", [1, 3])
def test_cudnn_fuse_path_training(dtype, ks):
    """``native_fuse=False``: the fuse conv through cuDNN (bias folded into the
    contraction for 16-bit outputs), every gradient within tolerance."""
    stats, fails = ddpm_parity((2, 24, 15, 17), ks, dtype, seed=7, input_seed=8,
                               native_fuse=False)
    _assert_ok(stats, fails)


def _training_step(model, x, y, g):
    for p in model.parameters():
        p.grad = None
    xi = x.detach().requires_grad_(True)
    yi = y.detach().requires_grad_(True)
    out = model(xi, yi)
    out.backward(g)
    return [out.detach().clone(), xi.grad.clone(), yi.grad.clone()] + [
        p.grad.clone() for p in model.parameters()]


def _update_in_place(model):
    with torch.no_grad():
        for p in model.parameters():
            p.mul_(0.75).add_(0.01)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_weight_update_between_steps_repacks(dtype):
    """After an in-place update (what an optimizer step does) the next training
    step must use the new weights, exactly like a module built with them."""
    from dynamicconvolutionoperator_b200 import DDPM

    torch.manual_seed(3)
    a = DDPM(32, 3, fused_generator_training=True).cuda().to(dtype)
    b = DDPM(32, 3, fused_generator_training=True).cuda().to(dtype)
    b.load_state_dict(a.state_dict())
    gen = torch.Generator().manual_seed(4)
    x, y, g = (torch.randn((1, 32, 24, 40), generator=gen).to(dtype).cuda() for _ in range(3))
    _training_step(a, x, y, g)
    _update_in_place(a)
    _update_in_place(b)
    got = _training_step(a, x, y, g)
    ref = _training_step(b, x, y, g)
    # dY is summed across CTAs with FP32 atomics (order not fixed), hence a small
    # tolerance; stale weights (scaled by 0.75) would be far outside it
    tol = 1e-5 if dtype == torch.float32 else 1.6e-2
    for u, v in zip(got, ref):
        torch.testing.assert_close(u.float(), v.float(), rtol=tol, atol=tol)


def test_graph_replay_sees_weight_updates():
    """A training step captured in a CUDA graph repacks the weights on every
    replay (nothing packed is cached at capture), so a replay after an
    in-place weight update matches an eager step with the new weights."""
    from dynamicconvolutionoperator_b200 import DDPM

    torch.manual_seed(5)
    model = DDPM(32, 3, fused_generator_training=True).cuda()
    fresh = DDPM(32, 3, fused_generator_training=True).cuda()
    gen = torch.Generator().manual_seed(6)
    x, y, g = (torch.randn((1, 32, 24, 40), generator=gen).cuda() for _ in range(3))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            _training_step(model, x, y, g)
    torch.cuda.current_stream().wait_stream(side)
    for p in model.parameters():
        p.grad = None
    graph = torch.cuda.CUDAGraph()
    xi = x.detach().requires_grad_(True)
    yi = y.detach().requires_grad_(True)
    with torch.cuda.graph(graph):
        out = model(xi, yi)
        out.backward(g)
    _update_in_place(model)
    fresh.load_state_dict(model.state_dict())
    for p in model.parameters():
        p.grad.zero_()
    xi.grad.zero_()
    yi.grad.zero_()
    graph.replay()
    torch.cuda.synchronize()
    got = [out.detach(), xi.grad, yi.grad] + [p.grad for p in model.parameters()]
    ref = _training_step(fresh, x, y, g)
    for u, v in zip(got, ref):
        torch.testing.assert_close(u, v, rtol=1e-5, atol=1e-5)
    del graph


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_weight_write_through_data_is_seen(dtype):
    """Writes through ``param.data`` leave the version counter untouched (what
    ``dist.broadcast(p.data)``, EMA or legacy optimizer code do): the next
    forward must still use the new weights, against the float64 oracle."""
    from dynamicconvolutionoperator_b200 import DDPM
    from oracle import ddpm_oracle as orc

    shape = (1, 32, 24, 40)
    first = orc.make_model(32, 3, dtype=dtype, seed=11)
    second = orc.make_model(32, 3, dtype=dtype, seed=12)
    dev = DDPM(32, 3, fused_generator_training=True).cuda().to(dtype)
    dev.load_state_dict(first.state_dict())
    x, y, g = orc.make_inputs(shape, dtype=dtype, seed=13, grad_seed=14)
    run_device(dev, x, y, g)  # a forward + backward with the first weights
    versions = [p._version for p in dev.parameters()]
    for p, q in zip(dev.parameters(), second.parameters()):
        p.data.copy_(q.detach().cuda())
    assert [p._version for p in dev.parameters()] == versions
    for grad in (None, g):
        out, grads = run_device(dev, x, y, grad)
        gold_out, gold_grads = orc.run_reference(second, x, y, grad=grad, dtype=torch.float64)
        stats, fails = compare(out, grads, gold_out, gold_grads, dtype)
        _assert_ok(stats, fails)


@pytest.mark.parametrize("ac_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("fused", [True, False])
def test_autocast_runs_the_native_kernels(ac_dtype, fused):
    """Under autocast the FP32 module runs in the autocast dtype on the native
    kernels (fused or materialised), returns that dtype, and its output and
    every gradient (x, y and the FP32 parameters) sit within the 16-bit
    tolerance of the float64 oracle. Inputs and weights are exactly
    representable in the autocast dtype, so the comparison measures the
    kernels, not the cast."""
    from dynamicconvolutionoperator_b200 import DDPM, _lib
    from oracle import ddpm_oracle as orc

    shape = (2, 24, 15, 17)
    ref = orc.make_model(24, 3, dtype=ac_dtype, seed=15)
    dev = DDPM(24, 3, fused_generator_training=fused, fused_generator_inference=fused).cuda()
    dev.load_state_dict({k: v.float() for k, v in ref.state_dict().items()})
    x, y, g = orc.make_inputs(shape, dtype=ac_dtype, seed=16, grad_seed=17)
    xd = x.float().cuda().requires_grad_(True)
    yd = y.float().cuda().requires_grad_(True)
    n0 = _lib.launch_count()
    with torch.autocast("cuda", dtype=ac_dtype):
        out = dev(xd, yd)
    assert out.dtype == ac_dtype
    names = ["x", "y"] + [n for n, _ in dev.named_parameters()]
    grads = torch.autograd.grad(out, [xd, yd, *dev.parameters()], g.cuda())
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 >= 4  # filter/generator and fuse kernels of the library
    assert all(gr.dtype == torch.float32 for gr in grads)
    gold_out, gold_grads = orc.run_reference(ref, x, y, grad=g, dtype=torch.float64)
    stats, fails = compare(out.detach().cpu(), {k: v.cpu() for k, v in zip(names, grads)},
                           gold_out, gold_grads, ac_dtype)
    _assert_ok(stats, fails)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_training_step_hands_the_generator_a_channel_last_gradient(dtype, monkeypatch):
    """At C=64 the fuse conv writes the gradient of the generator output
    channel-last and the generator backward reads it so (the *_nhwc entry
    points), within the oracle's tolerance (the cfg4 parity test covers the
    values at 256^2)."""
    from dynamicconvolutionoperator_b200 import _lib

    calls = []
    real = _lib.call

    def spy(name, *args):
        calls.append(name)
        return real(name, *args)

    monkeypatch.setattr(_lib, "call", spy)
    stats, fails = ddpm_parity((1, 64, 24, 40), 3, dtype, seed=60, input_seed=61,
                               fused_generator_training=True)
    _assert_ok(stats, fails)
    nhwc = {n for n in calls if n.endswith("_nhwc")}
    assert nhwc == {"ddpm_fuseconv_bwd_nhwc", "ddpm_gencat_bwd_x_staged_nhwc",
                    "ddpm_gencat_bwd_yw_staged_nhwc"}, calls


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_k5_training_takes_the_fused_forward_and_dx(dtype, monkeypatch):
    """K = 5 training through the fused path: the fused forward (writing the
    fuse conv's planes) and the fused dX kernel; for bf16 the fused dY + dW
    kernel with a channel-last gradient of the generator output, for FP32 dK
    from the filter backward (tap gradient only) and an NCHW gradient; every
    gradient within the oracle's tolerance."""
    from dynamicconvolutionoperator_b200 import _lib

    calls = []
    real = _lib.call

    def spy(name, *args):
        calls.append(name)
        return real(name, *args)

    monkeypatch.setattr(_lib, "call", spy)
    stats, fails = ddpm_parity((1, 64, 40, 48), 5, dtype, seed=62, input_seed=63,
                               fused_generator_training=True)
    _assert_ok(stats, fails)
    assert "ddpm_gencat_fwd_staged_planes" in calls and "ddpm_dyncat_fwd" not in calls, calls
    if dtype == torch.float32:
        assert {"ddpm_gencat_bwd_x_staged", "ddpm_dyncat_bwd"} <= set(calls), calls
        assert not any(n.endswith("_nhwc") for n in calls), calls
    else:
        assert {"ddpm_fuseconv_bwd_nhwc", "ddpm_gencat_bwd_x_staged_nhwc",
                "ddpm_gencat_bwd_yw_staged_nhwc"} <= set(calls), calls
        assert "ddpm_dyncat_bwd" not in calls, calls

