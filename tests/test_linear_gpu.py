"""BlockFHTLinear on the GPU against the oracle and the reference's golden outputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_linear_forward_backward_matches_golden(native_lib, golden):
    from latent_weight_lab import BlockFHTLinear

    layer = BlockFHTLinear(96, 40, bias=False, latent_dim=300, layers=3, seed=5, weight_scale=0.5).cuda()
    with torch.no_grad():
        layer.generator.latent.copy_(torch.from_numpy(golden["lin2_latent"]))
    x = torch.from_numpy(golden["lin2_x"]).cuda().requires_grad_(True)
    y = layer(x)
    y.backward(torch.from_numpy(golden["lin2_grad_y"]).cuda())
    assert rel_l2(y.detach().cpu().numpy(), golden["lin2_out"]) < 1e-5
    assert rel_l2(x.grad.cpu().numpy(), golden["lin2_grad_x"]) < 1e-5
    assert rel_l2(layer.generator.latent.grad.cpu().numpy(), golden["lin2_grad_latent"]) < 1e-5


def test_small_linear_with_bias_matches_golden(native_lib, golden):
    from latent_weight_lab import BlockFHTLinear

    layer = BlockFHTLinear(5, 3, bias=True, latent_dim=8, layers=2, seed=11).cuda()
    with torch.no_grad():
        layer.generator.latent.copy_(torch.from_numpy(golden["lin_latent"]))
        layer.bias.copy_(torch.from_numpy(golden["lin_bias"]))
    out = layer(torch.from_numpy(golden["lin_x"]).cuda())
    assert np.allclose(out.detach().cpu().numpy(), golden["lin_out"], atol=1e-6)
    assert np.allclose(layer.weight.detach().cpu().numpy(), golden["lin_weight"], atol=1e-7)


@pytest.mark.parametrize("dtype, tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2), (torch.float16, 1e-2)])
def test_gpt_shaped_linear_against_oracle(native_lib, dtype, tol):
    """768 -> 3072 with a 32768-value latent (blocks straddle weight rows)."""
    from latent_weight_lab import BlockFHTLinear

    torch.manual_seed(0)
    layer = BlockFHTLinear(768, 3072, latent_dim=32768, layers=3, seed=7).cuda().to(dtype)
    x = torch.randn(64, 768, device="cuda", dtype=dtype, requires_grad=True)
    y = layer(x)
    gy = torch.randn_like(y)
    y.backward(gy)
    z = layer.generator.latent.detach().float().cpu().numpy()
    ref_y = orc.linear_forward(x.detach().float().cpu().numpy(), z, 3072, 3, 7)
    assert rel_l2(y.detach().float().cpu().numpy(), ref_y) < tol
    gx, gz, _ = orc.linear_backward(gy.float().cpu().numpy(), x.detach().float().cpu().numpy(), z, 3072, 3, 7)
    assert rel_l2(x.grad.float().cpu().numpy(), gx) < tol
    assert rel_l2(layer.generator.latent.grad.float().cpu().numpy(), gz) < tol


def test_forward_fused_and_weight_cache(native_lib):
    from latent_weight_lab import (BlockFHTLinear, flush_block_fht_weight_cache, prepare_block_fht_weight_cache)

    torch.manual_seed(123)
    dyn = BlockFHTLinear(8, 6, bias=True, latent_dim=32, layers=2, seed=99, output_gain=True).cuda()
    cached = BlockFHTLinear(8, 6, bias=True, latent_dim=32, layers=2, seed=99, output_gain=True).cuda()
    cached.load_state_dict(dyn.state_dict())
    with torch.no_grad():
        dyn.output_gain.copy_(torch.linspace(0.5, 1.5, 6))
        cached.output_gain.copy_(torch.linspace(0.5, 1.5, 6))
    x = torch.randn(11, 8, device="cuda")
    assert torch.allclose(dyn.forward_fused(x), dyn(x), atol=2e-5)
    dyn(x).square().mean().backward()
    prepare_block_fht_weight_cache(cached)
    cached(x).square().mean().backward()
    flush_block_fht_weight_cache(cached)
    assert torch.allclose(cached.generator.latent.grad, dyn.generator.latent.grad, atol=1e-6)
    assert torch.allclose(cached.output_gain.grad, dyn.output_gain.grad, atol=1e-6)


def test_grouped_weight_cache_bf16(native_lib):
    from latent_weight_lab import BlockFHTLinear, prepare_block_fht_weight_cache

    torch.manual_seed(1)
    model = torch.nn.Sequential(*[BlockFHTLinear(768, 768, latent_dim=5898, layers=3, seed=s) for s in range(6)])
    model = model.cuda().bfloat16()
    prepare_block_fht_weight_cache(model)
    for m in model:
        assert torch.equal(m._cached_weight.detach(), m.weight.detach())


def test_block_fht_linear_forward_takes_fused_kernel_bf16(native_lib):
    """bf16 768 -> 3072: the drop-in forward runs the fused tcgen05 kernel (bit-identical
    to a direct call) and matches the oracle within the bf16 tolerance."""
    from latent_weight_lab import BlockFHTLinear, _native, block_fht_linear_forward

    torch.manual_seed(3)
    layer = BlockFHTLinear(768, 3072, bias=False, latent_dim=32768, layers=3, seed=21).cuda().bfloat16()
    x = torch.randn(2, 300, 768, device="cuda", dtype=torch.bfloat16)
    y = layer.forward_fused(x, weight_scale=0.5)
    direct = _native.linear_forward(x.reshape(-1, 768), layer.generator.latent, 3072, 3, 21, 0.5)
    assert direct is not None
    assert torch.equal(y.reshape(-1, 3072), direct)
    y2 = block_fht_linear_forward(x, layer.generator.latent, 3072, 3, 21, weight_scale=0.5)
    assert torch.equal(y, y2)
    z = layer.generator.latent.detach().float().cpu().numpy()
    ref = orc.linear_forward(x.reshape(-1, 768).float().cpu().numpy(), z, 3072, 3, 21) * 0.5
    assert rel_l2(y.reshape(-1, 3072).float().cpu().numpy(), ref) < 1e-2


@pytest.mark.parametrize("dtype, tol, K, N, L, scale", [(torch.float32, 1e-5, 96, 40, 300, 0.5),
                                                       (torch.float32, 1e-5, 768, 384, 40000, 1.0),
                                                       (torch.bfloat16, 1e-2, 768, 3072, 32768, 0.25),
                                                       (torch.float16, 1e-2, 256, 512, 5000, 1.0)])
def test_linear_backward_capi_matches_oracle(native_lib, dtype, tol, K, N, L, scale):
    """lwl_linear_backward (regenerated W, cuBLAS products, transform backward) against the
    oracle's _BlockFHTLinearFn.backward restatement."""
    from latent_weight_lab import _native

    torch.manual_seed(K + N)
    T = 129
    x = torch.randn(T, K, device="cuda").to(dtype)
    gy = torch.randn(T, N, device="cuda").to(dtype)
    z = (torch.randn(L, device="cuda") * 0.05).to(dtype)
    gx, gz = _native.linear_backward(x, gy, z, N, 3, 17, weight_scale=scale)
    rx, rz, _ = orc.linear_backward(gy.float().cpu().numpy(), x.float().cpu().numpy(), z.float().cpu().numpy(),
                                    N, 3, 17, scale)
    assert rel_l2(gx.float().cpu().numpy(), rx) < tol
    assert rel_l2(gz.float().cpu().numpy(), rz) < tol
    only_x, none_z = _native.linear_backward(x, gy, z, N, 3, 17, weight_scale=scale, need_latent=False)
    assert none_z is None and torch.equal(only_x, gx)
    none_x, only_z = _native.linear_backward(x, gy, z, N, 3, 17, weight_scale=scale, need_input=False)
    assert none_x is None and torch.equal(only_z, gz)


def test_linear_backward_capi_zero_tokens(native_lib):
    from latent_weight_lab import _native

    x = torch.zeros(0, 64, device="cuda")
    gy = torch.zeros(0, 32, device="cuda")
    z = torch.randn(100, device="cuda")
    gx, gz = _native.linear_backward(x, gy, z, 32, 2, 1)
    assert gx.shape == (0, 64) and torch.count_nonzero(gz) == 0


@pytest.mark.parametrize("gains, alpha", [("out", 0.0), ("in", 0.0), ("both", 0.02), ("both", 0.0)])
def test_forward_fused_with_gains_matches_materialised(native_lib, gains, alpha):
    """Gains and bias folded into the fused kernel equal the reference's
    materialised forward (F.linear with the module's weight) within bf16 tolerance."""
    from latent_weight_lab import BlockFHTLinear, _native

    torch.manual_seed(11)
    layer = BlockFHTLinear(768, 3072, bias=True, latent_dim=32768, layers=3, seed=4, weight_scale=0.7,
                           modulation_alpha=alpha, output_gain=gains in ("out", "both"),
                           input_gain=gains in ("in", "both")).cuda().bfloat16()
    with torch.no_grad():
        if layer.output_gain is not None:
            layer.output_gain.copy_(torch.rand(3072) + 0.5)
        if layer.input_gain is not None:
            layer.input_gain.copy_(torch.rand(768) + 0.5)
        layer.bias.copy_(torch.randn(3072) * 0.1)
    x = torch.randn(3, 111, 768, device="cuda", dtype=torch.bfloat16)
    calls = []
    orig = _native.linear_forward
    _native.linear_forward = lambda *a, **k: calls.append(1) or orig(*a, **k)
    try:
        y = layer.forward_fused(x, weight_scale=3.0)  # ignored with gains, as in the reference
    finally:
        _native.linear_forward = orig
    assert calls, "the fused kernel was not used"
    with torch.no_grad():
        ref = torch.nn.functional.linear(x.float(), layer.weight.float(), layer.bias.float())
    assert rel_l2(y.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("centered", [False, True])
def test_forward_fused_modulation_on_chip(native_lib, centered):
    """The modulation term (alpha * offset added to every weight element,
    block_fht.py:448-449) is added to the generated panel inside the fused
    kernel; without gains the call's weight_scale scales the generated part
    only, as in the reference's forward_fused (block_fht.py:482-501)."""
    from latent_weight_lab import BlockFHTLinear, _native

    torch.manual_seed(12)
    layer = BlockFHTLinear(768, 3072, bias=True, latent_dim=32768, layers=3, seed=6, weight_scale=0.7,
                           modulation_alpha=0.02, modulation_centered=centered).cuda().bfloat16()
    with torch.no_grad():
        layer.bias.copy_(torch.randn(3072) * 0.1)
    x = torch.randn(2, 300, 768, device="cuda", dtype=torch.bfloat16)
    calls = []
    orig = _native.linear_forward
    _native.linear_forward = lambda *a, **k: calls.append(k.get("weight_offset")) or orig(*a, **k)
    try:
        y = layer.forward_fused(x, weight_scale=0.5)
    finally:
        _native.linear_forward = orig
    assert calls and calls[0] is not None, "the modulation offset did not reach the fused kernel"
    with torch.no_grad():
        gen = layer.generator().float().view(3072, 768)
        c = (layer.modulation_alpha * layer._modulation_offset()).float()
        w = 0.5 * 0.7 * gen + c
        ref = torch.nn.functional.linear(x.float(), w, layer.bias.float())
    assert rel_l2(y.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


@pytest.mark.parametrize("gains, alpha, ws", [(False, 0.0, 0.5), (False, 0.02, 1.0), (True, 0.02, 3.0)])
def test_forward_fused_residual_base_one_gemm(native_lib, gains, alpha, ws):
    """A residual-base layer (base + s * generated, block_fht.py:451-452) runs as
    one fused GEMM: the base panel is added to the generated panel on chip.
    Checked against the materialised weight (with gains the call's
    weight_scale is ignored, as in the reference)."""
    from latent_weight_lab import BlockFHTLinear, _native

    torch.manual_seed(13)
    layer = BlockFHTLinear(768, 1024, bias=True, latent_dim=32768, layers=3, seed=8, weight_scale=0.7,
                           modulation_alpha=alpha, residual_base_scale=0.3, output_gain=gains,
                           input_gain=gains).cuda().bfloat16()
    with torch.no_grad():
        layer.bias.copy_(torch.randn(1024) * 0.1)
        if gains:
            layer.output_gain.copy_(torch.rand(1024) + 0.5)
            layer.input_gain.copy_(torch.rand(768) + 0.5)
    x = torch.randn(500, 768, device="cuda", dtype=torch.bfloat16)
    calls = []
    orig = _native.linear_forward
    _native.linear_forward = lambda *a, **k: calls.append(k.get("base")) or orig(*a, **k)
    try:
        y = layer.forward_fused(x, weight_scale=ws)
    finally:
        _native.linear_forward = orig
    assert calls and calls[0] is not None, "the residual base did not reach the fused kernel"
    with torch.no_grad():
        if gains:
            w = layer.weight.float()
        else:
            gen = layer.generator().float().view(1024, 768)
            c = (alpha * layer._modulation_offset()).float() if alpha else 0.0
            w = layer.residual_base_weight.float() + 0.3 * (ws * 0.7 * gen + c)
        ref = torch.nn.functional.linear(x.float(), w, layer.bias.float())
    assert rel_l2(y.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


def test_mlp_step_replays_as_cuda_graph(native_lib):
    """Forward + backward through BlockFHTLinear (generation, GEMMs, latent
    projections) captured in one CUDA graph gives the eager gradients."""
    from latent_weight_lab import BlockFHTLinear

    torch.manual_seed(7)
    up = BlockFHTLinear(768, 3072, latent_dim=32768, layers=3, seed=11).cuda().bfloat16()
    down = BlockFHTLinear(3072, 768, latent_dim=65536, layers=3, seed=12).cuda().bfloat16()  # large-block path
    x = torch.randn(512, 768, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    gy = torch.randn(512, 768, device="cuda", dtype=torch.bfloat16)

    def step():
        y = down(torch.nn.functional.gelu(up(x)))
        y.backward(gy)

    step()
    eager = [t.grad.clone() for t in (up.generator.latent, down.generator.latent, x)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        up.generator.latent.grad = down.generator.latent.grad = x.grad = None
        step()
    torch.cuda.current_stream().wait_stream(side)
    up.generator.latent.grad = down.generator.latent.grad = x.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    with torch.no_grad():
        x.mul_(1.0)  # inputs stay in place; the replay reads them
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    for ref, t in zip(eager, (up.generator.latent, down.generator.latent, x)):
        assert torch.equal(t.grad, ref)
