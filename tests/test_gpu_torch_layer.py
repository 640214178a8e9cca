"""The torch op contract on the GPU, restating python/test_torch_layer.py.

Differences from the reference's tests, by design of this build:
- ``device="cpu"`` raises instead of running a CPU rasterizer (there is no
  CPU path); the "CPU vs GPU gradients" checks compare against the CPU oracle.
- tensors stay on the GPU: CUDA params give CUDA outputs with no host copy.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_grads_close, assert_images_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
F = torch.nn.functional


@pytest.fixture(scope="module")
def tl():
    from diffrast import torch_layer

    assert torch.cuda.is_available()
    return torch_layer


def gen(seed):
    return torch.Generator().manual_seed(seed)


def test_output_shape_and_layout(tl):
    p = tl.random_params(3, 8, generator=gen(0))
    assert tl.rasterize(p, 16, 24).shape == (3, 3, 16, 24)
    assert tl.rasterize(p, 16, 24, channels_first=False).shape == (3, 16, 24, 3)
    a = tl.rasterize(p.cuda(), 16, 24)
    assert a.is_cuda and a.shape == (3, 3, 16, 24)
    b = tl.rasterize(p.cuda(), 16, 24, channels_first=False)
    assert torch.equal(a.permute(0, 2, 3, 1), b)


def test_render_is_differentiable(tl):
    p = tl.random_params(1, 4, generator=gen(0)).cuda().requires_grad_(True)
    tl.rasterize(p, 16, 16, sigma=0.03).sum().backward()
    assert p.grad is not None and p.grad.shape == p.shape
    assert torch.isfinite(p.grad).all()
    assert p.grad.abs().sum() > 0


def test_gradient_matches_numerical_differentiation(tl):
    # test_torch_layer.py:56-90: eps 5e-4, relative error < 2%, cosine > 0.999.
    eps, sigma = 5e-4, 0.03
    p = tl.random_params(1, 5, generator=gen(0)).cuda().requires_grad_(True)
    target = torch.rand(1, 3, 24, 24, generator=gen(1)).cuda()
    F.mse_loss(tl.rasterize(p, 24, 24, sigma=sigma), target).backward()
    analytic = p.grad.clone()
    numeric = torch.zeros_like(p)
    flat = numeric.view(-1)
    with torch.no_grad():
        base = p.detach().clone()
        for i in range(base.numel()):
            for sign in (1, -1):
                probe = base.clone().view(-1)
                probe[i] += sign * eps
                flat[i] += sign * F.mse_loss(tl.rasterize(probe.view_as(base), 24, 24, sigma=sigma),
                                             target)
        flat /= 2 * eps
    rel = ((analytic - numeric).norm() / numeric.norm()).item()
    cos = F.cosine_similarity(analytic.view(1, -1), numeric.view(1, -1)).item()
    assert rel < 0.02, rel
    assert cos > 0.999, cos


def test_gradient_descent_reduces_loss(tl):
    target = tl.rasterize(tl.random_params(1, 6, generator=gen(3)).cuda(), 32, 32,
                          sigma=0.002).detach()
    p = tl.random_params(1, 6, generator=gen(9)).cuda().requires_grad_(True)
    opt = torch.optim.Adam([p], lr=0.02)
    first = None
    for _ in range(60):
        opt.zero_grad()
        loss = F.mse_loss(tl.rasterize(p, 32, 32, sigma=0.03), target)
        loss.backward()
        opt.step()
        with torch.no_grad():
            p.copy_(tl.clamp_params(p))
        if first is None:
            first = loss.item()
    assert loss.item() < first * 0.7


def test_gradients_reach_an_upstream_network(tl):
    net = torch.nn.Linear(4, 6 * tl.N_PARAMS).cuda()
    params = net(torch.randn(2, 4, device="cuda")).view(2, 6, tl.N_PARAMS)
    tl.rasterize(params, 16, 16, sigma=0.03).mean().backward()
    assert net.weight.grad is not None
    assert torch.isfinite(net.weight.grad).all() and net.weight.grad.abs().sum() > 0


def test_rasterize_matches_the_cpu_oracle(tl, oracle):
    # Replaces test_rasterize_routes_to_the_requested_device: the CPU side of
    # the comparison is the oracle (the reference's CPU algorithm).
    p = tl.random_params(8, 128, generator=gen(0)).cuda().requires_grad_(True)
    out = tl.rasterize(p, 64, 64, sigma=0.02)
    assert tl.last_device() == "gpu"
    up = torch.randn_like(out) * 1e-3
    out.backward(up)
    pn = p.detach().cpu().numpy()
    ref = oracle.render_batch(pn, 64, 64, 0.02)
    assert_images_close(out.detach().permute(0, 2, 3, 1).cpu().numpy(), ref)
    up_hwc = up.permute(0, 2, 3, 1).contiguous().cpu().numpy()
    _, g_ref = oracle.backward_batch(pn, up_hwc, 0.02, mode=oracle.MODE_DIRECT_GRAD)
    assert_grads_close(p.grad.cpu().numpy(), g_ref)
    _, g_inv = oracle.backward_batch(pn, up_hwc, 0.02, mode=oracle.MODE_INVERT_GRAD)
    rel = np.abs(p.grad.cpu().numpy() - g_inv).max() / np.linalg.norm(g_inv)
    assert rel < 1e-3, rel  # the reference's CPU path inverts the gradient to a target


def test_cpu_device_is_an_error_not_a_fallback(tl):
    p = tl.random_params(2, 8, generator=gen(0))
    with pytest.raises(ValueError, match="no CPU rasterizer"):
        tl.rasterize(p, 16, 16, device="cpu")
    with pytest.raises(ValueError, match="no CPU rasterizer"):
        tl.fused_loss(p, torch.rand(2, 16, 16, 3), device="cpu")


def test_rejects_bad_shapes_and_sigma(tl):
    p = tl.random_params(1, 4, generator=gen(0))
    with pytest.raises(ValueError):
        tl.rasterize(p[..., :4], 16, 16)
    with pytest.raises(ValueError):
        tl.rasterize(p, 0, 16)
    with pytest.raises(ValueError):
        tl.rasterize(p, 16, 16, sigma=0.0)


def test_background_is_visible_where_nothing_is_drawn(tl):
    p = torch.tensor([[[5.0, 5.0, 5.1, 5.0, 5.05, 5.1, 1.0, 1.0, 1.0, 1.0]]])
    img = tl.rasterize(p, 8, 8, background=(0.25, 0.5, 0.75))
    assert abs(img[0, 0].mean().item() - 0.25) < 1e-5
    assert abs(img[0, 2].mean().item() - 0.75) < 1e-5


def test_fused_loss_matches_autograd_path(tl):
    p = tl.random_params(2, 5, generator=gen(0)).cuda()
    targets = torch.rand(2, 20, 20, 3, generator=gen(1)).cuda()
    losses, grads = tl.fused_loss(p, targets, sigma=0.03)
    pg = p.clone().requires_grad_(True)
    rendered = tl.rasterize(pg, 20, 20, sigma=0.03, channels_first=False)
    per_item = ((rendered - targets) ** 2).flatten(1).mean(1)
    per_item.sum().backward()
    torch.testing.assert_close(losses, per_item.detach(), rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(grads, pg.grad, rtol=1e-3, atol=1e-7)


def test_fused_loss_matches_the_cpu_oracle(tl, oracle):
    p = tl.random_params(8, 128, generator=gen(2)).cuda()
    targets = torch.rand(8, 64, 64, 3, generator=gen(3)).cuda()
    gpu_loss, gpu_grads = tl.fused_loss(p, targets, sigma=0.02)
    cpu_loss, cpu_grads = oracle.backward_batch(p.cpu().numpy(), targets.cpu().numpy(), 0.02)
    np.testing.assert_allclose(gpu_loss.cpu().numpy(), cpu_loss, rtol=1e-5, atol=1e-7)
    assert_grads_close(gpu_grads.cpu().numpy(), cpu_grads)
    rel = np.abs(cpu_grads - gpu_grads.cpu().numpy()).max() / np.linalg.norm(cpu_grads)
    assert rel < 1e-3
    # Bit-identical would mean one path silently ran the other's code.
    assert not np.array_equal(cpu_grads, gpu_grads.cpu().numpy())


def test_unknown_device_is_rejected(tl):
    p = tl.random_params(2, 8, generator=gen(0))
    with pytest.raises(ValueError):
        tl.fused_loss(p, torch.rand(2, 16, 16, 3), device="banana")


def test_rejects_bad_target_shape(tl):
    p = tl.random_params(1, 4, generator=gen(0))
    with pytest.raises(ValueError):
        tl.fused_loss(p, torch.rand(1, 3, 8, 8, 1))


def test_fused_mse_matches_rasterize_then_mse(tl):
    params = tl.random_params(4, 12, generator=gen(0)).cuda()
    target = tl.rasterize(tl.random_params(4, 12, generator=gen(1)).cuda(), 32, 32,
                          sigma=0.01).detach()
    a = params.clone().requires_grad_(True)
    F.mse_loss(tl.rasterize(a, 32, 32, sigma=0.01), target).backward()
    b = params.clone().requires_grad_(True)
    fused = tl.fused_mse(b, target, sigma=0.01)
    fused.backward()
    reference = F.mse_loss(tl.rasterize(params, 32, 32, sigma=0.01), target)
    assert abs(fused.item() - reference.item()) < 1e-6
    rel = (a.grad - b.grad).abs().max() / a.grad.norm().clamp_min(1e-12)
    assert rel.item() < 1e-4


def test_gradients_reach_a_network_through_the_fused_loss(tl):
    net = torch.nn.Linear(4, 6 * tl.N_PARAMS).cuda()
    target = torch.rand(2, 3, 16, 16, generator=gen(2)).cuda()
    tl.fused_mse(net(torch.randn(2, 4, device="cuda")).view(2, 6, tl.N_PARAMS), target,
                 sigma=0.02).backward()
    assert torch.isfinite(net.weight.grad).all() and net.weight.grad.abs().sum() > 0


def test_fused_mse_rejects_bad_shapes(tl):
    p = tl.random_params(2, 4, generator=gen(0))
    with pytest.raises(ValueError):
        tl.fused_mse(p, torch.rand(2, 16, 16, 3))
    with pytest.raises(ValueError):
        tl.fused_mse(p, torch.rand(2, 3, 16, 16), sigma=0.0)


def test_diffrast_rs_module_numpy_and_cuda_paths(oracle):
    import diffrast_rs

    p = np.ascontiguousarray(
        torch.cat([torch.rand(2, 6, 6), torch.rand(2, 6, 3), torch.rand(2, 6, 1) * 0.5 + 0.3],
                  -1).numpy(), dtype=np.float32)
    img = diffrast_rs.render_batch(p, 20, 24, 0.01, (0.1, 0.2, 0.3), "gpu")
    assert isinstance(img, np.ndarray) and img.shape == (2, 20, 24, 3)
    assert_images_close(img, oracle.render_batch(p, 20, 24, 0.01, (0.1, 0.2, 0.3)))
    targets = np.random.default_rng(0).uniform(0, 1, (2, 20, 24, 3)).astype(np.float32)
    losses, grads = diffrast_rs.fused_loss_backward(p, targets, 0.01, (0.1, 0.2, 0.3))
    ref_l, ref_g = oracle.backward_batch(p, targets, 0.01, (0.1, 0.2, 0.3))
    np.testing.assert_allclose(losses, ref_l, rtol=1e-5)
    assert_grads_close(grads, ref_g)
    g_in = np.random.default_rng(1).normal(0, 1e-4, (2, 20, 24, 3)).astype(np.float32)
    gb = diffrast_rs.backward_batch(p, g_in, 0.01, (0.1, 0.2, 0.3))
    _, ref_gb = oracle.backward_batch(p, g_in, 0.01, (0.1, 0.2, 0.3),
                                      mode=oracle.MODE_DIRECT_GRAD)
    assert_grads_close(gb, ref_gb)
    out = diffrast_rs.render_batch(torch.from_numpy(p).cuda(), 20, 24, 0.01, (0.1, 0.2, 0.3))
    assert out.is_cuda
    with pytest.raises(ValueError):
        diffrast_rs.render_batch(p, 20, 24, 0.0)
    with pytest.raises(ValueError):
        diffrast_rs.render_batch(p, 20, 24, 0.01, device="cpu")
    assert diffrast_rs.params_per_triangle() == 10
    assert diffrast_rs.gpu_adapter()


def test_config3_torch_op_path(tl, oracle):
    # Benchmark config 3: B=256, T=64, 128^2, params = activate(randn(seed 2)),
    # targets = random_params(seed 3) rendered at sigma 0.0015;
    # F.mse_loss(rasterize(params), targets).backward() vs the CPU op.
    raw = torch.randn(256, 64, 10, generator=gen(2))
    params = tl.activate(raw).cuda().requires_grad_(True)
    targets = tl.rasterize(tl.random_params(256, 64, generator=gen(3)).cuda(), 128, 128,
                           sigma=0.0015).detach()
    F.mse_loss(tl.rasterize(params, 128, 128, sigma=0.0015), targets).backward()
    pn = params.detach().cpu().numpy()
    n = 1.0 / (256 * 3 * 128 * 128)
    rendered = tl.rasterize(params.detach(), 128, 128, sigma=0.0015)
    up = (2.0 * n * (rendered - targets)).permute(0, 2, 3, 1).contiguous().cpu().numpy()
    _, g_ref = oracle.backward_batch(pn, up.astype(np.float32), 0.0015,
                                     mode=oracle.MODE_DIRECT_GRAD)
    assert_grads_close(params.grad.cpu().numpy(), g_ref, "config 3 grads")
    # Data-parallel form: 8 shards of 32 scenes, each loss scaled by B_local/B_global,
    # sum to the single-device gradient.
    total = torch.zeros_like(params.grad)
    for r in range(8):
        pr = params.detach()[32 * r:32 * (r + 1)].clone().requires_grad_(True)
        loss = F.mse_loss(tl.rasterize(pr, 128, 128, sigma=0.0015),
                          targets[32 * r:32 * (r + 1)]) * (32 / 256)
        loss.backward()
        total[32 * r:32 * (r + 1)] = pr.grad
    torch.testing.assert_close(total, params.grad, rtol=1e-4, atol=1e-8)  # atomic order
