"""The compact pixel tape (dr_render_taped / dr_grad_backward_taped).

The taped render must return exactly dr_render's image; the taped backward,
exactly dr_grad_backward's gradients (bit for bit, with deterministic sums),
by reading each pixel's forward running product back from the tape. Tampering
with the tape shows that it is read; its per-region flags make the backward
recompute where the tape cannot stand in (a NaN-alpha triangle, which
render() paints and the backward drops), and shapes that do not take the
region kernel recompute everywhere.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def native():
    # Deterministic sums, so that taped and recomputed gradients compare bit
    # for bit rather than to the float atomics' summation order.
    from diffrast import _native

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    _native.set_deterministic(True)
    yield _native
    _native.set_deterministic(False)


def headline_like(B=32, T=128, seed=3):
    from diffrast.scenes import config2_params

    p, _ = config2_params(B, T, 5)
    return torch.from_numpy(p).cuda()


def test_taped_pair_matches_the_untaped_pair(native):
    P = headline_like()
    assert native.query_path(32, 128, 256, 256) == native.PATH_REGION
    for layout in (native.LAYOUT_BHWC, native.LAYOUT_BCHW):
        img = native.render(P, 256, 256, 0.0015, (0.1, 0.2, 0.3), layout)
        img_t, tape = native.render_taped(P, 256, 256, 0.0015, (0.1, 0.2, 0.3), layout)
        assert torch.equal(img, img_t)
        g_in = torch.randn(img.shape, device="cuda",
                           generator=torch.Generator(device="cuda").manual_seed(1)) * 1e-3
        g = native.grad_backward(P, g_in, 0.0015, (0.1, 0.2, 0.3), layout)
        g_t = native.grad_backward_taped(P, g_in, tape, 0.0015, (0.1, 0.2, 0.3), layout)
        assert torch.equal(g_t, g)


def test_the_tape_is_read_and_its_flags_are_honoured(native):
    P = headline_like()
    _, tape = native.render_taped(P, 256, 256, 0.0015)
    g_in = torch.randn((32, 256, 256, 3), device="cuda",
                       generator=torch.Generator(device="cuda").manual_seed(2)) * 1e-3
    ref = native.grad_backward(P, g_in, 0.0015)
    header = native.pixel_tape_bytes(32, 256, 256) - 32 * 256 * 256 * 16
    body = tape[header:].view(torch.float32).view(32, 256, 256, 4)
    body[..., 0] *= 0.5  # every pixel's running product halved
    bent = native.grad_backward_taped(P, g_in, tape, 0.0015)
    assert not torch.allclose(bent, ref, rtol=1e-3, atol=1e-7)
    tape[:header].fill_(1)  # every region flagged: the backward recomputes
    back = native.grad_backward_taped(P, g_in, tape, 0.0015)
    assert torch.equal(back, ref)


def test_nan_alpha_regions_recompute(native):
    P = headline_like()
    P[3, 17, 9] = float("nan")  # render() paints it, the backward drops it
    img = native.render(P, 256, 256, 0.0015)
    img_t, tape = native.render_taped(P, 256, 256, 0.0015)
    assert torch.equal(torch.isnan(img), torch.isnan(img_t))
    ok = ~torch.isnan(img)
    assert torch.equal(img[ok], img_t[ok])
    header = native.pixel_tape_bytes(32, 256, 256) - 32 * 256 * 256 * 16
    assert int(tape[:header].view(torch.int32).ne(0).sum()) > 0  # its regions are flagged
    g_in = torch.randn((32, 256, 256, 3), device="cuda",
                       generator=torch.Generator(device="cuda").manual_seed(3)) * 1e-3
    g = native.grad_backward(P, g_in, 0.0015)
    g_t = native.grad_backward_taped(P, g_in, tape, 0.0015)
    assert torch.isfinite(g_t).all()
    assert torch.equal(g_t, g)


def test_shapes_off_the_region_kernel_recompute(native):
    from diffrast.scenes import uniform_scenes

    P = torch.from_numpy(uniform_scenes(3, 300, 5)).cuda()  # tile kernel
    assert native.query_path(3, 300, 96, 80) != native.PATH_REGION
    img = native.render(P, 96, 80, 0.003)
    img_t, tape = native.render_taped(P, 96, 80, 0.003)
    assert torch.equal(img, img_t)
    g_in = torch.randn((3, 96, 80, 3), device="cuda",
                       generator=torch.Generator(device="cuda").manual_seed(4)) * 1e-3
    g = native.grad_backward(P, g_in, 0.003)
    g_t = native.grad_backward_taped(P, g_in, tape, 0.003)
    assert torch.equal(g_t, g)
    with pytest.raises(ValueError):
        native.grad_backward_taped(P, g_in, tape[:16], 0.003)


def test_rasterize_backward_uses_the_tape(native, oracle):
    # torch_layer.rasterize keeps the tape when parameters need a gradient;
    # its gradients stay the oracle's.
    from diffrast import torch_layer

    from conftest import assert_grads_close

    p = headline_like(B=32, T=64)
    assert native.query_path(32, 64, 256, 256) == native.PATH_REGION  # the tape is kept
    target = torch.rand((32, 3, 256, 256), device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(5))
    q = p.clone().requires_grad_(True)
    loss = torch.nn.functional.mse_loss(torch_layer.rasterize(q, 256, 256, 0.0015), target)
    loss.backward()
    tgt_hwc = target.permute(0, 2, 3, 1).contiguous().cpu().numpy()
    ref_l, ref_g = oracle.backward_batch(p.cpu().numpy(), tgt_hwc, 0.0015)
    # F.mse_loss is the mean over B*3*H*W values; the oracle's per-scene MSE
    # gradients are per 3*H*W: scale by 1/B.
    assert_grads_close(q.grad.cpu().numpy(), ref_g / 32, "rasterize grads through the tape")
