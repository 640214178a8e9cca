"""The allocation-free entry point agrees with the regular one.

Some callers of this library cannot allocate GPU memory while they run:
cudaMalloc synchronizes the whole device and can stall for milliseconds, which
an interactive fit that steps once per displayed frame, or a serving loop with
a latency deadline, cannot afford; and some host applications hand out device
memory only from a fixed budget they manage themselves. For them the library
exports dr_loss_backward_noalloc, which takes its scratch from a static array
instead of a context's pool. These tests call it through the C ABI and check
its losses and gradients against dr_loss_backward's, on two calls in a row:
the second call reuses the array the first one left behind, so stale contents
(for example the per-scene tile counters) must not leak into its results.

The cases cover both image layouts, a background given or not (black), the
losses output given or not, scenes without triangles, and one launch large
enough (32 scenes of 256x256, 128 triangles) to take the region kernel, whose
per-region loss partials then live in the static array too.

The file name sorts last so that a stop-at-first-failure run has already run
every other test before this one.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import assert_grads_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


CASES = [
    # B, T, H, W, sigma, layout, background, want_losses
    (4, 96, 70, 90, 0.004, "bhwc", (0.1, 0.2, 0.3), True),
    (4, 96, 70, 90, 0.004, "bchw", (0.1, 0.2, 0.3), True),
    (3, 40, 33, 47, 0.01, "bhwc", None, True),
    (3, 40, 33, 47, 0.01, "bchw", None, False),
    (2, 0, 24, 20, 0.01, "bhwc", (0.3, 0.2, 0.1), True),
    (32, 128, 256, 256, 0.0015, "bhwc", None, True),
]


@pytest.mark.parametrize("B,T,H,W,sigma,layout,bg_values,want_losses", CASES)
def test_noalloc_matches_the_regular_entry_point_twice(B, T, H, W, sigma, layout, bg_values,
                                                        want_losses):
    from diffrast import _native
    from diffrast.scenes import uniform_scenes

    assert torch.cuda.is_available(), "GPU test"
    L = _native.lib()
    lay = _native.LAYOUT_BCHW if layout == "bchw" else _native.LAYOUT_BHWC
    bg = (ctypes.c_float * 3)(*bg_values) if bg_values is not None else None
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        params = (torch.from_numpy(uniform_scenes(B, T, 200 + call)).cuda() if T
                  else torch.zeros((B, 0, 10), device="cuda"))
        rng = np.random.default_rng(300 + call)
        shape = (B, 3, H, W) if lay == _native.LAYOUT_BCHW else (B, H, W, 3)
        target = torch.from_numpy(rng.uniform(0, 1, shape).astype(np.float32)).cuda()
        grads = torch.full((B, T, 10), float("nan"), device="cuda")
        losses = torch.full((B,), float("nan"), device="cuda") if want_losses else None
        status = L.dr_loss_backward_noalloc(
            _ptr(params), ctypes.cast(bg, ctypes.c_void_p) if bg is not None else None, B, T,
            H, W, sigma, _ptr(target), lay, _ptr(grads), _ptr(losses), ctypes.c_void_p(stream))
        assert status == _native.OK, L.dr_last_error().decode()
        ref_losses, ref_grads = _native.loss_backward(
            params, target, sigma, bg_values if bg_values is not None else (0.0, 0.0, 0.0),
            layout=lay)
        torch.cuda.synchronize()
        if want_losses:
            np.testing.assert_allclose(losses.cpu().numpy(), ref_losses.cpu().numpy(),
                                       rtol=1e-6)
        assert_grads_close(grads.cpu().numpy(), ref_grads.cpu().numpy(), f"call {call}")


def test_noalloc_rejects_work_beyond_its_static_scratch():
    from diffrast import _native

    L = _native.lib()
    B, T = 2, 16384  # B * T above DR_NOALLOC_MAX_TRIANGLES
    params = torch.zeros((B, T, 10), device="cuda")
    target = torch.zeros((B, 8, 8, 3), device="cuda")
    grads = torch.zeros((B, T, 10), device="cuda")
    status = L.dr_loss_backward_noalloc(_ptr(params), None, B, T, 8, 8, 0.01, _ptr(target),
                                        _native.LAYOUT_BHWC, _ptr(grads), None, None)
    assert status == _native.TOO_LARGE
    assert "DR_NOALLOC_MAX_TRIANGLES" in L.dr_last_error().decode()
