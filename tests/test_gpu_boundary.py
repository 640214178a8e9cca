"""The rest of GpuRasterizer's surface through the C ABI (diffrast-gpu/src/lib.rs):
single-scene backward with BackwardMode, the timed batched backward
(BackwardTimings), ReduceMode, is_discrete, tape/scratch sizes, the device
memory helpers bindings use, and the bounded host wait (POLL_TIMEOUT).
"""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

from conftest import assert_grads_close, assert_images_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def native():
    from diffrast import _native

    assert torch.cuda.is_available(), "GPU tests need CUDA"
    return _native


def test_single_scene_backward_in_both_modes(native, oracle):
    # backward / backward_with (lib.rs:503-604): Taped and Recompute give the
    # same results (the reference's own test, lib.rs:1279-1297), equal to the
    # oracle.
    from diffrast.scenes import uniform_scenes

    p = uniform_scenes(1, 60, 31)[0]
    target = oracle.render_batch(uniform_scenes(1, 60, 32), 41, 53, 0.004, (0.2, 0.1, 0.3))[0]
    P, Tg = torch.from_numpy(p).cuda(), torch.from_numpy(target).cuda()
    out = {}
    for mode in (native.BACKWARD_TAPED, native.BACKWARD_RECOMPUTE):
        out[mode] = native.backward_single(P, Tg, 0.004, (0.2, 0.1, 0.3), mode=mode,
                                           want_image=True)
    (lt, gt, it), (lr, gr, ir) = out[native.BACKWARD_TAPED], out[native.BACKWARD_RECOMPUTE]
    assert torch.equal(it, ir) and torch.equal(lt, lr)
    torch.testing.assert_close(gt, gr, rtol=1e-5, atol=1e-8)
    rl, rg, rimg = oracle.backward_batch(p[None], target[None], 0.004, (0.2, 0.1, 0.3),
                                         want_images=True)
    assert_images_close(ir.cpu().numpy()[None], rimg, "single-scene image")
    np.testing.assert_allclose(lr.cpu().numpy(), rl, rtol=1e-5)
    assert_grads_close(gr.cpu().numpy()[None], rg, "single-scene grads")
    with pytest.raises(ValueError):
        native.backward_single(P, Tg, 0.004, mode=7)


def test_timed_backward_reports_its_phases(native):
    # backward_many_timed (lib.rs:656-663): the same results as the untimed
    # host-buffer call, and a breakdown whose dispatch phase is the kernel.
    from diffrast.scenes import uniform_scenes

    p = torch.from_numpy(uniform_scenes(8, 128, 41)).pin_memory()
    tgt = torch.rand(8, 96, 96, 3, generator=torch.Generator().manual_seed(4)).pin_memory()
    l_ref, g_ref = native.loss_backward_host(p, tgt, 0.002)
    native.loss_backward_timed(p, tgt, 0.002)  # first call may grow the pool
    losses, grads, tm = native.loss_backward_timed(p, tgt, 0.002)
    torch.testing.assert_close(losses, l_ref, rtol=1e-6, atol=0)
    assert_grads_close(grads.numpy(), g_ref.numpy(), "timed vs pipelined")
    assert tm["pack_ms"] > 0 and tm["dispatch_ms"] > 0 and tm["readback_ms"] > 0
    assert tm["alloc_ms"] >= 0 and tm["loss_ms"] == 0
    assert abs(tm["total_ms"] - sum(v for k, v in tm.items() if k != "total_ms")) < 1e-3


def test_reduce_mode_is_accepted_and_changes_nothing(native):
    from diffrast.scenes import uniform_scenes

    P = torch.from_numpy(uniform_scenes(4, 50, 51)).cuda()
    tgt = torch.rand(4, 48, 40, 3, device="cuda")
    assert native.get_reduce_mode() == native.REDUCE_WORKGROUP
    la, ga = native.loss_backward(P, tgt, 0.005)
    try:
        native.set_reduce_mode(native.REDUCE_DIRECT)
        assert native.get_reduce_mode() == native.REDUCE_DIRECT
        lb, gb = native.loss_backward(P, tgt, 0.005)
    finally:
        native.set_reduce_mode(native.REDUCE_WORKGROUP)
    assert torch.equal(la, lb)
    torch.testing.assert_close(ga, gb, rtol=1e-5, atol=1e-8)
    with pytest.raises(ValueError):
        native.set_reduce_mode(5)


def test_device_queries_and_sizes(native):
    assert native.is_discrete(0)
    assert native.device_name(0)
    assert native.tape_bytes(128, 256, 256) == 128 * 256 * 256 * 12
    small = native.scratch_bytes(1, 64, 64, 64)   # one small scene: triangle split state
    large = native.scratch_bytes(32, 128, 256, 256)
    assert small > 0 and large > 0
    # 160-byte records and their 16-byte packed boxes, 8-byte loss partials per tile
    # and 4-byte counters per scene.
    assert large == 32 * 128 * (160 + 16) + 32 * 256 * 8 + 32 * 4


def test_device_memory_helpers_round_trip(native):
    # The calls a binding without its own CUDA runtime uses (the Rust shim).
    L = native.lib()
    dev = torch.device("cuda", 0)
    ctx = native.context(dev, torch.cuda.current_stream(dev).cuda_stream)
    src = np.arange(1000, dtype=np.float32)
    back = np.zeros_like(src)
    buf = ctypes.c_void_p()
    native.check(L.dr_device_alloc(ctx, src.nbytes, ctypes.byref(buf)))
    try:
        native.check(L.dr_memcpy(ctx, buf, src.ctypes.data_as(ctypes.c_void_p), src.nbytes,
                                 None))
        native.check(L.dr_memcpy(ctx, back.ctypes.data_as(ctypes.c_void_p), buf, src.nbytes,
                                 None))
        native.check(L.dr_stream_wait(None, 10.0))
    finally:
        native.check(L.dr_device_free(ctx, buf))
    assert np.array_equal(src, back)


def test_stream_wait_times_out_on_a_host_delay(native):
    # POLL_TIMEOUT semantics (lib.rs:223-229) without any GPU fault or spin:
    # a host function that sleeps 0.3 s is queued on the stream, so the stream
    # stays busy for that long with the device idle. A 0.05 s bounded wait must
    # return DR_TIMEOUT; a longer one then returns DR_OK.
    L = native.lib()
    cudart = None
    for name in ("libcudart.so.12", "libcudart.so"):
        try:
            cudart = ctypes.CDLL(name)
            break
        except OSError:
            continue
    if cudart is None:
        pytest.skip("no CUDA runtime library to queue a host function with")
    HOSTFN = ctypes.CFUNCTYPE(None, ctypes.c_void_p)

    @HOSTFN
    def sleeper(_):
        time.sleep(0.3)

    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    st = cudart.cudaLaunchHostFunc(ctypes.c_void_p(stream.cuda_stream), sleeper, None)
    assert st == 0
    t0 = time.perf_counter()
    assert L.dr_stream_wait(ctypes.c_void_p(stream.cuda_stream), 0.05) == native.TIMEOUT
    waited = time.perf_counter() - t0
    assert "did not finish" in L.dr_last_error().decode()
    assert L.dr_stream_wait(ctypes.c_void_p(stream.cuda_stream), 10.0) == native.OK
    assert 0.04 <= waited < 0.3
