"""ctypes binding of libdiffrast_cuda.so (the C ABI in include/diffrast_cuda.h).

Every hot-path call goes through here: torch supplies device memory and the
current CUDA stream; the library's sm_100a kernels do the work. There is no CPU
fallback. If the library is missing or no CUDA device is visible, the call
raises.
"""

from __future__ import annotations

import ctypes
import math
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdiffrast_cuda.so")

# dr_status (include/diffrast_cuda.h)
OK, INVALID_ARGUMENT, TOO_LARGE, NO_DEVICE, TIMEOUT, LAUNCH, COMM, OUT_OF_MEMORY, INTERNAL = range(9)
LAYOUT_BHWC, LAYOUT_BCHW = 0, 1
PATH_TILE, PATH_REGION, PATH_SPLIT, PATH_TILE_GATHER = 0, 1, 2, 3  # dr_path
BACKWARD_TAPED, BACKWARD_RECOMPUTE = 0, 1  # dr_backward_mode (BackwardMode)
REDUCE_DIRECT, REDUCE_WORKGROUP = 0, 1  # dr_reduce_mode (ReduceMode)
STOP_COMPLETED, STOP_CONVERGED, STOP_DIVERGED = 0, 1, 2
N_PARAMS = 10


class DiffrastError(RuntimeError):
    """A non-OK dr_status from the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class FitConfigC(ctypes.Structure):
    _fields_ = [
        ("iters", ctypes.c_int64),
        ("sigma_start", ctypes.c_float),
        ("sigma_end", ctypes.c_float),
        ("lr_pos", ctypes.c_float),
        ("lr_color", ctypes.c_float),
        ("lr_alpha", ctypes.c_float),
        ("patience", ctypes.c_int64),
        ("min_delta", ctypes.c_float),
    ]


class FitReportC(ctypes.Structure):
    _fields_ = [
        ("n_losses", ctypes.c_int64),
        ("best_iter", ctypes.c_int64),
        ("best_loss", ctypes.c_float),
        ("stop_reason", ctypes.c_int),
        ("config_error", ctypes.c_int),
    ]


class BackwardTimingsC(ctypes.Structure):
    """dr_backward_timings (BackwardTimings, diffrast-gpu/src/lib.rs:96-114)."""

    _fields_ = [("pack_ms", ctypes.c_float), ("alloc_ms", ctypes.c_float),
                ("dispatch_ms", ctypes.c_float), ("readback_ms", ctypes.c_float),
                ("loss_ms", ctypes.c_float)]


class PoolStatsC(ctypes.Structure):
    _fields_ = [("hits", ctypes.c_uint64), ("misses", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float

# name -> (restype, argtypes); kept in the order of include/diffrast_cuda.h.
SIGNATURES = {
    "dr_ctx_create": (_I, [_I, ctypes.POINTER(_P)]),
    "dr_ctx_destroy": (_I, [_P]),
    "dr_last_error": (ctypes.c_char_p, []),
    "dr_status_string": (ctypes.c_char_p, [_I]),
    "dr_params_per_triangle": (_I, []),
    "dr_version": (ctypes.c_char_p, []),
    "dr_device_name": (_I, [_I, ctypes.c_char_p, ctypes.c_size_t]),
    "dr_device_count": (_I, []),
    "dr_set_background_location": (_I, [_P, _I]),
    "dr_set_precision": (_I, [_P, _I]),
    "dr_set_triangle_split": (_I, [_P, _I]),
    "dr_query_path": (_I, [_P, _I, _I, _I, _I, ctypes.POINTER(_I)]),
    "dr_render": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
    "dr_loss_backward": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _P, _P]),
    "dr_loss_backward_host": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _P]),
    "dr_host_chunks": (_I, [_I, _P, _P]),
    "dr_grad_backward": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P]),
    "dr_loss_backward_sharded": (
        _I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _I, _I, _P, _P, _P]),
    "dr_triangle_block_forward": (
        _I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _I, _P, _P]),
    "dr_triangle_block_backward": (
        _I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _I, _P, _P, _I, _I, _P, _P, _P, _P]),
    "dr_mse_loss": (_I, [_P, _P, _P, _I, ctypes.c_int64, _P, _P]),
    "dr_adam_step": (
        _I, [_P, _P, _P, _P, _P, ctypes.c_int64, _F, _F, _F, ctypes.c_uint32, _F, _F, _F, _I, _P]),
    "dr_fit": (
        _I, [_P, _P, _I, _I, _P, _P, _I, ctypes.POINTER(FitConfigC), _P, _P, _P,
             ctypes.POINTER(FitReportC), _P]),
    "dr_loss_backward_noalloc": (
        _I, [_P, _P, _I, _I, _I, _I, _F, _P, _I, _P, _P, _P]),
    "dr_backward": (_I, [_P, _P, _P, _I, _I, _I, _F, _P, _I, _I, _P, _P, _P, _P]),
    "dr_set_reduce_mode": (_I, [_P, _I]),
    "dr_get_reduce_mode": (_I, [_P, ctypes.POINTER(_I)]),
    "dr_set_deterministic": (_I, [_P, _I]),
    "dr_pixel_tape_bytes": (ctypes.c_uint64, [_I, _I, _I]),
    "dr_render_taped": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _P, _P, _P]),
    "dr_grad_backward_taped": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _P]),
    "dr_get_deterministic": (_I, [_P, ctypes.POINTER(_I)]),
    "dr_loss_backward_timed": (
        _I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P,
             ctypes.POINTER(BackwardTimingsC), _P]),
    "dr_tape_bytes": (ctypes.c_uint64, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]),
    "dr_scratch_bytes": (ctypes.c_uint64, [_P, _I, _I, _I, _I]),
    "dr_is_discrete": (_I, [_I]),
    "dr_device_alloc": (_I, [_P, ctypes.c_size_t, ctypes.POINTER(_P)]),
    "dr_device_free": (_I, [_P, _P]),
    "dr_memcpy": (_I, [_P, _P, _P, ctypes.c_size_t, _P]),
    "dr_pool_stats_get": (_I, [_P, ctypes.POINTER(PoolStatsC)]),
    "dr_clear_pool": (_I, [_P]),
    "dr_stream_wait": (_I, [_P, ctypes.c_double]),
}

_lib = None
_lock = threading.Lock()
_ctxs: dict = {}


def lib():
    """The loaded library. Raises ImportError when it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python differentiable-rasterizer_b200/build_native.py` "
                        "(there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(status: int) -> None:
    if status == OK:
        return
    msg = lib().dr_last_error().decode(errors="replace")
    if status == INVALID_ARGUMENT or status == TOO_LARGE:
        raise ValueError(msg)
    raise DiffrastError(status, f"{lib().dr_status_string(status).decode()}: {msg}")


def device_count() -> int:
    return lib().dr_device_count()


def device_name(index: int = 0) -> str | None:
    buf = ctypes.create_string_buffer(256)
    if lib().dr_device_name(index, buf, 256) != OK:
        return None
    return buf.value.decode()


def _resolve_device(device: torch.device | None) -> torch.device:
    if device is None or device.type != "cuda":
        if device_count() == 0:
            raise DiffrastError(NO_DEVICE, "no CUDA device is visible (there is no CPU fallback)")
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cuda", device.index if device.index is not None else torch.cuda.current_device())


def context(device: torch.device, stream: int):
    """The dr_ctx for (device, stream): calls on one context share scratch, so
    each stream gets its own."""
    key = (device.index, stream)
    c = _ctxs.get(key)
    if c is None:
        with _lock:
            c = _ctxs.get(key)
            if c is None:
                h = _P()
                check(lib().dr_ctx_create(device.index, ctypes.byref(h)))
                if _precision != PRECISION_REFERENCE:
                    check(lib().dr_set_precision(h, _precision))
                if _split:
                    check(lib().dr_set_triangle_split(h, _split))
                if _deterministic:
                    check(lib().dr_set_deterministic(h, 1))
                _ctxs[key] = c = h
    return c


PRECISION_REFERENCE, PRECISION_STRICT, PRECISION_FAST = 0, 1, 2
_precision = PRECISION_REFERENCE


def set_precision(mode: int) -> None:
    """Soft-edge arithmetic for every context (dr_set_precision)."""
    global _precision
    _precision = int(mode)
    with _lock:
        for h in _ctxs.values():
            check(lib().dr_set_precision(h, _precision))


def get_precision() -> int:
    return _precision


_split = 0


def set_triangle_split(blocks: int) -> None:
    """Triangle-block split for every context (dr_set_triangle_split):
    0 automatic, 1 never, k exactly k blocks."""
    global _split
    _split = int(blocks)
    with _lock:
        for h in _ctxs.values():
            check(lib().dr_set_triangle_split(h, _split))


def query_path(B: int, T: int, height: int, width: int,
               device: torch.device | None = None) -> int:
    """dr_query_path: the kernel a loss/gradient call of this shape takes
    (PATH_TILE, PATH_REGION, PATH_SPLIT or PATH_TILE_GATHER)."""
    dev = _resolve_device(device)
    out = ctypes.c_int(-1)
    check(lib().dr_query_path(context(dev, _stream(dev)), B, T, height, width, ctypes.byref(out)))
    return out.value


def tape_bytes(n_tris: int, width: int, height: int) -> int:
    """dr_tape_bytes: what the reference's taped backward would store (this
    library stores no tape)."""
    return int(lib().dr_tape_bytes(n_tris, width, height))


def scratch_bytes(B: int, T: int, height: int, width: int,
                  device: torch.device | None = None) -> int:
    """dr_scratch_bytes: device scratch a loss/gradient call of this shape holds."""
    dev = _resolve_device(device)
    return int(lib().dr_scratch_bytes(context(dev, _stream(dev)), B, T, height, width))


def is_discrete(index: int = 0) -> bool:
    """dr_is_discrete (GpuRasterizer::is_discrete)."""
    v = lib().dr_is_discrete(index)
    if v < 0:
        raise DiffrastError(NO_DEVICE, f"no CUDA device {index}")
    return bool(v)


def set_reduce_mode(mode: int, device: torch.device | None = None) -> None:
    """dr_set_reduce_mode (ReduceMode): accepted for compatibility; both values
    run the same warp + shared-memory + one-atomic-per-CTA reduction."""
    dev = _resolve_device(device)
    check(lib().dr_set_reduce_mode(context(dev, _stream(dev)), int(mode)))


def get_reduce_mode(device: torch.device | None = None) -> int:
    dev = _resolve_device(device)
    out = ctypes.c_int(-1)
    check(lib().dr_get_reduce_mode(context(dev, _stream(dev)), ctypes.byref(out)))
    return out.value


_deterministic = False


def set_deterministic(on: bool) -> None:
    """Deterministic gradient sums for every context (dr_set_deterministic):
    bit-identical gradients call to call, fixed-point accumulation."""
    global _deterministic
    _deterministic = bool(on)
    with _lock:
        for h in _ctxs.values():
            check(lib().dr_set_deterministic(h, int(_deterministic)))


def get_deterministic() -> bool:
    return _deterministic


def shutdown() -> bool:
    """Destroy every context (diffrast_rs.shutdown_gpu, diffrast-py/src/lib.rs:435-444)."""
    if _lib is None:
        return False
    with _lock:
        had = bool(_ctxs)
        for h in _ctxs.values():
            _lib.dr_ctx_destroy(h)
        _ctxs.clear()
    return had


def pool_stats(device: torch.device | None = None):
    dev = _resolve_device(device)
    st = PoolStatsC()
    check(lib().dr_pool_stats_get(context(dev, _stream(dev)), ctypes.byref(st)))
    return {"hits": st.hits, "misses": st.misses, "bytes": st.bytes}


def clear_pool(device: torch.device | None = None) -> None:
    dev = _resolve_device(device)
    check(lib().dr_clear_pool(context(dev, _stream(dev))))


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _check_sigma(sigma: float) -> float:
    s = float(sigma)
    if not math.isfinite(s) or s <= 0.0:
        raise ValueError("sigma must be positive and finite")
    return s


def _bg_host(background, B: int):
    """Background as a host float array: 3 values, or (B, 3) per scene."""
    if isinstance(background, torch.Tensor):
        bg = background.detach().to("cpu", torch.float32).contiguous().reshape(-1)
    else:
        bg = torch.tensor(list(background) if not hasattr(background, "shape") else background,
                          dtype=torch.float32).reshape(-1)
    if bg.numel() == 3:
        return bg, 0
    if bg.numel() == 3 * B:
        return bg, 1
    raise ValueError("background must have 3 values or one RGB triple per scene")


def _as_cuda_f32(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    return t.detach().to(device=dev, dtype=torch.float32, non_blocking=True).contiguous()


# --- hot-path wrappers (tensors in, tensors out, all on one CUDA device) -----


def render(params: torch.Tensor, height: int, width: int, sigma: float, background=(0.0, 0.0, 0.0),
           layout: int = LAYOUT_BHWC, device: torch.device | None = None) -> torch.Tensor:
    """dr_render. Returns (B,H,W,3) or (B,3,H,W) f32 on the CUDA device."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device if device is not None else params.device)
    p = _as_cuda_f32(params, dev)
    B, T = p.shape[0], p.shape[1]
    shape = (B, 3, height, width) if layout == LAYOUT_BCHW else (B, height, width, 3)
    out = torch.empty(shape, dtype=torch.float32, device=dev)
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_render(context(dev, s), _ptr(p), _ptr(bg), per, B, T, height, width, sigma,
                          layout, _ptr(out), ctypes.c_void_p(s)))
    return out


def pixel_tape_bytes(B: int, height: int, width: int) -> int:
    """dr_pixel_tape_bytes: the compact forward tape's size."""
    return int(lib().dr_pixel_tape_bytes(B, height, width))


def render_taped(params: torch.Tensor, height: int, width: int, sigma: float,
                 background=(0.0, 0.0, 0.0), layout: int = LAYOUT_BHWC,
                 device: torch.device | None = None):
    """dr_render_taped: the image as `render` returns it, and the pixel tape
    (a uint8 device tensor) that `grad_backward_taped` reads back."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device if device is not None else params.device)
    p = _as_cuda_f32(params, dev)
    B, T = p.shape[0], p.shape[1]
    shape = (B, 3, height, width) if layout == LAYOUT_BCHW else (B, height, width, 3)
    out = torch.empty(shape, dtype=torch.float32, device=dev)
    tape = torch.empty(pixel_tape_bytes(B, height, width), dtype=torch.uint8, device=dev)
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_render_taped(context(dev, s), _ptr(p), _ptr(bg), per, B, T, height, width,
                                sigma, layout, _ptr(out), _ptr(tape), ctypes.c_void_p(s)))
    return out, tape


def grad_backward_taped(params: torch.Tensor, grad_images: torch.Tensor, tape: torch.Tensor,
                        sigma: float, background=(0.0, 0.0, 0.0), layout: int = LAYOUT_BHWC,
                        device: torch.device | None = None) -> torch.Tensor:
    """dr_grad_backward_taped: `grad_backward` with the forward read from the
    tape of `render_taped` (same params, sizes, sigma and background)."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device if device is not None else params.device)
    p = _as_cuda_f32(params, dev)
    g = _as_cuda_f32(grad_images, dev)
    B, T = p.shape[0], p.shape[1]
    if layout == LAYOUT_BCHW:
        H, W = g.shape[2], g.shape[3]
    else:
        H, W = g.shape[1], g.shape[2]
    if tape.device != dev or tape.numel() < pixel_tape_bytes(B, H, W):
        raise ValueError("tape does not belong to a render of this batch on this device")
    grads = torch.empty((B, T, N_PARAMS), dtype=torch.float32, device=dev)
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_grad_backward_taped(context(dev, s), _ptr(p), _ptr(bg), per, B, T, H, W,
                                       sigma, _ptr(g), layout, _ptr(tape), _ptr(grads),
                                       ctypes.c_void_p(s)))
    return grads


HOST_CHUNKS_MAX = 5  # DR_HOST_CHUNKS_MAX


def host_chunks(batch: int) -> list[tuple[int, int]]:
    """Scene ranges [lo, hi) that dr_loss_backward_host pipelines (dr_host_chunks):
    cuts at 1/16, 1/4, 1/2 and 3/4 of the batch (32 scenes: 2, 6, 8, 8, 8)."""
    lo = (ctypes.c_int * HOST_CHUNKS_MAX)()
    hi = (ctypes.c_int * HOST_CHUNKS_MAX)()
    n = lib().dr_host_chunks(int(batch), lo, hi)
    return [(lo[c], hi[c]) for c in range(n)]


def loss_backward_host(params: torch.Tensor, targets: torch.Tensor, sigma: float,
                       background=(0.0, 0.0, 0.0), layout: int = LAYOUT_BHWC,
                       device: torch.device | None = None):
    """dr_loss_backward_host: host tensors in, host tensors out.

    The library uploads the batch in scene chunks on a copy stream and runs
    each chunk's kernels and download as soon as its upload lands. Pinned
    inputs (``tensor.pin_memory()``) move at full PCIe rate, and the results
    then come back in pinned tensors. Returns (losses (B,), grads (B, T, 10))."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device)
    p = params.detach().to(torch.float32).contiguous()
    t = targets.detach().to(torch.float32).contiguous()
    if p.is_cuda or t.is_cuda:
        raise ValueError("loss_backward_host takes host tensors")
    B, T = p.shape[0], p.shape[1]
    H, W = (t.shape[2], t.shape[3]) if layout == LAYOUT_BCHW else (t.shape[1], t.shape[2])
    pin = p.is_pinned() and t.is_pinned()
    grads = torch.empty((B, T, N_PARAMS), dtype=torch.float32, pin_memory=pin)
    losses = torch.empty((B,), dtype=torch.float32, pin_memory=pin)
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_loss_backward_host(context(dev, s), _ptr(p), _ptr(bg), per, B, T, H, W, sigma,
                                      _ptr(t), layout, _ptr(grads), _ptr(losses),
                                      ctypes.c_void_p(s)))
    return losses, grads


def loss_backward(params: torch.Tensor, targets: torch.Tensor, sigma: float,
                  background=(0.0, 0.0, 0.0), layout: int = LAYOUT_BHWC, want_image: bool = False,
                  device: torch.device | None = None):
    """dr_loss_backward. Returns (losses (B,), grads (B,T,10)[, image]).

    With host tensors (and no image requested) the call runs on host buffers
    end to end (loss_backward_host, the upload pipelined with the
    computation) and returns host tensors."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device if device is not None else params.device)
    if (not want_image and not params.is_cuda and not targets.is_cuda and params.dim() == 3
            and params.shape[0] > 1 and params.shape[1] > 0):
        return loss_backward_host(params, targets, sigma, background, layout, dev)
    p = _as_cuda_f32(params, dev)
    t = _as_cuda_f32(targets, dev)
    B, T = p.shape[0], p.shape[1]
    if layout == LAYOUT_BCHW:
        H, W = t.shape[2], t.shape[3]
    else:
        H, W = t.shape[1], t.shape[2]
    grads = torch.empty((B, T, N_PARAMS), dtype=torch.float32, device=dev)
    losses = torch.empty((B,), dtype=torch.float32, device=dev)
    image = torch.empty_like(t) if want_image else None
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_loss_backward(context(dev, s), _ptr(p), _ptr(bg), per, B, T, H, W, sigma,
                                 _ptr(t), layout, _ptr(grads), _ptr(losses), _ptr(image),
                                 ctypes.c_void_p(s)))
    if want_image:
        return losses, grads, image
    return losses, grads


def backward_single(params: torch.Tensor, target: torch.Tensor, sigma: float,
                    background=(0.0, 0.0, 0.0), mode: int = BACKWARD_RECOMPUTE,
                    layout: int = LAYOUT_BHWC, want_image: bool = False,
                    device: torch.device | None = None):
    """dr_backward: one scene (T, 10) against one target (GpuRasterizer::backward_with).
    Returns (loss (1,), grads (T, 10)[, image])."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device if device is not None else params.device)
    p = _as_cuda_f32(params, dev)
    t = _as_cuda_f32(target, dev)
    if p.dim() != 2 or p.shape[1] != N_PARAMS:
        raise ValueError("params must be (T, 10)")
    T = p.shape[0]
    H, W = (t.shape[1], t.shape[2]) if layout == LAYOUT_BCHW else (t.shape[0], t.shape[1])
    grads = torch.empty((T, N_PARAMS), dtype=torch.float32, device=dev)
    loss = torch.empty((1,), dtype=torch.float32, device=dev)
    image = torch.empty_like(t) if want_image else None
    bg, _ = _bg_host(background, 1)
    s = _stream(dev)
    check(lib().dr_backward(context(dev, s), _ptr(p), _ptr(bg), T, H, W, sigma, _ptr(t), layout,
                            int(mode), _ptr(grads), _ptr(loss), _ptr(image), ctypes.c_void_p(s)))
    if want_image:
        return loss, grads, image
    return loss, grads


def loss_backward_timed(params: torch.Tensor, targets: torch.Tensor, sigma: float,
                        background=(0.0, 0.0, 0.0), layout: int = LAYOUT_BHWC,
                        device: torch.device | None = None):
    """dr_loss_backward_timed (backward_many_timed): host tensors in and out,
    phase by phase. Returns (losses, grads, timings dict in ms)."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device)
    p = params.detach().to(torch.float32).contiguous()
    t = targets.detach().to(torch.float32).contiguous()
    if p.is_cuda or t.is_cuda:
        raise ValueError("loss_backward_timed takes host tensors")
    B, T = p.shape[0], p.shape[1]
    H, W = (t.shape[2], t.shape[3]) if layout == LAYOUT_BCHW else (t.shape[1], t.shape[2])
    grads = torch.empty((B, T, N_PARAMS), dtype=torch.float32)
    losses = torch.empty((B,), dtype=torch.float32)
    bg, per = _bg_host(background, B)
    tm = BackwardTimingsC()
    s = _stream(dev)
    check(lib().dr_loss_backward_timed(context(dev, s), _ptr(p), _ptr(bg), per, B, T, H, W,
                                       sigma, _ptr(t), layout, _ptr(grads), _ptr(losses),
                                       ctypes.byref(tm), ctypes.c_void_p(s)))
    timings = {f: getattr(tm, f) for f, _ in BackwardTimingsC._fields_}
    timings["total_ms"] = sum(timings.values())
    return losses, grads, timings


def grad_backward(params: torch.Tensor, grad_images: torch.Tensor, sigma: float,
                  background=(0.0, 0.0, 0.0), layout: int = LAYOUT_BHWC,
                  device: torch.device | None = None) -> torch.Tensor:
    """dr_grad_backward. Returns grads (B,T,10)."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(device if device is not None else params.device)
    p = _as_cuda_f32(params, dev)
    g = _as_cuda_f32(grad_images, dev)
    B, T = p.shape[0], p.shape[1]
    if layout == LAYOUT_BCHW:
        H, W = g.shape[2], g.shape[3]
    else:
        H, W = g.shape[1], g.shape[2]
    grads = torch.empty((B, T, N_PARAMS), dtype=torch.float32, device=dev)
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_grad_backward(context(dev, s), _ptr(p), _ptr(bg), per, B, T, H, W, sigma,
                                 _ptr(g), layout, _ptr(grads), ctypes.c_void_p(s)))
    return grads


def loss_backward_sharded(params: torch.Tensor, targets: torch.Tensor, sigma: float, shard: int,
                          n_shards: int, background=(0.0, 0.0, 0.0), layout: int = LAYOUT_BHWC,
                          out=None):
    """dr_loss_backward_sharded. Returns (loss_sums (B,) f64, partial grads).

    ``out=(grads, sums)`` writes into caller-owned device tensors ((B, T, 10)
    f32 and (B,) f64, contiguous) instead of new ones."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(params.device)
    p = _as_cuda_f32(params, dev)
    t = _as_cuda_f32(targets, dev)
    B, T = p.shape[0], p.shape[1]
    H, W = (t.shape[2], t.shape[3]) if layout == LAYOUT_BCHW else (t.shape[1], t.shape[2])
    if out is None:
        grads = torch.empty((B, T, N_PARAMS), dtype=torch.float32, device=dev)
        sums = torch.empty((B,), dtype=torch.float64, device=dev)
    else:
        grads, sums = out
        if (grads.shape != (B, T, N_PARAMS) or grads.dtype != torch.float32
                or not grads.is_contiguous() or sums.shape != (B,)
                or sums.dtype != torch.float64 or not grads.is_cuda or not sums.is_cuda):
            raise ValueError("out must be ((B, T, 10) f32, (B,) f64) contiguous device tensors")
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_loss_backward_sharded(context(dev, s), _ptr(p), _ptr(bg), per, B, T, H, W,
                                         sigma, _ptr(t), layout, shard, n_shards, _ptr(grads),
                                         _ptr(sums), ctypes.c_void_p(s)))
    return sums, grads


TRIANGLE_BLOCK_STATE_FLOATS = 8  # DR_TRIANGLE_BLOCK_STATE_BYTES / 4


def triangle_block_state(params: torch.Tensor, height: int, width: int,
                         n_blocks: int) -> torch.Tensor:
    """A (n_blocks, B, H, W, 8) f32 buffer for the triangle-block calls."""
    dev = _resolve_device(params.device)
    B = params.shape[0]
    return torch.empty((n_blocks, B, height, width, TRIANGLE_BLOCK_STATE_FLOATS),
                       dtype=torch.float32, device=dev)


def triangle_block_forward(params: torch.Tensor, height: int, width: int, sigma: float,
                           n_blocks: int, block: int, state: torch.Tensor,
                           background=(0.0, 0.0, 0.0)) -> None:
    """dr_triangle_block_forward into state[block] (see triangle_block_state)."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(params.device)
    p = _as_cuda_f32(params, dev)
    B, T = p.shape[0], p.shape[1]
    if tuple(state.shape) != (n_blocks, B, height, width, TRIANGLE_BLOCK_STATE_FLOATS) or \
            not state.is_contiguous() or state.dtype != torch.float32 or state.device != dev:
        raise ValueError("state must come from triangle_block_state(params, H, W, n_blocks)")
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_triangle_block_forward(context(dev, s), _ptr(p), _ptr(bg), per, B, T, height,
                                          width, sigma, n_blocks, block, _ptr(state),
                                          ctypes.c_void_p(s)))


def triangle_block_backward(params: torch.Tensor, state: torch.Tensor, other: torch.Tensor,
                            sigma: float, n_blocks: int, block: int, background=(0.0, 0.0, 0.0),
                            layout: int = LAYOUT_BHWC, grad_input: bool = False,
                            want_image: bool = False):
    """dr_triangle_block_backward with every slice of `state` filled. Returns
    (losses (B,) or None, grads (B, T, 10) nonzero on block `block`[, image])."""
    sigma = _check_sigma(sigma)
    dev = _resolve_device(params.device)
    p = _as_cuda_f32(params, dev)
    o = _as_cuda_f32(other, dev)
    B, T = p.shape[0], p.shape[1]
    H, W = (o.shape[2], o.shape[3]) if layout == LAYOUT_BCHW else (o.shape[1], o.shape[2])
    if tuple(state.shape) != (n_blocks, B, H, W, TRIANGLE_BLOCK_STATE_FLOATS) or \
            not state.is_contiguous() or state.dtype != torch.float32 or state.device != dev:
        raise ValueError("state must come from triangle_block_state(params, H, W, n_blocks)")
    grads = torch.empty((B, T, N_PARAMS), dtype=torch.float32, device=dev)
    losses = None if grad_input else torch.empty((B,), dtype=torch.float32, device=dev)
    image = torch.empty_like(o) if want_image else None
    bg, per = _bg_host(background, B)
    s = _stream(dev)
    check(lib().dr_triangle_block_backward(context(dev, s), _ptr(p), _ptr(bg), per, B, T, H, W,
                                           sigma, n_blocks, block, _ptr(state), _ptr(o), layout,
                                           1 if grad_input else 0, _ptr(grads), _ptr(losses),
                                           _ptr(image), ctypes.c_void_p(s)))
    if want_image:
        return losses, grads, image
    return losses, grads


def mse_loss(images: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """dr_mse_loss over the leading (batch) dimension."""
    dev = _resolve_device(images.device)
    a = _as_cuda_f32(images, dev)
    b = _as_cuda_f32(targets, dev)
    if a.shape != b.shape:
        raise ValueError(f"shape mismatch {tuple(a.shape)} vs {tuple(b.shape)}")
    B = a.shape[0]
    n = a.numel() // max(B, 1)
    out = torch.empty((B,), dtype=torch.float32, device=dev)
    s = _stream(dev)
    check(lib().dr_mse_loss(context(dev, s), _ptr(a), _ptr(b), B, n, _ptr(out), ctypes.c_void_p(s)))
    return out


def adam_step(params: torch.Tensor, m: torch.Tensor, v: torch.Tensor, grads: torch.Tensor,
              step: int, lr_pos=0.004, lr_color=0.02, lr_alpha=0.01, beta1=0.9, beta2=0.999,
              eps=1e-8, project: bool = True) -> None:
    """dr_adam_step in place on contiguous f32 CUDA tensors."""
    for t in (params, m, v, grads):
        if t.device.type != "cuda" or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("adam_step needs contiguous float32 CUDA tensors")
    if not (params.numel() == m.numel() == v.numel() == grads.numel()):
        raise ValueError("gradient length mismatch")
    dev = params.device
    s = _stream(dev)
    check(lib().dr_adam_step(context(dev, s), _ptr(params), _ptr(m), _ptr(v), _ptr(grads),
                             params.numel(), lr_pos, lr_color, lr_alpha, step, beta1, beta2, eps,
                             1 if project else 0, ctypes.c_void_p(s)))


def fit(target: torch.Tensor, init_params: torch.Tensor, background, iters: int,
        sigma_start=0.02, sigma_end=0.0015, lr_pos=0.004, lr_color=0.02, lr_alpha=0.01,
        patience: int | None = 250, min_delta=1e-7):
    """dr_fit: the whole fit loop on the device. Returns a dict like FitReport."""
    dev = _resolve_device(target.device)
    t = _as_cuda_f32(target, dev)
    if t.dim() != 3 or t.shape[2] != 3:
        raise ValueError("target must be (H, W, 3)")
    p = _as_cuda_f32(init_params, dev).reshape(-1, N_PARAMS)
    T = p.shape[0]
    H, W = t.shape[0], t.shape[1]
    best = torch.empty_like(p)
    final = torch.empty_like(p)
    losses = torch.zeros(max(iters, 1), dtype=torch.float32)
    bg = torch.tensor(list(background), dtype=torch.float32)
    cfg = FitConfigC(iters, sigma_start, sigma_end, lr_pos, lr_color, lr_alpha,
                     -1 if patience is None else patience, min_delta)
    rep = FitReportC()
    s = _stream(dev)
    status = lib().dr_fit(context(dev, s), _ptr(t), H, W, _ptr(p), _ptr(bg), T, ctypes.byref(cfg),
                          _ptr(best), _ptr(final), ctypes.c_void_p(losses.data_ptr()),
                          ctypes.byref(rep), ctypes.c_void_p(s))
    check(status)
    n = rep.n_losses
    return {
        "losses": losses[:n].clone(),
        "best_params": best,
        "final_params": final,
        "best_iter": rep.best_iter,
        "best_loss": rep.best_loss,
        "stop_reason": rep.stop_reason,
    }
