"""The C ABI library loads and exports exactly what include/*.h declares.

CPU-only: no compute call is made. Without a GPU the context constructor must
report DR_NO_DEVICE rather than fall back to anything.
"""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO, has_gpu

HEADER_DIR = os.path.join(REPO, "include")


def declared_symbols():
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if fn.endswith(".h"):
            text = open(os.path.join(HEADER_DIR, fn)).read()
            names |= set(re.findall(r"^DR_API\s+[\w\s\*]+?\b(dr_\w+)\s*\(", text, re.M))
    return names


def test_header_declares_the_entry_points():
    names = declared_symbols()
    for required in ("dr_ctx_create", "dr_render", "dr_loss_backward", "dr_grad_backward",
                     "dr_mse_loss", "dr_adam_step", "dr_fit", "dr_loss_backward_sharded",
                     "dr_triangle_block_forward", "dr_triangle_block_backward",
                     "dr_loss_backward_host", "dr_host_chunks"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from diffrast import _native

    L = _native.lib()  # loads, and binds every signature in _native.SIGNATURES
    for name in declared_symbols():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert declared_symbols() <= exported
    # Nothing but the API leaks out of the library.
    assert all(n.startswith("dr_") for n in exported), sorted(n for n in exported
                                                             if not n.startswith("dr_"))


def test_python_binding_covers_the_header():
    from diffrast import _native

    assert declared_symbols() == set(_native.SIGNATURES)


def test_constants_and_strings():
    from diffrast import _native

    L = _native.lib()
    assert L.dr_params_per_triangle() == 10
    assert L.dr_version().decode()
    assert L.dr_status_string(_native.TIMEOUT).decode() == "timeout"


@pytest.mark.skipif(has_gpu(), reason="checks the no-device path")
def test_no_device_is_an_error_not_a_fallback():
    from diffrast import _native

    L = _native.lib()
    assert L.dr_device_count() == 0
    h = ctypes.c_void_p()
    st = L.dr_ctx_create(0, ctypes.byref(h))
    assert st == _native.NO_DEVICE
    assert L.dr_last_error().decode()


def test_argument_errors_need_no_device():
    from diffrast import _native

    L = _native.lib()
    # A null context is rejected before any CUDA call.
    assert L.dr_render(None, None, None, 0, 1, 1, 8, 8, 0.01, 0, None, None) == \
        _native.INVALID_ARGUMENT
    assert L.dr_adam_step(None, None, None, None, None, 1, 0.1, 0.1, 0.1, 1, 0.9, 0.999, 1e-8, 1,
                          None) == _native.INVALID_ARGUMENT
    assert L.dr_triangle_block_forward(None, None, None, 0, 1, 1, 8, 8, 0.01, 2, 0, None,
                                       None) == _native.INVALID_ARGUMENT
    assert L.dr_triangle_block_backward(None, None, None, 0, 1, 1, 8, 8, 0.01, 2, 1, None, None, 0,
                                        0, None, None, None, None) == _native.INVALID_ARGUMENT
    assert L.dr_loss_backward_host(None, None, None, 0, 1, 1, 8, 8, 0.01, None, 0, None, None,
                                   None) == _native.INVALID_ARGUMENT


def test_host_chunks_cover_the_batch_in_order():
    # dr_host_chunks is pure host logic: callable without a GPU.
    from diffrast._native import host_chunks

    assert host_chunks(0) == [] and host_chunks(1) == [(0, 1)]
    for b in range(2, 130):
        ch = host_chunks(b)
        assert ch[0][0] == 0 and ch[-1][1] == b
        assert all(lo < hi for lo, hi in ch)
        assert all(ch[i][1] == ch[i + 1][0] for i in range(len(ch) - 1))
        assert len(ch) <= 5
    assert [hi - lo for lo, hi in host_chunks(32)] == [2, 6, 8, 8, 8]


def test_reference_surface_without_a_device():
    # GpuRasterizer::tape_bytes is T * W * H * 3 * 4 (diffrast-gpu/src/lib.rs:391-393);
    # the other new entry points reject a null context before any CUDA call.
    from diffrast import _native

    L = _native.lib()
    assert L.dr_tape_bytes(512, 256, 256) == 512 * 256 * 256 * 3 * 4
    assert _native.tape_bytes(0, 8, 8) == 0
    assert L.dr_scratch_bytes(None, 1, 1, 8, 8) == 0
    assert L.dr_backward(None, None, None, 1, 8, 8, 0.01, None, 0, 0, None, None, None,
                         None) == _native.INVALID_ARGUMENT
    assert L.dr_set_reduce_mode(None, 0) == _native.INVALID_ARGUMENT
    tm = _native.BackwardTimingsC()
    assert L.dr_loss_backward_timed(None, None, None, 0, 1, 1, 8, 8, 0.01, None, 0, None, None,
                                    ctypes.byref(tm), None) == _native.INVALID_ARGUMENT
    assert L.dr_device_alloc(None, 16, ctypes.byref(ctypes.c_void_p())) == \
        _native.INVALID_ARGUMENT
    assert L.dr_memcpy(None, None, None, 4, None) == _native.INVALID_ARGUMENT
    if not has_gpu():
        assert L.dr_is_discrete(0) == -1


def _param_counts(text, pattern):
    out = {}
    for m in re.finditer(pattern, text, re.S | re.M):
        args = " ".join(m.group(2).split())
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def test_rust_ffi_block_matches_the_header():
    # bindings/rust/diffrast-cuda cannot be compiled in this image (no cargo);
    # its extern block must still declare every C entry point, each with the
    # header's number of parameters.
    header = open(os.path.join(HEADER_DIR, "diffrast_cuda.h")).read()
    ffi = open(os.path.join(REPO, "bindings", "rust", "diffrast-cuda", "src", "ffi.rs")).read()
    c = _param_counts(header, r"^DR_API\s+[\w\s\*]+?\b(dr_\w+)\s*\(([^)]*)\)")
    rs = _param_counts(ffi, r"pub fn (dr_\w+)\(([^)]*)\)")
    assert set(c) == declared_symbols()
    assert c == rs
