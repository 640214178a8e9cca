"""The soft-edge rounding helpers (csrc/dr_math.cuh) against CUDA's IEEE
operations, over 2^24 random inputs each.

div_rn_inv and sqrt_nr refine rcp.approx / rsqrt.approx with one Newton-Raphson
step and an FMA residual (Markstein's method): the refined value lies within
about 2^-44 of the exact result, so it rounds like __fdiv_rn / __fsqrt_rn except
for results that close to a rounding midpoint. sigmoid_rounded uses the fast
exponential, whose documented error grows with the argument (2 + 1.16 |x|
ulps); below zero the sigmoid is e / (1 + e) and inherits that error, above zero
it is 1 / (1 + e), where that error moves 1 + e by at most an ulp or two. The kernel evaluates the
sigmoid only for sd / sigma between about -14.2 (the reject line, ln(1e6) + 0.2)
and 16.8 (the accept line); farther out the line tests decide the pair. The test
bounds the sigmoid on that domain and reports the rest. The kernel is compiled here with nvcc from
tests/cuda/rounding_check.cu. Set DR_REPORT_DIR to write the counts as JSON.
"""

from __future__ import annotations

import ctypes
import json
import os
import shutil
import subprocess
import tempfile

import numpy as np
import pytest

from conftest import PKG, REPO

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

N = 1 << 24


def _build():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out = os.path.join(tempfile.mkdtemp(prefix="dr_rounding_"), "rounding_check.so")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "-shared", "-Xcompiler", "-fPIC", "-I", os.path.join(PKG, "csrc"), "-o", out,
                    os.path.join(REPO, "tests", "cuda", "rounding_check.cu")], check=True)
    lib = ctypes.CDLL(out)
    lib.rounding_check.restype = ctypes.c_int
    lib.rounding_check.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                   ctypes.c_void_p]
    return lib


def _ulps(got, ref):
    g = got.view(np.int32).astype(np.int64)
    r = ref.view(np.int32).astype(np.int64)
    # Map the sign-magnitude float bits onto a monotone integer line.
    g = np.where(g < 0, -(g & 0x7FFFFFFF), g)
    r = np.where(r < 0, -(r & 0x7FFFFFFF), r)
    return np.abs(g - r)


def test_rounding_helpers_against_ieee():
    assert torch.cuda.is_available()
    lib = _build()
    rng = np.random.default_rng(11)
    a = rng.normal(0.0, 1.0, N).astype(np.float32)
    # Divisors over many decades, both signs: the kernel divides by squared
    # edge lengths, distances down to 1e-9, sigma, and 1 + e in [1, 2].
    b = (rng.normal(0.0, 1.0, N) * np.exp(rng.uniform(-20, 20, N))).astype(np.float32)
    b[b == 0] = 1.0
    # One normal sample, scaled to the sigmoid's range of sd / sigma, is the
    # dividend, the square root's argument (its magnitude) and the sigmoid's.
    s = (a * 8.0).astype(np.float32)
    A = torch.from_numpy(s).cuda()
    Bt = torch.from_numpy(b).cuda()
    out = torch.empty(6 * N, dtype=torch.float32, device="cuda")
    assert lib.rounding_check(A.data_ptr(), Bt.data_ptr(), N, out.data_ptr()) == 0
    o = out.cpu().numpy().reshape(6, N)
    res = {}
    used = (s >= -14.5) & (s <= 17.0)  # the sigmoid's domain in the kernel
    for name, got, ref, sel in (("div_rn_inv", o[0], o[1], None), ("sqrt_nr", o[2], o[3], None),
                                ("sigmoid_rounded", o[4], o[5], used),
                                ("sigmoid_rounded x >= 0", o[4], o[5], used & (s >= 0)),
                                ("sigmoid_rounded all x", o[4], o[5], None)):
        keep = np.isfinite(ref) if sel is None else (np.isfinite(ref) & sel)
        assert np.array_equal(np.isfinite(got), np.isfinite(ref)), name
        u = _ulps(got[keep], ref[keep])
        res[name] = {"inputs": int(keep.sum()), "mismatches": int((u != 0).sum()),
                     "max_ulp": int(u.max())}
    # Below zero, the documented exponential error at the deepest argument used.
    neg = used & (s < 0)
    u_neg = _ulps(o[4][neg], o[5][neg])
    bound = 3 + np.floor(1.16 * np.abs(s[neg]))
    res["sigmoid_rounded x < 0 within 3 + 1.16|x| ulps"] = bool(np.all(u_neg <= bound))
    d = os.environ.get("DR_REPORT_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        with open(os.path.join(d, "rounding_helpers.json"), "w") as f:
            json.dump(res, f, indent=1)
    print(res)
    for name in ("div_rn_inv", "sqrt_nr"):
        assert res[name]["max_ulp"] <= 1, res
        assert res[name]["mismatches"] <= 1e-5 * N, res
    assert res["sigmoid_rounded x >= 0"]["max_ulp"] <= 2, res
    assert res["sigmoid_rounded x < 0 within 3 + 1.16|x| ulps"], res
