"""Generates the golden fixtures in this directory.

Run once where a checkout of the reference repository is available; the
fixtures are committed and travel with the tests (the checkout does not):

    python tests/golden/make_golden.py --reference <path to the reference checkout>

reference_torch_helpers.npz
    Outputs of the reference's own Python helpers, imported from the checkout:
    torch_layer.random_params / clamp_params / psnr
    (python/diffrast/torch_layer.py:256-303) and TriangleNet.activate
    (python/diffrast/model.py:162-175), on seeded inputs. torch_layer imports
    the compiled extension diffrast_rs when it loads; a stand-in module that
    only answers params_per_triangle() takes its place, since none of these
    helpers calls into the extension. model.py is loaded by file path, without
    the package __init__ (which pulls in plotting modules).

oracle_cases.npz
    The CPU oracle's outputs (f32 path, the reference's rounding) on the
    reference's test scenes (grad.rs:329-346, tests/integration.rs:12-17) and
    on seeded scenes of the benchmark distributions, including degenerate,
    NaN-vertex and zero/one-alpha triangles: rendered images, per-scene MSE
    losses and parameter gradients (MSE against a target). They pin the oracle
    run to run and give the GPU tests fixed vectors.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [REPO, os.path.join(REPO, "differentiable-rasterizer_b200")]


def _load(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def reference_helpers(ref: str) -> dict:
    import torch

    stub = types.ModuleType("diffrast_rs")
    stub.params_per_triangle = lambda: 10
    stub.shutdown_gpu = lambda: None  # registered with atexit by torch_layer
    sys.modules["diffrast_rs"] = stub
    tl = _load(os.path.join(ref, "python", "diffrast", "torch_layer.py"), "ref_torch_layer")
    model = _load(os.path.join(ref, "python", "diffrast", "model.py"), "ref_model")

    out = {}
    for seed, (b, t) in ((0, (2, 5)), (7, (3, 16)), (123, (1, 64))):
        g = torch.Generator().manual_seed(seed)
        out[f"random_params_s{seed}"] = tl.random_params(b, t, generator=g).numpy()
    g = torch.Generator().manual_seed(11)
    wild = (torch.rand(4, 9, 10, generator=g) * 3.0 - 1.0)
    wild[0, 0, 0] = float("nan")
    out["clamp_in"] = wild.numpy()
    out["clamp_out"] = tl.clamp_params(wild).numpy()
    g = torch.Generator().manual_seed(2)
    raw = torch.randn(3, 8, 10, generator=g) * 3.0
    out["activate_in"] = raw.numpy()
    for vr in (0.15, 0.0, 0.3):
        net = model.TriangleNet.__new__(model.TriangleNet)
        net.vertex_range = vr
        out[f"activate_out_vr{vr}"] = model.TriangleNet.activate(net, raw).numpy()
    g = torch.Generator().manual_seed(5)
    a = torch.rand(2, 3, 8, 8, generator=g)
    b = torch.rand(2, 3, 8, 8, generator=g)
    out["psnr_a"], out["psnr_b"] = a.numpy(), b.numpy()
    out["psnr_ab"] = np.float32(tl.psnr(a, b).item())
    out["psnr_aa"] = np.float32(tl.psnr(a, a).item())
    return out


def tri(verts, color, alpha):
    return np.array(list(np.ravel(verts)) + list(color) + [alpha], dtype=np.float32)


def cases() -> list[dict]:
    """Inputs of the oracle cases: params, target params, size, sigma, background."""
    from diffrast.scenes import config5_params, uniform_scenes

    out = []
    # grad.rs:329-346 (the gradient tests' scene pair), 48x48, sigma 0.03.
    scene = np.stack([tri([[0.21, 0.34], [0.77, 0.26], [0.58, 0.72]], [0.7, 0.4, 0.3], 0.7),
                      tri([[0.18, 0.55], [0.66, 0.69], [0.44, 0.24]], [0.3, 0.5, 0.8], 0.5)])
    target = np.stack([tri([[0.25, 0.30], [0.80, 0.22], [0.55, 0.78]], [0.9, 0.3, 0.2], 0.8),
                       tri([[0.15, 0.60], [0.70, 0.65], [0.40, 0.20]], [0.2, 0.6, 0.9], 0.6)])
    out.append(dict(name="grad_rs_pair", params=scene[None], target=target[None], h=48, w=48,
                    sigma=0.03, bg=(0.1, 0.12, 0.15)))
    # tests/integration.rs:12-17, 64x64 at the default sigma.
    ref = np.stack([tri([[0.20, 0.25], [0.80, 0.30], [0.50, 0.80]], [0.90, 0.30, 0.20], 0.9),
                    tri([[0.30, 0.55], [0.85, 0.60], [0.60, 0.15]], [0.20, 0.60, 0.90], 0.7)])
    out.append(dict(name="integration_scene", params=ref[None], target=scene[None], h=64, w=64,
                    sigma=0.0015, bg=(0.10, 0.11, 0.14)))
    # Benchmark distribution (config 2), small: B=3, T=40, 40x56 (not multiples of 16).
    out.append(dict(name="uniform_b3_t40", params=uniform_scenes(3, 40, 9001),
                    target=uniform_scenes(3, 40, 9002), h=40, w=56, sigma=0.0015,
                    bg=(0.0, 0.0, 0.0)))
    # Soft edges wide enough that most pixels are in a band, per-scene background.
    out.append(dict(name="uniform_wide_sigma", params=uniform_scenes(2, 24, 9003),
                    target=uniform_scenes(2, 24, 9004), h=33, w=47, sigma=0.02,
                    bg=np.array([[0.2, 0.3, 0.4], [0.9, 0.1, 0.5]], dtype=np.float32)))
    # Config 5 stress (degenerate, coincident, alpha 0 and 1), cropped to T=256.
    p5 = config5_params(1, 256, 5100)
    t5 = config5_params(1, 256, 5101)
    out.append(dict(name="stress_t256", params=p5, target=t5, h=64, w=64, sigma=0.0015,
                    bg=(0.0, 0.0, 0.0)))
    # Hand-made edge cases: NaN vertex, NaN alpha, off-screen, alpha 0 / 1 / tiny.
    e = uniform_scenes(1, 8, 9005)
    e[0, 0, 0] = np.nan
    e[0, 1, 9] = np.nan
    e[0, 2, :6] = [2.0, 2.0, 2.5, 2.0, 2.2, 2.6]
    e[0, 3, 9] = 0.0
    e[0, 4, 9] = 1.0
    e[0, 5, 9] = 5e-7
    out.append(dict(name="edge_cases", params=e, target=uniform_scenes(1, 8, 9006), h=24, w=20,
                    sigma=0.01, bg=(0.05, 0.05, 0.05)))
    return out


def oracle_cases() -> dict:
    import oracle

    oracle.build()
    out = {}
    for c in cases():
        n = c["name"]
        tgt = oracle.render_batch(c["target"], c["h"], c["w"], c["sigma"], c["bg"])
        img = oracle.render_batch(c["params"], c["h"], c["w"], c["sigma"], c["bg"])
        losses, grads = oracle.backward_batch(c["params"], tgt, c["sigma"], c["bg"])
        out[f"{n}/params"] = c["params"]
        out[f"{n}/target"] = tgt
        out[f"{n}/sigma"] = np.float32(c["sigma"])
        out[f"{n}/background"] = np.asarray(c["bg"], dtype=np.float32)
        out[f"{n}/image"] = img
        out[f"{n}/losses"] = losses
        out[f"{n}/grads"] = grads
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True, help="path to the reference checkout")
    args = ap.parse_args()
    np.savez_compressed(os.path.join(HERE, "reference_torch_helpers.npz"),
                        **reference_helpers(args.reference))
    np.savez_compressed(os.path.join(HERE, "oracle_cases.npz"), **oracle_cases())
    for f in ("reference_torch_helpers.npz", "oracle_cases.npz"):
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
