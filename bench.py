"""Benchmark: fwd+bwd pixel-triangle evaluations/s at B=32, T=128, 256x256.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward + per-image MSE + analytic backward over a batch of 32
seeded synthetic scenes (benchmark config 2's headline cell, sigma 0.0015),
through the C ABI (dr_loss_backward, the fused_loss_backward semantics). The
metric counts dense pairs B*T*H*W per step, as the reference's own
"fwd+bwd pixel*triangle evals/s" would.

Timing: W untimed warm-up steps; then K steps, each preceded by an untimed L2
flush (a 256 MiB write; the working set is smaller than the 126 MB L2), each
timed with CUDA events on the launching stream; barrier + synchronize around
the timed region; the MAX over ranks. Multi-GPU (torchrun): every rank runs its
own batch of 32 scenes (weak scaling, no data-path collective).

`e2e` is the same metric through the public torch API with host (pinned)
buffers: diffrast.torch_layer.fused_loss on CPU tensors, so every step copies
params + targets host->device and losses + grads device->host.

`--impl reference` times the reference's CPU algorithm (the C++ oracle port,
oracle/: the Rust crate cannot be built here) with every host thread, on the
same config and metric; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "differentiable-rasterizer_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

B, T, H, W, SIGMA = 32, 128, 256, 256, 0.0015
CELL = 5  # config 2 grid cell index for (T=128, 256^2)
METRIC = "fwd+bwd pixel*triangle evals/s (B=32,T=128,256^2)"
UNIT = "pair-evals/s"
FLOP_PER_PAIR = 170  # fwd 62 + bwd 108 FP32 FLOP per bounding-box pair
TRAFFIC_BYTES = 26_370_560  # DRAM bytes per raster launch (ncu, see roofline below)
REF_BUDGET_S = 120.0  # --impl reference: wall time all its steps share


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fit", action="store_true", help="skip the secondary fit metric")
    return ap.parse_args()


def dense_pairs(batch: int) -> int:
    return batch * T * H * W


def bbox_pairs(params: np.ndarray) -> int:
    """Bounding-box pairs (raster.rs:144-168 boxes of live triangles)."""
    from diffrast.scenes import bbox_pairs as count

    return count(params, W, H, SIGMA)


def inputs(rank: int):
    from diffrast.scenes import uniform_scenes

    params = uniform_scenes(B, T, 2000 + CELL + 1000 * rank)
    target_scenes = uniform_scenes(B, T, 3000 + CELL + 1000 * rank)
    return params, target_scenes


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r)
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows)}


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return {}


def cpu_reference_rate(params, target, threads: int = 0, max_scenes: int = B,
                       min_seconds: float = 10.0, max_steps: int = 50):
    """The oracle's fwd+loss+bwd on the host, whole steps repeated until
    min_seconds have passed (at most max_steps): (dense pairs/s, seconds,
    scenes per step, steps)."""
    import oracle

    oracle.build()
    p, t = params[:max_scenes], target[:max_scenes]
    steps = 0
    t0 = time.perf_counter()
    while steps < max_steps:
        oracle.backward_batch(p, t, SIGMA, threads=threads)
        steps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    dt = time.perf_counter() - t0
    return steps * dense_pairs(p.shape[0]) / dt, dt, p.shape[0], steps


def fit_metric(dev, with_cpu: bool):
    """Secondary benchmark metric: Adam fit iterations/s on config 1 (150
    triangles fitted to a 176x176 target for 800 iterations, FitConfig
    defaults), the whole loop on the device (dr_fit, one CUDA graph)."""
    import torch

    from diffrast import _native
    from diffrast.fit import mean_color, seed_colors
    from diffrast.scenes import config1_target_scene, seed_scene_geometry

    # The target is rendered by this library; the initial scene follows
    # fit.rs:356-385 (seed_colors / mean_color).
    t_dev = _native.render(torch.from_numpy(config1_target_scene(150, 0)).to(dev), 176, 176,
                           0.0015)[0].contiguous()
    target = t_dev.cpu().numpy()
    p = seed_scene_geometry(150, 1)
    seed_colors(target, p)
    bg = mean_color(target)
    p_dev = torch.from_numpy(p).to(dev)
    kw = dict(iters=800, patience=None)
    _native.fit(t_dev, p_dev, [float(v) for v in bg], **kw)  # capture + warm-up
    torch.cuda.synchronize(dev)
    reps = 3
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        rep = _native.fit(t_dev, p_dev, [float(v) for v in bg], **kw)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dt = e0.elapsed_time(e1) / 1e3 / reps
    out = {"metric": "Adam fit iters/s (config 1: T=150, 176x176, 800 iters)",
           "value": len(rep["losses"]) / dt, "unit": "iters/s",
           "timing": "CUDA events around dr_fit (one graph launch per 800-iteration fit)",
           "final_best_loss": rep["best_loss"]}
    if with_cpu:
        import oracle

        oracle.build()
        t0 = time.perf_counter()
        r = oracle.fit(target, p, bg, oracle.FitConfig(iters=200, patience=None))
        cdt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": len(r.losses) / cdt, "unit": "iters/s", "cores": 1,
                               "kind": "port", "sample": "first 200 of the 800 iterations, "
                                                         "single thread (Fitter is sequential)"}
    return out


def run_reference(args, rank: int, world: int):
    """--impl reference: the reference CPU algorithm, all host threads."""
    if rank != 0:
        return
    import oracle

    oracle.build()
    params, tscenes = inputs(0)
    target = oracle.render_batch(tscenes, H, W, SIGMA)
    threads = oracle.num_threads()
    # Each step is a bounded sample: the first n scenes of the batch, n chosen
    # from a timed full step so that all steps take about REF_BUDGET_S.
    t0 = time.perf_counter()
    oracle.backward_batch(params, target, SIGMA, threads=threads)
    full = time.perf_counter() - t0
    per_step = REF_BUDGET_S / max(args.steps + args.warmup, 1)
    n = max(1, min(B, int(B * per_step / max(full, 1e-9))))
    p_s, t_s = params[:n], target[:n]
    for _ in range(max(args.warmup, 0)):
        oracle.backward_batch(p_s, t_s, SIGMA, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.backward_batch(p_s, t_s, SIGMA, threads=threads)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    value = dense_pairs(n) / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded PCG64 scenes, config 2 distribution)",
        "config": {"workload": "config2 B=32 T=128 256x256 sigma=0.0015 fwd+mse+bwd",
                   "global_batch": B, "seq_len": None, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{n} of the {B} scenes per step (a full step takes "
                                   f"{full:.2f} s), {args.steps} steps"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference Rust crate cannot be built in this image (no cargo); timed the C++ "
                "restatement of its CPU path (oracle/diffrast_oracle.cpp)",
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        if args.impl == "ours":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))

    if args.impl == "reference":
        run_reference(args, rank, world)
        if dist is not None:
            dist.destroy_process_group()
        return

    from diffrast import _native
    from diffrast import torch_layer

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    params_np, tscenes_np = inputs(rank)
    P = torch.from_numpy(params_np).to(dev)
    TS = torch.from_numpy(tscenes_np).to(dev)
    target = _native.render(TS, H, W, SIGMA)  # targets = independent scenes rendered
    grads_dummy = None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return _native.loss_backward(P, target, SIGMA)

    for _ in range(max(args.warmup, 3)):
        grads_dummy = step()
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(local)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    times = []
    for _ in range(args.steps):
        flush.fill_(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        grads_dummy = step()
        e1.record(stream)
        times.append((e0, e1))
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clock_info = clocks.stop()
    total_ms = sum(a.elapsed_time(b) for a, b in times)
    t_ms = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t_ms, op=dist.ReduceOp.MAX)
    total_ms = float(t_ms.item())
    ms_per_step = total_ms / args.steps
    value = world * dense_pairs(B) / (ms_per_step / 1e3)
    del grads_dummy

    # e2e: public API with pinned host buffers (H2D of inputs, D2H of results).
    p_host = torch.from_numpy(params_np).pin_memory()
    t_host = target.cpu().pin_memory()
    # Warm-up creates the pipeline's streams, device buffers and pinned results.
    for _ in range(5):
        torch_layer.fused_loss(p_host, t_host, SIGMA)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    e2e_steps = max(3, min(args.steps, 50))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        losses_h, grads_h = torch_layer.fused_loss(p_host, t_host, SIGMA)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    h2d = p_host.numel() * 4 + t_host.numel() * 4
    d2h = losses_h.numel() * 4 + grads_h.numel() * 4

    if rank == 0:
        pk = peaks()
        n_bbox = bbox_pairs(params_np)
        sm_mhz = (clock_info or {}).get("sm_mhz") or pk.get("sm_max_mhz", 1965.0)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        fp32_peak = sms * 128 * 2 * sm_mhz * 1e6 / 1e12  # TFLOP/s at the sampled clock
        achieved = n_bbox * FLOP_PER_PAIR / (ms_per_step / 1e3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded PCG64 scenes, config 2 distribution)",
            "config": {"workload": "config2 B=32 T=128 256x256 sigma=0.0015 fwd+mse+bwd "
                                   "(dr_loss_backward)",
                       "global_batch": B * world, "seq_len": None,
                       "parallelism": f"batch-sharded x{world} (no collective)",
                       "l2": "flushed (256 MiB write) before every timed step"},
            "e2e": {"value": world * dense_pairs(B) / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "diffrast.torch_layer.fused_loss on pinned CPU tensors "
                           "(dr_loss_backward_host: chunked upload, kernels and download "
                           "in one call)"},
            "gpu_launches": 2 * args.steps,
            "roofline": {"bound": "fp32", "achieved": achieved, "peak": fp32_peak,
                         "unit": "TFLOP/s", "frac": achieved / fp32_peak,
                         # dram read + write of one raster launch, ncu capture in
                         # profiles/raster_kernel_config2_b32_t128_256.md
                         "traffic": TRAFFIC_BYTES,
                         "pairs_per_step": n_bbox, "flop_per_pair": FLOP_PER_PAIR,
                         "peak_source": f"nominal FP32 ({sms} SMs x 128 lanes x 2) at the "
                                        f"sampled SM clock {sm_mhz:.0f} MHz",
                         "timed": "whole step (set-up + raster kernels) per CUDA events"},
            "clocks": clock_info,
        }
        if not args.no_fit:
            line["secondary"] = fit_metric(dev, not args.no_cpu_baseline)
        if not args.no_cpu_baseline:
            import oracle

            tgt_np = target.cpu().numpy()
            thr = oracle.num_threads()
            rate, dt, ns, nsteps = cpu_reference_rate(params_np, tgt_np, threads=thr,
                                                      max_scenes=B)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": thr, "kind": "port",
                                    "sample": f"{nsteps} full steps of {ns} scenes ({dt:.1f} s "
                                              f"wall on {thr} threads), C++ restatement of the "
                                              "Rust CPU path"}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
